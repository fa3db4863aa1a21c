// Fused MoE expert path on compressed pages: rANS page decode -> SwiGLU GEMV.
//
// Reference math (runtime/layer_runner.py run_moe_mlp :347-394, _swiglu
// :185-190; runtime/quant.py matmul :431-444): per layer
//   h      = rms_norm(x, w_post_ln)                              (BF16)
//   logits = h @ Wr.T                                            (BF16 result)
//   probs  = softmax(fp32(logits)); top-k; optional renormalisation
//   for each routed expert e (first-appearance order over positions, top-k slots):
//     g = h_e @ Wg.T, u = h_e @ Wu.T  (BF16 results, fp32 accumulation)
//     a = bf16(bf16(bf16(sigmoid(g)) * g) * u)
//     y = a @ Wd.T                                               (BF16)
//     out[pos] = bf16(out[pos] + bf16(y * w_bf16))
//   x_out = bf16(x + out)
//
// Expert weights stay compressed in HBM as VRN1 frames with a checkpoint
// index (every 256 symbols).  A CTA takes one tile of a projection (whole
// rows) for one routed expert; each lane pair decodes one 256-element
// segment of a row straight into fp32 dot products with the routed tokens'
// activations (read through L1), so decoded weights never touch HBM.  Every
// segment must land exactly on its successor checkpoint (integrity of the
// compressed page; the tile CRC-32 was verified when the index was built).
// Partial row sums meet in shared memory; the CTA applies the reference's
// BF16 rounding points.  Kernels: router, route plan, gate/up (one projection
// tile per CTA), activation, down, ordered combine.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "rans_core.cuh"

using namespace voom;
using namespace voom::rans;

namespace {

constexpr int kThreads = 256;
constexpr int kTok = 8;          // tokens per expert pass
constexpr int kMaxTK = 512;      // T * top_k
constexpr int kMaxE = 1024;      // experts

struct Routes {
  uint32_t n_unique;
  uint32_t T, k, pad;
  uint32_t expert[kMaxTK];      // unique experts in first-appearance order
  uint32_t ntok[kMaxTK];        // tokens routed to unique expert u
  uint32_t uoff[kMaxTK + 1];    // first route row of unique expert u
  uint32_t upair[kMaxTK];       // [uoff[u] + i] -> token of the i-th route of u
  uint32_t tok_order[kMaxTK];   // [t*k + j] -> route row, sorted by u per token
  uint16_t w_bf16[kMaxTK];      // [route row] route weight in BF16
  uint16_t pad2[kMaxTK];
  uint32_t idx[kMaxTK];         // [t*k + j] expert
  float w[kMaxTK];              // [t*k + j] route weight (fp32)
};

__device__ __forceinline__ float bf2f(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ uint32_t f2bf(float f) {  // round to nearest even
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u) return (u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// ------------------------------------------------------------------ router
// Two kernels.  moe_router_logits: grid (ceil(E / 16), T); each CTA applies
// the RMSNorm (optional) to its token and computes 16 experts' logits =
// h @ Wr.T rounded to BF16 (+ optional bias), one warp per two experts, 8
// weights per lane per step; CTA 0 of a token also writes h (BF16) for the
// expert kernels.  moe_router_topk: one CTA per token, fp32 softmax, top-k
// (largest first; ties -> lower expert id) by k rounds of block arg-max,
// optional renormalisation.
constexpr int kMaxH = 8192;
constexpr int kRouterExperts = 4;  // experts per logits CTA: two warps per expert, one half of H each

__global__ void __launch_bounds__(kThreads) moe_router_logits(const uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ norm_w, float eps,
                                                              const uint16_t* __restrict__ wr,
                                                              const float* __restrict__ bias, uint32_t E,
                                                              uint32_t H, uint16_t* __restrict__ h,
                                                              float* __restrict__ logits) {
  __shared__ float s_h[kMaxH];
  __shared__ float s_red[kThreads / 32];
  __shared__ float s_scale;
  const uint32_t t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t* xt = x + size_t(t) * H;
  if (norm_w) {
    float ss = 0.f;
    for (uint32_t i = tid; i < H; i += kThreads) {
      const float v = bf2f(xt[i]);
      ss += v * v;
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < kThreads / 32; w++) tot += s_red[w];
      s_scale = rsqrtf(tot / float(H) + eps);
    }
    __syncthreads();
  }
  const bool write_h = blockIdx.x == 0;
  uint16_t* ht = h + size_t(t) * H;
  for (uint32_t i = tid; i < H; i += kThreads) {
    const uint32_t hb = norm_w ? f2bf(bf2f(xt[i]) * s_scale * bf2f(norm_w[i])) : xt[i];
    if (write_h) ht[i] = uint16_t(hb);
    s_h[i] = bf2f(hb);
  }
  __syncthreads();
  const uint32_t e = blockIdx.x * kRouterExperts + (warp & 3u), half = warp >> 2;
  const uint32_t hmid = (H / 16) * 8;  // split point, a multiple of 8
  __shared__ float s_part[kThreads / 32];
  if (e < E) {
    const uint16_t* we = wr + size_t(e) * H;
    float acc = 0.f;
    for (uint32_t i = (half ? hmid : 0u) + lane * 8; i < (half ? H : hmid); i += 256) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(we + i));
      acc = fmaf(bf2f(w.x & 0xFFFFu), s_h[i], acc);
      acc = fmaf(__uint_as_float(w.x & 0xFFFF0000u), s_h[i + 1], acc);
      acc = fmaf(bf2f(w.y & 0xFFFFu), s_h[i + 2], acc);
      acc = fmaf(__uint_as_float(w.y & 0xFFFF0000u), s_h[i + 3], acc);
      acc = fmaf(bf2f(w.z & 0xFFFFu), s_h[i + 4], acc);
      acc = fmaf(__uint_as_float(w.z & 0xFFFF0000u), s_h[i + 5], acc);
      acc = fmaf(bf2f(w.w & 0xFFFFu), s_h[i + 6], acc);
      acc = fmaf(__uint_as_float(w.w & 0xFFFF0000u), s_h[i + 7], acc);
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) s_part[warp] = acc;
  }
  __syncthreads();
  if (e < E && half == 0 && lane == 0)
    logits[size_t(t) * E + e] = rbf(s_part[warp] + s_part[warp + 4]) + (bias ? bias[e] : 0.f);
}

// One CTA per token: fp32 softmax (max and sum as one warp over lanes
// e % 32), then every expert's rank in (probability desc, id asc) order --
// each thread compares its experts against all others -- and the k first
// become the routes.  A NaN probability ranks below every number.
constexpr int kTopkThreads = 256;

__global__ void __launch_bounds__(kTopkThreads) moe_router_topk(const float* __restrict__ logits, uint32_t E,
                                                                uint32_t k, uint32_t norm_topk, Routes* routes) {
  __shared__ float s_p[kMaxE];
  __shared__ float s_key[kMaxE];
  __shared__ int s_pick[64];
  __shared__ float s_mx, s_sm;
  const uint32_t t = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  for (uint32_t e = tid; e < E; e += kTopkThreads) s_p[e] = logits[size_t(t) * E + e];
  __syncthreads();
  if (tid < 32) {
    float mx = -INFINITY;
    for (uint32_t e = lane; e < E; e += 32) mx = fmaxf(mx, s_p[e]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) s_mx = mx;
  }
  __syncthreads();
  const float mx = s_mx;
  for (uint32_t e = tid; e < E; e += kTopkThreads) {
    const float p = __expf(s_p[e] - mx);
    s_p[e] = p;
    s_key[e] = p == p ? p : -2.f;
  }
  __syncthreads();
  if (tid < 32) {
    float sm = 0.f;
    for (uint32_t e = lane; e < E; e += 32) sm += s_p[e];
    for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
    if (lane == 0) s_sm = sm;
  }
  for (uint32_t e = tid; e < E; e += kTopkThreads) {
    const float v = s_key[e];
    uint32_t rank = 0;
    for (uint32_t q = 0; q < E; q++) {
      const float w = s_key[q];
      rank += (w > v || (w == v && q < e)) ? 1u : 0u;
    }
    if (rank < k) s_pick[rank] = int(e);
  }
  __syncthreads();
  if (tid == 0) {
    const float sm = s_sm;
    float sel = 0.f;
    for (uint32_t j = 0; j < k; j++) sel += s_p[s_pick[j]] / sm;
    for (uint32_t j = 0; j < k; j++) {
      const float pw = s_p[s_pick[j]] / sm;
      routes->idx[t * k + j] = uint32_t(s_pick[j]);
      routes->w[t * k + j] = norm_topk ? pw / sel : pw;
    }
  }
}

// Route plan, one CTA of kMaxTK threads (thread p = route position t*k + j):
// unique experts in first-appearance order (positions, then slots), tokens per
// expert, route rows grouped by expert in position order, and each token's
// contributions ordered by that expert order (the order the reference
// accumulates them in).
__global__ void __launch_bounds__(kMaxTK) moe_route_plan(Routes* r, uint32_t T, uint32_t k) {
  __shared__ uint32_t s_first[kMaxE];  // first position of each expert
  __shared__ uint32_t s_cnt[kMaxE];    // routes per expert
  __shared__ uint32_t s_idx[kMaxTK];
  __shared__ uint32_t s_u[kMaxTK];     // unique index of position p's expert
  __shared__ uint32_t s_scan[kMaxTK];
  __shared__ uint32_t s_ntok[kMaxTK];  // routes of unique expert u
  __shared__ uint32_t s_warp[kMaxTK / 32];
  __shared__ uint32_t s_nu;
  const uint32_t p = threadIdx.x, n = T * k, lane = p & 31, warp = p >> 5;
  for (uint32_t e = p; e < kMaxE; e += blockDim.x) {
    s_first[e] = 0xFFFFFFFFu;
    s_cnt[e] = 0;
  }
  __syncthreads();
  const uint32_t e = p < n ? r->idx[p] : 0u;
  if (p < n) {
    s_idx[p] = e;
    atomicMin(&s_first[e], p);
    atomicAdd(&s_cnt[e], 1u);
  }
  __syncthreads();
  // exclusive scan of "p is its expert's first position" -> unique index
  const uint32_t flag = (p < n && s_first[e] == p) ? 1u : 0u;
  uint32_t v = flag;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  uint32_t before = 0;
  for (uint32_t w = 0; w < warp; w++) before += s_warp[w];
  s_scan[p] = before + v - flag;
  __syncthreads();
  const uint32_t u = p < n ? s_scan[s_first[e]] : 0u;
  if (p < n) s_u[p] = u;
  if (flag) {
    r->expert[u] = e;
    r->ntok[u] = s_cnt[e];
    s_ntok[u] = s_cnt[e];
  }
  if (p == blockDim.x - 1) {
    s_nu = before + v;
    r->n_unique = before + v;
    r->T = T;
    r->k = k;
  }
  __syncthreads();
  // uoff: exclusive scan of ntok in unique order (thread u holds ntok[u])
  const uint32_t nu = s_nu;
  const uint32_t cnt_u = p < nu ? s_ntok[p] : 0u;
  uint32_t c = cnt_u;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, c, o);
    if (lane >= o) c += t;
  }
  __syncthreads();
  if (lane == 31) s_warp[warp] = c;
  __syncthreads();
  uint32_t base = 0;
  for (uint32_t w = 0; w < warp; w++) base += s_warp[w];
  if (p < nu) s_scan[p] = base + c - cnt_u;
  if (p == 0) r->uoff[0] = 0;
  if (p < nu) r->uoff[p + 1] = base + c;
  __syncthreads();
  if (p < n) {
    // route row: uoff[u] + earlier positions with the same expert
    uint32_t rank = 0;
    for (uint32_t q = 0; q < p; q++) rank += (s_idx[q] == e) ? 1u : 0u;
    const uint32_t row = s_scan[u] + rank;
    r->upair[row] = p / k;
    r->w_bf16[row] = uint16_t(f2bf(r->w[p]));
    // this token's routes ordered by unique index (experts of a token are distinct)
    const uint32_t t = p / k, t0 = t * k;
    uint32_t pos = 0;
    for (uint32_t j = 0; j < k; j++) pos += (s_u[t0 + j] < u) ? 1u : 0u;
    r->tok_order[t0 + pos] = row;
  }
}

// Route rows for experts given by the host: uoff from ntok.
__global__ void moe_route_offsets(Routes* r, uint32_t n_unique, uint32_t T) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  r->n_unique = n_unique;
  r->T = T;
  r->uoff[0] = 0;
  for (uint32_t u = 0; u < n_unique; u++) r->uoff[u + 1] = r->uoff[u] + r->ntok[u];
}

// -------------------------------------------------------- fused decode-GEMV
struct GemvShared {
  uint32_t lut[2][4096];
  uint32_t cum[2][257];
  uint32_t red[8];
  uint32_t degenerate[2];
  float acc[1][128][kTok];  // [0][row in tile][token]
  uint32_t tok[kTok];
  uint32_t status;
};

// 8 BF16 weights (one uint4) times 8 activations at column k of each token.
template <int NT>
__device__ __forceinline__ void dot8(const uint4 w, const uint16_t* __restrict__ act, uint32_t ld,
                                     const uint32_t* tok, uint32_t ntk, uint32_t k, float* acc) {
  const float w0 = bf2f(w.x & 0xFFFFu), w1 = __uint_as_float(w.x & 0xFFFF0000u);
  const float w2 = bf2f(w.y & 0xFFFFu), w3 = __uint_as_float(w.y & 0xFFFF0000u);
  const float w4 = bf2f(w.z & 0xFFFFu), w5 = __uint_as_float(w.z & 0xFFFF0000u);
  const float w6 = bf2f(w.w & 0xFFFFu), w7 = __uint_as_float(w.w & 0xFFFF0000u);
#pragma unroll
  for (int j = 0; j < NT; j++) {
    if (j < int(ntk)) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(act + size_t(tok[j]) * ld + k));
      float s = acc[j];
      s = fmaf(w0, bf2f(a.x & 0xFFFFu), s);
      s = fmaf(w1, __uint_as_float(a.x & 0xFFFF0000u), s);
      s = fmaf(w2, bf2f(a.y & 0xFFFFu), s);
      s = fmaf(w3, __uint_as_float(a.y & 0xFFFF0000u), s);
      s = fmaf(w4, bf2f(a.z & 0xFFFFu), s);
      s = fmaf(w5, __uint_as_float(a.z & 0xFFFF0000u), s);
      s = fmaf(w6, bf2f(a.w & 0xFFFFu), s);
      s = fmaf(w7, __uint_as_float(a.w & 0xFFFF0000u), s);
      acc[j] = s;
    }
  }
}

// Decodes tile `t` of one projection for the CTA's tokens and adds every
// row's dot products into sh.acc[slot].  Rows of `cols` elements; each lane
// pair owns one `every`-element segment.  Returns nothing; errors -> sh.status.
template <int NT>
__device__ void gemv_tile(GemvShared& sh, const voom_expert_proj& P, uint32_t t, int slot,
                          const uint16_t* __restrict__ act, uint32_t ld, uint32_t ntk) {
  const voom_rans_tile tl = P.tiles[t];
  const uint32_t row_bytes = 2u * P.cols, every = P.every;
  const uint32_t rows = tl.raw_len / row_bytes;
  const uint32_t spr = P.cols / every;  // segments per row
  const uint32_t nseg = rows * spr;
  const uint32_t tid = threadIdx.x, lane = tid & 1u, p = tid >> 1;
  if (tl.mode == 1) {
    build_lut(sh.lut[0], sh.cum[0], sh.red, &sh.degenerate[0], P.src + tl.low_freq);
    build_lut(sh.lut[1], sh.cum[1], sh.red, &sh.degenerate[1], P.src + tl.high_freq);
  }
  float acc[NT];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j] = 0.f;
  uint32_t row_local = 0;
  if (p < nseg) {
    row_local = p / spr;
    const uint32_t k0 = (p % spr) * every;
    if (tl.mode == 0) {  // stored tile: weights read directly
      const uint8_t* wsrc = P.src + tl.src + size_t(p) * every * 2;
      for (uint32_t c = lane * 8; c < every; c += 16) {
        uint4 w;
        uint32_t v[4];
        for (int q = 0; q < 4; q++)
          v[q] = uint32_t(wsrc[2 * (c + 2 * q)]) | (uint32_t(wsrc[2 * (c + 2 * q) + 1]) << 8) |
                 (uint32_t(wsrc[2 * (c + 2 * q) + 2]) << 16) | (uint32_t(wsrc[2 * (c + 2 * q) + 3]) << 24);
        w = make_uint4(v[0], v[1], v[2], v[3]);
        dot8<NT>(w, act, ld, sh.tok, ntk, k0 + c, acc);
      }
    } else {
      const uint32_t* ck = P.ckpt + P.ckpt_base[t];
      PlaneRun r;
      if (p == 0) {
        plane_start(r, P.src, lane ? tl.high_freq : tl.low_freq, lane ? tl.high_payload : tl.low_payload, 0, 0,
                    false);
      } else {
        plane_start(r, P.src, lane ? tl.high_freq : tl.low_freq, lane ? tl.high_payload : tl.low_payload,
                    ck[(p - 1) * 4 + lane * 2], ck[(p - 1) * 4 + lane * 2 + 1], true);
      }
      const uint32_t lut_s = uint32_t(__cvta_generic_to_shared(&sh.lut[lane][0]));
      const unsigned mask = 0x3u << (tid & 30u);
      const bool degenerate = sh.degenerate[lane] != 0;
      const bool last = (p + 1 == nseg);
      const uint32_t x0 = r.x, c0 = r.cur;
      auto landed = [&]() {
        return last ? (r.cur == r.len) : (r.x == ck[p * 4 + lane * 2] && r.cur == ck[p * 4 + lane * 2 + 1]);
      };
      // Whole segment on the clamped window; a pair that does not land where
      // the exact decoder did (a stream that runs out of bytes) redoes the
      // segment on the exact path.
      bool exact = (every & 15u) || !__all_sync(mask, !degenerate && win_can_open(r));
      if (!exact) {
        Window W;
        win_open(W, r);
        uint32_t x = r.x;
        for (uint32_t done = 0; done < every; done += 16) {
          uint32_t a[4];
          win_decode16(lut_s, x, W, a);
          const uint4 w = exchange_pair16(lane, a[0], a[1], a[2], a[3], mask);
          dot8<NT>(w, act, ld, sh.tok, ntk, k0 + done + 8 * lane, acc);
        }
        r.x = x;
        r.cur = win_cur(W);
        if (__any_sync(mask, !landed())) {
          exact = true;
          r.x = x0;
          r.cur = c0;
#pragma unroll
          for (int j = 0; j < NT; j++) acc[j] = 0.f;
        }
      }
      if (exact) {  // lockstep pair: both planes decode `every` symbols
        for (uint32_t done = 0; done < every; done++) {
          const uint32_t s = rans_step_exact(lut_s, degenerate, r);
          const uint32_t o = __shfl_xor_sync(mask, s, 1);
          if (lane == 0) {
            const float w = bf2f(s | (o << 8));
#pragma unroll
            for (int j = 0; j < NT; j++)
              if (j < int(ntk)) acc[j] = fmaf(w, bf2f(act[size_t(sh.tok[j]) * ld + k0 + done]), acc[j]);
          }
        }
        if (!landed()) atomicOr(&sh.status, 1u);
      }
    }
  }
  // pair reduce, then rows meet in shared memory
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], 1);
  if (p < nseg && lane == 0) {
#pragma unroll
    for (int j = 0; j < NT; j++)
      if (j < int(ntk)) atomicAdd(&sh.acc[slot][row_local][j], acc[j]);
  }
  __syncthreads();
}

// Bit 2 of the status word: an expert has more route rows than the grid's
// token groups cover (more tokens than T for one expert).
constexpr uint32_t kStatusRoutes = 2u;

template <int NT>
__device__ __forceinline__ bool setup_tokens(GemvShared& sh, const Routes* R, uint32_t u, uint32_t grp,
                                             uint32_t* ntk_out, uint32_t* status) {
  if (u >= R->n_unique) return false;
  const uint32_t n = R->ntok[u];
  if (threadIdx.x == 0 && blockIdx.x == 0 && grp == 0 && n > gridDim.z * NT) atomicOr(status, kStatusRoutes);
  if (grp * NT >= n) return false;
  const uint32_t ntk = min(uint32_t(NT), n - grp * NT);
  if (threadIdx.x < NT)
    sh.tok[threadIdx.x] = threadIdx.x < ntk ? R->upair[R->uoff[u] + grp * NT + threadIdx.x] : 0;
  *ntk_out = ntk;
  return true;
}

// One gate or up tile of one routed expert (blockIdx.x = 2 * tile + proj) ->
// BF16 rows g (gate) or u (up) per token; moe_act combines them.  NT = tokens
// per CTA (1, 2, 4 or 8): registers scale with it.
template <int NT>
__global__ void __launch_bounds__(kThreads, 4) moe_gate_up(const voom_expert_pages* __restrict__ pages,
                                                           const Routes* __restrict__ R,
                                                           const uint16_t* __restrict__ h, uint32_t H, uint32_t I,
                                                           uint16_t* __restrict__ g_out,
                                                           uint16_t* __restrict__ u_out, uint32_t* status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  GemvShared& sh = *reinterpret_cast<GemvShared*>(smem_raw);
  const uint32_t t = blockIdx.x >> 1, proj = blockIdx.x & 1u, u = blockIdx.y, grp = blockIdx.z;
  uint32_t ntk;
  if (!setup_tokens<NT>(sh, R, u, grp, &ntk, status)) return;
  const voom_expert_pages& E = pages[R->expert[u]];
  const voom_expert_proj& P = proj ? E.up : E.gate;
  if (t >= P.n_tiles) return;
  for (int i = threadIdx.x; i < 128 * kTok; i += kThreads) (&sh.acc[0][0][0])[i] = 0.f;
  if (threadIdx.x == 0) sh.status = 0;
  __syncthreads();
  gemv_tile<NT>(sh, P, t, 0, h, H, ntk);
  const voom_rans_tile tl = P.tiles[t];
  const uint32_t rows = tl.raw_len / (2u * H), row0 = uint32_t(tl.dst / (2u * H));
  uint16_t* out = proj ? u_out : g_out;
  for (uint32_t q = threadIdx.x; q < rows * ntk; q += kThreads) {
    const uint32_t row = q / ntk, j = q % ntk;
    out[size_t(R->uoff[u] + grp * NT + j) * I + row0 + row] = uint16_t(f2bf(sh.acc[0][row][j]));
  }
  if (threadIdx.x == 0 && sh.status) atomicOr(status, 1u);
}

// SwiGLU of the route rows, in place over g: a = bf16(bf16(bf16(sigmoid(g)) * g) * u)
// (layer_runner.py _swiglu :185-190).  8 columns per thread.
__global__ void moe_act(const Routes* __restrict__ R, uint16_t* __restrict__ g, const uint16_t* __restrict__ up,
                        uint32_t I) {
  const uint32_t row = blockIdx.y;
  if (row >= R->uoff[R->n_unique]) return;
  const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 8u;
  if (c >= I) return;
  uint4* gp = reinterpret_cast<uint4*>(g + size_t(row) * I + c);
  const uint4 gv = *gp;
  const uint4 uv = *reinterpret_cast<const uint4*>(up + size_t(row) * I + c);
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t r = 0;
#pragma unroll
    for (int hlf = 0; hlf < 2; hlf++) {
      const float gf = bf2f((gw[q] >> (16 * hlf)) & 0xFFFFu), uf = bf2f((uw[q] >> (16 * hlf)) & 0xFFFFu);
      const float sg = rbf(1.f / (1.f + __expf(-gf)));
      r |= f2bf(rbf(rbf(sg * gf) * uf)) << (16 * hlf);
    }
    o[q] = r;
  }
  *gp = make_uint4(o[0], o[1], o[2], o[3]);
}

// down tile of one routed expert -> y rows (BF16) per token.
template <int NT>
__global__ void __launch_bounds__(kThreads, 4) moe_down(const voom_expert_pages* __restrict__ pages,
                                                        const Routes* __restrict__ R,
                                                        const uint16_t* __restrict__ act, uint32_t H, uint32_t I,
                                                        uint16_t* __restrict__ y_out, uint32_t* status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  GemvShared& sh = *reinterpret_cast<GemvShared*>(smem_raw);
  const uint32_t t = blockIdx.x, u = blockIdx.y, grp = blockIdx.z;
  uint32_t ntk;
  if (!setup_tokens<NT>(sh, R, u, grp, &ntk, status)) return;
  const voom_expert_pages& E = pages[R->expert[u]];
  if (t >= E.down.n_tiles) return;
  // the down projection reads this expert's activation rows
  if (threadIdx.x < NT) sh.tok[threadIdx.x] = R->uoff[u] + grp * NT + threadIdx.x;
  for (int i = threadIdx.x; i < 128 * kTok; i += kThreads) (&sh.acc[0][0][0])[i] = 0.f;
  if (threadIdx.x == 0) sh.status = 0;
  __syncthreads();
  gemv_tile<NT>(sh, E.down, t, 0, act, I, ntk);
  const voom_rans_tile tl = E.down.tiles[t];
  const uint32_t rows = tl.raw_len / (2u * I), row0 = uint32_t(tl.dst / (2u * I));
  for (uint32_t q = threadIdx.x; q < rows * ntk; q += kThreads) {
    const uint32_t row = q / ntk, j = q % ntk;
    y_out[size_t(R->uoff[u] + grp * NT + j) * H + row0 + row] = uint16_t(f2bf(sh.acc[0][row][j]));
  }
  if (threadIdx.x == 0 && sh.status) atomicOr(status, 1u);
}

// out[t] = ordered BF16 sum of bf16(y * w); x_out = bf16(x + out).
__global__ void moe_combine(const Routes* __restrict__ R, const uint16_t* __restrict__ y,
                            const uint16_t* __restrict__ x, uint16_t* __restrict__ x_out, uint32_t H,
                            uint32_t residual) {
  const uint32_t t = blockIdx.y;
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  const uint32_t k = R->k;
  float o = 0.f;
  for (uint32_t j = 0; j < k; j++) {
    const uint32_t q = R->tok_order[t * k + j];
    o = rbf(o + rbf(bf2f(y[size_t(q) * H + c]) * bf2f(R->w_bf16[q])));
  }
  const float base = residual ? bf2f(x[size_t(t) * H + c]) : 0.f;
  x_out[size_t(t) * H + c] = uint16_t(f2bf(base + o));
}

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct ScratchLayout {
  uint64_t routes, h, logits, act, y, total;
};

ScratchLayout layout(uint32_t T, uint32_t H, uint32_t I, uint32_t k) {
  ScratchLayout s;
  uint64_t o = 0;
  s.routes = o; o = align256(o + sizeof(Routes));
  s.h = o; o = align256(o + uint64_t(T) * H * 2 + 16);
  s.logits = o; o = align256(o + uint64_t(T) * kMaxE * 4);
  s.act = o; o = align256(o + uint64_t(T) * k * I * 2 + 16);
  s.y = o; o = align256(o + uint64_t(T) * k * (H > I ? H : I) * 2 + 16);  // u rows, then y rows
  s.total = o;
  return s;
}


template <int NT>
int launch_gemv_nt(const voom_expert_pages* d_pages, const Routes* R, const uint16_t* h, uint16_t* act,
                   uint16_t* ubuf, uint16_t* y, uint32_t T, uint32_t H, uint32_t I, uint32_t n_unique,
                   uint32_t max_rows, uint32_t gate_tiles, uint32_t down_tiles, uint32_t* d_status,
                   cudaStream_t st) {
  const uint32_t groups = (T + NT - 1) / NT;
  const size_t smem = sizeof(GemvShared);
  if (cudaFuncSetAttribute(moe_gate_up<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
          cudaSuccess ||
      cudaFuncSetAttribute(moe_down<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return VOOM_E_CUDA;
  moe_gate_up<NT><<<dim3(2 * gate_tiles, n_unique, groups), kThreads, smem, st>>>(d_pages, R, h, H, I, act, ubuf,
                                                                                   d_status);
  moe_act<<<dim3((I / 8 + 127) / 128, max_rows), 128, 0, st>>>(R, act, ubuf, I);
  moe_down<NT><<<dim3(down_tiles, n_unique, groups), kThreads, smem, st>>>(d_pages, R, act, H, I, y, d_status);
  return VOOM_OK;
}

// gate/up, activation, then down for every routed expert; tokens per CTA
// chosen from T (an expert sees at most T tokens).  ubuf holds max_rows x I.
int launch_gemv(const voom_expert_pages* d_pages, const Routes* R, const uint16_t* h, uint16_t* act,
                uint16_t* ubuf, uint16_t* y, uint32_t T, uint32_t H, uint32_t I, uint32_t n_unique,
                uint32_t max_rows, uint32_t gate_tiles, uint32_t down_tiles, uint32_t* d_status, cudaStream_t st) {
#define VOOM_GEMV(NT)                                                                                         \
  launch_gemv_nt<NT>(d_pages, R, h, act, ubuf, y, T, H, I, n_unique, max_rows, gate_tiles, down_tiles, d_status, \
                     st)
  if (T == 1) return VOOM_GEMV(1);
  if (T == 2) return VOOM_GEMV(2);
  if (T <= 4) return VOOM_GEMV(4);
  return VOOM_GEMV(8);
#undef VOOM_GEMV
}

}  // namespace

VOOM_API uint64_t voom_moe_scratch_bytes(uint32_t T, uint32_t H, uint32_t I, uint32_t top_k) {
  return layout(T, H, I, top_k).total;
}

static int moe_layer_impl(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                            const uint16_t* d_norm_w, float eps, const uint16_t* d_x, uint16_t* d_x_out, uint32_t T,
                            uint32_t H, uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                            uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                            uint32_t* d_status, void* stream) {
  if (!d_pages || !d_router_w || !d_x || !d_x_out || !d_scratch || !d_status) return VOOM_E_INVALID_ARG;
  if (T == 0 || top_k == 0 || top_k > 64 || uint64_t(T) * top_k > kMaxTK || n_experts > kMaxE ||
      top_k > n_experts || H % 8 || I % 8 || H > kMaxH)
    return VOOM_E_INVALID_ARG;
  const ScratchLayout L = layout(T, H, I, top_k);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* h = reinterpret_cast<uint16_t*>(s + L.h);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  uint16_t* y = reinterpret_cast<uint16_t*>(s + L.y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* logits = reinterpret_cast<float*>(s + L.logits);
  moe_router_logits<<<dim3((n_experts + kRouterExperts - 1) / kRouterExperts, T), kThreads, 0, st>>>(
      d_x, d_norm_w, eps, d_router_w, nullptr, n_experts, H, h, logits);
  moe_router_topk<<<T, kTopkThreads, 0, st>>>(logits, n_experts, top_k, norm_topk, R);
  moe_route_plan<<<1, kMaxTK, 0, st>>>(R, T, top_k);
  const uint32_t max_unique = min(n_experts, T * top_k);
  const int rc = launch_gemv(d_pages, R, h, act, y, y, T, H, I, max_unique, T * top_k, gate_tiles, down_tiles,
                             d_status, st);
  if (rc != VOOM_OK) return rc;
  moe_combine<<<dim3((H + 255) / 256, T), 256, 0, st>>>(R, y, d_x, d_x_out, H, residual);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API int voom_moe_layer(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                            const uint16_t* d_norm_w, float eps, const uint16_t* d_x, uint16_t* d_x_out, uint32_t T,
                            uint32_t H, uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                            uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                            uint32_t* d_status, void* stream) {
  return moe_layer_impl(d_pages, n_experts, d_router_w, d_norm_w, eps, d_x, d_x_out, T, H, I, top_k, norm_topk,
                        gate_tiles, down_tiles, residual, d_scratch, scratch_bytes, d_status, stream);
}

// Expert-parallel split of the layer: phase 1 leaves the unweighted expert
// outputs in d_y (T*top_k rows of H, route-row order; rows of experts whose
// pages have no tiles on this rank stay zero) and the routes in d_scratch;
// the caller sums d_y over ranks; phase 2 combines.
VOOM_API int voom_moe_experts(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                              const float* d_router_bias, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                              uint32_t T, uint32_t H,
                              uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                              uint32_t down_tiles, uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes,
                              uint32_t* d_status, void* stream) {
  if (!d_pages || !d_router_w || !d_x || !d_y || !d_scratch || !d_status) return VOOM_E_INVALID_ARG;
  if (T == 0 || top_k == 0 || top_k > 64 || uint64_t(T) * top_k > kMaxTK || n_experts > kMaxE ||
      top_k > n_experts || H % 8 || I % 8 || H > kMaxH)
    return VOOM_E_INVALID_ARG;
  const ScratchLayout L = layout(T, H, I, top_k);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* h = reinterpret_cast<uint16_t*>(s + L.h);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_y, 0, size_t(T) * top_k * H * 2, st) != cudaSuccess) return VOOM_E_CUDA;
  float* logits = reinterpret_cast<float*>(s + L.logits);
  moe_router_logits<<<dim3((n_experts + kRouterExperts - 1) / kRouterExperts, T), kThreads, 0, st>>>(
      d_x, d_norm_w, eps, d_router_w, d_router_bias, n_experts, H, h, logits);
  moe_router_topk<<<T, kTopkThreads, 0, st>>>(logits, n_experts, top_k, norm_topk, R);
  moe_route_plan<<<1, kMaxTK, 0, st>>>(R, T, top_k);
  const uint32_t max_unique = min(n_experts, T * top_k);
  uint16_t* ubuf = reinterpret_cast<uint16_t*>(s + L.y);
  const int rc = launch_gemv(d_pages, R, h, act, ubuf, d_y, T, H, I, max_unique, T * top_k, gate_tiles, down_tiles,
                             d_status, st);
  if (rc != VOOM_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API int voom_moe_combine(const void* d_scratch, const uint16_t* d_y, const uint16_t* d_x, uint16_t* d_x_out,
                              uint32_t T, uint32_t H, uint32_t residual, void* stream) {
  if (!d_scratch || !d_y || !d_x || !d_x_out || T == 0) return VOOM_E_INVALID_ARG;
  const Routes* R = reinterpret_cast<const Routes*>(d_scratch);  // routes sit at the start of the scratch
  moe_combine<<<dim3((H + 255) / 256, T), 256, 0, static_cast<cudaStream_t>(stream)>>>(R, d_y, d_x, d_x_out, H,
                                                                                        residual);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

// ------------------------------------------------------ no-allocation variant
// Scratch of voom_moe_layer_noalloc: one fixed device array per GPU, sized
// for T <= 64 tokens, T * top_k <= 256 routes, H <= 8192, I <= 4096.
namespace {
constexpr uint32_t kNoAllocMaxT = 64, kNoAllocMaxRoutes = 256, kNoAllocMaxH = 8192, kNoAllocMaxI = 4096;
constexpr uint64_t kNoAllocBytes =
    ((sizeof(Routes) + 255) & ~uint64_t(255)) +
    ((uint64_t(kNoAllocMaxT) * kNoAllocMaxH * 2 + 16 + 255) & ~uint64_t(255)) +
    uint64_t(kNoAllocMaxT) * kMaxE * 4 +
    ((uint64_t(kNoAllocMaxRoutes) * kNoAllocMaxI * 2 + 16 + 255) & ~uint64_t(255)) +
    ((uint64_t(kNoAllocMaxRoutes) * kNoAllocMaxH * 2 + 16 + 255) & ~uint64_t(255));

__device__ __align__(256) uint8_t g_moe_scratch[kNoAllocBytes];

// Device address of g_moe_scratch on the current device.  In host code the
// symbol names a host-side stand-in, so its address is looked up once per
// device (that device current) with cudaGetSymbolAddress and cached.
std::mutex g_noalloc_mu;
void* g_noalloc_addr[256];

int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return VOOM_E_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_moe_scratch) != cudaSuccess || !p) return VOOM_E_CUDA;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return VOOM_OK;
}
}  // namespace

VOOM_API int voom_moe_layer_noalloc(const voom_expert_pages* d_pages, uint32_t n_experts,
                                    const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps,
                                    const uint16_t* d_x, uint16_t* d_x_out, uint32_t T, uint32_t H, uint32_t I,
                                    uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles, uint32_t down_tiles,
                                    uint32_t residual, uint32_t* d_status, void* stream) {
  if (T > kNoAllocMaxT || uint64_t(T) * top_k > kNoAllocMaxRoutes || H > kNoAllocMaxH || I > kNoAllocMaxI)
    return VOOM_E_CAPACITY;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != VOOM_OK) return rc;
  return moe_layer_impl(d_pages, n_experts, d_router_w, d_norm_w, eps, d_x, d_x_out, T, H, I, top_k, norm_topk,
                        gate_tiles, down_tiles, residual, scratch, kNoAllocBytes, d_status, stream);
}

// Experts given by the host (routing already grouped, e.g. by
// consume_expert_batches): expert u takes tokens upair[off_u .. off_u +
// ntok[u]) (off_u = sum of earlier ntok); y row off_u + i receives expert u's
// output for its i-th token.  No combine.
VOOM_API int voom_expert_swiglu(const voom_expert_pages* d_pages, const uint32_t* d_expert_ids, uint32_t n_unique,
                                const uint32_t* d_ntok, const uint32_t* d_upair, uint32_t n_rows, uint32_t T,
                                const uint16_t* d_h,
                                uint32_t H, uint32_t I, uint32_t gate_tiles, uint32_t down_tiles, uint16_t* d_y,
                                void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  if (!d_pages || !d_expert_ids || !d_ntok || !d_upair || !d_h || !d_y || !d_scratch || !d_status)
    return VOOM_E_INVALID_ARG;
  if (T == 0 || n_unique == 0 || n_rows == 0 || n_rows > kMaxTK || n_unique > n_rows || H % 8 || I % 8)
    return VOOM_E_INVALID_ARG;
  const ScratchLayout L = layout(n_rows, H, I, 1);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  uint16_t* ubuf = reinterpret_cast<uint16_t*>(s + L.y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the route header lives in scratch: fill n_unique, T, expert, ntok, upair
  if (cudaMemcpyAsync(&R->expert[0], d_expert_ids, 4ull * n_unique, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(&R->ntok[0], d_ntok, 4ull * n_unique, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(&R->upair[0], d_upair, 4ull * n_rows, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return VOOM_E_CUDA;
  moe_route_offsets<<<1, 32, 0, st>>>(R, n_unique, T);
  const int rc = launch_gemv(d_pages, R, d_h, act, ubuf, d_y, T, H, I, n_unique, n_rows, gate_tiles, down_tiles,
                             d_status, st);
  if (rc != VOOM_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
