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
#include "moe_common.cuh"
#include "moe_proj.cuh"

using namespace voom;
using namespace voom::rans;

namespace {

using namespace voom::moe;

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

// Family differences: the qwen35 RMSNorm is zero-centred (weight 1 + w in
// fp32, qwen35.py:133-150); the GLM router computes fp32 logits from h and W
// cast to fp32 with no BF16 rounding and takes its bias in the top-k
// (glm.py:364-392); the generic / qwen35 logits are BF16 (quant.matmul)
// plus an optional fp32 bias.  Expert row E, when sg_w is given, is the
// qwen35 shared-expert gate: its BF16 logit goes through a sigmoid rounded
// to BF16 into R->sgate[t] (qwen35.py:637-638).
__global__ void __launch_bounds__(kThreads) moe_router_logits(const uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ norm_w, float eps,
                                                              const uint16_t* __restrict__ wr,
                                                              const float* __restrict__ bias, uint32_t E,
                                                              uint32_t H, uint16_t* __restrict__ h,
                                                              float* __restrict__ logits, uint32_t family,
                                                              const uint16_t* __restrict__ sg_w, Routes* R) {
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
  const float w_shift = family == VOOM_MOE_QWEN35 ? 1.f : 0.f;
  for (uint32_t i = tid; i < H; i += kThreads) {
    const uint32_t hb = norm_w ? f2bf(bf2f(xt[i]) * s_scale * (bf2f(norm_w[i]) + w_shift)) : xt[i];
    if (write_h) ht[i] = uint16_t(hb);
    s_h[i] = bf2f(hb);
  }
  __syncthreads();
  const uint32_t e = blockIdx.x * kRouterExperts + (warp & 3u), half = warp >> 2;
  const uint32_t hmid = (H / 16) * 8;  // split point, a multiple of 8
  const uint32_t rows = E + (sg_w ? 1u : 0u);
  __shared__ float s_part[kThreads / 32];
  if (e < rows) {
    const uint16_t* we = e < E ? wr + size_t(e) * H : sg_w;
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
  if (e < rows && half == 0 && lane == 0) {
    const float acc = s_part[warp] + s_part[warp + 4];
    if (e == E) {
      R->sgate[t] = uint16_t(f2bf(1.f / (1.f + expf(-rbf(acc)))));
    } else if (family == VOOM_MOE_GLM) {
      logits[size_t(t) * E + e] = acc;  // fp32 logits; the bias applies to the sigmoid scores
    } else {
      logits[size_t(t) * E + e] = rbf(acc) + (bias ? bias[e] : 0.f);
    }
  }
}

// One CTA per token.  generic / qwen35 (layer_runner.py:359-368,
// qwen35.py:584-593): fp32 softmax of the logits (max and sum as one warp
// over lanes e % 32), keys = probabilities, weights = the chosen
// probabilities, renormalised over the k chosen when norm_topk.  glm
// (glm.py:364-392): scores = sigmoid(fp32 logit), keys = scores + bias (the
// correction bias only decides the choice), weights = the chosen scores,
// divided by (their sum + 1e-20) when norm_topk, times routed_scale.  Every
// expert's rank in (key desc, id asc) order is counted by one thread against
// all others -- ties to the lower id, a NaN key ranks lowest -- and the k
// first become the routes.
constexpr int kTopkThreads = 256;

__global__ void __launch_bounds__(kTopkThreads) moe_router_topk(const float* __restrict__ logits, uint32_t E,
                                                                uint32_t k, uint32_t norm_topk, Routes* routes,
                                                                uint32_t family, const float* __restrict__ bias,
                                                                float routed_scale) {
  __shared__ float s_p[kMaxE];
  __shared__ float s_key[kMaxE];
  __shared__ int s_pick[64];
  __shared__ float s_mx, s_sm;
  const uint32_t t = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const bool glm = family == VOOM_MOE_GLM;
  for (uint32_t e = tid; e < E; e += kTopkThreads) s_p[e] = logits[size_t(t) * E + e];
  __syncthreads();
  if (glm) {
    for (uint32_t e = tid; e < E; e += kTopkThreads) {
      const float sc = 1.f / (1.f + expf(-s_p[e]));
      s_p[e] = sc;
      const float key = bias ? sc + bias[e] : sc;
      s_key[e] = key == key ? key : -INFINITY;
    }
    if (tid == 0) s_sm = 1.f;
  } else {
    if (tid < 32) {
      float mx = -INFINITY;
      for (uint32_t e = lane; e < E; e += 32) mx = fmaxf(mx, s_p[e]);
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      if (lane == 0) s_mx = mx;
    }
    __syncthreads();
    const float mx = s_mx;
    for (uint32_t e = tid; e < E; e += kTopkThreads) {
      const float p = expf(s_p[e] - mx);
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
  }
  __syncthreads();
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
    const float den = glm ? sel + 1e-20f : sel;
    for (uint32_t j = 0; j < k; j++) {
      const float pw = s_p[s_pick[j]] / sm;
      float w = norm_topk ? pw / den : pw;
      if (glm) w *= routed_scale;
      routes->idx[t * k + j] = uint32_t(s_pick[j]);
      routes->w[t * k + j] = w;
    }
  }
}

// Route plan, one CTA of kMaxTK threads (thread p = route position t*k + j).
// Unique experts are numbered in the order the family accumulates them:
// first appearance over (position, slot) for generic (layer_runner.py:
// 378-394), ascending id for qwen35 and glm (qwen35.py:617-633, glm.py:
// 455-480).  Then tokens per expert, route rows grouped by expert in
// position order, and each token's routes ordered by that expert order.
// With a shared expert (page-table index `shared`, kNoShared if none), it is
// appended as the last unique expert with one row per token (rows
// T*k .. T*k + T - 1, token order); the combine adds it after the routed sum.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  uint32_t incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= uint32_t(o)) incl += t;
  }
  __syncthreads();
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  uint32_t before = 0, all = 0;
  for (uint32_t w = 0; w < blockDim.x / 32; w++) {
    before += w < warp ? s_warp[w] : 0u;
    all += s_warp[w];
  }
  *total = all;
  return before + incl - v;
}

__global__ void __launch_bounds__(kMaxTK) moe_route_plan(Routes* r, uint32_t T, uint32_t k, uint32_t family,
                                                          uint32_t shared) {
  __shared__ uint32_t s_first[kMaxE];  // first position of each expert
  __shared__ uint32_t s_cnt[kMaxE];    // routes per expert
  __shared__ uint32_t s_uid[kMaxE];    // unique index of each expert (ascending order)
  __shared__ uint32_t s_idx[kMaxTK];
  __shared__ uint32_t s_u[kMaxTK];     // unique index of position p's expert
  __shared__ uint32_t s_scan[kMaxTK];
  __shared__ uint32_t s_ntok[kMaxU];   // routes of unique expert u
  __shared__ uint32_t s_warp[kMaxTK / 32];
  const uint32_t p = threadIdx.x, n = T * k;
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
  uint32_t nu = 0, u = 0;
  if (family == VOOM_MOE_GENERIC) {
    // exclusive scan of "p is its expert's first position" -> unique index
    const uint32_t flag = (p < n && s_first[e] == p) ? 1u : 0u;
    s_scan[p] = block_excl_scan(flag, s_warp, &nu);
    __syncthreads();
    u = p < n ? s_scan[s_first[e]] : 0u;
  } else {
    // exclusive scan of "expert is routed" over ids (two ids per thread)
    const uint32_t e0 = 2 * p, e1 = 2 * p + 1;
    const uint32_t f0 = s_first[e0] != 0xFFFFFFFFu, f1 = s_first[e1] != 0xFFFFFFFFu;
    const uint32_t b = block_excl_scan(f0 + f1, s_warp, &nu);
    s_uid[e0] = b;
    s_uid[e1] = b + f0;
    __syncthreads();
    u = p < n ? s_uid[e] : 0u;
  }
  if (p < n) {
    s_u[p] = u;
    if (s_first[e] == p) {
      r->expert[u] = e;
      r->ntok[u] = s_cnt[e];
      s_ntok[u] = s_cnt[e];
    }
  }
  const bool has_shared = shared != kNoShared;
  if (p == 0) {
    r->n_unique = nu + (has_shared ? 1u : 0u);
    r->T = T;
    r->k = k;
    r->family = family;
    r->shared_u = has_shared ? nu : kNoShared;
    r->n_rows = n + (has_shared ? T : 0u);
    if (has_shared) {
      r->expert[nu] = shared;
      r->ntok[nu] = T;
    }
  }
  __syncthreads();
  // uoff: exclusive scan of ntok in unique order (thread u holds ntok[u])
  uint32_t routed_rows = 0;
  const uint32_t cnt_u = p < nu ? s_ntok[p] : 0u;
  const uint32_t base = block_excl_scan(cnt_u, s_warp, &routed_rows);
  if (p < nu) s_scan[p] = base;
  if (p == 0) r->uoff[0] = 0;
  if (p < nu) r->uoff[p + 1] = base + cnt_u;
  if (has_shared && p == 0) r->uoff[nu + 1] = n + T;
  __syncthreads();
  if (p < n) {
    // route row: uoff[u] + earlier positions with the same expert
    uint32_t rank = 0;
    for (uint32_t q = 0; q < p; q++) rank += (s_idx[q] == e) ? 1u : 0u;
    const uint32_t row = s_scan[u] + rank;
    r->upair[row] = p / k;
    r->row_u[row] = uint16_t(u);
    r->w_bf16[row] = uint16_t(f2bf(r->w[p]));
    r->w_row[row] = r->w[p];
    // this token's routes ordered by unique index (experts of a token are distinct)
    const uint32_t t = p / k, t0 = t * k;
    uint32_t pos = 0;
    for (uint32_t j = 0; j < k; j++) pos += (s_u[t0 + j] < u) ? 1u : 0u;
    r->tok_order[t0 + pos] = row;
  }
  // every unique expert runs here unless moe_route_owners assigns owners
  for (uint32_t q = p; q < nu + (has_shared ? 1u : 0u); q += blockDim.x) {
    r->owned[q] = q;
    r->mine[q] = 1;
  }
  if (p == 0) r->n_owned = nu + (has_shared ? 1u : 0u);
  if (has_shared) {
    for (uint32_t t = p; t < T; t += blockDim.x) {
      r->row_u[n + t] = uint16_t(nu);
      r->upair[n + t] = t;
      r->w_bf16[n + t] = 0x3F80u;  // 1.0
      r->w_row[n + t] = 1.f;
    }
  }
}

// Route rows for experts given by the host: uoff from ntok.
__global__ void moe_route_offsets(Routes* r, uint32_t n_unique, uint32_t T) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  r->n_unique = n_unique;
  r->T = T;
  r->family = VOOM_MOE_GENERIC;
  r->shared_u = kNoShared;
  r->uoff[0] = 0;
  for (uint32_t u = 0; u < n_unique; u++) {
    r->uoff[u + 1] = r->uoff[u] + r->ntok[u];
    r->owned[u] = u;
    r->mine[u] = 1;
  }
  r->n_owned = n_unique;
  r->n_rows = r->uoff[n_unique];
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

// out[t] = ordered BF16 sum over the token's routes of the contribution
// bf16(y * w) -- w the BF16 route weight (generic, qwen35) or the fp32 one
// (glm, glm.py:469-473) -- in the route plan's expert order; then the shared
// expert's row: qwen35 adds bf16(sgate[t] * y_shared) (qwen35.py:636-638),
// glm adds y_shared (glm.py:484); x_out = bf16(x + out) with the residual.
__global__ void moe_combine(const Routes* __restrict__ R, const uint16_t* __restrict__ y,
                            const uint16_t* __restrict__ x, uint16_t* __restrict__ x_out, uint32_t H,
                            uint32_t residual) {
  const uint32_t t = blockIdx.y;
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  const uint32_t k = R->k;
  const bool fp32_w = R->family == VOOM_MOE_GLM;
  float o = 0.f;
  for (uint32_t j = 0; j < k; j++) {
    const uint32_t q = R->tok_order[t * k + j];
    const float w = fp32_w ? R->w_row[q] : bf2f(R->w_bf16[q]);
    o = rbf(o + rbf(bf2f(y[size_t(q) * H + c]) * w));
  }
  const uint32_t su = R->shared_u;
  if (su != kNoShared) {
    float ys = bf2f(y[size_t(R->uoff[su] + t) * H + c]);
    if (R->family == VOOM_MOE_QWEN35) ys = rbf(bf2f(R->sgate[t]) * ys);
    o = rbf(o + ys);
  }
  const float base = residual ? bf2f(x[size_t(t) * H + c]) : 0.f;
  x_out[size_t(t) * H + c] = uint16_t(f2bf(base + o));
}

// Expert parallelism: the rank that computes each unique expert's rows.  An
// expert whose pages one rank holds goes to that rank; an expert several ranks
// hold (a replicated hot expert) goes, in unique order after every
// single-holder expert is counted, to the least loaded of its holders (the
// lowest rank on a tie).  Every rank runs this on the same routes, so every
// route row is computed by exactly one rank.  Load of a unique expert = its
// page decode (kPageLoad) + its tokens.  holders[e] (e < n_experts, and
// n_experts for the shared expert): bit r = rank r holds the pages.  An
// expert nobody holds is computed nowhere (its rows stay zero) and flagged.
constexpr uint32_t kPageLoad = 16;

__global__ void moe_route_owners(Routes* r, const uint32_t* __restrict__ holders, uint32_t rank, uint32_t world,
                                 uint32_t* status) {
  __shared__ uint32_t s_owner[kMaxU];
  if (threadIdx.x == 0) {
    uint32_t load[32];
    for (uint32_t q = 0; q < 32; q++) load[q] = 0;
    const uint32_t nu = r->n_unique, mask = world >= 32 ? 0xFFFFFFFFu : (1u << world) - 1u;
    for (uint32_t u = 0; u < nu; u++) {
      const uint32_t h = holders[r->expert[u]] & mask;
      s_owner[u] = world;  // nobody (no holder), or decided in the second pass
      if (h && !(h & (h - 1u))) {
        const uint32_t o = uint32_t(__ffs(int(h))) - 1u;
        s_owner[u] = o;
        load[o] += kPageLoad + r->ntok[u];
      } else if (!h) {
        atomicOr(status, kStatusNoHolder);
      }
    }
    for (uint32_t u = 0; u < nu; u++) {
      uint32_t h = holders[r->expert[u]] & mask;
      if (!h || !(h & (h - 1u))) continue;
      uint32_t best = 0xFFFFFFFFu, bl = 0xFFFFFFFFu;
      for (; h; h &= h - 1u) {
        const uint32_t o = uint32_t(__ffs(int(h))) - 1u;
        if (load[o] < bl) {
          bl = load[o];
          best = o;
        }
      }
      s_owner[u] = best;
      load[best] += kPageLoad + r->ntok[u];
    }
    uint32_t n = 0;
    for (uint32_t u = 0; u < nu; u++) {
      const bool m = s_owner[u] == rank;
      r->mine[u] = m ? 1 : 0;
      if (m) r->owned[n++] = u;
    }
    r->n_owned = n;
  }
}

// Route rows in token-major order for the ranks' exchange: row t * rpt + j =
// token t's j-th route in the combine's order (j = top_k: the shared expert),
// zero when another rank computes it or t >= T (padding).  8 columns per thread.
__global__ void moe_rows_token_major(const Routes* __restrict__ R, const uint16_t* __restrict__ y,
                                     uint16_t* __restrict__ y_tm, uint32_t H) {
  const uint32_t row = blockIdx.y, c = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= H) return;
  const uint32_t k = R->k, rpt = k + (R->shared_u != kNoShared ? 1u : 0u);
  const uint32_t t = row / rpt, j = row - t * rpt;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (t < R->T) {
    const uint32_t q = j < k ? R->tok_order[t * k + j] : R->uoff[R->shared_u] + t;
    if (R->mine[R->row_u[q]]) v = *reinterpret_cast<const uint4*>(y + size_t(q) * H + c);
  }
  *reinterpret_cast<uint4*>(y_tm + size_t(row) * H + c) = v;
}

// moe_combine over tokens t0 .. t0 + gridDim.y - 1 from token-major rows
// (row (t - t0) * rpt + j); the same arithmetic, in the same order.  Rows of
// tokens past T write zeros.
__global__ void moe_combine_tm(const Routes* __restrict__ R, const uint16_t* __restrict__ y_tm,
                               const uint16_t* __restrict__ x, uint16_t* __restrict__ x_out, uint32_t t0, uint32_t H,
                               uint32_t residual) {
  const uint32_t tl = blockIdx.y, t = t0 + tl;
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  if (t >= R->T) {
    x_out[size_t(tl) * H + c] = 0;
    return;
  }
  const uint32_t k = R->k, rpt = k + (R->shared_u != kNoShared ? 1u : 0u);
  const bool fp32_w = R->family == VOOM_MOE_GLM;
  const uint16_t* yr = y_tm + size_t(tl) * rpt * H + c;
  float o = 0.f;
  for (uint32_t j = 0; j < k; j++) {
    const uint32_t q = R->tok_order[t * k + j];
    const float w = fp32_w ? R->w_row[q] : bf2f(R->w_bf16[q]);
    o = rbf(o + rbf(bf2f(yr[size_t(j) * H]) * w));
  }
  if (R->shared_u != kNoShared) {
    float ys = bf2f(yr[size_t(k) * H]);
    if (R->family == VOOM_MOE_QWEN35) ys = rbf(bf2f(R->sgate[t]) * ys);
    o = rbf(o + ys);
  }
  const float base = residual ? bf2f(x[size_t(t) * H + c]) : 0.f;
  x_out[size_t(tl) * H + c] = uint16_t(f2bf(base + o));
}

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct ScratchLayout {
  uint64_t routes, h, logits, act, y, seams, seam_bytes, total;
};

// Work counters (256 bytes) and seam cells of the CUDA-core kernel: two
// projections' worth of cells per unique expert.
constexpr uint64_t kCounterBytes = 256;
uint64_t seam_bytes(uint32_t max_unique) {
  return kCounterBytes + uint64_t(max_unique) * 2 * kSeams * sizeof(SeamCell);
}

// CTAs of the persistent CUDA-core kernel: four per SM of the current device.
uint32_t cc_grid() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148 * 4;
  if (!sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms[dev] = n;
  }
  return uint32_t(sms[dev]) * 4u;
}

ScratchLayout layout(uint32_t T, uint32_t H, uint32_t I, uint32_t k) {
  ScratchLayout s;
  uint64_t o = 0;
  s.routes = o; o = align256(o + sizeof(Routes));
  s.h = o; o = align256(o + uint64_t(T) * H * 2 + 16);
  s.logits = o; o = align256(o + uint64_t(T) * kMaxE * 4);
  s.act = o; o = align256(o + uint64_t(T) * k * I * 2 + 16);
  s.y = o; o = align256(o + uint64_t(T) * k * (H > I ? H : I) * 2 + 16);  // u rows, then y rows
  s.seams = o; s.seam_bytes = seam_bytes(min(uint64_t(T) * k, uint64_t(kMaxU))); o = align256(o + s.seam_bytes);
  s.total = o;
  return s;
}


// gate/up, activation, then down for every routed expert.  Experts with at
// most kTok tokens run on moe_proj_cc (NT picked from max_tok, the most
// tokens one expert can have); when max_tok > kTok the experts with more
// tokens run on moe_proj_mma (tensor cores), each page block decoded once.
// ubuf holds max_rows x I.
template <int NT>
int launch_cc(const voom_expert_pages* d_pages, const Routes* R, uint32_t which, const uint16_t* in, uint32_t ld_in,
              uint16_t* out0, uint16_t* out1, uint32_t ld_out, uint32_t nbpp, uint32_t n_proj, uint32_t cpt,
              uint32_t tiles, uint32_t n_unique, SeamCell* seams, uint32_t* counter, uint32_t* d_status,
              cudaStream_t st) {
  const size_t smem = sizeof(CcShared);
  if (cudaFuncSetAttribute(moe_proj_cc<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return VOOM_E_CUDA;
  const uint32_t items = n_unique * n_proj * nbpp;
  const uint32_t grid = min(cc_grid(), max(1u, items));
  moe_proj_cc<NT><<<grid, kThreads, smem, st>>>(d_pages, R, which, in, ld_in, out0, out1, ld_out, nbpp, n_proj, cpt,
                                                tiles, seams, counter, d_status);
  return VOOM_OK;
}

// One projection kind (gate and up, or down) of every unique expert: rows x
// cols, `tiles` = the largest tile count of any expert's frame of it.
int launch_proj(const voom_expert_pages* d_pages, const Routes* R, uint32_t which, const uint16_t* in,
                uint32_t ld_in, uint16_t* out0, uint16_t* out1, uint32_t ld_out, uint32_t rows, uint32_t cols,
                uint32_t tiles, uint32_t n_proj, uint32_t n_unique, uint32_t max_tok, SeamCell* seams,
                uint32_t* counter, uint32_t* d_status, cudaStream_t st) {
  const uint32_t t = max(1u, tiles);
  const uint32_t cpt = cc_chunks_per_tile(rows, cols, t), nbpp = t * cpt;
  const uint32_t ntok = min(max_tok, uint32_t(kTok));
  int rc;
  if (ntok <= 1)
    rc = launch_cc<1>(d_pages, R, which, in, ld_in, out0, out1, ld_out, nbpp, n_proj, cpt, t, n_unique, seams,
                      counter, d_status, st);
  else if (ntok <= 2)
    rc = launch_cc<2>(d_pages, R, which, in, ld_in, out0, out1, ld_out, nbpp, n_proj, cpt, t, n_unique, seams,
                      counter, d_status, st);
  else if (ntok <= 4)
    rc = launch_cc<4>(d_pages, R, which, in, ld_in, out0, out1, ld_out, nbpp, n_proj, cpt, t, n_unique, seams,
                      counter, d_status, st);
  else
    rc = launch_cc<8>(d_pages, R, which, in, ld_in, out0, out1, ld_out, nbpp, n_proj, cpt, t, n_unique, seams,
                      counter, d_status, st);
  if (rc != VOOM_OK || max_tok <= uint32_t(kTok)) return rc;
  const uint32_t ncap = (min(max_tok, kMmaMaxN) + 15u) & ~15u;
  const uint32_t zc = (max_tok + kMmaMaxN - 1) / kMmaMaxN;
  const uint32_t smem = mma_smem_bytes(ncap);
  if (cudaFuncSetAttribute(moe_proj_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return VOOM_E_CUDA;
  const uint32_t nbm = (rows + kMmaRows - 1) / kMmaRows;
  moe_proj_mma<<<dim3(n_proj * nbm, n_unique, zc), kThreads, smem, st>>>(d_pages, R, which, in, ld_in, out0, out1,
                                                                          ld_out, nbm, ncap, d_status);
  return VOOM_OK;
}

// gate/up, activation, then down for every routed expert.  Experts with at
// most kTok tokens run on moe_proj_cc, the others on moe_proj_mma (tensor
// cores); either way each page block is decoded once per call.  ubuf holds
// max_rows x I; seams = seam_bytes(n_unique) of scratch (cleared here).
int launch_gemv(const voom_expert_pages* d_pages, const Routes* R, const uint16_t* h, uint16_t* act,
                uint16_t* ubuf, uint16_t* y, uint32_t H, uint32_t I, uint32_t n_unique, uint32_t max_rows,
                uint32_t max_tok, uint32_t gate_tiles, uint32_t down_tiles, void* seams, uint32_t* d_status,
                cudaStream_t st) {
  if (cudaMemsetAsync(seams, 0, seam_bytes(n_unique), st) != cudaSuccess) return VOOM_E_CUDA;
  uint32_t* counters = static_cast<uint32_t*>(seams);
  SeamCell* sc = reinterpret_cast<SeamCell*>(static_cast<uint8_t*>(seams) + kCounterBytes);
  int rc = launch_proj(d_pages, R, 0, h, H, act, ubuf, I, I, H, gate_tiles, 2, n_unique, max_tok, sc, counters,
                       d_status, st);
  if (rc != VOOM_OK) return rc;
  moe_act<<<dim3((I / 8 + 127) / 128, max_rows), 128, 0, st>>>(R, act, ubuf, I);
  return launch_proj(d_pages, R, 1, act, I, y, y, H, H, I, down_tiles, 1, n_unique, max_tok, sc, counters + 1,
                     d_status, st);
}

// The generic family with no shared expert: what the variant-less entry
// points run.
voom_moe_variant generic_variant(uint32_t norm_topk, const float* bias) {
  voom_moe_variant v;
  v.family = VOOM_MOE_GENERIC;
  v.norm_topk = norm_topk;
  v.routed_scale = 1.f;
  v.shared_expert = -1;
  v.d_shared_gate_w = nullptr;
  v.d_router_bias = bias;
  return v;
}

uint32_t rows_per_token(const voom_moe_variant& v, uint32_t top_k) {
  return top_k + (v.shared_expert >= 0 ? 1u : 0u);
}

int check_variant(const voom_moe_variant* v, uint32_t n_experts) {
  if (!v || v->family > VOOM_MOE_GLM) return VOOM_E_INVALID_ARG;
  if (v->family == VOOM_MOE_QWEN35 && v->norm_topk != 1) return VOOM_E_INVALID_ARG;  // always renormalised
  if (v->shared_expert >= 0 && uint32_t(v->shared_expert) < n_experts) return VOOM_E_INVALID_ARG;
  if (v->d_shared_gate_w && (v->family != VOOM_MOE_QWEN35 || v->shared_expert < 0)) return VOOM_E_INVALID_ARG;
  return VOOM_OK;
}

// Router, top-k and route plan for T tokens: R, h and the logits in scratch.
int launch_front(const voom_moe_variant& v, const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps,
                 const uint16_t* d_x, uint32_t n_experts, uint32_t T, uint32_t H, uint32_t top_k, Routes* R,
                 uint16_t* h, float* logits, cudaStream_t st) {
  const uint32_t rows = n_experts + (v.d_shared_gate_w ? 1u : 0u);
  const float* logit_bias = v.family == VOOM_MOE_GLM ? nullptr : v.d_router_bias;
  moe_router_logits<<<dim3((rows + kRouterExperts - 1) / kRouterExperts, T), kThreads, 0, st>>>(
      d_x, d_norm_w, eps, d_router_w, logit_bias, n_experts, H, h, logits, v.family, v.d_shared_gate_w, R);
  moe_router_topk<<<T, kTopkThreads, 0, st>>>(logits, n_experts, top_k, v.norm_topk, R, v.family,
                                              v.family == VOOM_MOE_GLM ? v.d_router_bias : nullptr,
                                              v.routed_scale);
  moe_route_plan<<<1, kMaxTK, 0, st>>>(R, T, top_k, v.family,
                                       v.shared_expert >= 0 ? uint32_t(v.shared_expert) : kNoShared);
  return VOOM_OK;
}

int check_shape(uint32_t n_experts, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k) {
  if (T == 0 || top_k == 0 || top_k > 64 || uint64_t(T) * top_k > kMaxTK || n_experts > kMaxE ||
      top_k > n_experts || H % 8 || I % 8 || H > kMaxH)
    return VOOM_E_INVALID_ARG;
  return VOOM_OK;
}

int moe_layer_impl(const voom_moe_variant& v, const voom_expert_pages* d_pages, uint32_t n_experts,
                   const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                   uint16_t* d_x_out, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k, uint32_t gate_tiles,
                   uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                   uint32_t* d_status, void* stream) {
  if (!d_pages || !d_router_w || !d_x || !d_x_out || !d_scratch || !d_status) return VOOM_E_INVALID_ARG;
  int rc = check_shape(n_experts, T, H, I, top_k);
  if (rc != VOOM_OK) return rc;
  const uint32_t rpt = rows_per_token(v, top_k);
  const ScratchLayout L = layout(T, H, I, rpt);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* h = reinterpret_cast<uint16_t*>(s + L.h);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  uint16_t* y = reinterpret_cast<uint16_t*>(s + L.y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* logits = reinterpret_cast<float*>(s + L.logits);
  launch_front(v, d_router_w, d_norm_w, eps, d_x, n_experts, T, H, top_k, R, h, logits, st);
  const uint32_t max_unique = min(n_experts, T * top_k) + (v.shared_expert >= 0 ? 1u : 0u);
  rc = launch_gemv(d_pages, R, h, act, y, y, H, I, max_unique, T * rpt, T, gate_tiles, down_tiles, s + L.seams,
                   d_status, st);
  if (rc != VOOM_OK) return rc;
  moe_combine<<<dim3((H + 255) / 256, T), 256, 0, st>>>(R, y, d_x, d_x_out, H, residual);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

int moe_experts_impl(const voom_moe_variant& v, const voom_expert_pages* d_pages, uint32_t n_experts,
                     const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                     uint32_t T, uint32_t H, uint32_t I, uint32_t top_k, uint32_t gate_tiles, uint32_t down_tiles,
                     uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  if (!d_pages || !d_router_w || !d_x || !d_y || !d_scratch || !d_status) return VOOM_E_INVALID_ARG;
  int rc = check_shape(n_experts, T, H, I, top_k);
  if (rc != VOOM_OK) return rc;
  const uint32_t rpt = rows_per_token(v, top_k);
  const ScratchLayout L = layout(T, H, I, rpt);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* h = reinterpret_cast<uint16_t*>(s + L.h);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_y, 0, size_t(T) * rpt * H * 2, st) != cudaSuccess) return VOOM_E_CUDA;
  float* logits = reinterpret_cast<float*>(s + L.logits);
  launch_front(v, d_router_w, d_norm_w, eps, d_x, n_experts, T, H, top_k, R, h, logits, st);
  const uint32_t max_unique = min(n_experts, T * top_k) + (v.shared_expert >= 0 ? 1u : 0u);
  uint16_t* ubuf = reinterpret_cast<uint16_t*>(s + L.y);
  rc = launch_gemv(d_pages, R, h, act, ubuf, d_y, H, I, max_unique, T * rpt, T, gate_tiles, down_tiles, s + L.seams,
                   d_status, st);
  if (rc != VOOM_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

}  // namespace

VOOM_API uint64_t voom_moe_scratch_bytes(uint32_t T, uint32_t H, uint32_t I, uint32_t top_k) {
  return layout(T, H, I, top_k).total;
}

VOOM_API uint64_t voom_moe_scratch_bytes_v(const voom_moe_variant* v, uint32_t T, uint32_t H, uint32_t I,
                                           uint32_t top_k) {
  if (!v) return 0;
  return layout(T, H, I, rows_per_token(*v, top_k)).total;
}

VOOM_API int voom_moe_layer(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                            const uint16_t* d_norm_w, float eps, const uint16_t* d_x, uint16_t* d_x_out, uint32_t T,
                            uint32_t H, uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                            uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                            uint32_t* d_status, void* stream) {
  return moe_layer_impl(generic_variant(norm_topk, nullptr), d_pages, n_experts, d_router_w, d_norm_w, eps, d_x,
                        d_x_out, T, H, I, top_k, gate_tiles, down_tiles, residual, d_scratch, scratch_bytes,
                        d_status, stream);
}

VOOM_API int voom_moe_layer_v(const voom_moe_variant* v, const voom_expert_pages* d_pages, uint32_t n_experts,
                              const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                              uint16_t* d_x_out, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k,
                              uint32_t gate_tiles, uint32_t down_tiles, uint32_t residual, void* d_scratch,
                              uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  const int rc = check_variant(v, n_experts);
  if (rc != VOOM_OK) return rc;
  return moe_layer_impl(*v, d_pages, n_experts, d_router_w, d_norm_w, eps, d_x, d_x_out, T, H, I, top_k,
                        gate_tiles, down_tiles, residual, d_scratch, scratch_bytes, d_status, stream);
}

// Expert-parallel split of the layer: phase 1 leaves the unweighted expert
// outputs in d_y (route rows of H, route-row order; rows of experts whose
// pages have no tiles on this rank stay zero) and the routes in d_scratch;
// the caller sums d_y over ranks; phase 2 combines.
VOOM_API int voom_moe_experts(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                              const float* d_router_bias, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                              uint32_t T, uint32_t H,
                              uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                              uint32_t down_tiles, uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes,
                              uint32_t* d_status, void* stream) {
  return moe_experts_impl(generic_variant(norm_topk, d_router_bias), d_pages, n_experts, d_router_w, d_norm_w, eps,
                          d_x, T, H, I, top_k, gate_tiles, down_tiles, d_y, d_scratch, scratch_bytes, d_status,
                          stream);
}

VOOM_API int voom_moe_experts_v(const voom_moe_variant* v, const voom_expert_pages* d_pages, uint32_t n_experts,
                                const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps,
                                const uint16_t* d_x, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k,
                                uint32_t gate_tiles, uint32_t down_tiles, uint16_t* d_y, void* d_scratch,
                                uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  const int rc = check_variant(v, n_experts);
  if (rc != VOOM_OK) return rc;
  return moe_experts_impl(*v, d_pages, n_experts, d_router_w, d_norm_w, eps, d_x, T, H, I, top_k, gate_tiles,
                          down_tiles, d_y, d_scratch, scratch_bytes, d_status, stream);
}

VOOM_API int voom_moe_combine(const void* d_scratch, const uint16_t* d_y, const uint16_t* d_x, uint16_t* d_x_out,
                              uint32_t T, uint32_t H, uint32_t residual, void* stream) {
  if (!d_scratch || !d_y || !d_x || !d_x_out || T == 0) return VOOM_E_INVALID_ARG;
  const Routes* R = reinterpret_cast<const Routes*>(d_scratch);  // routes sit at the start of the scratch
  moe_combine<<<dim3((H + 255) / 256, T), 256, 0, static_cast<cudaStream_t>(stream)>>>(R, d_y, d_x, d_x_out, H,
                                                                                        residual);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

// Expert parallelism (one process per GPU): routing on every rank, each
// routed expert computed by one rank (moe_route_owners), the route rows
// returned in token-major order for a reduce-scatter over tokens; see the
// header.
VOOM_API int voom_moe_experts_ep(const voom_moe_variant* v, const voom_moe_ep* ep, const voom_expert_pages* d_pages,
                                 uint32_t n_experts, const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps,
                                 const uint16_t* d_x, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k,
                                 uint32_t gate_tiles, uint32_t down_tiles, uint16_t* d_y_tm, void* d_scratch,
                                 uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  int rc = check_variant(v, n_experts);
  if (rc != VOOM_OK) return rc;
  if (!ep || !ep->d_holders || ep->world == 0 || ep->world > 32 || ep->rank >= ep->world || ep->t_pad < T ||
      ep->t_pad % ep->world)
    return VOOM_E_INVALID_ARG;
  if (!d_pages || !d_router_w || !d_x || !d_y_tm || !d_scratch || !d_status) return VOOM_E_INVALID_ARG;
  rc = check_shape(n_experts, T, H, I, top_k);
  if (rc != VOOM_OK) return rc;
  const uint32_t rpt = rows_per_token(*v, top_k);
  const ScratchLayout L = layout(T, H, I, rpt);
  if (scratch_bytes < L.total) return VOOM_E_CAPACITY;
  uint8_t* s = static_cast<uint8_t*>(d_scratch);
  Routes* R = reinterpret_cast<Routes*>(s + L.routes);
  uint16_t* h = reinterpret_cast<uint16_t*>(s + L.h);
  uint16_t* act = reinterpret_cast<uint16_t*>(s + L.act);
  uint16_t* y = reinterpret_cast<uint16_t*>(s + L.y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* logits = reinterpret_cast<float*>(s + L.logits);
  launch_front(*v, d_router_w, d_norm_w, eps, d_x, n_experts, T, H, top_k, R, h, logits, st);
  moe_route_owners<<<1, 32, 0, st>>>(R, ep->d_holders, ep->rank, ep->world, d_status);
  const uint32_t max_unique = min(n_experts, T * top_k) + (v->shared_expert >= 0 ? 1u : 0u);
  rc = launch_gemv(d_pages, R, h, act, y, y, H, I, max_unique, T * rpt, T, gate_tiles, down_tiles, s + L.seams,
                   d_status, st);
  if (rc != VOOM_OK) return rc;
  moe_rows_token_major<<<dim3((H / 8 + 127) / 128, ep->t_pad * rpt), 128, 0, st>>>(R, y, d_y_tm, H);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API int voom_moe_combine_tm(const void* d_scratch, const uint16_t* d_y_shard, const uint16_t* d_x,
                                 uint16_t* d_out_shard, uint32_t t0, uint32_t t_count, uint32_t H, uint32_t residual,
                                 void* stream) {
  if (!d_scratch || !d_y_shard || !d_x || !d_out_shard || t_count == 0) return VOOM_E_INVALID_ARG;
  const Routes* R = reinterpret_cast<const Routes*>(d_scratch);  // routes sit at the start of the scratch
  moe_combine_tm<<<dim3((H + 255) / 256, t_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      R, d_y_shard, d_x, d_out_shard, t0, H, residual);
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
    ((uint64_t(kNoAllocMaxRoutes) * kNoAllocMaxH * 2 + 16 + 255) & ~uint64_t(255)) +
    ((256 + uint64_t(kNoAllocMaxRoutes) * 2 * kSeams * sizeof(SeamCell) + 255) & ~uint64_t(255));

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
  return moe_layer_impl(generic_variant(norm_topk, nullptr), d_pages, n_experts, d_router_w, d_norm_w, eps, d_x,
                        d_x_out, T, H, I, top_k, gate_tiles, down_tiles, residual, scratch, kNoAllocBytes,
                        d_status, stream);
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
  if (reinterpret_cast<uintptr_t>(d_h) & 15u) return VOOM_E_INVALID_ARG;  // rows are read 16 bytes at a time
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
  const int rc = launch_gemv(d_pages, R, d_h, act, ubuf, d_y, H, I, n_unique, n_rows, min(T, n_rows), gate_tiles,
                             down_tiles, s + L.seams, d_status, st);
  if (rc != VOOM_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
