// Fused rANS page decode + projection of the routed experts (the expert
// SwiGLU's three matmuls, runtime/layer_runner.py:185-190 _swiglu and
// runtime/quant.py:431-444 matmul: y = x @ W.T, BF16 out, fp32 sums).
//
// Every projection (rows x cols BF16, row-major) of every expert stays in HBM
// as a VRN1 frame with a checkpoint index: each `every`-symbol segment of a
// plane can be decoded on its own and must land exactly on the next
// checkpoint.  A row holds spr = cols / every consecutive segments.  Two
// kernels consume the pages, each decoding every page block ONCE per step,
// whatever the number of tokens routed to the expert:
//
//  moe_proj_cc   experts with at most 8 tokens.  CTA = a block of rows whose
//                segments (<= 128) are decoded by one lane pair each (lo and
//                hi plane) straight into fp32 dot products with the tokens'
//                activations (CUDA cores); per-segment partial sums meet in
//                shared memory and are added in segment order, so results do
//                not depend on scheduling.
//  moe_proj_mma  experts with more than 8 tokens (batched decode, prefill).
//                CTA = 128 rows.  Lane pair p decodes row p in K-steps of 64
//                elements into a shared-memory A tile laid out for UMMA
//                (K-major, no swizzle: 8 x 16-byte core matrices); the
//                tokens' activations form the B tile; one thread issues
//                tcgen05.mma (kind::f16, BF16 in, fp32 accumulator in TMEM,
//                M = 128 rows, N = tokens padded to 16) and commits to an
//                mbarrier; the next step's decode overlaps the MMA.  The
//                epilogue reads the accumulator with tcgen05.ld.
//
// Tiles may be any multiple of 2 * every bytes; a block of rows may span two
// tiles (their decode tables both sit in shared memory).  The tensor-core
// kernel needs tiles of at least 128 rows.  The segment length must follow
// the rule of every_rule() (the largest power of two dividing cols, up to 256,
// or 512 for projections of 4M weights or more), which fixes the row blocks on
// the host.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "moe_common.cuh"
#include "rans_core.cuh"

namespace voom {
namespace moe {

using namespace voom::rans;

#ifndef VOOM_EVERY_MAX
#define VOOM_EVERY_MAX 256
#endif
// projections of at least this many weights take segments of up to 2 x
// VOOM_EVERY_MAX symbols: they have work items enough to fill the GPU, and
// longer segments halve the per-segment setup; smaller projections keep the
// shorter chains, which is where their decode's parallelism comes from
#ifndef VOOM_EVERY_LARGE
#define VOOM_EVERY_LARGE (4u << 20)
#endif

constexpr int kPairs = kThreads / 2;   // lane pairs of a CTA: one segment each
constexpr uint32_t kStatusPage = 1u;      // a segment missed its checkpoint (damaged page)
constexpr uint32_t kStatusRoutes = 2u;    // an expert has more tokens than the launch covers
constexpr uint32_t kStatusGeometry = 4u;  // page geometry the kernels do not take
constexpr uint32_t kStatusTimeout = 8u;   // a tensor-core completion wait ran out
constexpr uint32_t kStatusNoHolder = 16u;  // expert parallelism: a routed expert no rank holds

__host__ __device__ inline uint32_t every_rule(uint32_t rows, uint32_t cols) {
  uint32_t e = uint64_t(rows) * cols >= VOOM_EVERY_LARGE ? 2u * VOOM_EVERY_MAX : VOOM_EVERY_MAX;
  while (e > 64 && cols % e) e >>= 1;
  return cols % e ? 0u : e;
}

// Rows per moe_proj_cc block: as many whole rows as 128 segments hold.
__host__ __device__ inline uint32_t cc_rows(uint32_t rows, uint32_t cols) {
  const uint32_t e = every_rule(rows, cols), spr = e ? cols / e : 1u;
  return spr >= uint32_t(kPairs) ? 1u : uint32_t(kPairs) / spr;
}

// ---------------------------------------------------------------- segments
__device__ __forceinline__ void seg_open(PlaneRun& r, const voom_expert_proj& P, const voom_rans_tile& tl,
                                         uint32_t t, uint32_t l, uint32_t lane) {
  const uint64_t fq = lane ? tl.high_freq : tl.low_freq;
  const uint32_t pl = lane ? tl.high_payload : tl.low_payload;
  if (l == 0) {
    plane_start(r, P.src, fq, pl, 0, 0, false);
  } else {
    const uint32_t* ck = P.ckpt + P.ckpt_base[t] + (l - 1u) * 4u + lane * 2u;
    plane_start(r, P.src, fq, pl, ck[0], ck[1], true);
  }
}

// True when plane `lane` of segment l of tile t ended where the encoder's
// stream did: on the next checkpoint, or at the payload end for the tile's
// last segment.
__device__ __forceinline__ bool seg_landed(const PlaneRun& r, const voom_expert_proj& P, uint32_t t, uint32_t l,
                                           uint32_t nseg_t, uint32_t lane) {
  if (l + 1u == nseg_t) return r.cur == r.len;
  const uint32_t* ck = P.ckpt + P.ckpt_base[t] + l * 4u + lane * 2u;
  return r.x == ck[0] && r.cur == ck[1];
}

// 8 weights (one uint4: BF16 k .. k+7) times the activations at columns
// k .. k+7 of the CTA's tokens.
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

// 16 stored (mode-0 tile) bytes = 8 BF16 weights, byte loads (any alignment).
__device__ __forceinline__ uint4 load_stored8(const uint8_t* p) {
  uint32_t v[4];
#pragma unroll
  for (int q = 0; q < 4; q++) v[q] = ld_u32_unaligned(p + 4 * q);
  return make_uint4(v[0], v[1], v[2], v[3]);
}

// Projection of work slot `bx`: gate (bx < nbpp) or up for which = 0, down
// for which = 1; *blk = the block within it.
__device__ __forceinline__ const voom_expert_proj& pick_proj(const voom_expert_pages& E, uint32_t which,
                                                             uint32_t nbpp, uint32_t bx, bool* second,
                                                             uint32_t* blk) {
  *second = which == 0 && bx >= nbpp;
  *blk = *second ? bx - nbpp : bx;
  return which ? E.down : (*second ? E.up : E.gate);
}

// ------------------------------------------------------------ CUDA-core path
// A CTA takes a chunk of one tile's segments: whole rows of the tile, at most
// 128 segments, so it holds one tile's decode tables (about 37 KB of shared
// memory: four CTAs per SM).  A row that a tile boundary cuts ("seam row")
// gets partial sums from the two tiles' chunks; each adds its sum into a
// seam cell in global memory and the second to arrive (an atomic counter,
// no waiting) writes the BF16 result and clears the cell.  With exactly two
// fp32 addends the sum does not depend on their order, so results stay
// deterministic.
constexpr uint32_t kSeams = 64;  // tile boundaries per projection the seam cells cover (<= 65 tiles)

struct SeamCell {
  float v[kTok];
  uint32_t count;
};

__host__ __device__ inline uint32_t cc_chunks_per_tile(uint32_t rows, uint32_t cols, uint32_t n_tiles) {
  const uint32_t rb = cc_rows(rows, cols);
  if (n_tiles <= 1) return (rows + rb - 1) / rb;
  const uint32_t rows_touch = (rows + n_tiles - 2) / (n_tiles - 1) + 2;  // rows meeting one tile, at most
  return (rows_touch + rb - 1) / rb;
}

struct CcShared {
  uint32_t lut[2][4096];     // [plane]
  uint32_t cum[257];
  uint32_t red[8];
  uint32_t degenerate[2];
  float part[kPairs][kTok];  // [segment of the chunk][token]
  uint32_t tok[kTok];
  uint32_t status;
  uint32_t seam_rows;        // number of seam rows in this chunk (0..2)
  uint32_t seam_id[2];       // their seam cell indices
  uint32_t seam_row[2];      // their row numbers
};

// One work item of the CUDA-core kernel: chunk slot `bx` (of n_proj x
// tiles x chunks per tile) of unique expert u.  act: the tokens' input rows
// (h for gate/up: token index; act for down: route row), ld_in columns;
// out0/out1: route rows x ld_out (gate / up or y).  Experts with more than
// kTok tokens are left to moe_proj_mma.  Ends with a block barrier.
template <int NT>
__device__ __forceinline__ void cc_item(CcShared& sh, const voom_expert_pages* __restrict__ pages,
                                        const Routes* __restrict__ R, uint32_t which, uint32_t u, uint32_t bx,
                                        const uint16_t* __restrict__ act, uint32_t ld_in,
                                        uint16_t* __restrict__ out0, uint16_t* __restrict__ out1, uint32_t ld_out,
                                        uint32_t nbpp, uint32_t cpt, uint32_t tiles_hint,
                                        SeamCell* __restrict__ seams, uint32_t* status) {
  const uint32_t n = R->ntok[u];
  if (n > uint32_t(kTok)) return;  // the tensor-core kernel serves this expert
  if (threadIdx.x == 0 && bx == 0 && n > uint32_t(NT)) atomicOr(status, kStatusRoutes);
  const uint32_t ntk = min(uint32_t(NT), n);
  bool second;
  uint32_t slot_blk;
  const voom_expert_proj& P = pick_proj(pages[R->expert[u]], which, nbpp, bx, &second, &slot_blk);
  if (P.n_tiles == 0) return;  // this expert's pages live on another GPU
  const uint32_t tid = threadIdx.x, lane = tid & 1u, p = tid >> 1;
  const uint32_t every = P.every, spr = P.cols / every, rb = cc_rows(P.rows, P.cols);
  const uint32_t spt = P.tiles[0].raw_len / (2u * every);
  if (P.n_tiles > tiles_hint || P.n_tiles > kSeams + 1 || every != every_rule(P.rows, P.cols) || spt < spr) {
    if (tid == 0 && slot_blk == 0) atomicOr(status, kStatusGeometry);
    return;
  }
  const uint32_t t = slot_blk / cpt, c = slot_blk - t * cpt;
  if (t >= P.n_tiles) return;
  const voom_rans_tile tl = P.tiles[t];
  const uint32_t ts0 = t * spt, ts1 = ts0 + tl.raw_len / (2u * every);
  const uint32_t ra = ts0 / spr;
  const uint32_t g0 = max(ts0, (ra + c * rb) * spr), g1 = min(ts1, (ra + (c + 1) * rb) * spr);
  if (g0 >= g1) return;
  const uint32_t nseg = g1 - g0;
  const uint32_t row_base = R->uoff[u];
  if (tid < uint32_t(NT)) sh.tok[tid] = tid < ntk ? (which ? row_base + tid : R->upair[row_base + tid]) : 0u;
  if (tid == 0) {
    sh.status = 0;
    uint32_t ns = 0;
    const uint32_t cell0 = (u * 2u + (second ? 1u : 0u)) * kSeams;
    if (g0 == ts0 && ts0 % spr) {  // first row began in the previous tile
      sh.seam_id[ns] = cell0 + t - 1u;
      sh.seam_row[ns++] = g0 / spr;
    }
    if (g1 == ts1 && ts1 % spr) {  // last row continues in the next tile
      sh.seam_id[ns] = cell0 + t;
      sh.seam_row[ns++] = (g1 - 1u) / spr;
    }
    sh.seam_rows = ns;
  }
  if (tl.mode == 1) {
    build_lut(sh.lut[0], sh.cum, sh.red, &sh.degenerate[0], P.src + tl.low_freq);
    build_lut(sh.lut[1], sh.cum, sh.red, &sh.degenerate[1], P.src + tl.high_freq);
  }
  __syncthreads();
  float acc[NT];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j] = 0.f;
  if (p < nseg) {
    const uint32_t g = g0 + p, l = g - ts0;
    const uint32_t k0 = (g % spr) * every;
    if (tl.mode == 0) {  // stored tile: weights read directly
      const uint8_t* wsrc = P.src + tl.src + size_t(l) * every * 2u;
      for (uint32_t cc = lane * 8u; cc < every; cc += 16u)
        dot8<NT>(load_stored8(wsrc + 2u * cc), act, ld_in, sh.tok, ntk, k0 + cc, acc);
    } else {
      const uint32_t nseg_t = ts1 - ts0;
      PlaneRun r;
      seg_open(r, P, tl, t, l, lane);
      const uint32_t lut_s = uint32_t(__cvta_generic_to_shared(&sh.lut[lane][0]));
      const unsigned mask = 0x3u << (tid & 30u);
      const bool degenerate = sh.degenerate[lane] != 0;
      const uint32_t x0 = r.x, c0 = r.cur;
      // whole segment on the clamped window; a pair that does not land where
      // the encoder's stream did redoes the segment on the exact path
      bool exact = (every & 15u) || !__all_sync(mask, !degenerate && win_can_open(r));
      if (!exact) {
        Window W;
        win_open(W, r);
        uint32_t x = r.x;
        for (uint32_t done = 0; done < every; done += 16) {
          uint32_t a[4];
          win_decode16(lut_s, x, W, a);
          const uint4 w = exchange_pair16(lane, a[0], a[1], a[2], a[3], mask);
          dot8<NT>(w, act, ld_in, sh.tok, ntk, k0 + done + 8u * lane, acc);
        }
        r.x = x;
        r.cur = win_cur(W);
        if (__any_sync(mask, !seg_landed(r, P, t, l, nseg_t, lane))) {
          exact = true;
          r.x = x0;
          r.cur = c0;
#pragma unroll
          for (int j = 0; j < NT; j++) acc[j] = 0.f;
        }
      }
      if (exact) {  // lockstep pair: both planes decode `every` symbols
        for (uint32_t done = 0; done < every; done++) {
          const uint32_t sym = rans_step_exact(lut_s, degenerate, r);
          const uint32_t other = __shfl_xor_sync(mask, sym, 1);
          if (lane == 0) {
            const float w = bf2f(sym | (other << 8));
#pragma unroll
            for (int j = 0; j < NT; j++)
              if (j < int(ntk)) acc[j] = fmaf(w, bf2f(act[size_t(sh.tok[j]) * ld_in + k0 + done]), acc[j]);
          }
        }
        if (!seg_landed(r, P, t, l, nseg_t, lane)) atomicOr(&sh.status, kStatusPage);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], 1);
  if (p < nseg && lane == 0) {
#pragma unroll
    for (int j = 0; j < NT; j++) sh.part[p][j] = acc[j];
  }
  __syncthreads();
  // rows of the chunk: the row's segments summed in order; whole rows are
  // written, seam rows add into their cell
  uint16_t* out = second ? out1 : out0;
  const uint32_t rfirst = g0 / spr, nrows = (g1 - 1u) / spr - rfirst + 1u;
  bool added = false;
  for (uint32_t q = tid; q < nrows * ntk; q += kThreads) {
    const uint32_t ri = q / ntk, j = q - ri * ntk, row = rfirst + ri;
    const uint32_t a = max(g0, row * spr), b = min(g1, (row + 1u) * spr);
    float sum = 0.f;
    for (uint32_t g = a; g < b; g++) sum += sh.part[g - g0][j];
    if (b - a == spr) {
      out[size_t(row_base + j) * ld_out + row] = uint16_t(f2bf(sum));
    } else {
      const uint32_t k = (sh.seam_rows > 1 && sh.seam_row[1] == row) ? 1u : 0u;
      atomicAdd(&seams[sh.seam_id[k]].v[j], sum);
      added = true;
    }
  }
  if (added) __threadfence();
  __syncthreads();
  if (tid == 0) {
    for (uint32_t k = 0; k < sh.seam_rows; k++) {  // the second chunk of a seam row finishes it
      SeamCell& cell = seams[sh.seam_id[k]];
      __threadfence();
      if (atomicAdd(&cell.count, 1u) == 1u) {
        __threadfence();
        for (uint32_t j = 0; j < ntk; j++)
          out[size_t(row_base + j) * ld_out + sh.seam_row[k]] = uint16_t(f2bf(atomicExch(&cell.v[j], 0.f)));
        atomicExch(&cell.count, 0u);
      }
    }
    if (sh.status) atomicOr(status, sh.status);
  }
  __syncthreads();  // the next item reuses the shared memory
}

// Persistent CUDA-core kernel: a grid of a few CTAs per SM pulls items
// (unique expert, chunk slot) from a global counter until none are left, so
// the uneven chunks of the routed experts spread evenly over the SMs.
// counter: zero before the launch.
template <int NT>
__global__ void __launch_bounds__(kThreads, 4) moe_proj_cc(const voom_expert_pages* __restrict__ pages,
                                                           const Routes* __restrict__ R, uint32_t which,
                                                           const uint16_t* __restrict__ act, uint32_t ld_in,
                                                           uint16_t* __restrict__ out0, uint16_t* __restrict__ out1,
                                                           uint32_t ld_out, uint32_t nbpp, uint32_t n_proj,
                                                           uint32_t cpt, uint32_t tiles_hint,
                                                           SeamCell* __restrict__ seams, uint32_t* counter,
                                                           uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  CcShared& sh = *reinterpret_cast<CcShared*>(smem_raw);
  __shared__ uint32_t s_item;
  const uint32_t per_u = n_proj * nbpp, total = R->n_owned * per_u;
  for (;;) {
    if (threadIdx.x == 0) s_item = atomicAdd(counter, 1u);
    __syncthreads();
    const uint32_t item = s_item;
    __syncthreads();
    if (item >= total) break;
    const uint32_t o = item / per_u;
    cc_item<NT>(sh, pages, R, which, R->owned[o], item - o * per_u, act, ld_in, out0, out1, ld_out, nbpp, cpt,
                tiles_hint, seams, status);
  }
}

// ------------------------------------------------------- tcgen05 primitives
constexpr uint32_t kMmaRows = 128;  // UMMA M: weight rows of a CTA, one per TMEM lane
constexpr uint32_t kMmaK = 64;      // K elements per shared-memory stage (small: two CTAs per SM)
constexpr uint32_t kMmaMaxN = 256;  // tokens per CTA (UMMA N <= 256)
constexpr uint32_t kMbarSpin = 1u << 20;  // bounded completion waits

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

// Shared-memory matrix descriptor (tcgen05): start address, leading and
// stride byte offsets (all >> 4), descriptor version 1, no swizzle.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor of kind::f16: fp32 accumulator, BF16 A and B, both
// K-major, no negation, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t M, uint32_t N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete; false after kMbarSpin tries.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMbarSpin; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 8 consecutive fp32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
  v[4] = __uint_as_float(r4);
  v[5] = __uint_as_float(r5);
  v[6] = __uint_as_float(r6);
  v[7] = __uint_as_float(r7);
}

// Byte offset of (row, k) in a K-major no-swizzle UMMA tile of kMmaK columns:
// 8-row x 16-byte core matrices, the kMmaK / 8 core matrices of a row group
// side by side (leading byte offset 128), row groups kMmaK * 16 bytes apart
// (stride byte offset).  k must be a multiple of 8 (one 16-byte chunk).
__device__ __forceinline__ uint32_t umma_off(uint32_t row, uint32_t k) {
  return (row >> 3) * (kMmaK * 16u) + (k >> 3) * 128u + (row & 7u) * 16u;
}

// ------------------------------------------------------ tensor-core path
struct MmaMisc {
  uint64_t mbar;
  uint32_t tmem_base;
  uint32_t redo;
  uint32_t status;
  uint32_t cum[257];
  uint32_t red[8];
  uint32_t degenerate[2][2];
  uint32_t tok[kMmaMaxN];
};

constexpr uint32_t kMmaLutBytes = 2u * 2u * 4096u * 4u;  // two tiles x two planes
constexpr uint32_t kMmaABytes = kMmaRows * kMmaK * 2u;

__host__ __device__ inline uint32_t mma_smem_bytes(uint32_t ncap) {
  return kMmaLutBytes + kMmaABytes + ncap * kMmaK * 2u + uint32_t(sizeof(MmaMisc));
}

__device__ __forceinline__ uint32_t tmem_cols(uint32_t n) {
  uint32_t c = 32;
  while (c < n) c <<= 1;
  return c;
}

// Same arguments as moe_proj_cc; ncap = the B tile's token capacity (a
// multiple of 16, <= 256) the launch sized shared memory for.  Grid: x = row
// blocks of 128 (gate then up for which = 0), y = unique experts, z = chunks
// of 256 tokens.
__global__ void __launch_bounds__(kThreads, 2) moe_proj_mma(const voom_expert_pages* __restrict__ pages,
                                                            const Routes* __restrict__ R, uint32_t which,
                                                            const uint16_t* __restrict__ act, uint32_t ld_in,
                                                            uint16_t* __restrict__ out0, uint16_t* __restrict__ out1,
                                                            uint32_t ld_out, uint32_t nbpp, uint32_t ncap,
                                                            uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (blockIdx.y >= R->n_owned) return;
  const uint32_t u = R->owned[blockIdx.y];
  const uint32_t n = R->ntok[u];
  if (n <= uint32_t(kTok)) return;  // moe_proj_cc serves this expert
  const uint32_t j0 = blockIdx.z * kMmaMaxN;
  if (j0 >= n) return;
  const uint32_t nz = min(n - j0, kMmaMaxN), N = (nz + 15u) & ~15u;
  bool second;
  uint32_t blk;
  const voom_expert_proj& P = pick_proj(pages[R->expert[u]], which, nbpp, blockIdx.x, &second, &blk);
  if (P.n_tiles == 0) return;
  const uint32_t r0 = blk * kMmaRows;
  if (r0 >= P.rows) return;
  const uint32_t r1 = min(P.rows, r0 + kMmaRows);
  const uint32_t every = P.every, K = P.cols, spr = K / every;
  const uint32_t KS = every < kMmaK ? every : kMmaK, steps = K / KS;
  const uint32_t spt = P.tiles[0].raw_len / (2u * every);
  const uint32_t t0 = spt ? (r0 * spr) / spt : 0u, t1 = spt ? (r1 * spr - 1u) / spt : 0u;
  const uint32_t tid = threadIdx.x, lane = tid & 1u, p = tid >> 1, warp = tid >> 5;
  if (N > ncap || spt == 0 || t1 - t0 > 1u || every != every_rule(P.rows, K) || (every & 15u)) {
    if (tid == 0) atomicOr(status, kStatusGeometry);
    return;
  }
  uint8_t* s_lut = smem_raw;
  uint8_t* s_a = smem_raw + kMmaLutBytes;
  uint8_t* s_b = s_a + kMmaABytes;
  MmaMisc& m = *reinterpret_cast<MmaMisc*>(s_b + ncap * kMmaK * 2u);
  const uint32_t bar = smem_u32(&m.mbar);
  const uint32_t ncols = tmem_cols(N);
  if (warp == 0) tmem_alloc(smem_u32(&m.tmem_base), ncols);
  if (tid == 0) {
    mbar_init(bar, 1);
    m.redo = 0;
    m.status = 0;
  }
  const uint32_t row_base = R->uoff[u] + j0;
  for (uint32_t j = tid; j < N; j += kThreads) m.tok[j] = j < nz ? (which ? row_base + j : R->upair[row_base + j]) : 0u;
  for (uint32_t k = 0; k <= t1 - t0; k++) {
    const voom_rans_tile& tl = P.tiles[t0 + k];
    if (tl.mode == 1) {
      uint32_t* lut = reinterpret_cast<uint32_t*>(s_lut) + k * 2u * 4096u;
      build_lut(lut, m.cum, m.red, &m.degenerate[k][0], P.src + tl.low_freq);
      build_lut(lut + 4096, m.cum, m.red, &m.degenerate[k][1], P.src + tl.high_freq);
    }
  }
  // rows past the block's end and tokens past nz stay zero in every stage
  for (uint32_t i = tid; i < (kMmaABytes + N * kMmaK * 2u) / 16u; i += kThreads)
    reinterpret_cast<uint4*>(s_a)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = m.tmem_base;
  const uint32_t idesc = umma_idesc_bf16(kMmaRows, N);
  const uint32_t a_s = smem_u32(s_a), b_s = smem_u32(s_b);
  const bool active = r0 + p < r1;
  const unsigned mask = 0x3u << (tid & 30u);
  uint32_t ncommit = 0;
  bool timeout = false;
  for (uint32_t mode = 0; mode < 2; mode++) {
    // segment state of this lane's plane, carried across the K-steps of a segment
    PlaneRun r;
    Window W;
    uint32_t x = 0, t = 0, l = 0, nseg_t = 0, lut_s = 0, tmode = 1;
    bool win = false, degenerate = false;
    for (uint32_t s = 0; s < steps; s++) {
      const uint32_t k0 = s * KS, c = k0 / every, o = k0 - c * every;
      if (active && o == 0) {  // open segment c of this row
        const uint32_t g = (r0 + p) * spr + c;
        t = g / spt;
        l = g - t * spt;
        const voom_rans_tile& tl = P.tiles[t];
        tmode = tl.mode;
        nseg_t = tl.raw_len / (2u * every);
        if (tmode == 1) {
          seg_open(r, P, tl, t, l, lane);
          lut_s = smem_u32(s_lut) + ((t - t0) * 2u + lane) * 16384u;
          degenerate = m.degenerate[t - t0][lane] != 0;
          win = __all_sync(mask, mode == 0 && !degenerate && win_can_open(r));
          if (win) {
            win_open(W, r);
            x = r.x;
          }
        }
      }
      uint4 wv[kMmaK / 16];
      if (active && tmode == 1 && win) {
#pragma unroll
        for (uint32_t q = 0; q < kMmaK / 16; q++) {
          if (q < KS / 16) {
            uint32_t a[4];
            win_decode16(lut_s, x, W, a);
            wv[q] = exchange_pair16(lane, a[0], a[1], a[2], a[3], mask);
          }
        }
      }
      // the previous step's MMAs must be done reading the tiles
      if (ncommit && !mbar_wait(bar, (ncommit - 1u) & 1u)) timeout = true;
      if (active) {
        if (tmode == 0) {
          const uint8_t* wsrc = P.src + P.tiles[t].src + (size_t(l) * every + o) * 2u;
          for (uint32_t q = lane; q < KS / 8u; q += 2u)
            *reinterpret_cast<uint4*>(s_a + umma_off(p, 8u * q)) = load_stored8(wsrc + 16u * q);
        } else if (win) {
#pragma unroll
          for (uint32_t q = 0; q < kMmaK / 16; q++)
            if (q < KS / 16) *reinterpret_cast<uint4*>(s_a + umma_off(p, 16u * q + 8u * lane)) = wv[q];
        } else {  // exact lockstep pair
          for (uint32_t i = 0; i < KS; i++) {
            const uint32_t sym = rans_step_exact(lut_s, degenerate, r);
            const uint32_t other = __shfl_xor_sync(mask, sym, 1);
            if (lane == 0)
              *reinterpret_cast<uint16_t*>(s_a + umma_off(p, i & ~7u) + 2u * (i & 7u)) = uint16_t(sym | (other << 8));
          }
        }
        if (tmode == 1 && o + KS == every) {  // segment end: landing check
          if (win) {
            r.x = x;
            r.cur = win_cur(W);
          }
          if (!seg_landed(r, P, t, l, nseg_t, lane)) atomicOr(&m.redo, 1u);
        }
      }
      // the tokens' activations for columns k0 .. k0 + KS
      for (uint32_t i = tid; i < nz * (KS / 8u); i += kThreads) {
        const uint32_t j = i / (KS / 8u), q = i - j * (KS / 8u);
        *reinterpret_cast<uint4*>(s_b + umma_off(j, 8u * q)) =
            __ldg(reinterpret_cast<const uint4*>(act + size_t(m.tok[j]) * ld_in + k0 + 8u * q));
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        for (uint32_t i = 0; i < KS / 16u; i++)
          umma_bf16(tmem, umma_desc(a_s + 256u * i, 128u, kMmaK * 16u), umma_desc(b_s + 256u * i, 128u, kMmaK * 16u),
                    idesc, (s > 0 || i > 0) ? 1u : 0u);
        umma_commit(bar);
      }
      ncommit++;
    }
    if (!mbar_wait(bar, (ncommit - 1u) & 1u)) timeout = true;
    tc_fence_after();
    __syncthreads();
    const uint32_t redo = m.redo;
    __syncthreads();
    if (!redo) break;
    if (mode == 1) {  // the exact decode misses too: the page is damaged
      if (tid == 0) m.status |= kStatusPage;
      break;
    }
    if (tid == 0) m.redo = 0;  // a segment left the window path: redo the block exactly
    __syncthreads();
  }
  // epilogue: TMEM lane = weight row, column = token
  if (warp < 4) {
    const uint32_t row = r0 + warp * 32u + (tid & 31u);
    uint16_t* out = second ? out1 : out0;
    for (uint32_t cb = 0; cb < N; cb += 8) {
      float v[8];
      tmem_ld8(tmem + ((warp * 32u) << 16) + cb, v);
      if (row < r1) {
#pragma unroll
        for (uint32_t i = 0; i < 8; i++)
          if (cb + i < nz) out[size_t(row_base + cb + i) * ld_out + row] = uint16_t(f2bf(v[i]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  if (tid == 0) {
    const uint32_t st = m.status | (timeout ? kStatusTimeout : 0u);
    if (st) atomicOr(status, st);
  }
}

}  // namespace moe
}  // namespace voom
