// BF16 NF12 exact sidecar on sm_100a: block decode and the fused decode +
// small-M linear.
//
// Layer stream (formats/bf16_nf12_sidecar.py:318-420 of the reference):
//   [header_bytes: one 16-byte header per 256-value block]
//   [384 bytes of 12-bit codes per block]
//   [3-byte patches (local index, exact bits) of every block]
// Header (little-endian): patch offset u32 (absolute in the stream), output
// offset u32, valid u16, exception count u16, modal high exponent nibble u8,
// flags u8, reserved u16.  A 12-bit code holds bits 0-10 of the BF16 value
// and its sign in bit 11; the value is code & 0x7FF | (code & 0x800) << 4 |
// mode << 11, unless a patch of the block names its local index (the first
// such patch wins, runtime/bf16_nf12_sidecar.py:73-81).
//
// Both kernels are HBM-bound: 400 bytes of stream per 256 values, read once.
//  - nf12_decode: one warp per block, 8 values per lane from 12 code bytes
//    (three aligned u32 loads), 16-byte stores; patches applied after a warp
//    barrier, first-wins resolved by an atomicMin in shared memory.
//  - nf12_linear<M, R>: out[p, n] = sum_k x[p, k] * w[n, k] for M <= 8
//    activation rows.  A warp owns R consecutive weight rows and walks their
//    K/256 blocks together: per block each lane takes 8 columns, loads the M
//    activation slices for them once (reused by the R rows), decodes 8
//    weights of each row and accumulates M x R fp32 partial sums; a split of
//    the K range over warps (when there are too few row groups to fill the
//    GPU) writes fp32 partials that nf12_reduce sums in a fixed order, so the
//    result does not depend on scheduling.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace {

constexpr uint32_t kBlockValues = 256;
constexpr uint32_t kCodeBytes = 384;
constexpr uint32_t kHeaderBytes = 16;
constexpr uint32_t kPatchBytes = 3;

struct Hdr {
  uint32_t patch_off, out_off, valid, count, mode;
};

__device__ __forceinline__ Hdr load_hdr(const uint8_t* enc, uint32_t blk) {
  const uint4 h = __ldg(reinterpret_cast<const uint4*>(enc + uint64_t(blk) * kHeaderBytes));
  Hdr r;
  r.patch_off = h.x;
  r.out_off = h.y;
  r.valid = h.z & 0xFFFFu;
  r.count = h.z >> 16;
  r.mode = h.w & 15u;
  return r;
}

// The 8 codes of lane `lane` in a block: bytes [12 lane, 12 lane + 12).
__device__ __forceinline__ void lane_codes(const uint8_t* codes_blk, uint32_t lane, uint32_t (&c)[8]) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(codes_blk + 12u * lane);
  const uint32_t a = __ldg(q), b = __ldg(q + 1), d = __ldg(q + 2);
  c[0] = a & 0xFFFu;
  c[1] = (a >> 12) & 0xFFFu;
  c[2] = __funnelshift_r(a, b, 24) & 0xFFFu;
  c[3] = (b >> 4) & 0xFFFu;
  c[4] = (b >> 16) & 0xFFFu;
  c[5] = __funnelshift_r(b, d, 28) & 0xFFFu;
  c[6] = (d >> 8) & 0xFFFu;
  c[7] = d >> 20;
}

__device__ __forceinline__ uint32_t restore(uint32_t code, uint32_t mode11) {
  return (code & 0x7FFu) | ((code & 0x800u) << 4) | mode11;
}

constexpr int kDecodeWarps = 8;

__global__ void __launch_bounds__(32 * kDecodeWarps) nf12_decode(const uint8_t* __restrict__ enc, uint64_t enc_bytes,
                                                                 uint64_t header_bytes, uint32_t first_block,
                                                                 uint32_t n_blocks, uint64_t output_base,
                                                                 uint16_t* __restrict__ out, uint64_t out_values,
                                                                 uint32_t* status) {
  __shared__ uint32_t s_win[kDecodeWarps][kBlockValues];
  const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
  for (uint32_t w = blockIdx.x * kDecodeWarps + wid; w < n_blocks; w += gridDim.x * kDecodeWarps) {
    const uint32_t blk = first_block + w;
    const Hdr h = load_hdr(enc, blk);
    const uint64_t o = uint64_t(h.out_off) - output_base;
    const bool bad = h.valid > kBlockValues || uint64_t(h.out_off) < output_base || o + h.valid > out_values ||
                     uint64_t(h.patch_off) + uint64_t(h.count) * kPatchBytes > enc_bytes;
    if (bad) {  // warp-uniform
      if (lane == 0) atomicOr(status, 1u);
      continue;
    }
    uint32_t c[8];
    lane_codes(enc + header_bytes + uint64_t(blk) * kCodeBytes, lane, c);
    const uint32_t m11 = h.mode << 11;
    const uint32_t l0 = lane * 8u;
    uint16_t* dst = out + o + l0;
    if (l0 + 8 <= h.valid && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
      uint4 v;
      v.x = restore(c[0], m11) | (restore(c[1], m11) << 16);
      v.y = restore(c[2], m11) | (restore(c[3], m11) << 16);
      v.z = restore(c[4], m11) | (restore(c[5], m11) << 16);
      v.w = restore(c[6], m11) | (restore(c[7], m11) << 16);
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
#pragma unroll
      for (uint32_t i = 0; i < 8; i++)
        if (l0 + i < h.valid) dst[i] = uint16_t(restore(c[i], m11));
    }
    if (h.count) {  // warp-uniform: first patch of a local index wins
      const uint8_t* pp = enc + h.patch_off;
      for (uint32_t i = lane; i < kBlockValues; i += 32) s_win[wid][i] = 0xFFFFFFFFu;
      __syncwarp();
      for (uint32_t p = lane; p < h.count; p += 32) {
        const uint32_t local = pp[kPatchBytes * p];
        if (local < h.valid) atomicMin(&s_win[wid][local], p);
      }
      __syncwarp();
      for (uint32_t p = lane; p < h.count; p += 32) {
        const uint32_t local = pp[kPatchBytes * p];
        if (local < h.valid && s_win[wid][local] == p)
          out[o + local] = uint16_t(pp[kPatchBytes * p + 1] | (uint32_t(pp[kPatchBytes * p + 2]) << 8));
      }
      __syncwarp();
    }
  }
}

constexpr int kLinWarps = 8;

template <int M>
struct Fix {
  float v[M];
};

// Exceptions of one block that fall in [lo, lo + len): the main loop used
// the weight decoded with the modal nibble, so each adds x * (exact -
// decoded) (the first patch of an index wins).  Kept out of line: it runs
// only for blocks with exceptions.
template <int M>
__device__ __noinline__ Fix<M> patch_fix(const uint8_t* __restrict__ enc, uint64_t codes_off, uint32_t poff,
                                         uint32_t cnt, uint32_t m27, uint32_t lo, uint32_t len,
                                         const uint16_t* __restrict__ xb, uint32_t K) {
  Fix<M> f;
#pragma unroll
  for (int p = 0; p < M; p++) f.v[p] = 0.f;
  const uint8_t* pp = enc + poff;
  for (uint32_t i = 0; i < cnt; i++) {
    const uint32_t local = pp[kPatchBytes * i];
    if (local < lo || local >= lo + len) continue;
    bool first = true;
    for (uint32_t j = 0; j < i; j++) first &= pp[kPatchBytes * j] != local;
    if (!first) continue;
    const uint8_t* cb = enc + codes_off + 3u * (local >> 1);
    const uint32_t pair = cb[0] | (uint32_t(cb[1]) << 8) | (uint32_t(cb[2]) << 16);
    const uint32_t code = (local & 1) ? pair >> 12 : pair & 0xFFFu;
    const float dec = __uint_as_float(((code & 0x7FFu) << 16) | ((code & 0x800u) << 20) | m27);
    const float ex = __uint_as_float((pp[kPatchBytes * i + 1] | (uint32_t(pp[kPatchBytes * i + 2]) << 8)) << 16);
#pragma unroll
    for (int p = 0; p < M; p++) {
      const float xv = __uint_as_float(uint32_t(xb[uint64_t(p) * K + local]) << 16);
      f.v[p] = fmaf(xv, ex, fmaf(-xv, dec, f.v[p]));
    }
  }
  return f;
}

// One weight matrix of a fused linear launch: out = x @ W.T with W the
// N x K tensor whose blocks start at first_block.  Warps [warp_begin,
// warp_begin + row_groups * splits) of the launch work on it; with splits > 1
// each writes fp32 partial sums of its K range to partial[split][M][N].
struct LinTask {
  const uint16_t* x;
  uint16_t* out;
  float* partial;
  uint32_t K, N, first_block, splits, row_groups, warp_begin;
};

constexpr int kMaxTasks = 16;

struct LinTasks {
  LinTask t[kMaxTasks];
  uint32_t n;
};

// Packed BF16 pair (low value in bits 0-15) of the 24-bit code pair at bits
// 0-23 of y: per value its low 11 code bits, its sign (code bit 11) at bit
// 15, and the modal nibble (m2 = mode << 11 | mode << 27) in bits 11-14.
__device__ __forceinline__ uint32_t pair_bf16x2(uint32_t y, uint32_t m2) {
  return (y & 0x7FFu) | ((y << 4) & 0x07FF8000u) | ((y << 8) & 0x80000000u) | m2;
}

// The 16 packed pairs of 48 code bytes (three uint4 = 12 words; every 3
// words hold 4 pairs).
__device__ __forceinline__ void pairs16(const uint4 (&q)[3], uint32_t m2, uint32_t (&pk)[16]) {
  const uint32_t w[12] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w,
                          q[2].x, q[2].y, q[2].z, q[2].w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t a = w[3 * i], b = w[3 * i + 1], d = w[3 * i + 2];
    pk[4 * i] = pair_bf16x2(a, m2);
    pk[4 * i + 1] = pair_bf16x2(__funnelshift_r(a, b, 24), m2);
    pk[4 * i + 2] = pair_bf16x2(__funnelshift_r(b, d, 16), m2);
    pk[4 * i + 3] = pair_bf16x2(d >> 8, m2);
  }
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Warp of a task: 16 weight rows [row0, row0 + 16) x all tokens, one 256-value
// block of each row per step, on the tensor cores (mma m16n8k16, BF16 in,
// fp32 accumulate): weight rows are the MMA's M dimension, the (up to 8)
// activation rows its N dimension.  Lane (g = lane / 4, t = lane % 4) decodes
// code pairs [32 t, 32 t + 32) of rows g and g + 8 (96 contiguous code bytes
// each) straight into A-fragment registers; because the sum over k may run
// in any order, MMA k-pairs t and t + 4 of slice s are the lane's own pairs
// 2 s and 2 s + 1, and the activation fragment (token g) is loaded with the
// same mapping.  Exceptions (decoded with the modal nibble) are corrected
// out of line.
template <int M>
__device__ __forceinline__ void linear_tile(const LinTask& T, uint32_t w, uint32_t lane, const uint8_t* __restrict__ enc,
                                            uint64_t enc_bytes, uint64_t header_bytes, uint32_t* status) {
  const uint32_t tiles = T.row_groups;
  const uint32_t tile = w % tiles, sp = w / tiles;
  const uint32_t N = T.N, K = T.K;
  const uint32_t g = lane >> 2, t = lane & 3u;
  const uint32_t r0 = tile * 16 + g, r1 = r0 + 8;
  const bool v0 = r0 < N, v1 = r1 < N;
  const uint32_t kblocks = K / kBlockValues;
  const uint32_t per = (kblocks + T.splits - 1) / T.splits;
  const uint32_t kb0 = sp * per, kb1 = min(kblocks, kb0 + per);
  const uint16_t* __restrict__ x = T.x;
  const bool xon = g < uint32_t(M);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  float e[4] = {0.f, 0.f, 0.f, 0.f};  // second accumulator: halves the MMA dependency chain
  float corr[2][M];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int p = 0; p < M; p++) corr[h][p] = 0.f;
  bool bad = false;
  for (uint32_t kb = kb0; kb < kb1; kb++) {
    const uint32_t blk0 = T.first_block + (v0 ? r0 : 0) * kblocks + kb;
    const uint32_t blk1 = T.first_block + (v1 ? r1 : 0) * kblocks + kb;
    const uint4 h0 = __ldg(reinterpret_cast<const uint4*>(enc + uint64_t(blk0) * kHeaderBytes));
    const uint4 h1 = __ldg(reinterpret_cast<const uint4*>(enc + uint64_t(blk1) * kHeaderBytes));
    uint4 q0[6], q1[6];
    const uint4* c0 = reinterpret_cast<const uint4*>(enc + header_bytes + uint64_t(blk0) * kCodeBytes + 96u * t);
    const uint4* c1 = reinterpret_cast<const uint4*>(enc + header_bytes + uint64_t(blk1) * kCodeBytes + 96u * t);
#pragma unroll
    for (int i = 0; i < 6; i++) {
      q0[i] = __ldg(c0 + i);
      q1[i] = __ldg(c1 + i);
    }
    const uint32_t mode0 = h0.w & 15u, mode1 = h1.w & 15u;
    bad |= (v0 && (h0.z & 0xFFFFu) != kBlockValues) || (v1 && (h1.z & 0xFFFFu) != kBlockValues);
    const uint32_t m20 = (mode0 << 11) | (mode0 << 27), m21 = (mode1 << 11) | (mode1 << 27);
    // activations of token g for k = kb * 256 + 64 t .. + 64, in two halves
    const uint4* xp = reinterpret_cast<const uint4*>(x + uint64_t(xon ? g : 0) * K + uint64_t(kb) * kBlockValues + 64u * t);
#pragma unroll
    for (int half = 0; half < 2; half++) {
      uint4 xv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) xv[i] = xon ? __ldg(xp + 4 * half + i) : make_uint4(0, 0, 0, 0);
      const uint4 qa[3] = {q0[3 * half], q0[3 * half + 1], q0[3 * half + 2]};
      const uint4 qb[3] = {q1[3 * half], q1[3 * half + 1], q1[3 * half + 2]};
      uint32_t a[16], b[16];
      pairs16(qa, m20, a);
      pairs16(qb, m21, b);
      const uint32_t xw[16] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w,
                               xv[2].x, xv[2].y, xv[2].z, xv[2].w, xv[3].x, xv[3].y, xv[3].z, xv[3].w};
#pragma unroll
      for (int s = 0; s < 8; s += 2) {
        mma_bf16_16816(d, a[2 * s], b[2 * s], a[2 * s + 1], b[2 * s + 1], xw[2 * s], xw[2 * s + 1]);
        mma_bf16_16816(e, a[2 * s + 2], b[2 * s + 2], a[2 * s + 3], b[2 * s + 3], xw[2 * s + 2], xw[2 * s + 3]);
      }
    }
    // rare: exceptions of rows g / g + 8 in this lane's 64 values
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const uint4 hd = hh ? h1 : h0;
      const bool vv = hh ? v1 : v0;
      const uint32_t cnt = hd.z >> 16;
      if (vv && cnt) {
        const uint32_t m27 = (hd.w & 15u) << 27;
        if (m27 == (15u << 27) || uint64_t(hd.x) + uint64_t(cnt) * kPatchBytes > enc_bytes) {
          bad = true;  // patches outside the stream, or a modal nibble of 15 (an exception may decode to Inf)
        } else {
          const uint32_t blk = hh ? blk1 : blk0;
          const Fix<M> f = patch_fix<M>(enc, header_bytes + uint64_t(blk) * kCodeBytes, hd.x, cnt, m27, 64u * t,
                                        64u, x + uint64_t(kb) * kBlockValues, K);
#pragma unroll
          for (int p = 0; p < M; p++) corr[hh][p] += f.v[p];
        }
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(status, 2u);
#pragma unroll
  for (int i = 0; i < 4; i++) d[i] += e[i];
  // corrections: sum over the 4 lanes of the row group, then each lane adds
  // those of its two tokens 2t, 2t + 1
#pragma unroll
  for (int hh = 0; hh < 2; hh++)
#pragma unroll
    for (int p = 0; p < M; p++) {
      corr[hh][p] += __shfl_xor_sync(0xFFFFFFFFu, corr[hh][p], 1);
      corr[hh][p] += __shfl_xor_sync(0xFFFFFFFFu, corr[hh][p], 2);
    }
#pragma unroll
  for (int p = 0; p < M; p++) {
    if (uint32_t(p) == 2 * t) {
      d[0] += corr[0][p];
      d[2] += corr[1][p];
    }
    if (uint32_t(p) == 2 * t + 1) {
      d[1] += corr[0][p];
      d[3] += corr[1][p];
    }
  }
  // D fragment: d0, d1 = rows r0, tokens 2t, 2t+1; d2, d3 = row r1
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t p = 2 * t + (i & 1);
    const uint32_t row = i < 2 ? r0 : r1;
    if (p >= uint32_t(M) || row >= N) continue;
    if (T.splits == 1) {
      T.out[uint64_t(p) * N + row] = __bfloat16_as_ushort(__float2bfloat16_rn(d[i]));
    } else {
      T.partial[(uint64_t(sp) * M + p) * N + row] = d[i];
    }
  }
}

template <int M>
__global__ void __launch_bounds__(32 * kLinWarps)
    nf12_linear(const LinTasks tasks, uint32_t total_warps, const uint8_t* __restrict__ enc, uint64_t enc_bytes,
                uint64_t header_bytes, uint32_t* status) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = blockIdx.x * kLinWarps + (threadIdx.x >> 5);
  if (warp >= total_warps) return;
  uint32_t i = 0;
  while (i + 1 < tasks.n && warp >= tasks.t[i + 1].warp_begin) i++;
  linear_tile<M>(tasks.t[i], warp - tasks.t[i].warp_begin, lane, enc, enc_bytes, header_bytes, status);
}

// Sums the split partials of every split task in split order.
__global__ void nf12_reduce(const LinTasks tasks, uint32_t M) {
  for (uint32_t ti = 0; ti < tasks.n; ti++) {
    const LinTask& T = tasks.t[ti];
    if (T.splits < 2) continue;
    const uint64_t n = uint64_t(M) * T.N;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
      float s = 0.f;
      for (uint32_t sp = 0; sp < T.splits; sp++) s += T.partial[uint64_t(sp) * n + i];
      T.out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(s));
    }
  }
}

int g_sms = 0;

int sm_count() {
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  return g_sms;
}

// Split plan of a launch: when the tasks' row groups are too few to keep
// about 16 warps resident per SM, every task's K range is split (at least 2
// groups of 4 blocks per split) and its fp32 partials take their place in the
// scratch, task after task.  Returns the scratch bytes needed.
uint64_t plan_tasks(LinTasks& L, uint32_t M) {
  uint64_t tiles = 0;
  for (uint32_t i = 0; i < L.n; i++) {
    L.t[i].row_groups = (L.t[i].N + 15) / 16;
    tiles += L.t[i].row_groups;
  }
  const uint64_t want = uint64_t(sm_count()) * 16;
  const uint32_t f = tiles >= want ? 1u : uint32_t((want + tiles - 1) / tiles);
  uint64_t scratch = 0;
  uint32_t warp = 0;
  for (uint32_t i = 0; i < L.n; i++) {
    LinTask& T = L.t[i];
    const uint32_t kblocks = T.K / kBlockValues;
    // at most 16 blocks of K per warp (long rows would otherwise set the
    // launch's tail), more splits while the launch has too few warps, at
    // least 4 blocks per split
    uint32_t sp = (kblocks + 15) / 16;
    sp = sp > f ? sp : f;
    sp = sp < kblocks / 4 ? sp : kblocks / 4;
    T.splits = sp < 1 ? 1 : sp;
    T.warp_begin = warp;
    warp += T.row_groups * T.splits;
    if (T.splits > 1) scratch += uint64_t(T.splits) * M * T.N * sizeof(float);
  }
  return scratch;
}

template <int M>
void launch_tasks(const LinTasks& L, const uint8_t* enc, uint64_t enc_bytes, uint64_t header_bytes, uint32_t* status,
                  cudaStream_t s) {
  const LinTask& last = L.t[L.n - 1];
  const uint32_t warps = last.warp_begin + last.row_groups * last.splits;
  nf12_linear<M><<<(warps + kLinWarps - 1) / kLinWarps, 32 * kLinWarps, 0, s>>>(L, warps, enc, enc_bytes,
                                                                                header_bytes, status);
}

int run_tasks(LinTasks& L, uint32_t M, const uint8_t* enc, uint64_t enc_bytes, uint64_t header_bytes, void* scratch,
              uint64_t scratch_bytes, uint32_t* status, cudaStream_t s) {
  const uint64_t need = plan_tasks(L, M);
  if (need && (!scratch || scratch_bytes < need)) return VOOM_E_CAPACITY;
  uint64_t off = 0;
  bool split = false;
  for (uint32_t i = 0; i < L.n; i++) {
    LinTask& T = L.t[i];
    if (T.splits > 1) {
      T.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + off);
      off += uint64_t(T.splits) * M * T.N * sizeof(float);
      split = true;
    } else {
      T.partial = nullptr;
    }
  }
  switch (M) {
    case 1: launch_tasks<1>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 2: launch_tasks<2>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 3: launch_tasks<3>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 4: launch_tasks<4>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 5: launch_tasks<5>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 6: launch_tasks<6>(L, enc, enc_bytes, header_bytes, status, s); break;
    case 7: launch_tasks<7>(L, enc, enc_bytes, header_bytes, status, s); break;
    default: launch_tasks<8>(L, enc, enc_bytes, header_bytes, status, s); break;
  }
  if (split) nf12_reduce<<<sm_count() * 2, 256, 0, s>>>(L, M);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

// Host checks of one task: shapes the kernel takes and its blocks inside the stream.
int check_task(const uint16_t* x, const uint16_t* out, uint32_t M, uint32_t K, uint32_t N, uint32_t first_block,
               uint64_t enc_bytes, uint64_t header_bytes) {
  if (!x || !out) return VOOM_E_INVALID_ARG;
  if (!M || M > 8 || !N || !K || K % 512 || N % 8) return VOOM_E_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(x) & 15u) return VOOM_E_INVALID_ARG;
  const uint64_t end = uint64_t(first_block) + uint64_t(N) * (K / kBlockValues);
  if (end * kHeaderBytes > header_bytes || header_bytes + end * kCodeBytes > enc_bytes) return VOOM_E_INVALID_ARG;
  return VOOM_OK;
}

}  // namespace

VOOM_API int voom_nf12_decode(const uint8_t* d_enc, uint64_t enc_bytes, uint64_t header_bytes, uint32_t first_block,
                              uint32_t n_blocks, uint64_t output_base, uint16_t* d_out, uint64_t out_values,
                              uint32_t* d_status, void* stream) {
  if (!d_enc || !d_out || !d_status) return VOOM_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(d_enc) & 15u) return VOOM_E_INVALID_ARG;
  if (header_bytes % kHeaderBytes) return VOOM_E_INVALID_ARG;
  const uint64_t end = uint64_t(first_block) + n_blocks;
  if (end * kHeaderBytes > header_bytes || header_bytes + end * kCodeBytes > enc_bytes) return VOOM_E_INVALID_ARG;
  if (!n_blocks) return VOOM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t grid = (n_blocks + kDecodeWarps - 1) / kDecodeWarps;
  const uint32_t cap = uint32_t(sm_count()) * 16;
  grid = grid < cap ? grid : cap;
  nf12_decode<<<grid, 32 * kDecodeWarps, 0, s>>>(d_enc, enc_bytes, header_bytes, first_block, n_blocks, output_base,
                                                 d_out, out_values, d_status);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API uint64_t voom_nf12_linear_scratch_bytes(uint32_t M, uint32_t K, uint32_t N) {
  if (!M || M > 8 || !N || !K || K % 512) return 0;
  LinTasks L{};
  L.n = 1;
  L.t[0].K = K;
  L.t[0].N = N;
  return plan_tasks(L, M);
}

VOOM_API int voom_nf12_linear(const uint16_t* d_x, uint32_t M, uint32_t K, uint32_t N, const uint8_t* d_enc,
                              uint64_t enc_bytes, uint64_t header_bytes, uint32_t first_block, void* d_scratch,
                              uint64_t scratch_bytes, uint16_t* d_out, uint32_t* d_status, void* stream) {
  if (!d_enc || !d_status || (reinterpret_cast<uintptr_t>(d_enc) & 15u) || header_bytes % kHeaderBytes)
    return VOOM_E_INVALID_ARG;
  const int rc = check_task(d_x, d_out, M, K, N, first_block, enc_bytes, header_bytes);
  if (rc != VOOM_OK) return rc;
  LinTasks L{};
  L.n = 1;
  L.t[0].x = d_x;
  L.t[0].out = d_out;
  L.t[0].K = K;
  L.t[0].N = N;
  L.t[0].first_block = first_block;
  return run_tasks(L, M, d_enc, enc_bytes, header_bytes, d_scratch, scratch_bytes, d_status,
                   static_cast<cudaStream_t>(stream));
}

VOOM_API uint64_t voom_nf12_linear_batch_scratch_bytes(const voom_nf12_linear_task* tasks, uint32_t n, uint32_t M) {
  if (!tasks || !n || n > kMaxTasks || !M || M > 8) return 0;
  LinTasks L{};
  L.n = n;
  for (uint32_t i = 0; i < n; i++) {
    if (!tasks[i].K || tasks[i].K % 512 || !tasks[i].N) return 0;
    L.t[i].K = tasks[i].K;
    L.t[i].N = tasks[i].N;
  }
  return plan_tasks(L, M);
}

VOOM_API int voom_nf12_linear_batch(const voom_nf12_linear_task* tasks, uint32_t n, uint32_t M, const uint8_t* d_enc,
                                    uint64_t enc_bytes, uint64_t header_bytes, void* d_scratch,
                                    uint64_t scratch_bytes, uint32_t* d_status, void* stream) {
  if (!tasks || !n || !d_enc || !d_status || (reinterpret_cast<uintptr_t>(d_enc) & 15u) ||
      header_bytes % kHeaderBytes)
    return VOOM_E_INVALID_ARG;
  if (n > kMaxTasks) return VOOM_E_CAPACITY;
  LinTasks L{};
  L.n = n;
  for (uint32_t i = 0; i < n; i++) {
    const voom_nf12_linear_task& t = tasks[i];
    const int rc = check_task(t.d_x, t.d_out, M, t.K, t.N, t.first_block, enc_bytes, header_bytes);
    if (rc != VOOM_OK) return rc;
    L.t[i].x = t.d_x;
    L.t[i].out = t.d_out;
    L.t[i].K = t.K;
    L.t[i].N = t.N;
    L.t[i].first_block = t.first_block;
  }
  return run_tasks(L, M, d_enc, enc_bytes, header_bytes, d_scratch, scratch_bytes, d_status,
                   static_cast<cudaStream_t>(stream));
}
