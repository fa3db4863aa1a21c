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

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

constexpr int kLinWarps = 8;

// Warp: rows [row0, row0 + R), K blocks [kb0, kb1) of each row.
template <int M, int R>
__global__ void __launch_bounds__(32 * kLinWarps) nf12_linear(const uint16_t* __restrict__ x, uint32_t K, uint32_t N,
                                                              const uint8_t* __restrict__ enc, uint64_t enc_bytes,
                                                              uint64_t header_bytes, uint32_t first_block,
                                                              uint32_t splits, float* __restrict__ partial,
                                                              uint16_t* __restrict__ out, uint32_t* status) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = blockIdx.x * kLinWarps + (threadIdx.x >> 5);
  const uint32_t groups = (N + R - 1) / R;
  if (warp >= groups * splits) return;
  const uint32_t g = warp % groups, sp = warp / groups;
  const uint32_t row0 = g * R;
  const uint32_t kblocks = K / kBlockValues;
  const uint32_t per = (kblocks + splits - 1) / splits;
  const uint32_t kb0 = sp * per, kb1 = min(kblocks, kb0 + per);
  float acc[M][R];
#pragma unroll
  for (int p = 0; p < M; p++)
#pragma unroll
    for (int r = 0; r < R; r++) acc[p][r] = 0.f;
  bool bad = false;
  for (uint32_t kb = kb0; kb < kb1; kb++) {
    const uint32_t k0 = kb * kBlockValues + lane * 8u;
    uint4 xv[M];
#pragma unroll
    for (int p = 0; p < M; p++) xv[p] = __ldg(reinterpret_cast<const uint4*>(x + uint64_t(p) * K + k0));
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t row = row0 + r;
      if (row >= N) break;
      const uint32_t blk = first_block + row * kblocks + kb;
      const Hdr h = load_hdr(enc, blk);
      uint32_t c[8];
      lane_codes(enc + header_bytes + uint64_t(blk) * kCodeBytes, lane, c);
      const uint32_t m11 = h.mode << 11;
      uint32_t wb[8];
#pragma unroll
      for (int i = 0; i < 8; i++) wb[i] = restore(c[i], m11);
      if (h.count) {  // rare: exceptions of this block, first patch of an index wins
        if (h.valid != kBlockValues || uint64_t(h.patch_off) + uint64_t(h.count) * kPatchBytes > enc_bytes) {
          bad = true;
        } else {
          const uint8_t* pp = enc + h.patch_off;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const uint32_t target = lane * 8u + uint32_t(i);
            for (uint32_t p = 0; p < h.count; p++) {
              if (pp[kPatchBytes * p] == target) {
                wb[i] = pp[kPatchBytes * p + 1] | (uint32_t(pp[kPatchBytes * p + 2]) << 8);
                break;
              }
            }
          }
        }
      } else if (h.valid != kBlockValues) {
        bad = true;
      }
      float w[8];
#pragma unroll
      for (int i = 0; i < 8; i++) w[i] = __uint_as_float(wb[i] << 16);
#pragma unroll
      for (int p = 0; p < M; p++) {
        float s = acc[p][r];
        s = fmaf(bf_lo(xv[p].x), w[0], s);
        s = fmaf(bf_hi(xv[p].x), w[1], s);
        s = fmaf(bf_lo(xv[p].y), w[2], s);
        s = fmaf(bf_hi(xv[p].y), w[3], s);
        s = fmaf(bf_lo(xv[p].z), w[4], s);
        s = fmaf(bf_hi(xv[p].z), w[5], s);
        s = fmaf(bf_lo(xv[p].w), w[6], s);
        s = fmaf(bf_hi(xv[p].w), w[7], s);
        acc[p][r] = s;
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(status, 2u);
#pragma unroll
  for (int p = 0; p < M; p++)
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[p][r] += __shfl_xor_sync(0xFFFFFFFFu, acc[p][r], o);
  if (lane == 0) {
#pragma unroll
    for (int p = 0; p < M; p++)
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t row = row0 + r;
        if (row >= N) continue;
        if (splits == 1) {
          out[uint64_t(p) * N + row] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[p][r]));
        } else {
          partial[(uint64_t(sp) * M + p) * N + row] = acc[p][r];
        }
      }
  }
}

__global__ void nf12_reduce(const float* __restrict__ partial, uint32_t splits, uint32_t M, uint32_t N,
                            uint16_t* __restrict__ out) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= uint64_t(M) * N) return;
  float s = 0.f;
  for (uint32_t sp = 0; sp < splits; sp++) s += partial[uint64_t(sp) * M * N + i];
  out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(s));
}

uint32_t rows_per_warp(uint32_t M) { return M <= 2 ? 2u : 4u; }

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

// K-range splits: enough warps to keep every SM busy (about 8 CTAs of 8 warps
// each), at least 2 blocks of K per split.
uint32_t pick_splits(uint32_t groups, uint32_t kblocks) {
  const uint64_t want = uint64_t(sm_count()) * 8 * kLinWarps;
  if (groups >= want) return 1;
  uint32_t s = uint32_t((want + groups - 1) / groups);
  s = s < kblocks / 2 ? s : kblocks / 2;
  return s < 1 ? 1 : s;
}

template <int M>
void launch_linear(uint32_t R, const uint16_t* x, uint32_t K, uint32_t N, const uint8_t* enc, uint64_t enc_bytes,
                   uint64_t header_bytes, uint32_t first_block, uint32_t splits, float* partial, uint16_t* out,
                   uint32_t* status, cudaStream_t s) {
  const uint32_t groups = (N + R - 1) / R;
  const uint32_t warps = groups * splits;
  const uint32_t grid = (warps + kLinWarps - 1) / kLinWarps;
  constexpr int kR = M <= 2 ? 2 : 4;  // rows per warp; matches rows_per_warp()
  (void)R;
  nf12_linear<M, kR><<<grid, 32 * kLinWarps, 0, s>>>(x, K, N, enc, enc_bytes, header_bytes, first_block, splits,
                                                      partial, out, status);
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
  const uint32_t R = rows_per_warp(M);
  const uint32_t splits = pick_splits((N + R - 1) / R, K / kBlockValues);
  return splits > 1 ? uint64_t(splits) * M * N * sizeof(float) : 0;
}

VOOM_API int voom_nf12_linear(const uint16_t* d_x, uint32_t M, uint32_t K, uint32_t N, const uint8_t* d_enc,
                              uint64_t enc_bytes, uint64_t header_bytes, uint32_t first_block, void* d_scratch,
                              uint64_t scratch_bytes, uint16_t* d_out, uint32_t* d_status, void* stream) {
  if (!d_x || !d_enc || !d_out || !d_status) return VOOM_E_INVALID_ARG;
  if (!M || M > 8 || !N || !K || K % 512 || N % 8) return VOOM_E_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(d_enc) & 15u) || (reinterpret_cast<uintptr_t>(d_x) & 15u))
    return VOOM_E_INVALID_ARG;
  if (header_bytes % kHeaderBytes) return VOOM_E_INVALID_ARG;
  const uint32_t kblocks = K / kBlockValues;
  const uint64_t end = uint64_t(first_block) + uint64_t(N) * kblocks;
  if (end * kHeaderBytes > header_bytes || header_bytes + end * kCodeBytes > enc_bytes) return VOOM_E_INVALID_ARG;
  const uint32_t R = rows_per_warp(M);
  const uint32_t splits = pick_splits((N + R - 1) / R, kblocks);
  const uint64_t need = splits > 1 ? uint64_t(splits) * M * N * sizeof(float) : 0;
  if (need && (!d_scratch || scratch_bytes < need)) return VOOM_E_CAPACITY;
  float* partial = static_cast<float*>(d_scratch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (M) {
    case 1: launch_linear<1>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 2: launch_linear<2>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 3: launch_linear<3>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 4: launch_linear<4>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 5: launch_linear<5>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 6: launch_linear<6>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    case 7: launch_linear<7>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
    default: launch_linear<8>(R, d_x, K, N, d_enc, enc_bytes, header_bytes, first_block, splits, partial, d_out, d_status, s); break;
  }
  if (splits > 1) {
    const uint64_t n = uint64_t(M) * N;
    nf12_reduce<<<uint32_t((n + 255) / 256), 256, 0, s>>>(partial, splits, M, N, d_out);
  }
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
