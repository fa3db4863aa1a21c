// Lane-pair rANS decode core for VRN1 planes (reference: formats/bf16_rans.py
// _decode_plane, :97-130), shared by the page decoder (rans.cu) and the fused
// expert kernels (expert.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace voom {
namespace rans {

constexpr uint32_t kRansL = 1u << 23;

__device__ __forceinline__ uint32_t ld_u8(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t* p) {
  return ld_u8(p) | (ld_u8(p + 1) << 8) | (ld_u8(p + 2) << 16) | (ld_u8(p + 3) << 24);
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// The 4 bytes at p as a big-endian word (first byte most significant), from
// two aligned L1-cached loads.  p[0..7] must be readable.
__device__ __forceinline__ uint32_t load4_be(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t v = __funnelshift_r(__ldg(w), __ldg(w + 1), uint32_t(a & 3u) * 8u);
  return __byte_perm(v, 0, 0x0123);
}

struct PlaneRun {
  const uint8_t* payload;  // plane payload: u32 initial state, renorm bytes
  uint32_t x, cur, len;
};

// One decoded symbol with the reference's exact renormalisation loop
// `while state < L and cursor < len` (bf16_rans.py:117-127).  Used near the
// end of a stream, for degenerate tables and for malformed states.
__device__ __forceinline__ uint32_t rans_step_exact(uint32_t lut_s, bool degenerate, PlaneRun& r) {
  uint32_t slot = r.x & 4095u, sym = 0;
  if (degenerate) {
    r.x = slot;  // all frequencies zero: symbol 0, frequency 0, cumulative 0
  } else {
    uint32_t e = lds32(lut_s + 4u * slot);
    r.x = (((e >> 8) & 4095u) + 1u) * (r.x >> 12) + (e >> 20);
    sym = e & 0xFFu;
  }
  while (r.x < kRansL && r.cur < r.len) {
    r.x = (r.x << 8) | ld_u8(r.payload + r.cur);
    r.cur++;
  }
  return sym;
}

// Branch-free symbol step for the bulk of a stream.  Preconditions: x >= L,
// non-degenerate table, at least 8 payload bytes left.  From x >= 2^23 and
// freq >= 1 the new state is >= 2^11, so at most two renormalisation bytes
// are needed: k = (x < 2^23) + (x < 2^15).
__device__ __forceinline__ uint32_t rans_step_fast(uint32_t lut_s, PlaneRun& r) {
  const uint32_t be = load4_be(r.payload + r.cur);
  const uint32_t e = lds32(lut_s + 4u * (r.x & 4095u));
  const uint32_t xs = r.x >> 12;
  uint32_t x = ((e >> 8) & 4095u) * xs + xs + (e >> 20);
  const uint32_t k = uint32_t(x < kRansL) + uint32_t(x < (kRansL >> 8));
  r.x = __funnelshift_l(be, x, 8u * k);
  r.cur += k;
  return e & 0xFFu;
}

// Renormalisation bytes of a fast run held in registers: a 64-bit window of
// the stream's next bytes (left-aligned, first byte most significant) plus one
// preloaded aligned word.  A step shifts k bytes out of the window; the window
// takes the preloaded word once 4 or fewer bytes remain, and only then is a
// new word loaded.  Per step about a third of a warp's lanes issue a load,
// against two unaligned loads per lane for load4_be, and the load result is
// not needed before the following refill.  Reads reach at most cur + 11.
struct Window {
  const uint32_t* words;  // next word to load
  uint64_t w;             // bytes [cur, cur + n) left-aligned
  uint32_t n;             // valid bytes in w: 5..8 before each step
  uint32_t nxt;           // big-endian word holding bytes [cur + n, cur + n + 4)
};

__device__ __forceinline__ uint32_t ldg_be32(const uint32_t* p) { return __byte_perm(__ldg(p), 0, 0x0123); }

// Opens a window at r.cur.  Payload bytes [cur - 3, cur + 12) must be readable.
__device__ __forceinline__ void win_open(Window& W, const PlaneRun& r) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(r.payload) + r.cur;
  const uint32_t* p = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t s = uint32_t(a & 3u);
  const uint64_t v = (uint64_t(ldg_be32(p)) << 32) | ldg_be32(p + 1);
  W.w = v << (8u * s);
  W.n = 8u - s;
  W.nxt = ldg_be32(p + 2);
  W.words = p + 3;
}

// Same arithmetic as rans_step_fast with the bytes taken from the window.
__device__ __forceinline__ uint32_t rans_step_win(uint32_t lut_s, PlaneRun& r, Window& W) {
  const uint32_t e = lds32(lut_s + 4u * (r.x & 4095u));
  const uint32_t xs = r.x >> 12;
  const uint32_t x = ((e >> 8) & 4095u) * xs + xs + (e >> 20);
  const uint32_t k = uint32_t(x < kRansL) + uint32_t(x < (kRansL >> 8));
  r.x = __funnelshift_l(uint32_t(W.w >> 32), x, 8u * k);
  W.w <<= 8u * k;
  W.n -= k;
  r.cur += k;
  if (W.n <= 4u) {
    W.w |= uint64_t(W.nxt) << (32u - 8u * W.n);
    W.n += 4u;
    W.nxt = ldg_be32(W.words);
    W.words++;
  }
  return e & 0xFFu;
}

// Bytes a fast 16-symbol chunk needs left in the stream: 32 consumed at most,
// plus the window's 12-byte reach.
constexpr uint32_t kWinGuard = 48;

// Builds the decode table of one plane from its 256 x u16 frequency table
// into lut[4096] (cum[257] and red[8] are shared scratch).  All 256 threads of
// the block participate.  *degenerate = 1 when every frequency is zero.
__device__ __forceinline__ void build_lut(uint32_t* lut, uint32_t* cum, uint32_t* red, uint32_t* degenerate,
                                          const uint8_t* freq) {
  const int tid = threadIdx.x;
  const uint32_t f = ld_u8(freq + 2 * tid) | (ld_u8(freq + 2 * tid + 1) << 8);  // kThreads == 256
  uint32_t v = f;
  const int lane = tid & 31, warp = tid >> 5;
  for (int o = 1; o < 32; o <<= 1) {  // requires blockDim.x == 256
    uint32_t n = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) red[warp] = v;
  __syncthreads();
  uint32_t base = 0;
  for (int w = 0; w < warp; w++) base += red[w];
  cum[tid] = base + v - f;
  if (tid == 255) cum[256] = base + v;
  __syncthreads();
  const uint32_t total = cum[256];
  if (tid == 0) *degenerate = (total == 0);
  if (total == 4096u) {
    // slot -> symbol without searching: mark each symbol's first slot, then a
    // block-wide running maximum over the 4096 slots (16 per thread).
    uint32_t* mark = lut;  // reused as the marker array, overwritten below
    const uint32_t base_slot = uint32_t(tid) * 16u;
#pragma unroll
    for (int j = 0; j < 16; j++) mark[base_slot + j] = 0;
    __syncthreads();
    if (f) mark[cum[tid]] = uint32_t(tid) + 1u;
    __syncthreads();
    uint32_t m[16];
    uint32_t run = 0;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      run = max(run, mark[base_slot + j]);
      m[j] = run;
    }
    // exclusive prefix maximum of the per-thread maxima
    uint32_t incl = run;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl = max(incl, n);
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    uint32_t before = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    if (lane == 0) before = 0;
    for (int w = 0; w < warp; w++) before = max(before, red[w]);
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const uint32_t s1 = max(before, m[j]);  // symbol + 1 owning this slot
      const uint32_t sym = s1 - 1u;
      const uint32_t c = cum[sym];
      const uint32_t fs = cum[sym + 1] - c;
      const uint32_t slot = base_slot + uint32_t(j);
      lut[slot] = sym | ((fs - 1u) << 8) | ((slot - c) << 20);
    }
  }
  __syncthreads();
}

// Interleaves this lane's 16 symbols (a0..a3) with its partner's: returns
// this lane's 16 output bytes of the 32-byte chunk (the low-plane lane gets
// BF16 elements 0..7, the high-plane lane elements 8..15).
__device__ __forceinline__ uint4 exchange_pair16(uint32_t lane, uint32_t a0, uint32_t a1, uint32_t a2,
                                                 uint32_t a3, unsigned mask) {
  uint32_t s0 = lane ? a0 : a2, s1 = lane ? a1 : a3;
  uint32_t r0 = __shfl_xor_sync(mask, s0, 1);
  uint32_t r1 = __shfl_xor_sync(mask, s1, 1);
  uint32_t lo0 = lane ? r0 : a0, lo1 = lane ? r1 : a1;
  uint32_t hi0 = lane ? a2 : r0, hi1 = lane ? a3 : r1;
  uint4 o;
  o.x = __byte_perm(lo0, hi0, 0x5140);
  o.y = __byte_perm(lo0, hi0, 0x7362);
  o.z = __byte_perm(lo1, hi1, 0x5140);
  o.w = __byte_perm(lo1, hi1, 0x7362);
  return o;
}

__device__ __forceinline__ void plane_start(PlaneRun& r, const uint8_t* src, uint64_t freq_off,
                                            uint32_t payload_len, uint32_t x0, uint32_t cur0,
                                            bool from_ckpt) {
  r.payload = src + freq_off + 512;
  r.len = payload_len;
  r.x = from_ckpt ? x0 : ld_u32_unaligned(r.payload);
  r.cur = from_ckpt ? cur0 : 4u;
}

}  // namespace rans
}  // namespace voom
