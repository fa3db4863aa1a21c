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

// Renormalisation bytes of a fast run held in registers: a 64-bit window
// (hi:lo) of the stream's next bytes, left-aligned, with nb valid bits, plus
// one preloaded aligned word (nxt).  A step shifts 8k bits out of the window;
// every second step the window takes nxt if 32 or fewer bits remain, and only
// then is the next word loaded.  Two steps use at most 32 bits, so the window
// never runs dry.  About a third of a warp's lanes load on a refill step, the
// load has two steps to land, and the bookkeeping is a few register ops.
struct Window {
  const uint32_t* words;  // aligned words of the stream; words[j] is loaded next
  uint32_t j;
  uint32_t jlast;         // last word holding a payload byte: loads clamp to it
  uint32_t hi, lo;        // window bits, first byte at the top of hi
  uint32_t nb;            // valid bits in (hi:lo), a multiple of 8
  uint32_t nxt;           // big-endian words[j - 1]: the bytes after the window
  uint32_t base;          // payload offset of words[0]
};

__device__ __forceinline__ uint32_t ldg_be32(const uint32_t* p) { return __byte_perm(__ldg(p), 0, 0x0123); }

// Opens a window at r.cur (requires 4 <= cur < len).  Loads never go past the
// aligned word that holds the payload's last byte, and an aligned word that
// holds a byte of a buffer lies inside that buffer's allocation, so every
// load is in bounds whatever the stream holds.  Bytes past the payload end
// enter the window only when a stream asks for more bytes than it has; the
// reference encoder's streams never do (they end at state L with every byte
// consumed), and callers detect it by the landing check (cursor past len).
__device__ __forceinline__ void win_open(Window& W, const PlaneRun& r) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(r.payload) + r.cur;
  const uint32_t s = uint32_t(a & 3u);
  W.words = reinterpret_cast<const uint32_t*>(a - s);
  W.base = r.cur - s;
  W.jlast = (r.len - 1u - W.base) >> 2;
  const uint32_t w0 = ldg_be32(W.words), w1 = ldg_be32(W.words + min(1u, W.jlast));
  W.hi = __funnelshift_l(w1, w0, 8u * s);
  W.lo = w1 << (8u * s);
  W.nb = 64u - 8u * s;
  W.nxt = ldg_be32(W.words + min(2u, W.jlast));
  W.j = 3;
}

// Stream position of the window's first byte.
__device__ __forceinline__ uint32_t win_cur(const Window& W) { return W.base + 4u * (W.j - 1u) - (W.nb >> 3); }

// True when the next 16 steps (8 refills) stay inside a payload of `len` bytes.
__device__ __forceinline__ bool win_room(const Window& W, uint32_t len) {
  return W.base + 4u * (W.j + 8u) <= len;
}

__device__ __forceinline__ void win_refill(Window& W) {
  const bool use = W.nb <= 32u;
  const uint32_t m = use ? 0xFFFFFFFFu : 0u;
  W.hi |= __funnelshift_rc(W.nxt, 0u, W.nb) & m;        // nxt >> nb
  W.lo |= __funnelshift_lc(0u, W.nxt, 32u - W.nb) & m;  // nxt << (32 - nb)
  W.nb += m & 32u;
  // predicated load (no branch): lanes that keep their window skip the access
  uint32_t raw = 0;
  asm(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p ld.global.nc.u32 %0, [%1];\n\t}"
      : "+r"(raw)
      : "l"(W.words + min(W.j, W.jlast)), "r"(m));
  W.nxt = use ? __byte_perm(raw, 0, 0x0123) : W.nxt;
  W.j += m & 1u;
}

// One symbol; returns the table entry (symbol in its low byte).  Requires
// L <= x < 2^31, which then holds after the step as well: the decoded state
// y lies in [2^11, 2^31) and 8k = (clz(y) - 1) & ~7 brings it back to
// [2^23, 2^31) -- the reference's byte-wise loop, k in {0, 1, 2}.
__device__ __forceinline__ uint32_t rans_step_win(uint32_t lut_s, uint32_t& x, Window& W) {
  const uint32_t e = lds32(lut_s + 4u * (x & 4095u));
  const uint32_t xs = x >> 12;
  const uint32_t y = ((e >> 8) & 4095u) * xs + xs + (e >> 20);
  const uint32_t sh = (uint32_t(__clz(y)) - 1u) & ~7u;
  x = __funnelshift_l(W.hi, y, sh);
  W.hi = __funnelshift_l(W.lo, W.hi, sh);
  W.lo <<= sh;
  W.nb -= sh;
  return e;
}

// Bytes 0 of four table entries, packed low to high.
__device__ __forceinline__ uint32_t pack4(uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3) {
  return __byte_perm(__byte_perm(e0, e1, 0x0040), __byte_perm(e2, e3, 0x0040), 0x5410);
}

// 16 symbols of one lane (4 words of 4 bytes), refilling every second step.
__device__ __forceinline__ void win_decode16(uint32_t lut_s, uint32_t& x, Window& W, uint32_t a[4]) {
#pragma unroll
  for (int q = 0; q < 4; q++) {
    win_refill(W);
    const uint32_t e0 = rans_step_win(lut_s, x, W);
    const uint32_t e1 = rans_step_win(lut_s, x, W);
    win_refill(W);
    const uint32_t e2 = rans_step_win(lut_s, x, W);
    const uint32_t e3 = rans_step_win(lut_s, x, W);
    a[q] = pack4(e0, e1, e2, e3);
  }
}

// Entry condition of a guarded windowed run (win_room checked per 16 steps).
__device__ __forceinline__ bool win_can_start(const PlaneRun& r) {
  return r.len >= r.cur + 48u && r.x >= kRansL && r.x < 0x80000000u;
}

// Entry condition of a clamped windowed run over a whole segment.
__device__ __forceinline__ bool win_can_open(const PlaneRun& r) {
  return r.cur >= 4u && r.len >= r.cur + 16u && r.x >= kRansL && r.x < 0x80000000u;
}

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
    // each warp fills the slots of every 8th symbol, 32 consecutive slots
    // per store (conflict-free); symbols are interleaved so the few large
    // ones land on different warps.
    for (int sym = warp; sym < 256; sym += 8) {
      const uint32_t c = cum[sym], fs = cum[sym + 1] - c;
      const uint32_t hdr = uint32_t(sym) | ((fs - 1u) << 8);
      for (uint32_t i = lane; i < fs; i += 32) lut[c + i] = hdr | (i << 20);
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
