// GPU decoder for vOOM "VRN1" BF16 rANS frames (reference: formats/bf16_rans.py).
//
// Format (bf16_rans.py:26-33): frame header <4sIII> (magic, raw_size,
// tile_bytes, tile_count); per tile <BIII> (mode, raw_len, payload_len, crc32);
// mode 1 = two planes (low = even bytes, high = odd bytes), each
// <I payload_len><256 x u16 freq (sum 4096)><u32 initial state><renorm bytes>.
//
// Parallelism: the format's independent unit is one (tile, plane) stream, a
// serial chain of 32-bit rANS states.  Lanes 2k and 2k+1 of a warp decode the
// low and high plane of the same range in lockstep, exchange 8 bytes by
// shuffle every 16 symbols and write the interleaved BF16 bytes with 128-bit
// stores.  The decode table (4096 slots, one u32 each:
// symbol | (freq-1) << 8 | (slot - cum) << 20) lives in shared memory, so a
// symbol costs one shared load; the renormalisation bytes at the stream
// cursor are fetched with two L1-cached aligned loads in parallel with it and
// folded in with one funnel shift.
//
// Cold kernel: one CTA per tile, one lane pair decodes the whole tile and can
// record a (state, cursor) checkpoint every `every` symbols.  Indexed kernel:
// with those checkpoints every segment is independent; one CTA decodes 128
// segment pairs of one tile, and the per-tile CRC-32 is assembled from the
// chunks' CRC registers (GF(2) shift to the tile end, XOR) by whichever CTA of
// the tile finishes last.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "rans_core.cuh"

namespace voom {
namespace {

using namespace voom::rans;
constexpr int kThreads = 256;
constexpr uint32_t kSegsPerChunk = kThreads / 2;

__device__ const CrcTables g_crc = make_crc_tables();
__device__ const CrcPow2 g_pow2 = make_crc_pow2();

// Position of each check inside a tile, in the order bf16_rans.py performs it.
enum : uint32_t {
  ORD_TILE_HEADER = 1,
  ORD_TILE_PAYLOAD = 2,
  ORD_RAW_SIZE = 3,
  ORD_LOW_HEADER = 4,
  ORD_LOW_PAYLOAD = 5,
  ORD_LOW_TOTAL = 6,
  ORD_LOW_TRAILING = 7,
  ORD_HIGH_HEADER = 8,
  ORD_HIGH_PAYLOAD = 9,
  ORD_HIGH_TOTAL = 10,
  ORD_HIGH_TRAILING = 11,
  ORD_TILE_TRAILING = 12,
  ORD_UNKNOWN_MODE = 13,
  ORD_CRC = 14
};

struct SharedPlanes {
  uint32_t lut[2][4096];  // reused as the CRC slicing table after decoding
  uint32_t cum[2][257];
  uint32_t pow2[64];
  uint32_t red[kThreads / 32];
  uint32_t flags;
  uint32_t degenerate[2];
  uint32_t last;
};

__device__ __forceinline__ void record_ckpt(uint32_t* ckpt, uint32_t done, uint32_t every,
                                            uint32_t limit_k, uint32_t plane, const PlaneRun& r) {
  if ((done & (every - 1)) == 0) {
    const uint32_t k = done / every;
    if (k >= 1 && k <= limit_k) {
      ckpt[(k - 1) * 4 + plane * 2] = r.x;
      ckpt[(k - 1) * 4 + plane * 2 + 1] = r.cur;
    }
  }
}

// Decodes `n` symbols of one plane with one byte store per symbol (stride 2)
// and exact reference semantics.  Used for stream ends, unaligned tiles,
// degenerate planes and partial tiles.
__device__ __forceinline__ void decode_generic(uint32_t lut_s, bool degenerate, PlaneRun& r,
                                               uint32_t n, uint32_t first, uint8_t* out,
                                               uint32_t* ckpt, uint32_t every, uint32_t limit_k,
                                               uint32_t plane) {
  for (uint32_t i = 0; i < n; i++) {
    out[2u * i] = uint8_t(rans_step_exact(lut_s, degenerate, r));
    if (ckpt) record_ckpt(ckpt, first + i + 1, every, limit_k, plane, r);
  }
}

// Lockstep pair decode of up to `nchunks` x 16 symbols (low plane on the even
// lane, high plane on the odd lane, both non-degenerate, `out` 16-byte
// aligned) on the windowed step.  The pair starts only when both lanes can
// (win_can_start) and continues while both windows have room for 16 more
// steps; the caller finishes each plane with decode_generic.  Returns chunks
// done, with r.x / r.cur advanced past them.
__device__ __forceinline__ uint32_t decode_pair_fast(uint32_t lut_s, PlaneRun& r, uint32_t nchunks,
                                                     uint32_t first, uint8_t* out, uint32_t lane,
                                                     uint32_t* ckpt, uint32_t every,
                                                     uint32_t limit_k, unsigned mask) {
  uint32_t c = 0;
  if (nchunks == 0 || !__all_sync(mask, win_can_start(r))) return 0;
  Window W;
  win_open(W, r);
  uint32_t x = r.x;
  for (;;) {
    if ((c & 3u) == 0) asm volatile("prefetch.global.L1 [%0];" ::"l"(W.words + W.j + 64));
    uint32_t a[4];
    win_decode16(lut_s, x, W, a);
    *reinterpret_cast<uint4*>(out + 32u * c + 16u * lane) = exchange_pair16(lane, a[0], a[1], a[2], a[3], mask);
    c++;
    if (ckpt) {
      r.x = x;
      r.cur = win_cur(W);
      record_ckpt(ckpt, first + 16u * c, every, limit_k, lane, r);
    }
    if (c == nchunks || !__all_sync(mask, win_room(W, r.len))) break;
  }
  r.x = x;
  r.cur = win_cur(W);
  return c;
}

// One full segment (`every` symbols, a multiple of 16) of a lane pair on the
// clamped window (win_can_open holds for both lanes; `out` 16-byte aligned).
// r.x / r.cur end where the window stopped; the caller checks the landing.
__device__ __forceinline__ void decode_pair_seg(uint32_t lut_s, PlaneRun& r, uint32_t every, uint8_t* out,
                                                uint32_t lane, unsigned mask) {
  Window W;
  win_open(W, r);
  uint32_t x = r.x;
  for (uint32_t c = 0; c < every / 16u; c++) {
    uint32_t a[4];
    win_decode16(lut_s, x, W, a);
    *reinterpret_cast<uint4*>(out + 32u * c + 16u * lane) = exchange_pair16(lane, a[0], a[1], a[2], a[3], mask);
  }
  r.x = x;
  r.cur = win_cur(W);
}

__device__ __forceinline__ void load_crc_tables(SharedPlanes& sh) {
  uint32_t* t = &sh.lut[0][0];
  const uint32_t* g = &g_crc.t[0][0];
  for (int i = threadIdx.x; i < 8 * 256; i += kThreads) t[i] = g[i];
  if (threadIdx.x < 64) sh.pow2[threadIdx.x] = g_pow2.p[threadIdx.x];
  __syncthreads();
}

__device__ __forceinline__ const uint32_t (*crc_tab(SharedPlanes& sh))[256] {
  return reinterpret_cast<const uint32_t(*)[256]>(&sh.lut[0][0]);
}

__device__ __forceinline__ void copy_stored(const uint8_t* src, uint8_t* dst, uint64_t n) {
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0) {
    uint64_t nv = n >> 4;
    for (uint64_t i = threadIdx.x; i < nv; i += kThreads)
      reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    for (uint64_t i = (nv << 4) + threadIdx.x; i < n; i += kThreads) dst[i] = src[i];
  } else {
    for (uint64_t i = threadIdx.x; i < n; i += kThreads) dst[i] = src[i];
  }
}

// Whole-tile status for one-CTA tiles: trailing flags, then CRC.
__device__ __forceinline__ void finish_whole_tile(SharedPlanes& sh, const voom_rans_tile& tl,
                                                  const uint8_t* src, uint8_t* out, uint32_t* status,
                                                  uint32_t tile) {
  __syncthreads();  // decoded bytes visible, LUT no longer needed
  uint32_t st = sh.flags;
  if ((tl.flags & VOOM_RANS_DO_CRC) && !(st & (VOOM_RANS_ST_LOW_TRAILING | VOOM_RANS_ST_HIGH_TRAILING))) {
    load_crc_tables(sh);
    const uint8_t* p = tl.mode == 0 ? src + tl.src : out + tl.dst;
    if (block_crc32(crc_tab(sh), sh.pow2, p, tl.raw_len, sh.red) != tl.crc32) st |= VOOM_RANS_ST_CRC_MISMATCH;
  }
  if (threadIdx.x == 0) status[tile] = st;
}

__global__ void __launch_bounds__(kThreads, 1) rans_cold_kernel(const uint8_t* __restrict__ src,
                                                                const voom_rans_tile* __restrict__ tiles,
                                                                uint8_t* __restrict__ out,
                                                                uint32_t* __restrict__ status,
                                                                uint32_t* __restrict__ ckpt,
                                                                const uint32_t* __restrict__ ckpt_base,
                                                                uint32_t every) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SharedPlanes& sh = *reinterpret_cast<SharedPlanes*>(smem_raw);
  const voom_rans_tile tl = tiles[blockIdx.x];
  if (threadIdx.x == 0) sh.flags = 0;
  if (tl.mode == 0) {
    if (tl.flags & VOOM_RANS_DO_COPY) copy_stored(src + tl.src, out + tl.dst, tl.raw_len);
    finish_whole_tile(sh, tl, src, out, status, blockIdx.x);
    return;
  }
  const bool do_low = tl.flags & VOOM_RANS_DO_LOW, do_high = tl.flags & VOOM_RANS_DO_HIGH;
  if (do_low) build_lut(sh.lut[0], sh.cum[0], sh.red, &sh.degenerate[0], src + tl.low_freq);
  if (do_high) build_lut(sh.lut[1], sh.cum[1], sh.red, &sh.degenerate[1], src + tl.high_freq);
  const uint32_t n_low = (tl.raw_len + 1) / 2, n_high = tl.raw_len / 2;
  uint32_t* ck = ckpt ? ckpt + ckpt_base[blockIdx.x] : nullptr;
  const uint32_t nseg = n_low ? (n_low + every - 1) / every : 1;
  const uint32_t limit_k = nseg - 1;
  if (threadIdx.x < 2) {
    const uint32_t lane = threadIdx.x;
    const bool active = lane ? do_high : do_low;
    if (active) {
      PlaneRun r;
      plane_start(r, src, lane ? tl.high_freq : tl.low_freq, lane ? tl.high_payload : tl.low_payload, 0, 0,
                  false);
      const uint32_t n = lane ? n_high : n_low;
      const uint32_t lut_s = uint32_t(__cvta_generic_to_shared(&sh.lut[lane][0]));
      const bool fast = do_low && do_high && !sh.degenerate[0] && !sh.degenerate[1] &&
                        ((reinterpret_cast<uintptr_t>(out + tl.dst) & 15u) == 0);
      uint32_t done = 0;
      if (fast) done = 16u * decode_pair_fast(lut_s, r, n_high / 16, 0, out + tl.dst, lane, ck, every, limit_k, 0x3u);
      decode_generic(lut_s, sh.degenerate[lane], r, n - done, done, out + tl.dst + lane + 2 * done, ck, every,
                     limit_k, lane);
      if (r.cur != r.len) atomicOr(&sh.flags, lane ? VOOM_RANS_ST_HIGH_TRAILING : VOOM_RANS_ST_LOW_TRAILING);
    }
  }
  finish_whole_tile(sh, tl, src, out, status, blockIdx.x);
}

__global__ void __launch_bounds__(kThreads, 2) rans_indexed_kernel(
    const uint8_t* __restrict__ src, const voom_rans_tile* __restrict__ tiles,
    const voom_rans_chunk* __restrict__ chunks, uint8_t* __restrict__ out, uint32_t* __restrict__ status,
    const uint32_t* __restrict__ ckpt, const uint32_t* __restrict__ ckpt_base, uint32_t every,
    uint32_t* __restrict__ tile_scratch) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SharedPlanes& sh = *reinterpret_cast<SharedPlanes*>(smem_raw);
  const voom_rans_chunk ch = chunks[blockIdx.x];
  const voom_rans_tile tl = tiles[ch.tile];
  if (threadIdx.x == 0) sh.flags = 0;
  if (tl.mode == 0) {  // stored tile: always a single chunk
    if (tl.flags & VOOM_RANS_DO_COPY) copy_stored(src + tl.src, out + tl.dst, tl.raw_len);
    finish_whole_tile(sh, tl, src, out, status, ch.tile);
    return;
  }
  const bool do_low = tl.flags & VOOM_RANS_DO_LOW, do_high = tl.flags & VOOM_RANS_DO_HIGH;
  if (do_low) build_lut(sh.lut[0], sh.cum[0], sh.red, &sh.degenerate[0], src + tl.low_freq);
  if (do_high) build_lut(sh.lut[1], sh.cum[1], sh.red, &sh.degenerate[1], src + tl.high_freq);
  const uint32_t n_low = (tl.raw_len + 1) / 2, n_high = tl.raw_len / 2;
  const uint32_t nseg = n_low ? (n_low + every - 1) / every : 1;
  const uint32_t nb = nseg - 1;  // checkpoint boundaries 1..nb
  const uint32_t* ck = ckpt + ckpt_base[ch.tile];
  const uint32_t lane = threadIdx.x & 1u;
  const unsigned mask = 0x3u << (threadIdx.x & 30u);
  const bool aligned = ((reinterpret_cast<uintptr_t>(out + tl.dst) & 15u) == 0);
  const bool fast_ok = do_low && do_high && !sh.degenerate[0] && !sh.degenerate[1] && aligned;
  const bool active = lane ? do_high : do_low;
  const uint32_t n = lane ? n_high : n_low;
  const uint32_t lut_s = uint32_t(__cvta_generic_to_shared(&sh.lut[lane][0]));
  uint32_t bad = 0;
  const uint32_t seg = ch.seg_begin + (threadIdx.x >> 1);
  if (seg < ch.seg_end) {
    const uint32_t first = seg * every;
    const uint32_t cnt = first < n ? min(every, n - first) : 0u;
    PlaneRun r;
    if (active) {
      uint32_t x0 = 0, c0 = 0;
      if (seg) {
        x0 = ck[(seg - 1) * 4 + lane * 2];
        c0 = ck[(seg - 1) * 4 + lane * 2 + 1];
      }
      plane_start(r, src, lane ? tl.high_freq : tl.low_freq, lane ? tl.high_payload : tl.low_payload, x0,
                  c0, seg != 0);
    }
    // The pair decodes a full segment on the clamped window when both planes
    // have one; a pair that does not land where the exact decoder did (a
    // stream that runs out of bytes) redoes it, like every partial segment,
    // on the exact path.
    const uint32_t cnt_high = first < n_high ? min(every, n_high - first) : 0u;
    const bool last = (seg + 1 > nb) || ((seg + 1) * every > n);
    uint32_t done = 0;
    if (fast_ok && cnt_high == every && (every & 15u) == 0 && __all_sync(mask, win_can_open(r))) {
      const uint32_t x0 = r.x, c0 = r.cur;
      decode_pair_seg(lut_s, r, every, out + tl.dst + 2u * first, lane, mask);
      const bool landed = last ? (r.cur == r.len)
                               : (r.x == ck[seg * 4 + lane * 2] && r.cur == ck[seg * 4 + lane * 2 + 1]);
      if (__any_sync(mask, !landed)) {
        r.x = x0;
        r.cur = c0;
      } else {
        done = every;
      }
    }
    if (active) {
      decode_generic(lut_s, sh.degenerate[lane], r, cnt - done, first + done,
                     out + tl.dst + lane + 2u * (first + done), nullptr, every, 0, lane);
      if (last) {
        if (r.cur != r.len) bad |= lane ? VOOM_RANS_ST_HIGH_TRAILING : VOOM_RANS_ST_LOW_TRAILING;
      } else if (r.x != ck[seg * 4 + lane * 2] || r.cur != ck[seg * 4 + lane * 2 + 1]) {
        bad |= lane ? VOOM_RANS_ST_HIGH_TRAILING : VOOM_RANS_ST_LOW_TRAILING;
      }
    }
  }
  if (bad) atomicOr(&sh.flags, bad);
  __syncthreads();  // this chunk's bytes are written; LUT no longer needed
  // CRC register of this chunk's byte range, moved to the end of the tile.
  const uint64_t b = min(uint64_t(2) * ch.seg_begin * every, uint64_t(tl.raw_len));
  const uint64_t e = min(uint64_t(2) * ch.seg_end * every, uint64_t(tl.raw_len));
  uint32_t contrib = 0;
  if (tl.flags & VOOM_RANS_DO_CRC) {
    load_crc_tables(sh);
    contrib = block_crc_reg(crc_tab(sh), sh.pow2, out + tl.dst + b, e - b, b == 0 ? 0xFFFFFFFFu : 0u, sh.red);
    if (tl.raw_len - e) contrib = gf2_mulmod(crc_zeros_op(sh.pow2, tl.raw_len - e), contrib);
  }
  uint32_t* ts = tile_scratch + 4u * ch.tile;  // [0] CRC xor, [1] finished chunks, [2] flags
  if (threadIdx.x == 0) {
    if (contrib) atomicXor(&ts[0], contrib);
    if (sh.flags) atomicOr(&ts[2], sh.flags);
    __threadfence();
    sh.last = (atomicAdd(&ts[1], 1u) == ch.n_in_tile - 1);
  }
  __syncthreads();
  if (sh.last && threadIdx.x == 0) {
    __threadfence();
    const uint32_t reg = atomicExch(&ts[0], 0u);
    uint32_t st = atomicExch(&ts[2], 0u);
    atomicExch(&ts[1], 0u);
    if ((tl.flags & VOOM_RANS_DO_CRC) && !(st & (VOOM_RANS_ST_LOW_TRAILING | VOOM_RANS_ST_HIGH_TRAILING)) &&
        (reg ^ 0xFFFFFFFFu) != tl.crc32)
      st |= VOOM_RANS_ST_CRC_MISMATCH;
    status[ch.tile] = st;
  }
}

inline uint32_t rd32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

bool valid_every(uint32_t e) { return e >= 64 && (e & (e - 1)) == 0; }

uint32_t tile_segments(uint32_t raw_len, uint32_t every) {
  const uint32_t n_low = (raw_len + 1) / 2;
  return n_low ? (n_low + every - 1) / every : 1;
}

}  // namespace
}  // namespace voom

using namespace voom;

VOOM_API uint64_t voom_rans_ckpt_words(uint32_t raw_len, uint32_t every) {
  if (!valid_every(every)) return 0;
  return 4ull * (tile_segments(raw_len, every) - 1);
}

VOOM_API int voom_rans_chunks(const voom_rans_tile* tiles, uint32_t n_tiles, uint32_t every,
                              voom_rans_chunk* chunks, uint32_t max_chunks, uint32_t* n_chunks) {
  if (!n_chunks || (n_tiles && !tiles) || !valid_every(every)) return VOOM_E_INVALID_ARG;
  uint32_t k = 0;
  for (uint32_t t = 0; t < n_tiles; t++) {
    const uint32_t nseg = tiles[t].mode == 0 ? 1 : tile_segments(tiles[t].raw_len, every);
    const uint32_t nc = tiles[t].mode == 0 ? 1 : (nseg + kSegsPerChunk - 1) / kSegsPerChunk;
    for (uint32_t c = 0; c < nc; c++, k++) {
      if (chunks && k < max_chunks) {
        chunks[k].tile = t;
        chunks[k].seg_begin = c * kSegsPerChunk;
        chunks[k].seg_end = min((c + 1) * kSegsPerChunk, nseg);
        chunks[k].n_in_tile = nc;
      }
    }
  }
  *n_chunks = k;
  return (chunks && k > max_chunks) ? VOOM_E_CAPACITY : VOOM_OK;
}

VOOM_API int voom_rans_plan(const uint8_t* f, uint64_t n, uint64_t src_base, uint64_t dst_base,
                            voom_rans_tile* tiles, uint32_t max_tiles, voom_rans_plan_info* info) {
  if (!info || (!f && n)) return VOOM_E_INVALID_ARG;
  memset(info, 0, sizeof(*info));
  uint32_t planned = 0;
  auto emit = [&](const voom_rans_tile& d) {
    if (tiles && planned < max_tiles) tiles[planned] = d;
    planned++;
  };
  auto fail = [&](int code, uint32_t tile, uint32_t ord) {
    info->struct_error = code;
    info->struct_tile = tile;
    info->struct_ordinal = ord;
  };
  auto freq_total = [&](uint64_t at) {
    uint64_t tot = 0;
    for (int s = 0; s < 256; s++) tot += uint32_t(f[at + 2 * s]) | (uint32_t(f[at + 2 * s + 1]) << 8);
    return tot;
  };
  if (n < 16) {
    fail(VOOM_RANS_TRUNC_FRAME, 0, 0);
  } else if (memcmp(f, "VRN1", 4) != 0) {
    fail(VOOM_RANS_NOT_FRAME, 0, 0);
  } else {
    info->raw_size = rd32(f + 4);
    info->tile_bytes = rd32(f + 8);
    info->tile_count = rd32(f + 12);
    uint64_t pos = 16, out = 0;
    bool broke = false;
    for (uint64_t t = 0; t < info->tile_count && !broke; t++) {
      const uint32_t ti = uint32_t(t);
      if (pos + 13 > n) { fail(VOOM_RANS_TRUNC_TILE_HEADER, ti, ORD_TILE_HEADER); broke = true; break; }
      const uint32_t mode = f[pos];
      const uint32_t raw = rd32(f + pos + 1), pay = rd32(f + pos + 5), crc = rd32(f + pos + 9);
      pos += 13;
      const uint64_t end = pos + pay;
      if (end > n) { fail(VOOM_RANS_TRUNC_TILE_PAYLOAD, ti, ORD_TILE_PAYLOAD); broke = true; break; }
      voom_rans_tile d;
      memset(&d, 0, sizeof d);
      d.dst = dst_base + out;
      d.raw_len = raw;
      d.crc32 = crc;
      d.mode = mode;
      if (mode == 0) {
        if (pay != raw) { fail(VOOM_RANS_RAW_SIZE_MISMATCH, ti, ORD_RAW_SIZE); broke = true; break; }
        d.src = src_base + pos;
        d.flags = VOOM_RANS_DO_COPY | VOOM_RANS_DO_CRC;
      } else if (mode == 1) {
        // low plane (bf16_rans.py:97-114)
        const uint64_t avail = pay, p = pos;
        if (avail < 516) { fail(VOOM_RANS_TRUNC_PLANE_HEADER, ti, ORD_LOW_HEADER); broke = true; break; }
        const uint64_t psz = rd32(f + p);
        if (psz < 4 || 516 + psz > avail) { fail(VOOM_RANS_TRUNC_PLANE_PAYLOAD, ti, ORD_LOW_PAYLOAD); broke = true; break; }
        const uint64_t tot = freq_total(p + 4);
        if (tot != 0 && tot != 4096) { fail(VOOM_RANS_BAD_FREQ_TOTAL, ti, ORD_LOW_TOTAL); broke = true; break; }
        d.low_freq = src_base + p + 4;
        d.low_payload = uint32_t(psz);
        d.flags = VOOM_RANS_DO_LOW;
        const uint64_t used = 516 + psz;
        // high plane: failures here come after the low plane's decode
        const uint64_t avail2 = avail - used, p2 = pos + used;
        int err = 0;
        uint32_t ord = 0;
        uint64_t psz2 = 0;
        if (avail2 < 516) { err = VOOM_RANS_TRUNC_PLANE_HEADER; ord = ORD_HIGH_HEADER; }
        else {
          psz2 = rd32(f + p2);
          if (psz2 < 4 || 516 + psz2 > avail2) { err = VOOM_RANS_TRUNC_PLANE_PAYLOAD; ord = ORD_HIGH_PAYLOAD; }
          else {
            const uint64_t tot2 = freq_total(p2 + 4);
            if (tot2 != 0 && tot2 != 4096) { err = VOOM_RANS_BAD_FREQ_TOTAL; ord = ORD_HIGH_TOTAL; }
          }
        }
        if (!err) {
          d.high_freq = src_base + p2 + 4;
          d.high_payload = uint32_t(psz2);
          d.flags |= VOOM_RANS_DO_HIGH;
          if (used + 516 + psz2 != pay) { err = VOOM_RANS_TILE_TRAILING; ord = ORD_TILE_TRAILING; }
        }
        if (err) {
          fail(err, ti, ord);
          emit(d);
          out += raw;
          broke = true;
          break;
        }
        d.flags |= VOOM_RANS_DO_CRC;
      } else {
        fail(VOOM_RANS_UNKNOWN_MODE, ti, ORD_UNKNOWN_MODE);
        info->bad_mode = mode;
        broke = true;
        break;
      }
      emit(d);
      out += raw;
      pos = end;
    }
    info->out_bytes = out;
    if (!broke) {
      info->frame_end = 1;
      if (pos != n || out != info->raw_size) fail(VOOM_RANS_LENGTH_MISMATCH, info->tile_count, 0);
    }
  }
  info->n_tiles = planned;
  if (tiles && planned > max_tiles) return VOOM_E_CAPACITY;
  return VOOM_OK;
}

VOOM_API int voom_rans_resolve(const voom_rans_plan_info* info, const uint32_t* st, uint32_t n_tiles,
                               uint32_t* err_tile) {
  if (!info || (n_tiles && !st)) return VOOM_E_INVALID_ARG;
  uint32_t dummy;
  if (!err_tile) err_tile = &dummy;
  *err_tile = 0;
  for (uint32_t t = 0; t < n_tiles; t++) {
    const bool here = info->struct_error && t == info->struct_tile;
    const uint32_t lim = here ? info->struct_ordinal : 0xFFFFFFFFu;
    *err_tile = t;
    if ((st[t] & VOOM_RANS_ST_LOW_TRAILING) && ORD_LOW_TRAILING < lim) return VOOM_RANS_TRAILING_RENORM;
    if ((st[t] & VOOM_RANS_ST_HIGH_TRAILING) && ORD_HIGH_TRAILING < lim) return VOOM_RANS_TRAILING_RENORM;
    if ((st[t] & VOOM_RANS_ST_CRC_MISMATCH) && ORD_CRC < lim) return VOOM_RANS_CHECKSUM;
    if (here) return info->struct_error;
  }
  if (info->struct_error) {
    *err_tile = info->struct_tile;
    return info->struct_error;
  }
  return VOOM_OK;
}

VOOM_API int voom_rans_decode(const uint8_t* d_src, const voom_rans_tile* d_tiles, uint32_t n_tiles,
                              uint8_t* d_out, uint32_t* d_status, uint32_t* d_ckpt,
                              const uint32_t* d_ckpt_base, uint32_t ckpt_every, void* stream) {
  if (n_tiles == 0) return VOOM_OK;
  if (!d_src || !d_tiles || !d_out || !d_status) return VOOM_E_INVALID_ARG;
  if (d_ckpt && (!d_ckpt_base || !valid_every(ckpt_every))) return VOOM_E_INVALID_ARG;
  const size_t smem = sizeof(SharedPlanes);
  if (cudaFuncSetAttribute(rans_cold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return VOOM_E_CUDA;
  rans_cold_kernel<<<n_tiles, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      d_src, d_tiles, d_out, d_status, d_ckpt, d_ckpt_base, d_ckpt ? ckpt_every : 64u);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API int voom_rans_decode_indexed(const uint8_t* d_src, const voom_rans_tile* d_tiles,
                                      const voom_rans_chunk* d_chunks, uint32_t n_chunks, uint8_t* d_out,
                                      uint32_t* d_status, const uint32_t* d_ckpt,
                                      const uint32_t* d_ckpt_base, uint32_t ckpt_every,
                                      uint32_t* d_tile_scratch, void* stream) {
  if (n_chunks == 0) return VOOM_OK;
  if (!d_src || !d_tiles || !d_chunks || !d_out || !d_status || !d_ckpt || !d_ckpt_base || !d_tile_scratch ||
      !valid_every(ckpt_every))
    return VOOM_E_INVALID_ARG;
  const size_t smem = sizeof(SharedPlanes);
  if (cudaFuncSetAttribute(rans_indexed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return VOOM_E_CUDA;
  rans_indexed_kernel<<<n_chunks, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      d_src, d_tiles, d_chunks, d_out, d_status, d_ckpt, d_ckpt_base, ckpt_every, d_tile_scratch);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
