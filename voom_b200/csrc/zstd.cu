// GPU Zstandard (RFC 8878) decoder for vpack hi planes and kv_paged pages.
//
// Pipeline over a planned batch of jobs (host plan: zstd_plan.cpp):
//   K0 block literals - one CTA per block, a warp per Huffman stream: the
//                      literals section staged in shared memory, 32 lanes per
//                      stream on spans that settle on codeword boundaries (on a
//                      side stream, beside K1).
//   K1 block decode  - one warp per block builds the LL/OF/ML FSE tables and
//                      walks the sequence bitstream, storing each sequence's
//                      literal length, match length and offset value.
//   K1b seq scan     - one CTA per block: repeat-offset rules on symbolic slots
//                      (each of the 3 repeat slots as "block-start slot minus
//                      d" or a constant) and output / literal positions by a
//                      block scan over sequence chunks; the block's output size
//                      and repeat transform, so blocks need no serial pass.
//   K2 job scan      - one thread per job: block output positions (prefix sum
//                      of block sizes) and the repeat offsets every block starts
//                      with (composition of the transforms); size checks.
//   K3 block execute - one CTA per block: concrete offsets from the block's
//                      start state, then every output byte is written as either
//                      a resolved literal (bit 31 set | byte) or the position it
//                      copies.
//   K4 resolve       - pointer jumping over the decoded space: each pass
//                      follows up to 16 copy links per byte with path
//                      compression, so chains of any length resolve in
//                      log16(length) passes; later passes only touch output
//                      tiles that still had unresolved bytes.
//   K5 output        - resolved bytes, interleaved with the raw lo plane for
//                      vpack bodies (out[2k] = lo[k], out[2k+1] = hi[k]).
//   K6 checksum      - XXH64 of frames that carry a content checksum.
// No step waits on another CTA; the host loop is fixed (no host sync).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "zstd_plan.h"

using namespace voom;
using namespace voom::zstd;

namespace {

constexpr uint32_t kResolved = 0x80000000u;
constexpr int kResolvePasses = 6;
constexpr int kHops = 16;

__constant__ uint32_t c_ll_base[36] = {0,  1,  2,  3,  4,  5,  6,  7,  8,   9,   10,  11,
                                       12, 13, 14, 15, 16, 18, 20, 22, 24,  28,  32,  40,
                                       48, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768, 65536};
__constant__ uint8_t c_ll_bits[36] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1,
                                      1, 1, 2, 2, 3, 3, 4, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16};
__constant__ uint32_t c_ml_base[53] = {3,  4,  5,  6,  7,  8,  9,  10, 11, 12, 13, 14, 15, 16,
                                       17, 18, 19, 20, 21, 22, 23, 24, 25, 26, 27, 28, 29, 30,
                                       31, 32, 33, 34, 35, 37, 39, 41, 43, 47, 51, 59, 67, 83,
                                       99, 131, 259, 515, 1027, 2051, 4099, 8195, 16387, 32771, 65539};
__constant__ uint8_t c_ml_bits[53] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                                      0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1,
                                      2, 2, 3, 3, 4, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16};

struct View {
  const ZPlanHeader* h;
  const ZJob* jobs;
  const ZFrame* frames;
  const ZBlock* blocks;
  const ZHuf* huf;
  const ZFse* fse;
  const ZOutTile* tiles;
  uint32_t* res;
  uint8_t* lit;
  ZSeq* seq;
  ZBlockRt* rt;
  uint32_t* dirty;
  uint2* list;  // two resolve worklists of (Z position, tile)
};

__device__ __forceinline__ View make_view(const uint8_t* img, uint8_t* scratch) {
  View v;
  v.h = reinterpret_cast<const ZPlanHeader*>(img);
  v.jobs = reinterpret_cast<const ZJob*>(img + v.h->off_jobs);
  v.frames = reinterpret_cast<const ZFrame*>(img + v.h->off_frames);
  v.blocks = reinterpret_cast<const ZBlock*>(img + v.h->off_blocks);
  v.huf = reinterpret_cast<const ZHuf*>(img + v.h->off_huf);
  v.fse = reinterpret_cast<const ZFse*>(img + v.h->off_fse);
  v.tiles = reinterpret_cast<const ZOutTile*>(img + v.h->off_tiles);
  v.res = reinterpret_cast<uint32_t*>(scratch + v.h->s_res);
  v.lit = scratch + v.h->s_lit;
  v.seq = reinterpret_cast<ZSeq*>(scratch + v.h->s_seq);
  v.rt = reinterpret_cast<ZBlockRt*>(scratch + v.h->s_blk);
  v.dirty = reinterpret_cast<uint32_t*>(scratch + v.h->s_ctr);
  v.list = reinterpret_cast<uint2*>(scratch + v.h->s_list);
  return v;
}

// 8 bytes starting at p (any alignment) from two aligned loads; the source
// buffer is 8-byte aligned at its start and padded by 16 bytes at its end.
__device__ __forceinline__ uint64_t load8(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint64_t* q = reinterpret_cast<const uint64_t*>(a & ~uintptr_t(7));
  const uint32_t sh = uint32_t(a & 7u) * 8u;
  const uint64_t lo = __ldg(q), hi = __ldg(q + 1);
  return sh ? (lo >> sh) | (hi << (64u - sh)) : lo;
}

__device__ __forceinline__ uint32_t bfe32(uint32_t v, uint32_t pos, uint32_t len) {
  uint32_t r;
  asm("bfe.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(pos), "r"(len));
  return r;
}

// Register window over a backward bitstream for one lane: the unread bits
// just below position P, left-aligned in (hi:lo) with vb of them valid,
// refilled 32 bits at a time from aligned words that are loaded two refills
// ahead (q0, q1), so a lane's loads are in flight long before they are needed
// and do not depend on L1 keeping the line.  Words below the stream start
// read as zero, as do the bits of word 0 below the stream's first byte.
struct DownWin {
  const uint32_t* w;
  uint32_t mask0;  // keeps the stream's bits of word 0
  uint32_t hi, lo, vb;
  uint32_t q0, q1;
  int32_t nidx;    // next word to load
  int32_t P;       // unread stream bits

  __device__ __forceinline__ uint32_t word(int32_t i) const {
    const uint32_t v = __ldg(w + max(i, 0));
    return i < 0 ? 0u : (i == 0 ? v & mask0 : v);
  }
  __device__ __forceinline__ void init(const uint8_t* s, int32_t P0) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(s);
    w = reinterpret_cast<const uint32_t*>(s - (a & 3u));
    const uint32_t boff = uint32_t(a & 3u) * 8u;
    mask0 = ~((1u << boff) - 1u);
    P = P0;
    const int32_t A = P0 + int32_t(boff);  // aligned bit position, >= 1
    const int32_t m = (A - 1) >> 5;
    const uint32_t sh = uint32_t(32 * (m + 1) - A);  // 0..31
    const uint32_t wm = word(m), wm1 = word(m - 1);
    hi = __funnelshift_l(wm1, wm, sh);
    lo = wm1 << sh;
    vb = 64u - sh;
    q0 = word(m - 2);
    q1 = word(m - 3);
    nidx = m - 4;
  }
  __device__ __forceinline__ void consume(uint32_t n) {  // n <= 31
    hi = __funnelshift_l(lo, hi, n);
    lo <<= n;
    vb -= n;
    P -= int32_t(n);
  }
  // afterwards at least 32 bits are valid
  __device__ __forceinline__ void refill() {
    const bool use = vb <= 32u;
    const uint32_t m = use ? 0xFFFFFFFFu : 0u;
    hi |= __funnelshift_rc(q0, 0u, vb) & m;
    lo |= __funnelshift_lc(0u, q0, 32u - vb) & m;
    vb += m & 32u;
    if (use) {
      q0 = q1;
      q1 = word(nidx);
      nidx--;
    }
  }
};

// Window over a backward bitstream staged in shared memory, for one lane: the
// 32 bits just below position P are read afresh for every lookup (two word
// loads and a funnel shift), so the lane keeps no refill queue and the warp
// has no divergent refill branch.  Same interface as DownWin for huf_run.
// The stage has a zero chunk below and above the staged bytes, so the reads
// near either end of a stream stay inside it (P >= -43 in every decode loop,
// and the stream starts at least 128 bits above the stage's first bit).
struct PosWin {
  const uint32_t* w;  // stage words
  int32_t boff;       // stage bit of the stream's first bit
  int32_t P;          // unread stream bits
  uint32_t hi;        // stream bits [P - 32, P), bit P - 1 at the top

  __device__ __forceinline__ void init(const uint32_t* stage_words, int32_t first_bit, int32_t P0) {
    w = stage_words;
    boff = first_bit;
    P = P0;
  }
  __device__ __forceinline__ void refill() {
    const int32_t A = boff + P;
    const int32_t k = A >> 5;
    hi = __funnelshift_r(w[k - 1], w[k], uint32_t(A));
  }
  __device__ __forceinline__ void consume(uint32_t n) { P -= int32_t(n); }
};

// Asynchronous 16-byte global -> shared copies (cp.async, per thread groups).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// DownWin for one lane reading its own stream through a ring of 32 words (4
// quarters of 8) in shared memory, filled by cp.async.  Async-copy groups are
// tracked per warp, so a lane waiting for its own copy would wait for every
// lane's: the decode therefore runs in warp-uniform rounds (at most 8 ring
// words, one quarter, per lane per round), and at each round start every
// lane commits one group (possibly empty) and waits only for the groups of
// earlier rounds.  A lane keeps the three quarters below the one it reads
// from issued (the whole ring at the start), so every quarter it reads in a
// round was issued at least two rounds earlier.  Words are counted from the
// 16-byte boundary at or below the stream start; bits below the stream start
// read as whatever precedes it, which cannot change a decode that ends
// exactly on the stream's first bit (and one that does not is rejected either
// way).
constexpr int kRingStride = 36;  // words per lane row (16-byte aligned rows)
constexpr int kRingRound = 8;    // ring words a lane may read per round

struct RingWin {
  const uint8_t* g;
  uint32_t* ring;
  uint32_t nchunk;  // 16-byte chunks from g that hold stream bytes (0: lane idle)
  uint32_t hi, lo, vb;
  uint32_t q0, q1;
  int32_t nidx;
  int32_t pc;     // unread stream bits = vb + pc + 32 * nidx (kept out of the per-symbol chain)
  int32_t nextq;  // next quarter to issue

  __device__ __forceinline__ uint32_t word(int32_t i) const { return i < 0 ? 0u : ring[i & 31]; }
  __device__ __forceinline__ void fetch(int32_t h) {  // words [8h, 8h + 8) into their ring slots
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const uint32_t c = 2u * uint32_t(h) + uint32_t(k);
      if (h >= 0 && c < nchunk) cp_async16(ring + ((8 * h + 4 * k) & 31), g + 16ull * c);
    }
  }
  // every lane of the warp calls this (an idle lane passes slen = 0)
  __device__ __forceinline__ void init(const uint8_t* s, uint32_t slen, int32_t P0, uint32_t* lane_ring) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(s);
    g = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(15));
    const uint32_t off = uint32_t(a & 15u);
    ring = lane_ring;
    nchunk = slen ? (off + slen + 15) / 16 : 0u;
    const int32_t A = slen ? P0 + int32_t(8 * off) : 1;
    const int32_t m = (A - 1) >> 5;
    for (int k = 0; k < 4; k++) fetch((m >> 3) - k);  // the whole ring
    nextq = (m >> 3) - 4;
    cp_async_commit();
    cp_async_wait_all();
    const uint32_t sh = uint32_t(32 * (m + 1) - A);
    const uint32_t wm = word(m), wm1 = word(m - 1);
    hi = __funnelshift_l(wm1, wm, sh);
    lo = wm1 << sh;
    vb = 64u - sh;
    q0 = word(m - 2);
    q1 = word(m - 3);
    nidx = m - 4;
    pc = P0 - int32_t(vb) - 32 * nidx;
  }
  // unread stream bits (negative after an overrun)
  __device__ __forceinline__ int32_t pos() const { return int32_t(vb) + pc + 32 * nidx; }
  // round start (after the warp's wait): issue the quarters down to three
  // below the one the next read falls in
  __device__ __forceinline__ void top_up() {
    const int32_t target = (nidx >> 3) - 3;
    while (nextq >= target && nextq >= 0) fetch(nextq--);
  }
  // e = a table entry whose low 5 bits are the code length (1..11): the
  // funnel shifts use the amount modulo 32 and the counter masks it
  __device__ __forceinline__ void consume_entry(uint32_t e) {
    hi = __funnelshift_l(lo, hi, e);
    lo = __funnelshift_l(0u, lo, e);
    vb -= e & 31u;
  }
  __device__ __forceinline__ void refill() {
    const bool use = vb <= 32u;
    const uint32_t mk = use ? 0xFFFFFFFFu : 0u;
    hi |= __funnelshift_rc(q0, 0u, vb) & mk;
    lo |= __funnelshift_lc(0u, q0, 32u - vb) & mk;
    vb += mk & 32u;
    if (use) {
      q0 = q1;
      q1 = word(nidx);
      nidx--;
    }
  }
};

// FSE decode table (RFC 8878 4.1.1): cell = symbol | nbBits << 8 | base << 16,
// built by one warp.  S = stride of the table in u32 words (2 when it is the x
// word of a uint2 cell array); `next` and `start` are 64-entry scratch.
//  - "less than 1" symbols (count -1) take the top cells in symbol order;
//  - the other symbols' occurrences, in symbol order, go to the cells the
//    spread walk pos_k = (k * step) & mask visits, skipping cells above
//    `high`: lane l walks its own range of k, a warp scan of the valid counts
//    gives each lane its first occurrence index, and a binary search of the
//    symbols' first occurrence indices gives each occurrence's symbol;
//  - a cell's state counter x is the symbol's count plus the number of its
//    cells below it: cells are taken 32 at a time in increasing order and
//    lanes holding the same symbol rank themselves with match_any.
template <int S>
__device__ void fse_build_warp(const ZFse& f, uint32_t* t, uint16_t* next, uint16_t* start, int* al_out) {
  const int lane = threadIdx.x & 31;
  if (f.rle) {
    if (lane == 0) {
      t[0] = f.rle_sym;
      *al_out = 0;
    }
    __syncwarp();
    return;
  }
  const int al = f.al, size = 1 << al, nsym = f.nsym;
  const uint32_t lt = (1u << lane) - 1u;
  const int c0 = lane < nsym ? f.norm[lane] : 0, c1 = lane + 32 < nsym ? f.norm[lane + 32] : 0;
  const uint32_t lp0 = __ballot_sync(0xFFFFFFFFu, c0 == -1), lp1 = __ballot_sync(0xFFFFFFFFu, c1 == -1);
  const int n_lp = __popc(lp0) + __popc(lp1);
  const int high = size - 1 - n_lp;
  if (c0 == -1) t[S * (size - 1 - __popc(lp0 & lt))] = uint32_t(lane);
  if (c1 == -1) t[S * (size - 1 - __popc(lp0) - __popc(lp1 & lt))] = uint32_t(lane + 32);
  // first occurrence index of every symbol (prefix sums of the positive counts)
  const int p0 = c0 > 0 ? c0 : 0, p1 = c1 > 0 ? c1 : 0;
  int i0 = p0, i1 = p1;
  for (int o = 1; o < 32; o <<= 1) {
    const int a0 = __shfl_up_sync(0xFFFFFFFFu, i0, o), a1 = __shfl_up_sync(0xFFFFFFFFu, i1, o);
    if (lane >= o) {
      i0 += a0;
      i1 += a1;
    }
  }
  const int tot0 = __shfl_sync(0xFFFFFFFFu, i0, 31);
  start[lane] = uint16_t(i0 - p0);
  start[lane + 32] = uint16_t(tot0 + i1 - p1);
  next[lane] = uint16_t(c0 == -1 ? 1 : p0);
  next[lane + 32] = uint16_t(c1 == -1 ? 1 : p1);
  __syncwarp();
  // spread: lane l takes k in [l * per, (l + 1) * per)
  const int per = size >> 5, step = (size >> 1) + (size >> 3) + 3, mask = size - 1;
  const int k0 = lane * per;
  int valid = 0;
  for (int k = k0; k < k0 + per; k++) valid += ((k * step) & mask) <= high;
  int before = valid;
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xFFFFFFFFu, before, o);
    if (lane >= o) before += a;
  }
  int j = before - valid;
  const int ns = nsym < 64 ? nsym : 64;
  for (int k = k0; k < k0 + per; k++) {
    const int pos = (k * step) & mask;
    if (pos > high) continue;
    // last symbol whose first occurrence index is <= j
    int lo = 0, hi = ns - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (int(start[mid]) <= j) lo = mid;
      else hi = mid - 1;
    }
    t[S * pos] = uint32_t(lo);
    j++;
  }
  __syncwarp();
  for (int base = 0; base < size; base += 32) {
    const int u = base + lane;
    const uint32_t sym = t[S * u] & 0xFFu;
    const uint32_t m = __match_any_sync(0xFFFFFFFFu, sym);
    const uint32_t x = uint32_t(next[sym]) + uint32_t(__popc(m & lt));
    __syncwarp();
    if ((m & lt) == 0) next[sym] = uint16_t(next[sym] + __popc(m));
    const uint32_t nb = uint32_t(al - (31 - __clz(x)));
    t[S * u] = sym | (nb << 8) | (((x << nb) - uint32_t(size)) << 16);
    __syncwarp();
  }
  if (lane == 0) *al_out = al;
  __syncwarp();
}

// Shared memory of the literal decode (K0: Huffman tables) and of the
// sequence walk (K1: FSE tables, bitstream ring, batch positions).
constexpr int kSeqRing = 256;  // ring entries (16 B each)
struct K1Walk {
  // FSE cells (RFC 8878 3.1.1.3.2.1.1), one per state.  LL / ML: x = extra
  // bits | state bits << 6 | baseline << 11, y = byte offset of the next
  // state's first cell.  OF: offset code | state bits << 6 | byte offset of
  // the next state's first cell << 16.  The low 11 bits of three cells add
  // without carries between the fields: extra bits <= 63, state bits <= 26.
  uint2 ll2[512], ml2[512];
  uint32_t of[256];
  uint4 sring[kSeqRing];  // sequence bitstream: entry i = words i..i+3, ring indexed by i & 255
  uint4 skeep[32];        // per sequence of the current batch: bit position, LL, ML, OF cell offsets
  uint16_t next[3][64];
  uint16_t fse_start[64];
  int al[3];
};
struct K1Lit {
  uint32_t huf3[2048];  // up to 3 symbols per lookup: s0|s1<<8|s2<<16|bits<<24|count<<28
  uint16_t huf[2048];
  uint16_t sstart[256];
};
// K0 (zstd_block_literals): a block's literals section is copied into
// shared memory first, then decoded from there by one warp per stream.
constexpr int kLitWarps = 4;               // one warp per Huffman stream
constexpr uint32_t kLitStage = 34 * 1024;  // bytes of a literals section decoded from shared memory
struct K0Shared {
  K1Lit l;
  uint4 stage[kLitStage / 16 + 2];  // a zero chunk, the section's chunks, a zero chunk
};
constexpr int32_t kLitMargin = 128;  // bits decoded to synchronise a span's entry

// Write-combining byte output of one lane: bytes gather in a 64-bit register
// and leave as aligned 8-byte stores; the partial first and last words go out
// byte by byte, so a lane never writes outside its own range.  (A warp's lanes
// write far-apart ranges, so byte stores would cost one L1 wavefront per lane
// per byte.)
struct ByteSink {
  uint64_t* wp;   // aligned word being filled
  uint64_t acc;
  uint32_t k;     // bytes of the word filled (from its aligned start)
  uint32_t k0;    // first byte of ours in the first word; 0 after it
  __device__ __forceinline__ void init(uint8_t* dst) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst);
    wp = reinterpret_cast<uint64_t*>(a & ~uintptr_t(7));
    k = k0 = uint32_t(a & 7u);
    acc = 0;
  }
  __device__ __forceinline__ void flush_bytes(uint32_t from, uint32_t to) {
    uint8_t* b = reinterpret_cast<uint8_t*>(wp);
    for (uint32_t j = from; j < to; j++) b[j] = uint8_t(acc >> (8 * j));
  }
  // append the c (1..3) bytes of `syms` (low first)
  __device__ __forceinline__ void put(uint32_t syms, uint32_t c) {
    const uint64_t v = uint64_t(syms & (0xFFFFFFu >> (8 * (3 - c))));
    acc |= v << (8 * k);
    const uint64_t spill = k ? v >> (64 - 8 * k) : 0ull;  // bytes past the word
    k += c;
    if (k >= 8) {
      if (k0) {
        flush_bytes(k0, 8);
        k0 = 0;
      } else {
        *wp = acc;
      }
      wp++;
      acc = spill;
      k -= 8;
    }
  }
  __device__ __forceinline__ void finish() { flush_bytes(k0, k); }
};

// Huffman decode of one backward stream by one lane, from W.P down to the
// first codeword boundary at or below `stop` (want < 0; out may be null to
// count only), or of exactly `want` symbols.  Multi-symbol lookups never
// cross `stop` (one lookup spans at most maxbits bits), so the exit is the
// first true boundary at or below it whatever the grouping; in counted mode
// they run while >= 3 symbols remain, like the serial decoder.  Returns the
// symbols decoded.
template <class Win>
__device__ __forceinline__ uint32_t huf_run(const K1Lit& sh, Win& W, int32_t stop, uint32_t maxbits,
                                            uint8_t* out, int32_t want) {
  const uint32_t shift = 32u - maxbits;
  uint32_t n = 0;
  ByteSink bs;
  if (out) bs.init(out);
  if (want < 0) {  // every code is >= 1 bit (the planner checks the weights), so P falls
    while (W.P - int32_t(maxbits) > stop) {
      W.refill();
      const uint32_t e = sh.huf3[W.hi >> shift];
      const uint32_t c = e >> 28;
      if (out) bs.put(e, c);
      n += c;
      W.consume(max(1u, (e >> 24) & 15u));
    }
    while (W.P > stop) {
      W.refill();
      const uint32_t e = sh.huf[W.hi >> shift];
      if (out) bs.put(e, 1);
      n++;
      W.consume(max(1u, e >> 8));
    }
    if (out) bs.finish();
    return n;
  }
  const uint32_t w = uint32_t(want);
  while (n + 3 <= w && W.P >= -32) {
    W.refill();
    const uint32_t e = sh.huf3[W.hi >> shift];
    const uint32_t c = e >> 28;
    bs.put(e, c);
    n += c;
    W.consume(max(1u, (e >> 24) & 15u));
  }
  for (; n < w && W.P >= -32; n++) {
    W.refill();
    const uint32_t e = sh.huf[W.hi >> shift];
    bs.put(e, 1);
    W.consume(max(1u, e >> 8));
  }
  bs.finish();
  return n;
}

// Literals section (RFC 8878 3.1.1.3.1) by the literal warps: raw / RLE by
// all of them; Huffman streams one warp each.  A stream of B bits is cut into
// 32 spans; lane j starts at the top of span j and decodes to the first
// codeword boundary at or below the span's end (its exit).  Lane j+1 then
// restarts at lane j's exit, and the pass repeats until no start moves: lane
// 0 starts on the true first codeword, so after pass k lanes 0..k-1 are
// exact, and Huffman codes resynchronise within a few codewords, so two
// passes usually settle every lane.  A last pass writes each lane's symbols at
// its prefix offset; the last lane decodes exactly the remaining count and
// must end on bit 0 (the serial decoder's check).
template <bool kStaged>
__device__ void decode_literals(const uint8_t* src, const View& v, const ZBlock& b, K1Lit& sh, uint8_t* lit,
                                const uint32_t* stage, uint64_t stage_off, uint32_t* status) {
  using Win = typename std::conditional<kStaged, PosWin, DownWin>::type;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (b.lit_type == 0) {
    for (uint32_t i = tid; i < b.lit_regen; i += 32 * kLitWarps) lit[i] = __ldg(src + b.src + i);
    return;
  }
  if (b.lit_type == 1) {
    const uint8_t c = __ldg(src + b.src);
    for (uint32_t i = tid; i < b.lit_regen; i += 32 * kLitWarps) lit[i] = c;
    return;
  }
  const ZHuf& H = v.huf[b.huf];
  const int maxbits = H.maxbits, nsym = H.nsym;
  if (tid == 0) {
    uint32_t count[13] = {0}, start[13];
    for (int s = 0; s < nsym; s++) count[H.w[s]]++;
    uint32_t pos = 0;
    for (int k = 1; k <= maxbits; k++) {
      start[k] = pos;
      pos += count[k] << (k - 1);
    }
    for (int s = 0; s < nsym; s++) {
      const int w = H.w[s];
      if (!w) continue;
      sh.sstart[s] = uint16_t(start[w]);
      start[w] += 1u << (w - 1);
    }
  }
  __syncthreads();
  for (int s = tid; s < nsym; s += 32 * kLitWarps) {
    const int w = H.w[s];
    if (!w) continue;
    const uint16_t e = uint16_t(s | ((maxbits + 1 - w) << 8));
    const uint32_t st = sh.sstart[s], len = 1u << (w - 1);
    for (uint32_t i = 0; i < len; i++) sh.huf[st + i] = e;
  }
  __syncthreads();
  // multi-symbol entries: greedily chain codes while they fit in maxbits
  const uint32_t tsize = 1u << maxbits, mask = tsize - 1;
  for (uint32_t i = tid; i < tsize; i += 32 * kLitWarps) {
    uint32_t e0 = sh.huf[i], l0 = e0 >> 8, bits = l0, cnt = 1, syms = e0 & 0xFFu;
    const uint32_t e1 = sh.huf[(i << l0) & mask], l1 = e1 >> 8;
    if (bits + l1 <= uint32_t(maxbits)) {
      syms |= (e1 & 0xFFu) << 8;
      bits += l1;
      cnt = 2;
      const uint32_t e2 = sh.huf[(i << bits) & mask], l2 = e2 >> 8;
      if (bits + l2 <= uint32_t(maxbits)) {
        syms |= (e2 & 0xFFu) << 16;
        bits += l2;
        cnt = 3;
      }
    }
    sh.huf3[i] = syms | (bits << 24) | (cnt << 28);
  }
  __syncthreads();
  const int streams = int(b.lit_streams);
  if (warp >= streams) return;
  const uint32_t seg = streams == 1 ? b.lit_regen : (b.lit_regen + 3) / 4;
  const uint32_t count = (streams == 1 || warp < 3) ? seg : b.lit_regen - 3 * seg;
  uint64_t off = b.src;
  for (int k = 0; k < warp; k++) off += b.lit_len[k];
  uint8_t* out = lit + uint32_t(warp) * seg;
  const uint8_t* sp = src + off;
  // stage bit of the stream's first bit (staged sections: global byte g is stage byte g - stage_off)
  const int32_t first_bit = int32_t(8 * (off - stage_off));
  const uint32_t slen = b.lit_len[warp];
  const uint32_t lastb =
      slen ? (kStaged ? (stage[(off - stage_off + slen - 1) >> 2] >> (8 * ((off - stage_off + slen - 1) & 3))) & 0xFFu
                      : uint32_t(__ldg(sp + slen - 1)))
           : 0u;
  bool ok = lastb != 0;
  auto win_init = [&](Win& W, int32_t P0) {
    if constexpr (kStaged) W.init(stage, first_bit, P0);
    else W.init(sp, P0);
  };
  if (ok) {
    const int32_t B = int32_t(8 * (slen - 1) + (31 - __clz(lastb)));
    // spans: one lane for short streams, else 32
    const int nl = B >= 32 * 256 ? 32 : 1;
    const int32_t span = (B + nl - 1) / nl;
    const bool active = lane < nl;
    const bool last = lane == nl - 1;
    const int32_t stop = last ? 0 : B - (lane + 1) * span;
    int32_t start = active ? B - lane * span : 0;
    if (active && lane > 0) {
      // Enter the span synchronised: decode from kLitMargin bits above its
      // top down to the first boundary at or below it.  Huffman codes
      // resynchronise within a few codewords, so this is usually the previous
      // lane's exit and the first counting pass is already exact.
      Win W;
      win_init(W, min(B, start + kLitMargin));
      huf_run(sh, W, start, uint32_t(maxbits), nullptr, -1);
      start = W.P;
    }
    uint32_t n = 0;
    for (int pass = 0; pass <= nl; pass++) {
      int32_t exitp = start;
      n = 0;
      if (active && !last) {
        Win W;
        win_init(W, start);
        n = huf_run(sh, W, stop, uint32_t(maxbits), nullptr, -1);
        exitp = W.P;
      }
      int32_t next = __shfl_up_sync(0xFFFFFFFFu, exitp, 1);
      if (lane == 0 || !active) next = start;
      if (!__any_sync(0xFFFFFFFFu, next != start)) break;
      start = next;
    }
    // offsets: exclusive prefix of the non-last lanes' counts
    uint32_t incl = (active && !last) ? n : 0u;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t excl = incl - ((active && !last) ? n : 0u);
    bool lane_ok = true;
    if (active) {
      Win W;
      win_init(W, start);
      if (!last) {
        lane_ok = excl + n <= count;  // a damaged stream may decode more symbols than it holds
        if (lane_ok) huf_run(sh, W, stop, uint32_t(maxbits), out + excl, -1);
      } else if (excl <= count) {
        const uint32_t got = huf_run(sh, W, 0, uint32_t(maxbits), out + excl, int32_t(count - excl));
        lane_ok = (got == count - excl) && W.P == 0;
      } else {
        lane_ok = false;
      }
    }
    ok = __all_sync(0xFFFFFFFFu, lane_ok);
  }
  if (!ok && lane == 0) atomicOr(status + b.job, VOOM_ZSTD_ST_LITERALS);
}

// Huffman literals of direct jobs' blocks (no sequences: the literals are the
// output), one lane per stream.  Spans of one stream decoded in parallel enter
// their span speculatively and need another pass for every lane whose entry
// did not resynchronise; literals close to uniform (the low bytes of BF16
// activations) resynchronise slowly, so here every stream is decoded once,
// serially, and the parallelism comes from the number of streams: a warp
// takes 8 blocks, lanes 4g..4g+3 the (up to) 4 streams of block g, with the
// block's single-symbol decode table (2^maxbits u16 entries) in shared memory.
constexpr int kDlBlocksPerWarp = 8;
constexpr uint32_t kHufTab = 1u << 11;  // RFC 8878 caps Huffman codes at 11 bits

__global__ void __launch_bounds__(32) zstd_direct_literals(const uint8_t* __restrict__ src, const uint8_t* img,
                                                           uint8_t* scratch, uint8_t* __restrict__ out,
                                                           uint32_t* status) {
  __shared__ uint16_t s_tab[kDlBlocksPerWarp][kHufTab];
  __shared__ __align__(16) uint32_t s_ring[32][kRingStride];
  const View v = make_view(img, scratch);
  const uint32_t* dlit = reinterpret_cast<const uint32_t*>(img + v.h->off_dlit);
  const uint32_t lane = threadIdx.x, g = lane >> 2, q = lane & 3u;
  const uint32_t slot = blockIdx.x * kDlBlocksPerWarp + g;
  const bool on = slot < v.h->n_dlit;
  ZBlock b;
  uint32_t maxbits = 1, nsym = 0;
  const ZHuf* H = nullptr;
  if (on) {
    b = v.blocks[dlit[slot]];
    H = v.huf + b.huf;
    maxbits = H->maxbits;
    nsym = H->nsym;
  }
  // table build: lane q of the group places symbols [64q, 64q + 64); codes are
  // canonical (weight ascending, then symbol order), so every weight's first
  // position is the sum over lighter weights and a lane's offset within a
  // weight is the count of that weight in the lanes before it
  // this lane's 64 weights as 16 independent 4-byte loads (ZHuf rows are
  // 4-byte aligned); weights past nsym read as 0
  const uint32_t s0 = 64 * q, s1 = min(nsym, s0 + 64);
  uint32_t wv[16];
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const uint32_t sy = s0 + 4u * uint32_t(k);
    uint32_t x = sy < s1 ? __ldg(reinterpret_cast<const uint32_t*>(H->w + sy)) : 0u;
    if (sy + 4 > s1 && sy < s1) x &= 0xFFFFFFFFu >> (8 * (sy + 4 - s1));
    wv[k] = x;
  }
  uint32_t cnt[12];
#pragma unroll
  for (int k = 0; k < 12; k++) cnt[k] = 0;
#pragma unroll
  for (int k = 0; k < 16; k++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint32_t w = (wv[k] >> (8 * c)) & 0xFFu;
#pragma unroll
      for (int t = 1; t < 12; t++) cnt[t] += (w == uint32_t(t));
    }
  uint32_t pos[12];
  uint32_t start = 0;
#pragma unroll
  for (int k = 1; k < 12; k++) {
    uint32_t incl = cnt[k];
    uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, 1, 4);
    if (q >= 1) incl += t;
    t = __shfl_up_sync(0xFFFFFFFFu, incl, 2, 4);
    if (q >= 2) incl += t;
    const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 3, 4);
    pos[k] = start + ((incl - cnt[k]) << (k - 1));
    start += total << (k - 1);
  }
  // a complete code fills the table exactly (the same for the group's lanes)
  bool ok = start == (1u << maxbits);
  // entry = code length | symbol << 8: the funnel shift that consumes a code
  // takes its amount from the low 5 bits, so no extraction sits in the chain
  uint16_t* tab = s_tab[g];
  if (ok) {
#pragma unroll
    for (int k4 = 0; k4 < 64; k4++) {  // unrolled: wv stays in registers
      const uint32_t w = (wv[k4 >> 2] >> (8 * (k4 & 3))) & 0xFFu;
      if (w) {
        uint32_t p = 0;
#pragma unroll
        for (int k = 1; k < 12; k++)
          if (w == uint32_t(k)) {
            p = pos[k];
            pos[k] += 1u << (k - 1);
          }
        const uint16_t e = uint16_t((maxbits + 1 - w) | ((s0 + uint32_t(k4)) << 8));
        const uint32_t len = 1u << (w - 1);
        for (uint32_t i = 0; i < len; i++)
          if (p + i < kHufTab) tab[p + i] = e;
      }
    }
  }
  __syncwarp();
  // From here every lane stays to the end: the rounds below are warp-uniform.
  const int streams = on ? int(b.lit_streams) : 0;
  const bool act = on && int(q) < streams;
  uint32_t seg = 0, count = 0, slen = 0;
  const uint8_t* sp = src;
  uint8_t* dst = out;
  int32_t B = 0;
  if (act) {
    const ZJob& job = v.jobs[b.job];
    seg = streams == 1 ? b.lit_regen : (b.lit_regen + 3) / 4;
    count = (streams == 1 || q < 3) ? seg : b.lit_regen - 3 * seg;
    uint64_t off = b.src;
    slen = b.lit_len[0];
#pragma unroll
    for (uint32_t k = 1; k < 4; k++)
      if (k <= q) {
        off += slen;
        slen = b.lit_len[k];
      }
    sp = src + off;
    const uint32_t lastb = slen ? __ldg(sp + slen - 1) : 0u;
    ok = ok && lastb != 0 && seg * uint64_t(q) <= b.lit_regen;
    if (ok) B = int32_t(8 * (slen - 1) + (31 - __clz(lastb)));
    dst = out + job.dst + b.out_off + uint64_t(q) * seg;
  }
  ok = act && ok;
  RingWin W;
  W.init(sp, ok ? slen : 0u, B, s_ring[lane]);
  const uint32_t shift = 32u - maxbits;
  uint32_t n = 0;
  // one symbol: a refill leaves >= 32 valid bits, a code is <= 11
  auto one = [&]() -> uint32_t {
    W.refill();
    const uint32_t e = tab[W.hi >> shift];
    W.consume_entry(e);
    return e >> 8;
  };
  // head: single symbols up to a 4-byte boundary of the output (within the
  // ring's initial four quarters: at most 3 refills)
  if (ok) {
    const uint32_t head = min(count, uint32_t(4u - (reinterpret_cast<uintptr_t>(dst) & 3u)) & 3u);
    for (; n < head; n++) dst[n] = uint8_t(one());
  }
  uint32_t* d32 = reinterpret_cast<uint32_t*>(dst + n);
  // the count bounds every loop; a damaged stream that runs past its start reads
  // zero words and is rejected by the final position check
  bool live = ok && n + 4 <= count;
  while (__any_sync(0xFFFFFFFFu, live)) {
    cp_async_wait_prev();
    if (live) W.top_up();
    cp_async_commit();
    // 4 symbols (two refills, at most 2 ring words) and one 32-bit store per step
#pragma unroll 2
    for (int r = 0; r < kRingRound / 2; r++) {
      if (live) {
        W.refill();
        const uint32_t e0 = tab[W.hi >> shift];
        W.consume_entry(e0);
        const uint32_t e1 = tab[W.hi >> shift];
        W.consume_entry(e1);
        W.refill();
        const uint32_t e2 = tab[W.hi >> shift];
        W.consume_entry(e2);
        const uint32_t e3 = tab[W.hi >> shift];
        W.consume_entry(e3);
        // symbols are byte 1 of each entry
        *d32++ = __byte_perm(__byte_perm(e0, e1, 0x0051), __byte_perm(e2, e3, 0x0051), 0x5410);
        n += 4;
        live = n + 4 <= count;
      }
    }
  }
  // every copy complete: the tail below may read from the quarter issued last,
  // and no copy may still target shared memory when the CTA exits
  cp_async_wait_all();
  if (ok)  // tail: fewer than 4 symbols (at most 3 more ring words)
    for (; n < count; n++) dst[n] = uint8_t(one());
  ok = ok && n == count && W.pos() == 0;
  if (act && !ok) atomicOr(status + b.job, VOOM_ZSTD_ST_LITERALS);
}

// Symbolic repeat-offset slot: kind 0..2 = the block's input slot minus d,
// kind 3 = the constant d.
struct RepSlots {
  uint32_t k[3], d[3];
};

__device__ __forceinline__ void rep_sub(uint32_t& k, uint32_t& d, uint32_t kk, uint32_t dd, uint32_t delta) {
  k = kk;
  d = kk == 3 ? dd - delta : dd + delta;
}

// One sequence's repeat-offset rule (RFC 8878 3.1.2.5) applied to symbolic
// slots; returns the offset it uses.
__device__ __forceinline__ void rep_step(RepSlots& r, uint32_t ofv, uint32_t ll, uint32_t& ok, uint32_t& ov) {
  if (ofv > 3) {
    ok = 3;
    ov = ofv - 3;
  } else {
    const uint32_t idx = ofv - 1 + (ll == 0);
    if (idx == 0) {
      ok = r.k[0]; ov = r.d[0];
      return;
    }
    if (idx == 1) {
      ok = r.k[1]; ov = r.d[1];
      r.k[1] = r.k[0]; r.d[1] = r.d[0];
      r.k[0] = ok; r.d[0] = ov;
      return;
    }
    if (idx == 2) {
      ok = r.k[2]; ov = r.d[2];
    } else {
      rep_sub(ok, ov, r.k[0], r.d[0], 1);
    }
  }
  r.k[2] = r.k[1]; r.d[2] = r.d[1];
  r.k[1] = r.k[0]; r.d[1] = r.d[0];
  r.k[0] = ok; r.d[0] = ov;
}

// Slots after transform t applied to slots s (t is symbolic in its own input).
__device__ __forceinline__ RepSlots rep_compose(const RepSlots& s, const RepSlots& t) {
  RepSlots o;
#pragma unroll
  for (int q = 0; q < 3; q++) {
    if (t.k[q] == 3) {
      o.k[q] = 3;
      o.d[q] = t.d[q];
    } else {
      const uint32_t src = t.k[q];
      const uint32_t sk = src == 0 ? s.k[0] : (src == 1 ? s.k[1] : s.k[2]);
      const uint32_t sd = src == 0 ? s.d[0] : (src == 1 ? s.d[1] : s.d[2]);
      rep_sub(o.k[q], o.d[q], sk, sd, t.d[q]);
    }
  }
  return o;
}

// Sequences section (RFC 8878 3.1.1.3.2.2) by a K1 walker warp.  All 32
// lanes run the FSE walk in lockstep (same values; shared-memory reads are
// broadcasts).  Each sequence reads its fields from fixed positions below the
// current bit position P -- offset extra bits, match-length extra, literal-
// length extra, then the LL, ML and OF state bits.  The walk carries only the
// state chain and records each sequence's position and cells; every 32
// sequences lane j extracts the fields of the batch's sequence j and stores
// its literal length, match length and offset value.  zstd_seq_scan resolves
// repeat offsets and output positions in parallel afterwards.  Returns the
// section's status bits.
__device__ uint32_t decode_sequences(const uint8_t* src, const View& v, const ZBlock& b, K1Walk& sh) {
  const int lane = threadIdx.x & 31;
  // tables are built in the x words of their cell arrays
  fse_build_warp<2>(v.fse[b.fse[0]], reinterpret_cast<uint32_t*>(sh.ll2), sh.next[0], sh.fse_start, &sh.al[0]);
  fse_build_warp<1>(v.fse[b.fse[1]], sh.of, sh.next[1], sh.fse_start, &sh.al[1]);
  fse_build_warp<2>(v.fse[b.fse[2]], reinterpret_cast<uint32_t*>(sh.ml2), sh.next[2], sh.fse_start, &sh.al[2]);
  {
    const uint32_t nll = 1u << sh.al[0], nof = 1u << sh.al[1], nml = 1u << sh.al[2];
    for (uint32_t u = lane; u < nll; u += 32) {
      const uint32_t t = sh.ll2[u].x, c = min(t & 0xFFu, 35u), nb = (t >> 8) & 0xFFu;
      sh.ll2[u] = make_uint2(uint32_t(c_ll_bits[c]) | (nb << 6) | (c_ll_base[c] << 11), (t >> 16) << 3);
    }
    for (uint32_t u = lane; u < nml; u += 32) {
      const uint32_t t = sh.ml2[u].x, c = min(t & 0xFFu, 52u), nb = (t >> 8) & 0xFFu;
      sh.ml2[u] = make_uint2(uint32_t(c_ml_bits[c]) | (nb << 6) | (c_ml_base[c] << 11), (t >> 16) << 3);
    }
    for (uint32_t u = lane; u < nof; u += 32) {
      const uint32_t t = sh.of[u], nb = (t >> 8) & 0xFFu;
      sh.of[u] = min(t & 0xFFu, 31u) | (nb << 6) | (((t >> 16) << 2) << 16);
    }
  }
  __syncwarp();
  ZSeq* out = v.seq + b.seq_off;
  uint32_t st = 0;
  const uint8_t* p = src + b.seq_src;
  const uint32_t len = b.seq_len;
  const uint32_t lastb = len ? __ldg(p + len - 1) : 0u;
  if (!lastb) return VOOM_ZSTD_ST_SEQUENCES;
  // Aligned words of the stream: word k holds aligned bits [32k, 32k+32);
  // stream bit q is aligned bit q + boff.  Ring entry i holds words i..i+3
  // (128 bits from word i), so any 96-bit window is one 16-byte read.
  const uintptr_t pa = reinterpret_cast<uintptr_t>(p);
  const uint32_t* wbase = reinterpret_cast<const uint32_t*>(pa & ~uintptr_t(3));
  const int32_t boff = int32_t(pa & 3u) * 8;
  auto gword = [&](int32_t k) -> uint32_t { return k >= 0 ? __ldg(wbase + k) : 0u; };
  // entries [e0, e0 + 32) from words e0 .. e0 + 34 (the top three words of
  // the batch come from `above`, the words just over it)
  auto fill32 = [&](int32_t e0, uint32_t w_l, uint3 above) {
    const uint32_t n1 = __shfl_down_sync(0xFFFFFFFFu, w_l, 1), n2 = __shfl_down_sync(0xFFFFFFFFu, w_l, 2),
                   n3 = __shfl_down_sync(0xFFFFFFFFu, w_l, 3);
    const uint32_t w1 = lane < 31 ? n1 : above.x;
    const uint32_t w2 = lane < 30 ? n2 : (lane == 30 ? above.x : above.y);
    const uint32_t w3 = lane < 29 ? n3 : (lane == 29 ? above.x : (lane == 30 ? above.y : above.z));
    sh.sring[(e0 + lane) & (kSeqRing - 1)] = make_uint4(w_l, w1, w2, w3);
  };
  const int32_t Pa0 = int32_t(8 * (len - 1) + (31 - __clz(lastb))) + boff;  // aligned position
  int32_t Pa = Pa0;
  // the ring covers entries [lo_w, lo_w + kSeqRing); reads touch entries at or below (Pa - 1) >> 5
  int32_t lo_w = ((Pa0 - 1) >> 5) + 1 - kSeqRing;
  {
    const int32_t topw = lo_w + kSeqRing;
    uint3 above = make_uint3(gword(topw), gword(topw + 1), gword(topw + 2));
    for (int j = kSeqRing / 32 - 1; j >= 0; j--) {
      const int32_t e0 = lo_w + 32 * j;
      const uint32_t w_l = gword(e0 + lane);
      fill32(e0, w_l, above);
      above = make_uint3(__shfl_sync(0xFFFFFFFFu, w_l, 0), __shfl_sync(0xFFFFFFFFu, w_l, 1),
                         __shfl_sync(0xFFFFFFFFu, w_l, 2));
    }
  }
  uint32_t pre = gword(lo_w - 32 + lane);  // next batch, loaded one refill ahead
  __syncwarp();
  const char* ring = reinterpret_cast<const char*>(sh.sring);
  // stream bits [a, a + 32) at aligned position a (entry (a >> 5) & 255 at byte offset 16 x that)
  auto at = [&](int32_t a) -> uint32_t {
    const uint4 e = *reinterpret_cast<const uint4*>(ring + ((uint32_t(a) >> 1) & 0xFF0u));
    return __funnelshift_r(e.x, e.y, uint32_t(a));  // shifts by a & 31
  };
  const uint32_t a0 = sh.al[0], a1 = sh.al[1], a2 = sh.al[2];
  const char* cll = reinterpret_cast<const char*>(sh.ll2);
  const char* cml = reinterpret_cast<const char*>(sh.ml2);
  const char* cof = reinterpret_cast<const char*>(sh.of);
  if (Pa - boff < int32_t(a0 + a1 + a2)) return VOOM_ZSTD_ST_SEQUENCES;
  // cell byte offsets of the current LL, ML and OF states
  uint32_t oll, oml, oof;
  {
    const uint32_t init = at(Pa - int32_t(a0 + a1 + a2));
    oml = bfe32(init, 0, a2) << 3;
    oof = bfe32(init, a2, a1) << 2;
    oll = bfe32(init, a1 + a2, a0) << 3;
    Pa -= int32_t(a0 + a1 + a2);
  }
  const uint32_t nseq = b.nseq;
  // after every batch of up to 32 sequences: lane j's record from skeep[j].
  // The batch's positions stay inside the ring (a sequence spans at most 89
  // bits; refills move the ring down 32 entries at a time).
  auto flush = [&](uint32_t first, uint32_t count) {
    __syncwarp();
    if (uint32_t(lane) < count) {
      const uint4 k = sh.skeep[lane];
      const int32_t myPa = int32_t(k.x);
      const uint32_t xL = reinterpret_cast<const uint2*>(cll + k.y)->x;
      const uint32_t xM = reinterpret_cast<const uint2*>(cml + k.z)->x;
      const uint32_t xO = *reinterpret_cast<const uint32_t*>(cof + k.w);
      const uint32_t ofc = xO & 63u, mlb = xM & 63u, llb = xL & 63u;
      // offset extra (<= 31 bits) at the top of the word below the position,
      // ML then LL extras (<= 32 bits together) under it; a field of n bits is
      // the top n bits of its window (n = 0: the clamped funnel shift by 32
      // gives 0)
      const uint32_t w1 = at(myPa - 32), w2 = at(myPa - int32_t(ofc) - 32);
      const uint32_t ofv = (1u << ofc) + __funnelshift_rc(w1, 0u, 32u - ofc);
      const uint32_t ml = (xM >> 11) + __funnelshift_rc(w2, 0u, 32u - mlb);
      const uint32_t ll = (xL >> 11) + __funnelshift_rc(w2 << mlb, 0u, 32u - llb);
      ZSeq* r = out + first + lane;  // raw record; zstd_seq_scan fills offsets and positions
      *reinterpret_cast<uint2*>(&r->ll) = make_uint2(ll, ml);
      r->oval = ofv;
    }
    __syncwarp();
  };
  // Checked before every group of up to 8 sequences: refill while Pa - 96 -
  // 7 x 89 (the lowest window read of the group) would fall under the ring;
  // one refill of 32 entries (1024 bits) covers a group (<= 712 bits).
  constexpr int32_t kSlack = 96 + 7 * 89;
  int32_t refill_at = 32 * lo_w + kSlack;
  auto refill = [&]() {
    if (Pa < refill_at) {
      const uint4 e = sh.sring[lo_w & (kSeqRing - 1)];
      fill32(lo_w - 32, pre, make_uint3(e.x, e.y, e.z));
      lo_w -= 32;
      refill_at -= 32 * 32;
      pre = gword(lo_w - 32 + lane);
      __syncwarp();
    }
  };
  // One sequence that reads state bits (every sequence but the last).  The
  // 96 stream bits under the position come from one ring entry read beside
  // the three cells (its address depends on the position only), so the chain
  // from one state to the next holds a single shared-memory read: cells ->
  // the extra-bit count (one add of the three x words) -> the 32 bits under
  // the extras -> the three state fields -> the next cells' offsets.
  auto step = [&](uint4* keep) {
    const uint2 cL = *reinterpret_cast<const uint2*>(cll + oll);
    const uint2 cM = *reinterpret_cast<const uint2*>(cml + oml);
    const uint32_t cO = *reinterpret_cast<const uint32_t*>(cof + oof);
    const uint32_t p96 = uint32_t(Pa - 96);  // >= 32 * lo_w (refill invariant)
    const uint4 e = *reinterpret_cast<const uint4*>(ring + ((p96 >> 1) & 0xFF0u));
    *keep = make_uint4(uint32_t(Pa), oll, oml, oof);  // same value from every lane
    // stream bits [Pa - 96, Pa) as lo | mid | hi (funnel shifts by p96 & 31)
    const uint32_t lo = __funnelshift_r(e.x, e.y, p96), mid = __funnelshift_r(e.y, e.z, p96),
                   hi = __funnelshift_r(e.z, e.w, p96);
    // bits 0-5: the extra bits (<= 63), bits 6-10: the state bits (<= 26)
    const uint32_t S = cL.x + cM.x + cO;
    // the 32 bits under the extras (the LL, ML, OF state bits at the top);
    // funnel shifts take S modulo 32
    const uint32_t w = (S & 32u) ? __funnelshift_l(lo, mid, S) : __funnelshift_l(mid, hi, S);
    // state-bit counts in the low 5 bits (the baselines above are shifted out
    // modulo 32): top n bits of a word = high word of (0:word) << n
    const uint32_t nL = cL.x >> 6, nM = cM.x >> 6, nO = cO >> 6;
    const uint32_t bL = __funnelshift_l(w, 0u, nL);
    const uint32_t bM = __funnelshift_l(__funnelshift_l(0u, w, nL), 0u, nM);
    const uint32_t bO = __funnelshift_l(__funnelshift_l(0u, w, nL + nM), 0u, nO);
    oll = cL.y + (bL << 3);
    oml = cM.y + (bM << 3);
    oof = (cO >> 16) + (bO << 2);
    // A stream that runs out reads zero words below its start (never memory
    // outside it) and ends with Pa below boff: checked once below.
    Pa -= int32_t((S & 63u) + ((S >> 6) & 31u));
  };
  for (uint32_t first = 0; first + 1 < nseq; first += 32) {
    const uint32_t cnt = min(32u, nseq - 1 - first);
    if (cnt == 32) {
      for (uint32_t g = 0; g < 32; g += 8) {
        refill();
#pragma unroll
        for (uint32_t jj = 0; jj < 8; jj++) step(sh.skeep + g + jj);
      }
    } else {
      for (uint32_t jj = 0; jj < cnt; jj++) {
        refill();
        step(sh.skeep + jj);
      }
    }
    flush(first, cnt);
  }
  if (nseq) {  // the last sequence: extra bits only
    refill();
    sh.skeep[0] = make_uint4(uint32_t(Pa), oll, oml, oof);
    const uint32_t S = reinterpret_cast<const uint2*>(cll + oll)->x + reinterpret_cast<const uint2*>(cml + oml)->x +
                       *reinterpret_cast<const uint32_t*>(cof + oof);
    Pa -= int32_t(S & 63u);
    flush(nseq - 1, 1);
  }
  if (Pa != boff) st = VOOM_ZSTD_ST_SEQUENCES;  // overrun (Pa < boff) or bits left over
  return st;
}

// K0: the literals section of every block of the segment's block list (one
// CTA per block, a warp per stream).  The section is first copied into shared
// memory with coalesced 16-byte loads: the 32 lanes of a stream's warp each
// decode their own span, and reading the words from global memory made every
// lookup wait on a load that missed L1.  Sections larger than the stage are
// decoded from global memory.  Raw and RLE sections are copied; direct jobs'
// Huffman literals are zstd_direct_literals' work.
__global__ void __launch_bounds__(32 * kLitWarps) zstd_block_literals(const uint8_t* __restrict__ src,
                                                                      const uint8_t* img, uint8_t* scratch,
                                                                      uint8_t* out, uint32_t* status, uint32_t bl0) {
  __shared__ K0Shared sh;
  const View v = make_view(img, scratch);
  const uint32_t bi = reinterpret_cast<const uint32_t*>(img + v.h->off_blist)[bl0 + blockIdx.x];
  const ZBlock b = v.blocks[bi];
  if (b.type != 2) return;
  const ZJob& job = v.jobs[b.job];
  if (job.bad || (job.direct && b.lit_type == 2)) return;
  // a direct job's literals are its output bytes
  uint8_t* lit = job.direct ? out + job.dst + b.out_off : v.lit + b.lit_off;
  uint64_t len = 0;
  if (b.lit_type == 2)
    for (uint32_t q = 0; q < b.lit_streams; q++) len += b.lit_len[q];
  const uint64_t base = b.src & ~uint64_t(15);
  const uint64_t chunks = (b.src + len - base + 15) / 16;  // the source has 16 readable bytes past its end
  if (b.lit_type == 2 && chunks <= kLitStage / 16) {
    const uint4* g = reinterpret_cast<const uint4*>(src + base);
    for (uint32_t i = threadIdx.x; i < chunks; i += blockDim.x) sh.stage[1 + i] = __ldg(g + i);
    if (threadIdx.x == 0) {
      sh.stage[0] = make_uint4(0u, 0u, 0u, 0u);
      sh.stage[chunks + 1] = make_uint4(0u, 0u, 0u, 0u);
    }
    // (the table build in decode_literals synchronises the CTA before any read)
    decode_literals<true>(src, v, b, sh.l, lit, reinterpret_cast<const uint32_t*>(sh.stage), base - 16, status);
  } else {
    decode_literals<false>(src, v, b, sh.l, lit, nullptr, 0, status);
  }
}

// K1: the sequences section of every block of the segment's block list, one
// warp per block, and every block's runtime record.  One-warp CTAs take the
// SMs' warp slots in launch order, so the first `wave` CTAs (4 per SM) get a
// scheduler each and the rest pair up with them; CTA c < wave walks the c-th
// longest block and CTA wave + i the i-th shortest, so a long walk shares its
// scheduler with a short one and then runs alone (a walk sharing its scheduler
// takes about 120 cycles per sequence, alone about 90).
__global__ void __launch_bounds__(32) zstd_block_decode(const uint8_t* __restrict__ src, const uint8_t* img,
                                                        uint8_t* scratch, uint32_t bl0, uint32_t n_bl,
                                                        uint32_t wave) {
  __shared__ K1Walk sh;
  const View v = make_view(img, scratch);
  const uint32_t c = blockIdx.x, pos = c < wave ? c : n_bl - 1u - (c - wave);
  const uint32_t bi = reinterpret_cast<const uint32_t*>(img + v.h->off_k1list)[bl0 + pos];
  const ZBlock b = v.blocks[bi];
  ZBlockRt* rt = v.rt + bi;
  uint32_t st = 0;
  if (b.type == 2 && b.nseq) st = decode_sequences(src, v, b, sh);
  if (threadIdx.x == 0) {
    // blocks with sequences get out_size and the repeat transform from
    // zstd_seq_scan; a damaged literals section flags its job in K0
    if (b.type == 2 && !b.nseq && b.lit_regen > b.max_out) st |= VOOM_ZSTD_ST_SIZE;
    rt->out_size = b.type == 2 ? b.lit_regen : b.size;
    rt->status = st;
    for (int k = 0; k < 3; k++) {
      rt->rep_kind[k] = uint32_t(k);
      rt->rep_val[k] = 0;
    }
  }
}

// Per compressed block with sequences, after zstd_block_decode: the repeat-
// offset rules and output / literal positions of every sequence (RFC 8878
// 3.1.2.5).  Rounds of 128 x 4 consecutive records: each thread applies the
// rules of its 4 records to symbolic slots (slot = block-start slot minus d,
// or a constant), giving its transform and length sums; warps scan the
// transforms, the 4 warp totals are scanned by warp 0, and each thread,
// starting from its carry-in (all earlier records composed), replays its 4
// records on those slots to get each one's offset and positions.  Also the
// block's output size, its repeat transform for the job scan, and the
// literal-count check.
constexpr int kSeqScanThreads = 128;  // 8 CTAs per SM at 61 registers
constexpr int kSeqPerThread = 4;

__global__ void __launch_bounds__(kSeqScanThreads) zstd_seq_scan(const uint8_t* img, uint8_t* scratch,
                                                                 uint32_t bl0) {
  constexpr int kW = kSeqScanThreads / 32;
  __shared__ uint32_t s_k[kW][3], s_d[kW][3];
  __shared__ uint32_t s_ll[kW], s_ml[kW];
  // per warp: carry-in slots and length sums; entry [kW] = the round total
  __shared__ uint32_t s_ck[kW + 1][3], s_cd[kW + 1][3];
  __shared__ uint32_t s_cl[kW + 1], s_cm[kW + 1];
  const View v = make_view(img, scratch);
  // blocks in walk order (most sequences first): the CTAs of the longest
  // blocks start in the first wave
  const uint32_t bi = reinterpret_cast<const uint32_t*>(img + v.h->off_k1list)[bl0 + blockIdx.x];
  const ZBlock b = v.blocks[bi];
  if (b.type != 2 || b.nseq == 0) return;
  ZBlockRt* rt = v.rt + bi;
  if (rt->status) return;  // the block failed in K1; its job is reported bad
  ZSeq* seq = v.seq + b.seq_off;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5, n = b.nseq;
  RepSlots C;  // slots at the start of the round (relative to the block start)
#pragma unroll
  for (int q = 0; q < 3; q++) {
    C.k[q] = uint32_t(q);
    C.d[q] = 0;
  }
  uint32_t cll = 0, cml = 0;  // literal and match bytes before the round
  for (uint32_t base = 0; base < n; base += kSeqScanThreads * kSeqPerThread) {
    const uint32_t i0 = base + tid * kSeqPerThread;
    uint32_t ll[kSeqPerThread], ml[kSeqPerThread], ofv[kSeqPerThread];
#pragma unroll
    for (int r = 0; r < kSeqPerThread; r++) {
      ll[r] = ml[r] = 0;
      ofv[r] = 4;
      if (i0 + r < n) {
        const uint2 lm = *reinterpret_cast<const uint2*>(&seq[i0 + r].ll);
        ll[r] = lm.x;
        ml[r] = lm.y;
        ofv[r] = seq[i0 + r].oval;
      }
    }
    // this thread's transform: its records' rules on identity slots
    RepSlots incl;
#pragma unroll
    for (int q = 0; q < 3; q++) {
      incl.k[q] = uint32_t(q);
      incl.d[q] = 0;
    }
    uint32_t ill = 0, iml = 0;
#pragma unroll
    for (int r = 0; r < kSeqPerThread; r++) {
      uint32_t uk, ud;
      if (i0 + r < n) rep_step(incl, ofv[r], ll[r], uk, ud);
      ill += ll[r];
      iml += ml[r];
    }
    for (int o = 1; o < 32; o <<= 1) {
      RepSlots prev;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        prev.k[q] = __shfl_up_sync(0xFFFFFFFFu, incl.k[q], o);
        prev.d[q] = __shfl_up_sync(0xFFFFFFFFu, incl.d[q], o);
      }
      const uint32_t pl = __shfl_up_sync(0xFFFFFFFFu, ill, o), pm = __shfl_up_sync(0xFFFFFFFFu, iml, o);
      if (lane >= o) {
        incl = rep_compose(prev, incl);
        ill += pl;
        iml += pm;
      }
    }
    if (lane == 31) {
#pragma unroll
      for (int q = 0; q < 3; q++) {
        s_k[warp][q] = incl.k[q];
        s_d[warp][q] = incl.d[q];
      }
      s_ll[warp] = ill;
      s_ml[warp] = iml;
    }
    __syncthreads();
    // warp 0 scans the warp totals (lane w holds warp w's), starting from the
    // round's carry-in C, and publishes each warp's carry-in and the total
    if (warp == 0) {
      RepSlots x;
      uint32_t xl = 0, xm = 0;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        x.k[q] = lane < kW ? s_k[lane][q] : uint32_t(q);
        x.d[q] = lane < kW ? s_d[lane][q] : 0u;
      }
      if (lane < kW) {
        xl = s_ll[lane];
        xm = s_ml[lane];
      }
      for (int o = 1; o < kW; o <<= 1) {
        RepSlots prev;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          prev.k[q] = __shfl_up_sync(0xFFFFFFFFu, x.k[q], o);
          prev.d[q] = __shfl_up_sync(0xFFFFFFFFu, x.d[q], o);
        }
        const uint32_t pl = __shfl_up_sync(0xFFFFFFFFu, xl, o), pm = __shfl_up_sync(0xFFFFFFFFu, xm, o);
        if (lane >= o) {
          x = rep_compose(prev, x);
          xl += pl;
          xm += pm;
        }
      }
      // exclusive: carry-in of warp `lane` = C composed with warps 0..lane-1
      RepSlots e;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        e.k[q] = __shfl_up_sync(0xFFFFFFFFu, x.k[q], 1);
        e.d[q] = __shfl_up_sync(0xFFFFFFFFu, x.d[q], 1);
        if (lane == 0) {
          e.k[q] = uint32_t(q);
          e.d[q] = 0;
        }
      }
      uint32_t el = __shfl_up_sync(0xFFFFFFFFu, xl, 1), em = __shfl_up_sync(0xFFFFFFFFu, xm, 1);
      if (lane == 0) el = em = 0;
      const RepSlots cin = rep_compose(C, e);
      if (lane < kW) {
#pragma unroll
        for (int q = 0; q < 3; q++) {
          s_ck[lane][q] = cin.k[q];
          s_cd[lane][q] = cin.d[q];
        }
        s_cl[lane] = cll + el;
        s_cm[lane] = cml + em;
      }
      if (lane == kW - 1) {
        const RepSlots tot = rep_compose(C, x);
#pragma unroll
        for (int q = 0; q < 3; q++) {
          s_ck[kW][q] = tot.k[q];
          s_cd[kW][q] = tot.d[q];
        }
        s_cl[kW] = cll + xl;
        s_cm[kW] = cml + xm;
      }
    }
    __syncthreads();
    RepSlots cw, all;
#pragma unroll
    for (int q = 0; q < 3; q++) {
      cw.k[q] = s_ck[warp][q];
      cw.d[q] = s_cd[warp][q];
      all.k[q] = s_ck[kW][q];
      all.d[q] = s_cd[kW][q];
    }
    const uint32_t wll = s_cl[warp], wml = s_cm[warp];
    const uint32_t tll = s_cl[kW], tml = s_cm[kW];
    __syncthreads();  // the shared totals are rewritten next round
    // exclusive within the warp: the lanes below this one
    RepSlots ex;
#pragma unroll
    for (int q = 0; q < 3; q++) {
      ex.k[q] = __shfl_up_sync(0xFFFFFFFFu, incl.k[q], 1);
      ex.d[q] = __shfl_up_sync(0xFFFFFFFFu, incl.d[q], 1);
      if (lane == 0) {
        ex.k[q] = uint32_t(q);
        ex.d[q] = 0;
      }
    }
    uint32_t ell = __shfl_up_sync(0xFFFFFFFFu, ill, 1), eml = __shfl_up_sync(0xFFFFFFFFu, iml, 1);
    if (lane == 0) ell = eml = 0;
    // replay this thread's records on the slots in force before its first
    RepSlots cur = rep_compose(cw, ex);
    uint32_t lit = wll + ell, dst = lit + wml + eml;
#pragma unroll
    for (int r = 0; r < kSeqPerThread; r++) {
      if (i0 + r < n) {
        uint32_t ok, ov;
        rep_step(cur, ofv[r], ll[r], ok, ov);
        // records are 24 bytes: (oval, okind) and (dst, lit) are 8-byte aligned pairs
        *reinterpret_cast<uint2*>(&seq[i0 + r].oval) = make_uint2(ov, ok);
        *reinterpret_cast<uint2*>(&seq[i0 + r].dst) = make_uint2(dst, lit);
      }
      lit += ll[r];
      dst += ll[r] + ml[r];
    }
    C = all;
    cll = tll;
    cml = tml;
  }
  if (tid == 0) {
    uint32_t st = 0;
    if (cll > b.lit_regen) st |= VOOM_ZSTD_ST_SEQUENCES;
    const uint32_t out_size = b.lit_regen + cml;
    if (out_size > b.max_out) st |= VOOM_ZSTD_ST_SIZE;
    rt->out_size = out_size;
    rt->status = st;
    for (int k = 0; k < 3; k++) {
      rt->rep_kind[k] = C.k[k];
      rt->rep_val[k] = C.d[k];
    }
  }
}

// K2, one warp per job: the blocks of each frame 32 at a time -- a warp scan
// of their output sizes gives every block's Z position, and a scan of their
// symbolic repeat-offset transforms (composed in block order) applied to the
// repeat offsets at the start of the chunk gives every block's initial repeat
// offsets; the chunk's totals carry into the next 32.
constexpr int kJobScanWarps = 4;

__device__ __forceinline__ uint32_t rep_apply(const RepSlots& t, const uint32_t (&in)[3], int q) {
  const uint32_t src = t.k[q] == 0 ? in[0] : (t.k[q] == 1 ? in[1] : in[2]);
  return t.k[q] == 3 ? t.d[q] : src - t.d[q];
}

__global__ void __launch_bounds__(32 * kJobScanWarps) zstd_job_scan(const uint8_t* img, uint8_t* scratch,
                                                                     uint32_t* status, uint32_t job0,
                                                                     uint32_t n_jobs) {
  const View v = make_view(img, scratch);
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t jr = blockIdx.x * kJobScanWarps + (threadIdx.x >> 5);
  if (jr >= n_jobs) return;
  const uint32_t j = job0 + jr;
  const ZJob job = v.jobs[j];
  // direct jobs: sizes were checked by the planner, literal faults are
  // reported by the literal decoders themselves
  if (job.bad || job.direct) return;
  uint64_t z = job.zoff;
  uint32_t st = 0;
  for (uint32_t f = job.frame_first; f < job.frame_first + job.n_frames; f++) {
    const ZFrame fr = v.frames[f];
    uint32_t rep[3] = {1, 4, 8};
    const uint64_t fz = z;
    for (uint32_t c = 0; c < fr.n_blocks; c += 32) {
      const uint32_t bi = fr.block_first + c + lane;
      const bool on = c + lane < fr.n_blocks;
      uint32_t size = 0;
      RepSlots T;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        T.k[q] = uint32_t(q);
        T.d[q] = 0;
      }
      if (on) {
        const ZBlockRt& rt = v.rt[bi];
        size = rt.out_size;
        st |= rt.status;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          T.k[q] = rt.rep_kind[q];
          T.d[q] = rt.rep_val[q];
        }
      }
      // inclusive scans of sizes and transforms over the lanes
      uint64_t incl = size;
      RepSlots X = T;
      for (int o = 1; o < 32; o <<= 1) {
        const uint64_t ps = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        RepSlots prev;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          prev.k[q] = __shfl_up_sync(0xFFFFFFFFu, X.k[q], o);
          prev.d[q] = __shfl_up_sync(0xFFFFFFFFu, X.d[q], o);
        }
        if (lane >= uint32_t(o)) {
          incl += ps;
          X = rep_compose(prev, X);
        }
      }
      // exclusive: the transform of the lanes below this one
      RepSlots E;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        E.k[q] = __shfl_up_sync(0xFFFFFFFFu, X.k[q], 1);
        E.d[q] = __shfl_up_sync(0xFFFFFFFFu, X.d[q], 1);
        if (lane == 0) {
          E.k[q] = uint32_t(q);
          E.d[q] = 0;
        }
      }
      if (on) {
        ZBlockRt* rt = v.rt + bi;
        rt->zstart = z + incl - size;
        rt->frame_zstart = fz;
#pragma unroll
        for (int q = 0; q < 3; q++) rt->init_rep[q] = rep_apply(E, rep, q);
      }
      // carry: the chunk's total size and composed transform (lane 31)
      z += __shfl_sync(0xFFFFFFFFu, incl, 31);
      RepSlots A;
#pragma unroll
      for (int q = 0; q < 3; q++) {
        A.k[q] = __shfl_sync(0xFFFFFFFFu, X.k[q], 31);
        A.d[q] = __shfl_sync(0xFFFFFFFFu, X.d[q], 31);
      }
      uint32_t nr[3];
#pragma unroll
      for (int q = 0; q < 3; q++) nr[q] = rep_apply(A, rep, q);
#pragma unroll
      for (int q = 0; q < 3; q++) rep[q] = nr[q];
    }
    if (fr.fcs != ~0ull && z - fz != fr.fcs) st |= VOOM_ZSTD_ST_SIZE;
  }
  for (int o = 16; o; o >>= 1) st |= __shfl_xor_sync(0xFFFFFFFFu, st, o);
  if (z - job.zoff != job.dst_len) st |= VOOM_ZSTD_ST_SIZE;
  if (st && lane == 0) atomicOr(status + j, st);
}

// Output chunk of K3: its entries are built in shared memory, then written out
// with coalesced stores (a sequence's bytes are contiguous, but a warp's
// sequences are not).
constexpr uint32_t kExecChunk = 4096;
constexpr uint32_t kExecMaxChunks = (128 * 1024) / kExecChunk + 1;

constexpr uint32_t kLongLit = 64;  // literal runs longer than this are copied by the whole CTA

__global__ void __launch_bounds__(256) zstd_block_execute(const uint8_t* __restrict__ src, const uint8_t* img,
                                                          uint8_t* scratch, uint8_t* __restrict__ out,
                                                          uint32_t* status, uint32_t bl0) {
  __shared__ uint32_t s_out[kExecChunk];
  __shared__ uint32_t s_first[kExecMaxChunks];
  __shared__ uint3 s_long[kExecChunk / (kLongLit + 1) + 1];  // (first, end, literal position) per long run
  __shared__ uint32_t s_nlong;
  const View v = make_view(img, scratch);
  const uint32_t bi = reinterpret_cast<const uint32_t*>(img + v.h->off_blist)[bl0 + blockIdx.x];
  const ZBlock b = v.blocks[bi];
  const ZJob& job = v.jobs[b.job];
  if (job.bad) return;
  if (job.direct) {  // raw / RLE bytes straight to the output; literals were written by K1
    uint8_t* d = out + job.dst + b.out_off;
    if (b.type == 0) {
      for (uint32_t i = threadIdx.x; i < b.size; i += blockDim.x) d[i] = __ldg(src + b.src + i);
    } else if (b.type == 1) {
      const uint8_t c = __ldg(src + b.src);
      for (uint32_t i = threadIdx.x; i < b.size; i += blockDim.x) d[i] = c;
    }
    return;
  }
  const ZBlockRt rt = v.rt[bi];
  // A job's Z-space holds exactly dst_len words.  Blocks whose decoded sizes
  // add up to more (no content size, a damaged stream, a wrong dst_len) were
  // flagged by the job scan; none of their bytes may be written, or they
  // would land in the next job's words or past the scratch.
  if ((status[b.job] & VOOM_ZSTD_ST_SIZE) || rt.zstart < job.zoff ||
      rt.zstart + rt.out_size > job.zoff + job.dst_len)
    return;
  uint32_t* res = v.res + rt.zstart;
  if (b.type == 0) {
    for (uint32_t i = threadIdx.x; i < b.size; i += blockDim.x) res[i] = kResolved | __ldg(src + b.src + i);
    return;
  }
  if (b.type == 1) {
    const uint32_t c = kResolved | __ldg(src + b.src);
    for (uint32_t i = threadIdx.x; i < b.size; i += blockDim.x) res[i] = c;
    return;
  }
  if (rt.status) return;  // the job already failed in K1 / K1b
  const ZSeq* seq = v.seq + b.seq_off;
  const uint8_t* lit = v.lit + b.lit_off;
  const uint64_t before = rt.zstart - rt.frame_zstart;
  const uint32_t n = b.nseq, out_size = rt.out_size;
  if (out_size > b.max_out) return;  // reported by K1b
  const uint32_t nchunks = (out_size + kExecChunk - 1) / kExecChunk;
  // the literal tail after the last sequence is record n
  uint32_t tail_dst = 0, tail_lit = 0;
  if (n) {
    const ZSeq last = seq[n - 1];
    tail_dst = last.dst + last.ll + last.ml;
    tail_lit = last.lit + last.ll;
  }
  // s_first[c] = the record holding chunk c's first byte
  for (uint32_t c = threadIdx.x; c < nchunks; c += blockDim.x) s_first[c] = n;
  if (threadIdx.x == 0) s_nlong = 0;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const ZSeq s = seq[i];
    const uint32_t len = s.ll + s.ml;
    for (uint32_t c = (s.dst + kExecChunk - 1) / kExecChunk; c * kExecChunk < s.dst + len && c < nchunks; c++)
      s_first[c] = i;
  }
  __syncthreads();
  uint32_t bad = 0;
  for (uint32_t c = 0; c < nchunks; c++) {
    const uint32_t c0 = c * kExecChunk, c1 = min(out_size, c0 + kExecChunk);
    for (uint32_t i = s_first[c] + threadIdx.x; i <= n; i += blockDim.x) {
      uint32_t dst, ll, ml, lp, off = 0;
      bool ok = true;
      if (i < n) {
        const ZSeq s = seq[i];
        dst = s.dst;
        ll = s.ll;
        ml = s.ml;
        lp = s.lit;
        const uint32_t rep = s.okind == 0 ? rt.init_rep[0] : (s.okind == 1 ? rt.init_rep[1] : rt.init_rep[2]);
        off = s.okind == 3 ? s.oval : rep - s.oval;
        ok = off != 0 && uint64_t(off) <= before + dst + ll;
      } else {
        dst = tail_dst;
        ll = b.lit_regen - tail_lit;
        ml = 0;
        lp = tail_lit;
      }
      if (dst >= c1) break;  // records are in output order
      bad |= !ok;
      const uint32_t a0 = max(dst, c0), a1 = min(dst + ll, c1);
      if (a1 > a0 + kLongLit) {  // a long run: queued for the CTA-wide copy below
        s_long[atomicAdd(&s_nlong, 1u)] = make_uint3(a0, a1, lp + (a0 - dst));
      } else {  // literal bytes, 8 loads in flight at a time (read-only global loads)
        uint32_t p = a0;
        for (; p + 8 <= a1; p += 8) {
          const uint8_t* q = lit + lp + (p - dst);
          uint32_t bv[8];
#pragma unroll
          for (int k = 0; k < 8; k++) bv[k] = __ldg(q + k);
#pragma unroll
          for (int k = 0; k < 8; k++) s_out[p - c0 + k] = kResolved | bv[k];
        }
        for (; p < a1; p++) s_out[p - c0] = kResolved | __ldg(lit + lp + (p - dst));
      }
      const uint64_t m = rt.zstart + dst + ll;
      const uint32_t b0 = max(dst + ll, c0), b1 = min(dst + ll + ml, c1);
      {  // match bytes: a link to the source, or -- when the source lies in an
         // earlier chunk of this block, whose words this CTA wrote before the
         // last barrier -- that word itself (its byte, or its own link: one hop
         // of the output pass's chase done here); 8 loads in flight at a time
        uint32_t p = b0;
        for (; p + 8 <= b1; p += 8) {
          uint32_t vv[8];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint32_t q = p + k;
            vv[k] = ok ? uint32_t(m + (q - dst - ll) - off) : kResolved;
            if (ok && off <= q && q - off < c0) vv[k] = res[q - off];
          }
#pragma unroll
          for (int k = 0; k < 8; k++) s_out[p - c0 + k] = vv[k];
        }
        for (; p < b1; p++) {
          uint32_t val = ok ? uint32_t(m + (p - dst - ll) - off) : kResolved;
          if (ok && off <= p && p - off < c0) val = res[p - off];
          s_out[p - c0] = val;
        }
      }
    }
    __syncthreads();
    const uint32_t nlong = s_nlong;
    for (uint32_t r = 0; r < nlong; r++) {  // long literal runs, coalesced over the CTA
      const uint3 L = s_long[r];
      for (uint32_t p = L.x + threadIdx.x; p < L.y; p += blockDim.x)
        s_out[p - c0] = kResolved | __ldg(lit + L.z + (p - L.x));
    }
    __syncthreads();
    if (threadIdx.x == 0) s_nlong = 0;
    for (uint32_t p = c0 + threadIdx.x; p < c1; p += blockDim.x) res[p] = s_out[p - c0];
    __syncthreads();
  }
  if (bad) atomicOr(status + b.job, VOOM_ZSTD_ST_OFFSET);
}

// Match links left by block execution are resolved in three steps.
//  zstd_output (one CTA per output tile) streams the tile's link words, follows
//    each unresolved byte's links up to kHops times (the links of 8
//    neighbouring bytes in lockstep, so their loads are in flight together),
//    stores what it reached back (path compression: chains through the byte
//    stop there) and writes every resolved byte to the output, interleaved
//    with the lo plane.  A byte still unresolved goes on worklist 0; its
//    output byte is written later.
//  zstd_resolve passes 1 .. kResolvePasses-1 follow the links of the worklist
//    entries (list p-1 in, list p out; lists 1 and 2 alternate).
//  zstd_patch writes the output byte of every worklist-0 entry, or flags the
//    job when its chain is still unresolved.
// If worklist 0 overflows, the passes rescan the tiles that had unresolved
// bytes and zstd_patch rewrites those tiles whole.  Later lists cannot
// overflow: a pass pushes at most one entry per entry it reads.
// Counters after the tile flags: [0] worklist-0 overflow, [1 + p] entries
// pushed by pass p.  A tile flag holds kPatch | unresolved count.
static_assert(kResolvePasses > 1, "at least one list pass");
constexpr uint32_t kPatch = 0x80000000u;

__device__ __forceinline__ uint2* list_at(const View& v, int pass) {
  return v.list + uint64_t(pass == 0 ? 0 : 1 + ((pass - 1) & 1)) * v.h->list_cap;
}

__device__ __forceinline__ void list_push(const View& v, uint32_t* ctr, int pass, uint32_t z, uint32_t tile) {
  const uint32_t i = atomicAdd(&ctr[1 + pass], 1u);
  if (i < v.h->list_cap) list_at(v, pass)[i] = make_uint2(z, tile);
  else atomicOr(&ctr[0], 1u);
}

// Follows up to kHops copy links from u; returns the last value reached.
__device__ __forceinline__ uint32_t chase(const View& v, uint32_t u, uint64_t zmax) {
  for (int h = 0; h < kHops && !(u & kResolved); h++) {
    if (u >= zmax) return kResolved;  // out-of-range link (only from a damaged stream)
    u = v.res[u];
  }
  return u;
}

// chase() of 8 links in lockstep rounds: the loads of one round are
// independent, so up to 8 are in flight per thread.
__device__ __forceinline__ void chase8(const View& v, uint32_t (&u)[8], uint64_t zmax) {
  for (int h = 0; h < kHops; h++) {
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (!(u[i] & kResolved)) u[i] = u[i] < zmax ? v.res[u[i]] : kResolved;
    if (u[0] & u[1] & u[2] & u[3] & u[4] & u[5] & u[6] & u[7] & kResolved) return;
  }
}

// Output bytes of job bytes k .. k+7 (hi0 = bytes 0-3, hi1 = bytes 4-7):
// interleaved with the body's lo plane (vpack) or stored as they are.
__device__ __forceinline__ void emit8(const ZJob& job, const uint8_t* __restrict__ src, uint8_t* __restrict__ out,
                                      uint64_t k, uint32_t hi0, uint32_t hi1) {
  if (job.flags & VOOM_ZSTD_INTERLEAVE) {
    const uint64_t lo = load8(src + job.lo_src + k);
    const uint32_t lo0 = uint32_t(lo), lo1 = uint32_t(lo >> 32);
    uint4 o;
    o.x = __byte_perm(lo0, hi0, 0x5140);
    o.y = __byte_perm(lo0, hi0, 0x7362);
    o.z = __byte_perm(lo1, hi1, 0x5140);
    o.w = __byte_perm(lo1, hi1, 0x7362);
    uint8_t* d = out + job.dst + 2 * k;
    if ((job.dst & 15u) == 0) {
      *reinterpret_cast<uint4*>(d) = o;
    } else {
      const uint32_t wv[4] = {o.x, o.y, o.z, o.w};
      for (int i = 0; i < 16; i++) d[i] = uint8_t(wv[i >> 2] >> (8 * (i & 3)));
    }
  } else {
    uint8_t* d = out + job.dst + k;
    if ((reinterpret_cast<uintptr_t>(d) & 7u) == 0) {
      *reinterpret_cast<uint2*>(d) = make_uint2(hi0, hi1);
    } else {
      for (int i = 0; i < 8; i++) d[i] = uint8_t((i < 4 ? hi0 : hi1) >> (8 * (i & 3)));
    }
  }
}

__device__ __forceinline__ void emit1(const ZJob& job, const uint8_t* __restrict__ src, uint8_t* __restrict__ out,
                                      uint64_t k, uint8_t hb, bool lo_too) {
  if (job.flags & VOOM_ZSTD_INTERLEAVE) {
    if (lo_too) out[job.dst + 2 * k] = __ldg(src + job.lo_src + k);
    out[job.dst + 2 * k + 1] = hb;
  } else {
    out[job.dst + k] = hb;
  }
}

__device__ __forceinline__ uint32_t low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

__global__ void __launch_bounds__(256) zstd_output(const uint8_t* __restrict__ src, const uint8_t* img,
                                                   uint8_t* scratch, uint8_t* __restrict__ out, uint32_t tile0) {
  __shared__ uint32_t s_unres;
  const View v = make_view(img, scratch);
  const uint32_t ti = tile0 + blockIdx.x;
  const ZOutTile t = v.tiles[ti];
  const ZJob job = v.jobs[t.job];
  if (job.bad) return;
  if (threadIdx.x == 0) s_unres = 0;
  __syncthreads();
  uint32_t* ctr = v.dirty + v.h->n_tiles;
  const uint64_t zmax = v.h->zbytes;
  const uint64_t end = t.begin + t.len;
  uint32_t unres = 0;
  // The tile is walked in block-wide steps of 8 bytes per thread (no barrier
  // between steps: links into the block's own earlier chunks were already
  // followed once by the block execute pass).  Each thread loads its next
  // link words before chasing the current ones; only the owning thread ever
  // writes a position here, so the early load is exact.
  const uint32_t step = 8u * blockDim.x;
  uint4 n0 = make_uint4(0, 0, 0, 0), n1 = n0;
  if (t.begin + 8u * threadIdx.x + 8 <= end) {
    n0 = *reinterpret_cast<const uint4*>(v.res + job.zoff + t.begin + 8u * threadIdx.x);
    n1 = *reinterpret_cast<const uint4*>(v.res + job.zoff + t.begin + 8u * threadIdx.x + 4);
  }
  for (uint64_t base = t.begin; base < end; base += step) {
    const uint64_t k = base + 8u * threadIdx.x;
    const uint64_t z = job.zoff + k;
    const uint4 r0 = n0, r1 = n1;
    if (k + step + 8 <= end) {
      n0 = *reinterpret_cast<const uint4*>(v.res + z + step);
      n1 = *reinterpret_cast<const uint4*>(v.res + z + step + 4);
    }
    if (k + 8 <= end) {
      uint32_t u[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
      if (!(u[0] & u[1] & u[2] & u[3] & u[4] & u[5] & u[6] & u[7] & kResolved)) {
        chase8(v, u, zmax);
        // path compression: later chains through these bytes stop here
        *reinterpret_cast<uint4*>(v.res + z) = make_uint4(u[0], u[1], u[2], u[3]);
        *reinterpret_cast<uint4*>(v.res + z + 4) = make_uint4(u[4], u[5], u[6], u[7]);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          if (!(u[i] & kResolved)) {
            unres++;
            list_push(v, ctr, 0, uint32_t(z + i), ti);
          }
        }
      }
      emit8(job, src, out, k, low_bytes(u[0], u[1], u[2], u[3]), low_bytes(u[4], u[5], u[6], u[7]));
    } else if (k < end) {
      for (uint32_t i = 0; i < uint32_t(end - k); i++) {
        uint32_t u = v.res[z + i];
        if (!(u & kResolved)) {
          u = chase(v, u, zmax);
          v.res[z + i] = u;
          if (!(u & kResolved)) {
            unres++;
            list_push(v, ctr, 0, uint32_t(z + i), ti);
          }
        }
        emit1(job, src, out, k + i, uint8_t(u), true);
      }
    }
  }
  if (unres) atomicAdd(&s_unres, unres);
  __syncthreads();
  if (threadIdx.x == 0) v.dirty[ti] = s_unres ? (kPatch | s_unres) : 0u;
}

// One resolve pass.  Grid-stride over the worklist, or (worklist 0
// overflowed) over the segment's tiles: a few CTAs per SM, so a pass over an
// empty list costs one small launch.
__global__ void __launch_bounds__(256) zstd_resolve(const uint8_t* img, uint8_t* scratch, int pass,
                                                    uint32_t tile0, uint32_t n_tiles) {
  __shared__ uint32_t s_unres;
  const View v = make_view(img, scratch);
  uint32_t* ctr = v.dirty + v.h->n_tiles;
  const uint64_t zmax = v.h->zbytes;
  if (!*reinterpret_cast<volatile uint32_t*>(&ctr[0])) {
    const uint64_t left = ctr[pass], cap = v.h->list_cap;  // pushed by pass - 1
    const uint64_t n_in = left < cap ? left : cap;
    const uint2* in = list_at(v, pass - 1);
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n_in;
         e += uint64_t(gridDim.x) * blockDim.x) {
      const uint2 ent = in[e];
      if (ent.x >= zmax || ent.y >= v.h->n_tiles) continue;
      const uint32_t u = chase(v, v.res[ent.x], zmax);
      v.res[ent.x] = u;
      if (!(u & kResolved) && pass + 1 < kResolvePasses) list_push(v, ctr, pass, ent.x, ent.y);
    }
    return;
  }
  for (uint32_t ti = tile0 + blockIdx.x; ti < tile0 + n_tiles; ti += gridDim.x) {
    const ZOutTile t = v.tiles[ti];
    const ZJob job = v.jobs[t.job];
    if (job.bad || !(v.dirty[ti] & ~kPatch)) continue;  // the same for every thread
    if (threadIdx.x == 0) s_unres = 0;
    __syncthreads();
    uint32_t unres = 0;
    for (uint64_t k = t.begin + threadIdx.x; k < t.begin + t.len; k += blockDim.x) {
      const uint64_t z = job.zoff + k;
      uint32_t u = v.res[z];
      if (u & kResolved) continue;
      u = chase(v, u, zmax);
      v.res[z] = u;
      unres += !(u & kResolved);
    }
    if (unres) atomicAdd(&s_unres, unres);
    __syncthreads();
    if (threadIdx.x == 0) v.dirty[ti] = kPatch | s_unres;
    __syncthreads();  // s_unres is reused for the next tile
  }
}

__global__ void __launch_bounds__(256) zstd_patch(const uint8_t* __restrict__ src, const uint8_t* img,
                                                  uint8_t* scratch, uint8_t* __restrict__ out, uint32_t* status,
                                                  uint32_t tile0) {
  const View v = make_view(img, scratch);
  uint32_t* ctr = v.dirty + v.h->n_tiles;
  const uint64_t zmax = v.h->zbytes;
  if (!*reinterpret_cast<volatile uint32_t*>(&ctr[0])) {
    const uint64_t left = ctr[1], cap = v.h->list_cap;
    const uint64_t n_in = left < cap ? left : cap;
    const uint2* in = list_at(v, 0);
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n_in;
         e += uint64_t(gridDim.x) * blockDim.x) {
      const uint2 ent = in[e];
      if (ent.x >= zmax || ent.y >= v.h->n_tiles) continue;
      const uint32_t j = v.tiles[ent.y].job;
      const uint32_t u = v.res[ent.x];
      if (!(u & kResolved)) {
        atomicOr(status + j, VOOM_ZSTD_ST_UNRESOLVED);
        continue;
      }
      const ZJob& job = v.jobs[j];
      emit1(job, src, out, ent.x - job.zoff, uint8_t(u), false);
    }
    return;
  }
  const uint32_t ti = tile0 + blockIdx.x;
  const ZOutTile t = v.tiles[ti];
  const ZJob job = v.jobs[t.job];
  if (job.bad || !(v.dirty[ti] & kPatch)) return;
  if (v.dirty[ti] & ~kPatch) {
    if (threadIdx.x == 0) atomicOr(status + t.job, VOOM_ZSTD_ST_UNRESOLVED);
    return;
  }
  const uint64_t end = t.begin + t.len;
  for (uint64_t k = t.begin + 8u * threadIdx.x; k < end; k += 8u * blockDim.x) {
    const uint64_t z = job.zoff + k;
    const uint32_t cnt = uint32_t((end - k) < 8 ? (end - k) : 8);
    if (cnt == 8) {
      const uint4 r0 = *reinterpret_cast<const uint4*>(v.res + z);
      const uint4 r1 = *reinterpret_cast<const uint4*>(v.res + z + 4);
      emit8(job, src, out, k, low_bytes(r0.x, r0.y, r0.z, r0.w), low_bytes(r1.x, r1.y, r1.z, r1.w));
    } else {
      for (uint32_t i = 0; i < cnt; i++) emit1(job, src, out, k + i, uint8_t(v.res[z + i]), true);
    }
  }
}

// XXH64 (xxHash specification) of a frame's decoded bytes, one thread per frame.
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

// The bytes are read back from the output (hi bytes of an interleaved body).
__global__ void zstd_checksum(const uint8_t* img, uint8_t* scratch, const uint8_t* __restrict__ out,
                              uint32_t* status) {
  const View v = make_view(img, scratch);
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= v.h->n_frames) return;
  const ZFrame fr = v.frames[f];
  const ZJob& job = v.jobs[fr.job];
  if (!fr.csum_flag || job.bad || status[fr.job]) return;
  const uint64_t P1 = 0x9E3779B185EBCA87ull, P2 = 0xC2B2AE3D27D4EB4Full, P3 = 0x165667B19E3779F9ull,
                 P4 = 0x85EBCA77C2B2AE63ull, P5 = 0x27D4EB2F165667C5ull;
  uint64_t z0 = 0, n = 0;
  if (fr.n_blocks) {
    const ZBlockRt& a = v.rt[fr.block_first];
    const ZBlockRt& l = v.rt[fr.block_first + fr.n_blocks - 1];
    z0 = a.zstart;
    n = l.zstart + l.out_size - z0;
  }
  if (z0 < job.zoff || z0 + n > job.zoff + job.dst_len) {  // never read past the job's output
    atomicOr(status + fr.job, VOOM_ZSTD_ST_SIZE);
    return;
  }
  const bool inter = job.flags & VOOM_ZSTD_INTERLEAVE;
  const uint8_t* r = out + job.dst + (inter ? 2 * (z0 - job.zoff) + 1 : z0 - job.zoff);
  const uint32_t stride = inter ? 2u : 1u;
  auto byte = [&](uint64_t i) { return uint64_t(r[stride * i]); };
  auto rd = [&](uint64_t i, int nb) {
    uint64_t x = 0;
    for (int k = 0; k < nb; k++) x |= byte(i + k) << (8 * k);
    return x;
  };
  auto round = [&](uint64_t acc, uint64_t in) { return rotl64(acc + in * P2, 31) * P1; };
  uint64_t h, i = 0;
  if (n >= 32) {
    uint64_t v1 = P1 + P2, v2 = P2, v3 = 0, v4 = 0 - P1;
    for (; i + 32 <= n; i += 32) {
      v1 = round(v1, rd(i, 8));
      v2 = round(v2, rd(i + 8, 8));
      v3 = round(v3, rd(i + 16, 8));
      v4 = round(v4, rd(i + 24, 8));
    }
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = (h ^ round(0, v1)) * P1 + P4;
    h = (h ^ round(0, v2)) * P1 + P4;
    h = (h ^ round(0, v3)) * P1 + P4;
    h = (h ^ round(0, v4)) * P1 + P4;
  } else {
    h = P5;
  }
  h += n;
  for (; i + 8 <= n; i += 8) {
    h ^= round(0, rd(i, 8));
    h = rotl64(h, 27) * P1 + P4;
  }
  if (i + 4 <= n) {
    h ^= rd(i, 4) * P1;
    h = rotl64(h, 23) * P2 + P3;
    i += 4;
  }
  for (; i < n; i++) {
    h ^= byte(i) * P5;
    h = rotl64(h, 11) * P1;
  }
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  if (uint32_t(h) != fr.csum) atomicOr(status + fr.job, VOOM_ZSTD_ST_CHECKSUM);
}

}  // namespace

// Host side: counts come from the host plan handle (zstd_plan.cpp).
namespace voom {
namespace zstd {
bool plan_counts(const void* plan, ZPlanHeader* out, std::vector<ZSegment>* segs);
}
}  // namespace voom

// Optional per-kernel timing of voom_zstd_decode (diagnostics): when on, an
// event is recorded on the launch stream after every launch, with the id of
// the kernel it closes; voom_zstd_kernel_times returns the intervals of the
// last decode.  Events belong to the device current when timing was enabled.
namespace {
constexpr int kMaxTimed = 96;
bool g_time_on = false;
int g_time_dev = -1;  // device the events were created on
cudaEvent_t g_tev[kMaxTimed + 1];
uint32_t g_tid[kMaxTimed];
int g_ntev = 0;
// Timing applies to decodes on the device the events belong to; a decode on
// any other device records nothing.
bool timing_here() {
  if (!g_time_on) return false;
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess && dev == g_time_dev;
}
void tmark(cudaStream_t s, uint32_t id) {
  if (g_ntev > kMaxTimed || !timing_here()) return;
  if (g_ntev > 0) g_tid[g_ntev - 1] = id;
  cudaEventRecord(g_tev[g_ntev++], s);
}
// First-wave size of zstd_block_decode: 4 one-warp CTAs per SM of the current
// device (one per scheduler), at most the block count.
uint32_t k1_wave(uint32_t n_bl) {
  static int sms[64] = {0};
  int dev = 0;
  int n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms[dev] = 0;
    if (sms[dev] > 0) n = sms[dev];
  }
  return std::min<uint32_t>(n_bl, 4u * uint32_t(n));
}

// The literal decode (K0) runs on a side stream beside the sequence walk
// (K1): the walks are one warp per block and bound by their serial chains, so
// K0's CTAs use the SMs' spare issue slots instead of adding their time.  One
// side stream and a fork / join event pair per device, made on first use; the
// enqueue sequence holds a lock so that concurrent callers' events do not mix.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool tried = false, ok = false;
};
SideStream g_side[64];
std::mutex g_side_mu;

SideStream* side_stream_locked() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStream& ss = g_side[dev];
  if (!ss.tried) {
    ss.tried = true;
    ss.ok = cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) == cudaSuccess;
  }
  return ss.ok ? &ss : nullptr;
}
}  // namespace

// n bytes from device-mapped pinned host memory into device memory, read by
// the SMs: unlike cudaMemcpyAsync it does not queue on a copy engine behind
// earlier transfers (a small plan image would otherwise wait for every body
// upload enqueued before it).
__global__ void __launch_bounds__(256) zstd_copy_mapped(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                                        uint64_t n) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0) {
    const uint64_t n16 = n / 16;
    for (uint64_t i = t; i < n16; i += stride)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    for (uint64_t i = n16 * 16 + t; i < n; i += stride) dst[i] = src[i];
  } else {
    for (uint64_t i = t; i < n; i += stride) dst[i] = src[i];
  }
}

VOOM_API int voom_copy_from_host(void* d_dst, const void* h_src, uint64_t n, void* stream) {
  if (!n) return VOOM_OK;
  if (!d_dst || !h_src) return VOOM_E_INVALID_ARG;
  // the whole range must lie in one pinned allocation mapped into this device
  cudaPointerAttributes a{};
  void* d_src = nullptr;
  if (cudaPointerGetAttributes(&a, h_src) != cudaSuccess || a.type != cudaMemoryTypeHost ||
      cudaHostGetDevicePointer(&d_src, const_cast<void*>(h_src), 0) != cudaSuccess || !d_src) {
    cudaGetLastError();  // clear the lookup's error: the caller falls back to a plain copy
    return VOOM_E_INVALID_ARG;
  }
  void* d_last = nullptr;
  if (cudaHostGetDevicePointer(&d_last, static_cast<uint8_t*>(const_cast<void*>(h_src)) + (n - 1), 0) != cudaSuccess ||
      static_cast<uint8_t*>(d_last) != static_cast<uint8_t*>(d_src) + (n - 1)) {
    cudaGetLastError();
    return VOOM_E_INVALID_ARG;
  }
  const uint64_t blocks = std::min<uint64_t>((n + 16 * 256 - 1) / (16 * 256), 148 * 2);
  zstd_copy_mapped<<<uint32_t(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(d_dst), static_cast<const uint8_t*>(d_src), n);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API int voom_zstd_set_timing(int on) {
  if (on && !g_time_on) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return VOOM_E_CUDA;
    for (int i = 0; i <= kMaxTimed; i++) {
      if (cudaEventCreate(&g_tev[i]) != cudaSuccess) {
        for (int q = 0; q < i; q++) cudaEventDestroy(g_tev[q]);  // nothing stays half made
        return VOOM_E_CUDA;
      }
    }
    g_time_dev = dev;
  } else if (!on && g_time_on) {
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(g_time_dev);
    cudaDeviceSynchronize();
    for (int i = 0; i <= kMaxTimed; i++) cudaEventDestroy(g_tev[i]);
    if (cur >= 0) cudaSetDevice(cur);
    g_time_dev = -1;
  }
  g_time_on = on != 0;
  g_ntev = 0;
  return VOOM_OK;
}

VOOM_API int voom_zstd_kernel_times(float* ms, uint32_t* ids, int cap) {
  if (!g_time_on || g_ntev < 2) return 0;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != g_time_dev) return 0;
  if (cudaEventSynchronize(g_tev[g_ntev - 1]) != cudaSuccess) return VOOM_E_CUDA;
  int n = 0;
  for (int i = 1; i < g_ntev && n < cap; i++, n++) {
    if (cudaEventElapsedTime(&ms[n], g_tev[i - 1], g_tev[i]) != cudaSuccess) return VOOM_E_CUDA;
    ids[n] = g_tid[i - 1];
  }
  return n;
}

VOOM_API int voom_zstd_decode(const uint8_t* d_src, const void* d_plan, const void* h_plan, void* d_scratch,
                              uint8_t* d_out, uint32_t* d_status, void* stream) {
  if (!d_src || !d_plan || !h_plan || !d_scratch || !d_out || !d_status) return VOOM_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(d_src) & 15u) return VOOM_E_INVALID_ARG;  // streams are read in 16-byte chunks
  ZPlanHeader h;
  std::vector<ZSegment> segs;
  if (!voom::zstd::plan_counts(h_plan, &h, &segs)) return VOOM_E_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* img = static_cast<const uint8_t*>(d_plan);
  uint8_t* scr = static_cast<uint8_t*>(d_scratch);
  if (timing_here()) g_ntev = 0;
  tmark(s, 0);
  if (h.n_dlit) {
    zstd_direct_literals<<<(h.n_dlit + kDlBlocksPerWarp - 1) / kDlBlocksPerWarp, 32, 0, s>>>(d_src, img, scr,
                                                                                            d_out, d_status);
    tmark(s, VOOM_ZSTD_K_DIRECT_LITERALS);
  }
  // One pass of the pipeline per Z-space segment; the link-word scratch and
  // the resolve worklists are reused, everything else is indexed globally.
  for (const ZSegment& g : segs) {
    // resolve worklist counters (after the tile flags)
    if (cudaMemsetAsync(scr + h.s_ctr + 4ull * h.n_tiles, 0, 32, s) != cudaSuccess) return VOOM_E_CUDA;
    if (g.n_bl) {
      {
        std::lock_guard<std::mutex> lock(g_side_mu);
        SideStream* ss = side_stream_locked();
        if (ss) {  // K1 on the caller's stream (dispatched first), K0 beside it
          if (cudaEventRecord(ss->fork, s) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess)
            return VOOM_E_CUDA;
          zstd_block_decode<<<g.n_bl, 32, 0, s>>>(d_src, img, scr, g.bl0, g.n_bl, k1_wave(g.n_bl));
          zstd_block_literals<<<g.n_bl, 32 * kLitWarps, 0, ss->s>>>(d_src, img, scr, d_out, d_status, g.bl0);
          if (cudaEventRecord(ss->join, ss->s) != cudaSuccess || cudaStreamWaitEvent(s, ss->join, 0) != cudaSuccess)
            return VOOM_E_CUDA;
        } else {
          zstd_block_literals<<<g.n_bl, 32 * kLitWarps, 0, s>>>(d_src, img, scr, d_out, d_status, g.bl0);
          zstd_block_decode<<<g.n_bl, 32, 0, s>>>(d_src, img, scr, g.bl0, g.n_bl, k1_wave(g.n_bl));
        }
      }
      tmark(s, VOOM_ZSTD_K_BLOCK_DECODE);  // literals and sequences together
      zstd_seq_scan<<<g.n_bl, kSeqScanThreads, 0, s>>>(img, scr, g.bl0);
      tmark(s, VOOM_ZSTD_K_SEQ_SCAN);
      zstd_job_scan<<<(g.n_jobs + kJobScanWarps - 1) / kJobScanWarps, 32 * kJobScanWarps, 0, s>>>(
          img, scr, d_status, g.job0, g.n_jobs);
      tmark(s, VOOM_ZSTD_K_JOB_SCAN);
      zstd_block_execute<<<g.n_bl, 256, 0, s>>>(d_src, img, scr, d_out, d_status, g.bl0);
      tmark(s, VOOM_ZSTD_K_BLOCK_EXECUTE);
    }
    if (g.n_tiles) {
      zstd_output<<<g.n_tiles, 256, 0, s>>>(d_src, img, scr, d_out, g.tile0);
      tmark(s, VOOM_ZSTD_K_OUTPUT);
      const uint32_t rgrid = std::min<uint32_t>(g.n_tiles, k1_wave(g.n_tiles));  // <= 4 CTAs per SM
      for (int p = 1; p < kResolvePasses; p++) zstd_resolve<<<rgrid, 256, 0, s>>>(img, scr, p, g.tile0, g.n_tiles);
      tmark(s, VOOM_ZSTD_K_RESOLVE);
      zstd_patch<<<g.n_tiles, 256, 0, s>>>(d_src, img, scr, d_out, d_status, g.tile0);
      tmark(s, VOOM_ZSTD_K_PATCH);
    }
  }
  if (h.n_frames) {
    zstd_checksum<<<(h.n_frames + 63) / 64, 64, 0, s>>>(img, scr, d_out, d_status);
    tmark(s, VOOM_ZSTD_K_CHECKSUM);
  }
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
