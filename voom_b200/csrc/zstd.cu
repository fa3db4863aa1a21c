// GPU Zstandard (RFC 8878) decoder for vpack hi planes and kv_paged pages.
//
// Pipeline over a planned batch of jobs (host plan: zstd_plan.cpp):
//   K1 block decode  - one CTA per block.  Warp 0 builds the Huffman table in
//                      shared memory and decodes the (1 or 4) literal streams,
//                      one lane per stream; warp 1 builds the LL/OF/ML FSE
//                      tables (one lane each) and lane 0 decodes the sequence
//                      bitstream, recording (literal length, match length,
//                      offset value) and the block's repeat-offset transform
//                      (each of the 3 repeat slots as "input slot minus d" or
//                      a constant) so blocks need no serial pass.
//   K2 job scan      - one thread per job: block output positions (prefix sum
//                      of block sizes) and the repeat offsets every block starts
//                      with (composition of the transforms); size checks.
//   K3 block execute - one CTA per block: concrete offsets (serial replay of
//                      the repeat-offset rules from the block's start state),
//                      then every output byte is written as either a resolved
//                      literal (bit 31 set | byte) or the position it copies.
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

// Backward bit reader (RFC 8878 4.1: a stream is read from its last byte
// towards its first, after the final byte's leading zeros and 1 marker): the next unread bits are left-aligned in a 64-bit
// window (stream bit pos-1 at bit 63); `vb` valid bits; refilled 32 bits at a
// time.  Reading n <= 32 bits is a shift of the window's high word.
struct BitIn {
  const uint8_t* p;
  int32_t pos;  // unread bits left in the stream
  int32_t vb;   // valid bits at the top of w (vb <= pos + 32 near the start)
  uint64_t w;

  __device__ __forceinline__ uint32_t bits32_at(int32_t q) const {  // stream bits [q, q+32), zeros below 0
    if (q >= 0) return uint32_t(load8(p + (q >> 3)) >> (q & 7));
    if (q <= -32) return 0u;
    return uint32_t(load8(p) << (-q));
  }
  __device__ __forceinline__ bool init(const uint8_t* s, uint32_t len) {
    p = s;
    if (len == 0) return false;
    const uint32_t last = __ldg(s + len - 1);
    if (!last) return false;
    pos = int32_t(8 * (len - 1) + (31 - __clz(last)));
    w = 0;
    vb = 0;
    refill();
    refill();
    return true;
  }
  __device__ __forceinline__ void refill() {  // requires vb <= 32
    w |= uint64_t(bits32_at(pos - vb - 32)) << (32 - vb);
    vb += 32;
  }
  __device__ __forceinline__ void ensure(int n) {
    if (vb < n) refill();
  }
  __device__ __forceinline__ uint32_t top(int n) const {  // 1 <= n <= 32
    return uint32_t(w >> 32) >> (32 - n);
  }
  __device__ __forceinline__ void skip(int n) {
    w <<= n;
    vb -= n;
    pos -= n;
  }
  __device__ __forceinline__ uint32_t read(int n) {  // 0 <= n <= 32
    if (n == 0) return 0;
    const uint32_t v = top(n);
    skip(n);
    return v;
  }
};

// FSE decode table (RFC 8878 4.1.1): cell = symbol | nbBits << 8 | base << 16.
__device__ void fse_build_dev(const ZFse& f, uint32_t* t, uint16_t* next, int* al_out) {
  if (f.rle) {
    t[0] = f.rle_sym;
    *al_out = 0;
    return;
  }
  const int al = f.al, size = 1 << al, nsym = f.nsym;
  int high = size - 1;
  for (int s = 0; s < nsym; s++) {
    const int c = f.norm[s];
    if (c == -1) {
      t[high--] = uint32_t(s);
      next[s] = 1;
    } else {
      next[s] = uint16_t(c > 0 ? c : 0);
    }
  }
  const int step = (size >> 1) + (size >> 3) + 3, mask = size - 1;
  int pos = 0;
  for (int s = 0; s < nsym; s++) {
    const int c = f.norm[s];
    for (int i = 0; i < c; i++) {
      t[pos] = uint32_t(s);
      do pos = (pos + step) & mask; while (pos > high);
    }
  }
  for (int u = 0; u < size; u++) {
    const uint32_t s = t[u] & 0xFFu;
    const uint32_t x = next[s]++;
    const uint32_t nb = uint32_t(al - (31 - __clz(x)));
    t[u] = s | (nb << 8) | (((x << nb) - uint32_t(size)) << 16);
  }
  *al_out = al;
}

struct K1Shared {
  uint32_t huf3[2048];  // up to 3 symbols per lookup: s0|s1<<8|s2<<16|bits<<24|count<<28
  uint16_t huf[2048];
  uint16_t sstart[256];
  uint32_t ll[512], of[256], ml[512];
  uint16_t next[3][64];
  int al[3];
  uint32_t st;
  uint32_t out_size;
  uint32_t rep_kind[3], rep_val[3];
};

__device__ void decode_literals(const uint8_t* src, const View& v, const ZBlock& b, K1Shared& sh,
                                uint8_t* lit) {
  const int lane = threadIdx.x & 31;
  if (b.lit_type == 0) {
    for (uint32_t i = lane; i < b.lit_regen; i += 32) lit[i] = __ldg(src + b.src + i);
    return;
  }
  if (b.lit_type == 1) {
    const uint8_t c = __ldg(src + b.src);
    for (uint32_t i = lane; i < b.lit_regen; i += 32) lit[i] = c;
    return;
  }
  const ZHuf& H = v.huf[b.huf];
  const int maxbits = H.maxbits, nsym = H.nsym;
  if (lane == 0) {
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
  __syncwarp();
  for (int s = lane; s < nsym; s += 32) {
    const int w = H.w[s];
    if (!w) continue;
    const uint16_t e = uint16_t(s | ((maxbits + 1 - w) << 8));
    const uint32_t st = sh.sstart[s], len = 1u << (w - 1);
    for (uint32_t i = 0; i < len; i++) sh.huf[st + i] = e;
  }
  __syncwarp();
  // multi-symbol entries: greedily chain codes while they fit in maxbits
  const uint32_t tsize = 1u << maxbits, mask = tsize - 1;
  for (uint32_t i = lane; i < tsize; i += 32) {
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
  __syncwarp();
  const int streams = int(b.lit_streams);
  if (lane < streams) {
    const uint32_t seg = streams == 1 ? b.lit_regen : (b.lit_regen + 3) / 4;
    const uint32_t count = (streams == 1 || lane < 3) ? seg : b.lit_regen - 3 * seg;
    uint64_t off = b.src;
    for (int k = 0; k < lane; k++) off += b.lit_len[k];
    uint8_t* out = lit + uint32_t(lane) * seg;
    BitIn r;
    bool ok = r.init(src + off, b.lit_len[lane]);
    if (ok) {
      uint32_t i = 0;
      while (i + 3 <= count) {
        r.ensure(maxbits);
        const uint32_t e = sh.huf3[r.top(maxbits)];
        const uint32_t c = e >> 28;
        out[i] = uint8_t(e);
        if (c > 1) out[i + 1] = uint8_t(e >> 8);
        if (c > 2) out[i + 2] = uint8_t(e >> 16);
        i += c;
        r.skip(int((e >> 24) & 15u));
        if (r.pos < -32) break;
      }
      for (; i < count && r.pos >= -32; i++) {
        r.ensure(maxbits);
        const uint32_t e = sh.huf[r.top(maxbits)];
        out[i] = uint8_t(e);
        r.skip(int(e >> 8));
      }
      ok = (r.pos == 0);
    }
    if (!ok) atomicOr(&sh.st, VOOM_ZSTD_ST_LITERALS);
  }
}

__device__ void decode_sequences(const uint8_t* src, const View& v, const ZBlock& b, K1Shared& sh) {
  const int lane = threadIdx.x & 31;
  if (lane < 3) fse_build_dev(v.fse[b.fse[lane]], lane == 0 ? sh.ll : (lane == 1 ? sh.of : sh.ml), sh.next[lane],
                              &sh.al[lane]);
  __syncwarp();
  if (lane != 0) return;
  uint32_t rk[3] = {0, 1, 2}, rv[3] = {0, 0, 0};
  uint32_t sum_ml = 0, sum_ll = 0, st = 0;
  BitIn r;
  if (!r.init(src + b.seq_src, b.seq_len)) {
    st = VOOM_ZSTD_ST_SEQUENCES;
  } else {
    r.ensure(26);
    uint32_t sll = r.read(sh.al[0]), sof = r.read(sh.al[1]), sml = r.read(sh.al[2]);
    ZSeq* out = v.seq + b.seq_off;
    uint32_t dst = 0;
    for (uint32_t i = 0; i < b.nseq; i++) {
      const uint32_t eLL = sh.ll[sll], eOF = sh.of[sof], eML = sh.ml[sml];
      const uint32_t ofc = eOF & 0xFFu, mlc = eML & 0xFFu, llc = eLL & 0xFFu;
      r.ensure(31);
      const uint32_t ofv = (1u << ofc) + r.read(int(ofc));
      r.ensure(32);
      const uint32_t ml = c_ml_base[mlc] + r.read(c_ml_bits[mlc]);
      const uint32_t ll = c_ll_base[llc] + r.read(c_ll_bits[llc]);
      // repeat-offset rules (RFC 8878 3.1.2.5) on symbolic slots
      uint32_t ok, ov;
      if (ofv > 3) {
        ok = 3;
        ov = ofv - 3;
        rk[2] = rk[1]; rv[2] = rv[1];
        rk[1] = rk[0]; rv[1] = rv[0];
        rk[0] = ok; rv[0] = ov;
      } else {
        const uint32_t idx = ofv - 1 + (ll == 0);
        if (idx == 0) {
          ok = rk[0]; ov = rv[0];
        } else if (idx == 1) {
          ok = rk[1]; ov = rv[1];
          rk[1] = rk[0]; rv[1] = rv[0];
          rk[0] = ok; rv[0] = ov;
        } else if (idx == 2) {
          ok = rk[2]; ov = rv[2];
          rk[2] = rk[1]; rv[2] = rv[1];
          rk[1] = rk[0]; rv[1] = rv[0];
          rk[0] = ok; rv[0] = ov;
        } else {
          ok = rk[0]; ov = rk[0] == 3 ? rv[0] - 1 : rv[0] + 1;
          rk[2] = rk[1]; rv[2] = rv[1];
          rk[1] = rk[0]; rv[1] = rv[0];
          rk[0] = ok; rv[0] = ov;
        }
      }
      ZSeq s;
      s.ll = ll;
      s.ml = ml;
      s.oval = ov;
      s.okind = ok;
      s.dst = dst;
      s.lit = sum_ll;
      out[i] = s;
      dst += ll + ml;
      sum_ml += ml;
      sum_ll += ll;
      if (i + 1 < b.nseq) {
        r.ensure(26);
        sll = (eLL >> 16) + r.read(int((eLL >> 8) & 0xFFu));
        sml = (eML >> 16) + r.read(int((eML >> 8) & 0xFFu));
        sof = (eOF >> 16) + r.read(int((eOF >> 8) & 0xFFu));
      }
      if (r.pos < -32) break;
    }
    if (r.pos != 0) st = VOOM_ZSTD_ST_SEQUENCES;
  }
  if (sum_ll > b.lit_regen) st |= VOOM_ZSTD_ST_SEQUENCES;
  if (st) atomicOr(&sh.st, st);
  sh.out_size = b.lit_regen + sum_ml;
  for (int k = 0; k < 3; k++) {
    sh.rep_kind[k] = rk[k];
    sh.rep_val[k] = rv[k];
  }
}

__global__ void __launch_bounds__(64) zstd_block_decode(const uint8_t* __restrict__ src, const uint8_t* img,
                                                        uint8_t* scratch) {
  __shared__ K1Shared sh;
  const View v = make_view(img, scratch);
  const ZBlock b = v.blocks[blockIdx.x];
  ZBlockRt* rt = v.rt + blockIdx.x;
  if (b.type != 2) {
    if (threadIdx.x == 0) {
      rt->out_size = b.size;
      rt->status = 0;
      for (int k = 0; k < 3; k++) {
        rt->rep_kind[k] = uint32_t(k);
        rt->rep_val[k] = 0;
      }
    }
    return;
  }
  if (threadIdx.x == 0) {
    sh.st = 0;
    sh.out_size = b.lit_regen;
    for (int k = 0; k < 3; k++) {
      sh.rep_kind[k] = uint32_t(k);
      sh.rep_val[k] = 0;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) decode_literals(src, v, b, sh, v.lit + b.lit_off);
  else if (b.nseq) decode_sequences(src, v, b, sh);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t st = sh.st;
    if (sh.out_size > b.max_out) st |= VOOM_ZSTD_ST_SIZE;
    rt->out_size = sh.out_size;
    rt->status = st;
    for (int k = 0; k < 3; k++) {
      rt->rep_kind[k] = sh.rep_kind[k];
      rt->rep_val[k] = sh.rep_val[k];
    }
  }
}

__global__ void zstd_job_scan(const uint8_t* img, uint8_t* scratch, uint32_t* status) {
  const View v = make_view(img, scratch);
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= v.h->n_jobs) return;
  const ZJob job = v.jobs[j];
  if (job.bad) return;
  uint64_t z = job.zoff;
  uint32_t st = 0;
  for (uint32_t f = job.frame_first; f < job.frame_first + job.n_frames; f++) {
    const ZFrame fr = v.frames[f];
    uint32_t rep[3] = {1, 4, 8};
    const uint64_t fz = z;
    for (uint32_t bi = fr.block_first; bi < fr.block_first + fr.n_blocks; bi++) {
      ZBlockRt* rt = v.rt + bi;
      rt->zstart = z;
      rt->frame_zstart = fz;
      for (int k = 0; k < 3; k++) rt->init_rep[k] = rep[k];
      st |= rt->status;
      z += rt->out_size;
      uint32_t nr[3];
      for (int k = 0; k < 3; k++) nr[k] = rt->rep_kind[k] == 3 ? rt->rep_val[k] : rep[rt->rep_kind[k]] - rt->rep_val[k];
      for (int k = 0; k < 3; k++) rep[k] = nr[k];
    }
    if (fr.fcs != ~0ull && z - fz != fr.fcs) st |= VOOM_ZSTD_ST_SIZE;
  }
  if (z - job.zoff != job.dst_len) st |= VOOM_ZSTD_ST_SIZE;
  if (st) atomicOr(status + j, st);
}

__global__ void __launch_bounds__(128) zstd_block_execute(const uint8_t* __restrict__ src, const uint8_t* img,
                                                          uint8_t* scratch, uint32_t* status) {
  __shared__ uint32_t s_end[2];
  const View v = make_view(img, scratch);
  const ZBlock b = v.blocks[blockIdx.x];
  if (v.jobs[b.job].bad) return;
  const ZBlockRt rt = v.rt[blockIdx.x];
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
  if (rt.status) return;  // the job already failed in K1
  const ZSeq* seq = v.seq + b.seq_off;
  const uint8_t* lit = v.lit + b.lit_off;
  const uint64_t before = rt.zstart - rt.frame_zstart;
  uint32_t bad = 0;
  for (uint32_t i = threadIdx.x; i < b.nseq; i += blockDim.x) {
    const ZSeq s = seq[i];
    const uint32_t off = s.okind == 3 ? s.oval : rt.init_rep[s.okind] - s.oval;
    const bool ok = off != 0 && uint64_t(off) <= before + s.dst + s.ll;
    bad |= !ok;
    for (uint32_t k = 0; k < s.ll; k++) res[s.dst + k] = kResolved | lit[s.lit + k];
    const uint64_t m = rt.zstart + s.dst + s.ll;
    for (uint32_t k = 0; k < s.ml; k++) res[s.dst + s.ll + k] = ok ? uint32_t(m + k - off) : kResolved;
    if (i + 1 == b.nseq && threadIdx.x == (b.nseq - 1) % blockDim.x) {
      s_end[0] = s.dst + s.ll + s.ml;
      s_end[1] = s.lit + s.ll;
    }
  }
  if (threadIdx.x == 0 && b.nseq == 0) {
    s_end[0] = 0;
    s_end[1] = 0;
  }
  if (bad) atomicOr(status + b.job, VOOM_ZSTD_ST_OFFSET);
  __syncthreads();
  const uint32_t pos = s_end[0], litp = s_end[1];
  for (uint32_t k = threadIdx.x; k < b.lit_regen - litp; k += blockDim.x) res[pos + k] = kResolved | lit[litp + k];
}

__global__ void __launch_bounds__(256) zstd_resolve(const uint8_t* img, uint8_t* scratch, uint32_t* status,
                                                    int first_pass) {
  __shared__ uint32_t s_unres;
  const View v = make_view(img, scratch);
  const ZOutTile t = v.tiles[blockIdx.x];
  if (!first_pass && !v.dirty[blockIdx.x]) return;
  const ZJob job = v.jobs[t.job];
  if (job.bad) return;
  if (threadIdx.x == 0) s_unres = 0;
  __syncthreads();
  const uint64_t zmax = v.h->zbytes;
  uint32_t unres = 0;
  for (uint64_t k = t.begin + threadIdx.x; k < t.begin + t.len; k += blockDim.x) {
    const uint64_t z = job.zoff + k;
    uint32_t u = v.res[z];
    if (u & kResolved) continue;
    for (int h = 0; h < kHops && !(u & kResolved); h++) {
      if (u >= zmax) {
        u = kResolved;
        break;
      }
      u = v.res[u];
    }
    v.res[z] = u;
    unres += !(u & kResolved);
  }
  if (unres) atomicAdd(&s_unres, unres);
  __syncthreads();
  if (threadIdx.x == 0) v.dirty[blockIdx.x] = s_unres;
}

__global__ void __launch_bounds__(256) zstd_output(const uint8_t* __restrict__ src, const uint8_t* img,
                                                   uint8_t* scratch, uint8_t* __restrict__ out, uint32_t* status) {
  const View v = make_view(img, scratch);
  const ZOutTile t = v.tiles[blockIdx.x];
  const ZJob job = v.jobs[t.job];
  if (job.bad) return;
  if (v.dirty[blockIdx.x]) {
    if (threadIdx.x == 0) atomicOr(status + t.job, VOOM_ZSTD_ST_UNRESOLVED);
    return;
  }
  const bool inter = job.flags & VOOM_ZSTD_INTERLEAVE;
  const bool vec = ((job.dst & 15u) == 0);
  const uint64_t end = t.begin + t.len;
  for (uint64_t k = t.begin + 8u * threadIdx.x; k < end; k += 8u * blockDim.x) {
    const uint64_t z = job.zoff + k;
    const uint32_t cnt = uint32_t((end - k) < 8 ? (end - k) : 8);
    if (cnt == 8) {
      const uint4 r0 = *reinterpret_cast<const uint4*>(v.res + z);
      const uint4 r1 = *reinterpret_cast<const uint4*>(v.res + z + 4);
      const uint32_t hi0 = __byte_perm(__byte_perm(r0.x, r0.y, 0x0040), __byte_perm(r0.z, r0.w, 0x0040), 0x5410);
      const uint32_t hi1 = __byte_perm(__byte_perm(r1.x, r1.y, 0x0040), __byte_perm(r1.z, r1.w, 0x0040), 0x5410);
      if (inter) {
        const uint64_t lo = load8(src + job.lo_src + k);
        const uint32_t lo0 = uint32_t(lo), lo1 = uint32_t(lo >> 32);
        uint4 o;
        o.x = __byte_perm(lo0, hi0, 0x5140);
        o.y = __byte_perm(lo0, hi0, 0x7362);
        o.z = __byte_perm(lo1, hi1, 0x5140);
        o.w = __byte_perm(lo1, hi1, 0x7362);
        uint8_t* d = out + job.dst + 2 * k;
        if (vec) {
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
    } else {
      for (uint32_t i = 0; i < cnt; i++) {
        const uint8_t hb = uint8_t(v.res[z + i]);
        if (inter) {
          out[job.dst + 2 * (k + i)] = __ldg(src + job.lo_src + k + i);
          out[job.dst + 2 * (k + i) + 1] = hb;
        } else {
          out[job.dst + k + i] = hb;
        }
      }
    }
  }
}

// XXH64 (xxHash specification) of a frame's decoded bytes, one thread per frame.
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

__global__ void zstd_checksum(const uint8_t* img, uint8_t* scratch, uint32_t* status) {
  const View v = make_view(img, scratch);
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= v.h->n_frames) return;
  const ZFrame fr = v.frames[f];
  if (!fr.csum_flag || v.jobs[fr.job].bad || status[fr.job]) return;
  const uint64_t P1 = 0x9E3779B185EBCA87ull, P2 = 0xC2B2AE3D27D4EB4Full, P3 = 0x165667B19E3779F9ull,
                 P4 = 0x85EBCA77C2B2AE63ull, P5 = 0x27D4EB2F165667C5ull;
  uint64_t z0 = 0, n = 0;
  if (fr.n_blocks) {
    const ZBlockRt& a = v.rt[fr.block_first];
    const ZBlockRt& l = v.rt[fr.block_first + fr.n_blocks - 1];
    z0 = a.zstart;
    n = l.zstart + l.out_size - z0;
  }
  const uint32_t* r = v.res + z0;
  auto byte = [&](uint64_t i) { return uint64_t(r[i] & 0xFFu); };
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
bool plan_counts(const void* plan, ZPlanHeader* out);
}
}  // namespace voom

VOOM_API int voom_zstd_decode(const uint8_t* d_src, const void* d_plan, const void* h_plan, void* d_scratch,
                              uint8_t* d_out, uint32_t* d_status, void* stream) {
  if (!d_src || !d_plan || !h_plan || !d_scratch || !d_out || !d_status) return VOOM_E_INVALID_ARG;
  ZPlanHeader h;
  if (!voom::zstd::plan_counts(h_plan, &h)) return VOOM_E_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* img = static_cast<const uint8_t*>(d_plan);
  uint8_t* scr = static_cast<uint8_t*>(d_scratch);
  if (h.n_blocks) {
    zstd_block_decode<<<h.n_blocks, 64, 0, s>>>(d_src, img, scr);
    zstd_job_scan<<<(h.n_jobs + 127) / 128, 128, 0, s>>>(img, scr, d_status);
    zstd_block_execute<<<h.n_blocks, 128, 0, s>>>(d_src, img, scr, d_status);
  }
  if (h.n_tiles) {
    for (int p = 0; p < kResolvePasses; p++)
      zstd_resolve<<<h.n_tiles, 256, 0, s>>>(img, scr, d_status, p == 0);
    zstd_output<<<h.n_tiles, 256, 0, s>>>(d_src, img, scr, d_out, d_status);
  }
  if (h.n_frames) zstd_checksum<<<(h.n_frames + 63) / 64, 64, 0, s>>>(img, scr, d_status);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
