// Host planner for the GPU zstd decoder.
//
// Walks every job's frames exactly as RFC 8878 lays them out -- frame header
// (3.1.1.1), block headers (3.1.1.2), the literals section header and Huffman
// tree description (3.1.1.3.1, 4.2.1), the sequences section header and FSE
// table descriptions (3.1.1.3.2, 4.1.1) -- and records where each block's
// entropy-coded payloads start.  Those payloads (Huffman literal streams, the
// FSE sequence bitstream) and everything after them are decoded on the GPU.
// Jobs are planned on a pool of host threads; each job is independent.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <new>
#include <atomic>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/voom_b200.h"
#include "zstd_plan.h"

#define VOOM_API extern "C" __attribute__((visibility("default")))

using namespace voom::zstd;

namespace {

constexpr uint32_t kPredef = 0x80000000u;  // local marker: predefined table k

inline int hb32(uint32_t v) { return 31 - __builtin_clz(v); }

inline uint64_t le(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = 0; i < n; i++) v |= uint64_t(p[i]) << (8 * i);
  return v;
}

// ------------------------------------------------ table-description readers
// little-endian bit field [q, q + nb) of p[0..n) (zero past n), nb <= 32
inline uint32_t bitfield(const uint8_t* p, size_t n, uint64_t q, int nb) {
  if (nb <= 0) return 0;
  const uint64_t byte = q >> 3;
  uint64_t v = 0;
  if (byte + 8 <= n) {
    memcpy(&v, p + byte, 8);
  } else {
    for (uint64_t k = 0; k < 8 && byte + k < n; k++) v |= uint64_t(p[byte + k]) << (8 * k);
  }
  v >>= (q & 7);
  return uint32_t(v & ((uint64_t(1) << nb) - 1));
}
struct FwdBits {
  const uint8_t* p;
  size_t n;
  uint64_t pos = 0;
  uint32_t peek(int nb) const { return bitfield(p, n, pos, nb); }
  uint32_t get(int nb) {
    const uint32_t v = peek(nb);
    pos += uint64_t(nb);
    return v;
  }
};

// FSE normalized counts (RFC 8878 4.1.1).  Returns the symbol count or -1.
int read_ncount(const uint8_t* p, size_t n, int max_al, int max_sym, int16_t* norm, int* al_out,
                size_t* used) {
  if (n == 0) return -1;
  FwdBits r{p, n};
  const int al = int(r.get(4)) + 5;
  if (al > max_al) return -1;
  int remaining = (1 << al) + 1, threshold = 1 << al, nb = al + 1, sym = 0;
  for (int i = 0; i <= max_sym; i++) norm[i] = 0;
  while (remaining > 1) {
    if (sym > max_sym) return -1;
    const int mx = (2 * threshold - 1) - remaining;
    int count;
    const uint32_t low = r.peek(nb - 1);
    if (int(low) < mx) {
      count = int(low);
      r.pos += uint64_t(nb - 1);
    } else {
      uint32_t v = r.peek(nb);
      if (int(v) >= threshold) v -= uint32_t(mx);
      count = int(v);
      r.pos += uint64_t(nb);
    }
    count -= 1;
    remaining -= count < 0 ? -count : count;
    norm[sym++] = int16_t(count);
    if (count == 0) {
      for (;;) {
        const uint32_t rep = r.get(2);
        for (uint32_t k = 0; k < rep; k++) {
          if (sym > max_sym) return -1;
          norm[sym++] = 0;
        }
        if (rep != 3) break;
      }
    }
    while (remaining < threshold) {
      nb--;
      threshold >>= 1;
    }
  }
  if (remaining != 1 || r.pos > 8 * uint64_t(n)) return -1;
  *used = size_t((r.pos + 7) / 8);
  *al_out = al;
  return sym;
}

struct FseCell {
  uint8_t sym, nb;
  uint16_t base;
};

bool fse_build(const int16_t* norm, int nsym, int al, FseCell* t) {
  const int size = 1 << al;
  int high = size - 1;
  uint32_t next[256];
  uint8_t symtab[512];
  for (int s = 0; s < nsym; s++) {
    if (norm[s] == -1) {
      symtab[high--] = uint8_t(s);
      next[s] = 1;
    } else {
      next[s] = uint32_t(std::max<int>(norm[s], 0));
    }
  }
  int pos = 0;
  const int step = (size >> 1) + (size >> 3) + 3, mask = size - 1;
  for (int s = 0; s < nsym; s++)
    for (int i = 0; i < norm[s]; i++) {
      symtab[pos] = uint8_t(s);
      do pos = (pos + step) & mask; while (pos > high);
    }
  if (pos != 0) return false;
  for (int u = 0; u < size; u++) {
    const int s = symtab[u];
    const uint32_t x = next[s]++;
    const int nbits = al - hb32(x);
    t[u].sym = uint8_t(s);
    t[u].nb = uint8_t(nbits);
    t[u].base = uint16_t((x << nbits) - uint32_t(size));
  }
  return true;
}

// Backward bit reader over a small buffer (Huffman weight streams only).
struct BwdBits {
  const uint8_t* p;
  size_t n;
  int64_t pos;
  bool init(const uint8_t* b, size_t len) {
    if (len == 0 || b[len - 1] == 0) return false;
    p = b;
    n = len;
    pos = int64_t(8 * (len - 1)) + hb32(b[len - 1]);
    return true;
  }
  // the nb bits below pos (bits below the stream start read as 0)
  uint32_t read(int nb) {
    const int64_t q = pos - nb;
    uint32_t v = 0;
    if (q >= 0)
      v = bitfield(p, n, uint64_t(q), nb);
    else if (pos > 0)
      v = bitfield(p, n, 0, int(pos)) << int(-q);
    pos -= nb;
    return v;
  }
};


// Huffman tree description (RFC 8878 4.2.1) -> weights of every symbol.
bool read_huffman(const uint8_t* p, size_t n, ZHuf* h, size_t* used) {
  uint8_t w[256];
  int nw = 0;
  if (n < 1) return false;
  const int hbyte = p[0];
  if (hbyte >= 128) {
    nw = hbyte - 127;
    const size_t bytes = size_t(nw + 1) / 2;
    if (1 + bytes > n) return false;
    for (int i = 0; i < nw; i++) w[i] = (i % 2 == 0) ? p[1 + i / 2] >> 4 : p[1 + i / 2] & 15;
    *used = 1 + bytes;
  } else {
    if (hbyte == 0 || size_t(1 + hbyte) > n) return false;
    const uint8_t* q = p + 1;
    int16_t norm[256];
    int al;
    size_t hdr;
    const int ns = read_ncount(q, size_t(hbyte), 6, 255, norm, &al, &hdr);
    if (ns < 0 || hdr >= size_t(hbyte)) return false;
    FseCell ft[64];
    if (!fse_build(norm, ns, al, ft)) return false;
    BwdBits r;
    if (!r.init(q + hdr, size_t(hbyte) - hdr)) return false;
    uint32_t s1 = r.read(al), s2 = r.read(al);
    for (;;) {
      if (nw > 253) return false;
      w[nw++] = ft[s1].sym;
      s1 = ft[s1].base + r.read(ft[s1].nb);
      if (r.pos < 0) { w[nw++] = ft[s2].sym; break; }
      w[nw++] = ft[s2].sym;
      s2 = ft[s2].base + r.read(ft[s2].nb);
      if (r.pos < 0) { w[nw++] = ft[s1].sym; break; }
    }
    *used = 1 + size_t(hbyte);
  }
  uint32_t total = 0;
  for (int i = 0; i < nw; i++) {
    if (w[i] > 11) return false;
    if (w[i]) total += 1u << (w[i] - 1);
  }
  if (total == 0) return false;
  const int maxbits = hb32(total) + 1;
  if (maxbits > 11) return false;
  const uint32_t rest = (1u << maxbits) - total;
  if (rest & (rest - 1)) return false;
  w[nw++] = uint8_t(hb32(rest) + 1);
  memset(h, 0, sizeof(*h));
  memcpy(h->w, w, size_t(nw));
  h->nsym = uint16_t(nw);
  h->maxbits = uint8_t(maxbits);
  return true;
}

// --------------------------------------------------------------- job plan
struct JobPlan {
  std::vector<ZFrame> frames;
  std::vector<ZBlock> blocks;
  std::vector<ZHuf> huf;
  std::vector<ZFse> fse;
  bool bad = false;
};

// Tables a compressed block declares: its own Huffman description or none
// (treeless literals reuse the frame's previous table), and per sequence
// code either the predefined table (0), its own RLE / compressed table (1)
// or the previous block's (2, repeat mode).  Filled in parallel; the
// references are resolved per frame afterwards (resolve_job).
struct BlockTables {
  bool huf_own = false, treeless = false;
  ZHuf huf;
  int fse_kind[3] = {0, 0, 0};
  ZFse fse[3];
};

bool plan_compressed(const uint8_t* base, uint64_t at, size_t n, ZBlock& b, BlockTables& T) {
  const uint8_t* p = base + at;
  if (n < 1) return false;
  // literals section header (RFC 8878 3.1.1.3.1.1)
  const int type = p[0] & 3, sf = (p[0] >> 2) & 3;
  size_t used;
  if (type <= 1) {
    size_t regen, hsz;
    if (sf == 0 || sf == 2) { regen = p[0] >> 3; hsz = 1; }
    else if (sf == 1) { if (n < 2) return false; regen = (p[0] >> 4) + (size_t(p[1]) << 4); hsz = 2; }
    else { if (n < 3) return false; regen = (p[0] >> 4) + (size_t(p[1]) << 4) + (size_t(p[2]) << 12); hsz = 3; }
    if (regen > kBlockMax) return false;
    b.lit_type = uint32_t(type);
    b.lit_regen = uint32_t(regen);
    b.src = at + hsz;
    if (type == 0) {
      if (hsz + regen > n) return false;
      used = hsz + regen;
    } else {
      if (hsz + 1 > n) return false;
      used = hsz + 1;
    }
    b.lit_streams = 0;
  } else {
    const int streams = sf == 0 ? 1 : 4;
    const int hsz = sf <= 1 ? 3 : (sf == 2 ? 4 : 5);
    const int bits = sf <= 1 ? 10 : (sf == 2 ? 14 : 18);
    if (size_t(hsz) > n) return false;
    const uint64_t hv = le(p, hsz);
    const size_t regen = size_t((hv >> 4) & ((1u << bits) - 1));
    const size_t csize = size_t((hv >> (4 + bits)) & ((1u << bits) - 1));
    if (regen > kBlockMax || size_t(hsz) + csize > n) return false;
    size_t q = size_t(hsz), avail = csize;
    if (type == 2) {
      size_t wu;
      if (!read_huffman(p + q, avail, &T.huf, &wu)) return false;
      T.huf_own = true;
      q += wu;
      avail -= wu;
    } else {
      T.treeless = true;  // needs the frame's previous table
    }
    b.lit_type = 2;
    b.lit_regen = uint32_t(regen);
    b.lit_streams = uint32_t(streams);
    if (streams == 1) {
      if (avail == 0) return false;
      b.src = at + q;
      b.lit_len[0] = uint32_t(avail);
    } else {
      if (avail < 10) return false;
      const size_t s1 = p[q] | (p[q + 1] << 8), s2 = p[q + 2] | (p[q + 3] << 8), s3 = p[q + 4] | (p[q + 5] << 8);
      if (6 + s1 + s2 + s3 >= avail || !s1 || !s2 || !s3) return false;
      const size_t seg = (regen + 3) / 4;
      if (3 * seg > regen) return false;
      b.src = at + q + 6;
      b.lit_len[0] = uint32_t(s1);
      b.lit_len[1] = uint32_t(s2);
      b.lit_len[2] = uint32_t(s3);
      b.lit_len[3] = uint32_t(avail - 6 - s1 - s2 - s3);
    }
    used = size_t(hsz) + csize;
  }
  // sequences section header (RFC 8878 3.1.1.3.2.1)
  p += used;
  at += used;
  n -= used;
  if (n < 1) return false;
  size_t nseq, hsz;
  if (p[0] == 0) {
    if (n != 1) return false;
    b.nseq = 0;
    return true;
  } else if (p[0] < 128) {
    nseq = p[0];
    hsz = 1;
  } else if (p[0] < 255) {
    if (n < 2) return false;
    nseq = (size_t(p[0] - 128) << 8) + p[1];
    hsz = 2;
  } else {
    if (n < 3) return false;
    nseq = p[1] + (size_t(p[2]) << 8) + 0x7F00;
    hsz = 3;
  }
  if (hsz >= n) return false;
  const uint8_t modes = p[hsz++];
  if (modes & 3) return false;
  static const int kMaxAl[3] = {9, 8, 9}, kMaxSym[3] = {35, 31, 52};
  const int mode[3] = {modes >> 6, (modes >> 4) & 3, (modes >> 2) & 3};  // LL, OF, ML
  for (int k = 0; k < 3; k++) {
    if (mode[k] == 0) {
      T.fse_kind[k] = 0;
    } else if (mode[k] == 1) {
      if (hsz >= n || p[hsz] > kMaxSym[k]) return false;
      ZFse& f = T.fse[k];
      memset(&f, 0, sizeof f);
      f.rle = 1;
      f.rle_sym = p[hsz++];
      T.fse_kind[k] = 1;
    } else if (mode[k] == 2) {
      ZFse& f = T.fse[k];
      memset(&f, 0, sizeof f);
      int al;
      size_t u;
      // counts that read_ncount accepts fill the table exactly, so the spread
      // always closes (its step is odd, hence coprime with the table size):
      // the device builds the decode table from them
      const int ns = read_ncount(p + hsz, n - hsz, kMaxAl[k], kMaxSym[k], f.norm, &al, &u);
      if (ns < 0) return false;
      f.nsym = uint16_t(ns);
      f.al = uint8_t(al);
      T.fse_kind[k] = 1;
      hsz += u;
    } else {
      T.fse_kind[k] = 2;
    }
  }
  if (hsz >= n || p[n - 1] == 0) return false;
  b.nseq = uint32_t(nseq);
  b.seq_src = at + hsz;
  b.seq_len = uint32_t(n - hsz);
  return true;
}

// Frame and block walk of one job (sequential: block headers chain); the
// compressed blocks' sections are parsed later in parallel.
void walk_job(const uint8_t* base, const voom_zstd_job& job, JobPlan& jp) {
  uint64_t pos = job.src;
  const uint64_t end = job.src + job.src_len;
  if (job.src_len == 0) { jp.bad = true; return; }
  while (pos < end) {
    if (end - pos < 4) { jp.bad = true; return; }
    const uint32_t magic = uint32_t(le(base + pos, 4));
    if ((magic & 0xFFFFFFF0u) == 0x184D2A50u) {  // skippable frame
      if (end - pos < 8) { jp.bad = true; return; }
      const uint64_t sz = le(base + pos + 4, 4);
      if (pos + 8 + sz > end) { jp.bad = true; return; }
      pos += 8 + sz;
      continue;
    }
    if (magic != 0xFD2FB528u) { jp.bad = true; return; }
    pos += 4;
    if (pos >= end) { jp.bad = true; return; }
    const uint8_t fhd = base[pos++];
    const int fcs_flag = fhd >> 6, single = (fhd >> 5) & 1, csum = (fhd >> 2) & 1, did = fhd & 3;
    if (fhd & 8) { jp.bad = true; return; }
    uint64_t wsize = 0;
    if (!single) {
      if (pos >= end) { jp.bad = true; return; }
      const uint8_t wd = base[pos++];
      const uint64_t wbase = 1ull << (10 + (wd >> 3));
      wsize = wbase + (wbase / 8) * (wd & 7);
    }
    static const int kDid[4] = {0, 1, 2, 4};
    if (pos + uint64_t(kDid[did]) > end) { jp.bad = true; return; }
    if (kDid[did] && le(base + pos, kDid[did]) != 0) { jp.bad = true; return; }  // no dictionaries
    pos += uint64_t(kDid[did]);
    const int fcs_sz = fcs_flag == 0 ? (single ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
    if (pos + uint64_t(fcs_sz) > end) { jp.bad = true; return; }
    ZFrame fr;
    memset(&fr, 0, sizeof fr);
    fr.fcs = fcs_sz ? le(base + pos, fcs_sz) + (fcs_sz == 2 ? 256 : 0) : ~0ull;
    pos += uint64_t(fcs_sz);
    if (single) wsize = fr.fcs;
    const uint64_t block_max = std::min<uint64_t>(wsize, kBlockMax);
    fr.block_first = uint32_t(jp.blocks.size());
    const uint32_t frame_index = uint32_t(jp.frames.size());
    for (;;) {
      if (pos + 3 > end) { jp.bad = true; return; }
      const uint32_t bh = uint32_t(le(base + pos, 3));
      pos += 3;
      const int last = bh & 1, type = (bh >> 1) & 3;
      const uint64_t bs = bh >> 3;
      if (type == 3 || bs > block_max) { jp.bad = true; return; }
      ZBlock b;
      memset(&b, 0, sizeof b);
      b.type = uint32_t(type);
      b.frame = frame_index;
      b.huf = kNone;
      b.fse[0] = b.fse[1] = b.fse[2] = kNone;
      b.max_out = uint32_t(block_max);
      if (type == 0) {
        if (pos + bs > end) { jp.bad = true; return; }
        b.src = pos;
        b.size = uint32_t(bs);
        pos += bs;
      } else if (type == 1) {
        if (pos + 1 > end) { jp.bad = true; return; }
        b.src = pos;
        b.size = uint32_t(bs);
        pos += 1;
      } else {
        if (pos + bs > end) { jp.bad = true; return; }
        b.src = pos;
        b.size = uint32_t(bs);  // compressed size until parsed
        pos += bs;
      }
      jp.blocks.push_back(b);
      if (last) break;
    }
    fr.n_blocks = uint32_t(jp.blocks.size()) - fr.block_first;
    fr.csum_flag = uint32_t(csum);
    if (csum) {
      if (pos + 4 > end) { jp.bad = true; return; }
      fr.csum = uint32_t(le(base + pos, 4));
      pos += 4;
    }
    jp.frames.push_back(fr);
  }
}

// A job is direct when it is not interleaved and none of its blocks has
// sequences: every block's decoded size is then known here (raw / RLE size,
// or the literals' regenerated size), so each block's output offset is too.
// The sizes must add up to the job length and match every recorded frame
// content size; otherwise the job takes the general path, which reports the
// mismatch.
bool make_direct(JobPlan& jp, const voom_zstd_job& job) {
  if (jp.bad || (job.flags & VOOM_ZSTD_INTERLEAVE)) return false;
  uint64_t off = 0;
  for (const ZFrame& fr : jp.frames) {
    const uint64_t f0 = off;
    for (uint32_t i = fr.block_first; i < fr.block_first + fr.n_blocks; i++) {
      const ZBlock& b = jp.blocks[i];
      if (b.type == 2 && b.nseq) return false;
      const uint64_t sz = b.type == 2 ? b.lit_regen : b.size;
      if (sz > b.max_out) return false;
      off += sz;
    }
    if (fr.fcs != ~0ull && off - f0 != fr.fcs) return false;
  }
  if (off != job.dst_len) return false;
  off = 0;
  for (ZBlock& b : jp.blocks) {
    b.out_off = off;
    off += b.type == 2 ? b.lit_regen : b.size;
  }
  return true;
}

// Table references of one job's compressed blocks, frame by frame: own
// tables are appended, treeless / repeat blocks take the previous ones
// (RFC 8878 3.1.1.3.1.1, 3.1.1.3.2.1.1).
void resolve_job(JobPlan& jp, const BlockTables* tabs, const uint8_t* ok) {
  for (const ZFrame& fr : jp.frames) {
    uint32_t last_huf = kNone, last_fse[3] = {kNone, kNone, kNone};
    for (uint32_t i = fr.block_first; i < fr.block_first + fr.n_blocks; i++) {
      ZBlock& b = jp.blocks[i];
      if (b.type != 2) continue;
      if (!ok[i]) { jp.bad = true; return; }
      const BlockTables& T = tabs[i];
      if (b.lit_type == 2) {
        if (T.huf_own) {
          last_huf = uint32_t(jp.huf.size());
          jp.huf.push_back(T.huf);
        } else if (last_huf == kNone) {
          jp.bad = true;  // treeless literals without a previous table
          return;
        }
        b.huf = last_huf;
      }
      if (b.nseq) {
        for (int k = 0; k < 3; k++) {
          if (T.fse_kind[k] == 0) {
            b.fse[k] = kPredef | uint32_t(k);
          } else if (T.fse_kind[k] == 1) {
            b.fse[k] = uint32_t(jp.fse.size());
            jp.fse.push_back(T.fse[k]);
          } else {
            if (last_fse[k] == kNone) { jp.bad = true; return; }
            b.fse[k] = last_fse[k];
          }
          last_fse[k] = b.fse[k];
        }
      }
    }
  }
}

// Per-job counts (filled in parallel) and first indices in the plan arrays
// (a serial prefix pass): the arrays are then filled in parallel, straight
// into the image.
struct JobSpan {
  uint32_t nf, nb, nh, ns, nt, ndl, nbl;
  uint64_t lit, nseq;
};
struct JobBase {
  uint32_t f, b, h, s, t, dl, bl;
  uint64_t lit, seq;
};

struct Plan {
  std::vector<ZSegment> segs;
  std::vector<uint32_t> status;
  std::unique_ptr<uint8_t[]> image;  // header + arrays, ready to copy to the device
  ZPlanHeader hdr;
  uint64_t image_bytes = 0;
  uint64_t decoded = 0;
  uint32_t n_bad = 0, n_direct = 0;
};

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

const int16_t kLLDef[36] = {4, 3, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 1, 1, 1, 2, 2,
                            2, 2, 2, 2, 2, 2, 2, 3, 2, 1, 1, 1, 1, 1, -1, -1, -1, -1};
const int16_t kOFDef[29] = {1, 1, 1, 1, 1, 1, 2, 2, 2, 1, 1, 1, 1, 1, 1,
                            1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1};
const int16_t kMLDef[53] = {1, 4, 3, 2, 2, 2, 2, 2, 2, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                            1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                            1, 1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1, -1, -1};

}  // namespace

VOOM_API void* voom_zstd_plan_create(const uint8_t* h_src, uint64_t src_len, const voom_zstd_job* jobs,
                                     uint32_t n_jobs, int threads) {
  if ((!h_src && src_len) || (!jobs && n_jobs)) return nullptr;
  Plan* P = new (std::nothrow) Plan();
  if (!P) return nullptr;
  std::vector<JobPlan> jp(n_jobs);
  // threads: every core by default, but each thread takes at least a grain
  // of work (starting a thread costs about as much as planning a few dozen
  // blocks: 16 threads on a 1,147-block batch measured slower than 8)
  const int nt_all = threads > 0 ? threads : int(std::max(1u, std::thread::hardware_concurrency()));
  // runs f(i) for i in [0, n) on up to nt_all threads, at least `grain`
  // items each (dynamic assignment)
  auto parallel = [&](uint64_t n, uint64_t grain, auto&& f) {
    const int nt = int(std::max<uint64_t>(1, std::min<uint64_t>(uint64_t(nt_all), n / grain)));
    std::atomic<uint64_t> next{0};
    auto run = [&]() {
      for (uint64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) f(i);
    };
    std::vector<std::thread> pool;
    for (int w = 1; w < nt; w++) pool.emplace_back(run);
    run();
    for (auto& t : pool) t.join();
  };
  // 1. frame / block walk per job
  parallel(n_jobs, 256, [&](uint64_t j) {
    if (jobs[j].src + jobs[j].src_len > src_len) { jp[j].bad = true; return; }
    walk_job(h_src, jobs[j], jp[j]);
  });
  // 2. per job: every compressed block's sections, table references, the
  // direct check and the job's counts
  std::vector<uint64_t> bstart(n_jobs + 1, 0);
  for (uint32_t j = 0; j < n_jobs; j++) bstart[j + 1] = bstart[j] + (jp[j].bad ? 0 : jp[j].blocks.size());
  // uninitialised here: each block's entry is initialised by the thread that
  // plans it (one thread touching ~700 bytes per block cost milliseconds)
  static_assert(std::is_trivially_destructible<BlockTables>::value, "freed without destructors");
  struct FreeTabs {
    void operator()(BlockTables* t) const { ::operator delete[](t); }
  };
  std::unique_ptr<BlockTables, FreeTabs> tabs(static_cast<BlockTables*>(
      ::operator new[](sizeof(BlockTables) * std::max<uint64_t>(1, bstart[n_jobs]))));
  std::unique_ptr<uint8_t[]> okb(new uint8_t[std::max<uint64_t>(1, bstart[n_jobs])]);
  std::vector<uint8_t> direct(n_jobs, 0);
  std::vector<JobSpan> span(n_jobs);
  // the blocks' sections in parallel over all blocks (one large job would
  // otherwise hold a thread for all of its blocks)
  std::vector<uint32_t> bjob(bstart[n_jobs]);
  for (uint32_t j = 0; j < n_jobs; j++)
    for (uint64_t g = bstart[j]; g < bstart[j + 1]; g++) bjob[g] = j;
  parallel(bstart[n_jobs], 128, [&](uint64_t g) {
    const uint32_t j = bjob[g];
    ZBlock& b = jp[j].blocks[g - bstart[j]];
    new (tabs.get() + g) BlockTables();
    okb[g] = 1;
    if (b.type != 2) return;
    const uint64_t at = b.src;
    const size_t bs = b.size;
    b.src = 0;
    b.size = 0;
    okb[g] = plan_compressed(h_src, at, bs, b, tabs.get()[g]) ? 1 : 0;
  });
  parallel(n_jobs, 256, [&](uint64_t j) {
    JobPlan& q = jp[j];
    JobSpan& c = span[j];
    memset(&c, 0, sizeof c);
    if (q.bad) return;
    BlockTables* T = tabs.get() + bstart[j];
    uint8_t* ok = okb.get() + bstart[j];
    resolve_job(q, T, ok);
    direct[j] = make_direct(q, jobs[j]) ? 1 : 0;
    if (q.bad) return;
    c.nf = uint32_t(q.frames.size());
    c.nb = uint32_t(q.blocks.size());
    c.nh = uint32_t(q.huf.size());
    c.ns = uint32_t(q.fse.size());
    c.nt = direct[j] ? 0u : uint32_t((jobs[j].dst_len + kOutTile - 1) / kOutTile);
    for (const ZBlock& b : q.blocks) {
      if (b.type == 2 && direct[j] && b.lit_type == 2) c.ndl++;
      else c.nbl++;
      if (b.type == 2 && !direct[j]) {
        c.lit += align_up(b.lit_regen, 16);
        c.nseq += b.nseq;
      }
    }
  });
  tabs.reset();
  okb.reset();

  // 3. serial prefix: Z-space offsets, segments, statuses, array bases
  std::vector<JobBase> base(n_jobs);
  std::vector<uint64_t> zoffs(n_jobs, 0);
  std::vector<uint8_t> bad(n_jobs, 0);
  JobBase run;
  memset(&run, 0, sizeof run);
  run.s = 3;  // predefined sequence tables occupy fse[0..2]
  uint64_t zoff = 0, zmax = 0;
  P->status.assign(n_jobs, 0);
  ZSegment seg;
  memset(&seg, 0, sizeof seg);
  auto close_segment = [&](uint32_t j_end) {
    seg.n_jobs = j_end - seg.job0;
    seg.n_frames = run.f - seg.frame0;
    seg.n_blocks = run.b - seg.block0;
    seg.n_tiles = run.t - seg.tile0;
    seg.n_bl = run.bl - seg.bl0;
    seg.zbytes = zoff;
    zmax = std::max(zmax, zoff);
    if (seg.n_jobs) P->segs.push_back(seg);
    seg.job0 = j_end;
    seg.frame0 = run.f;
    seg.block0 = run.b;
    seg.tile0 = run.t;
    seg.bl0 = run.bl;
    zoff = 0;
  };
  for (uint32_t j = 0; j < n_jobs; j++) {
    const bool qbad = jp[j].bad;
    const uint64_t zneed = (qbad || direct[j]) ? 0 : align_up(jobs[j].dst_len, 16);
    if (zneed > kZJobMax) {
      bad[j] = 1;
      zoffs[j] = zoff;
      P->status[j] = VOOM_ZSTD_ST_TOO_LARGE;
      P->n_bad++;
      continue;
    }
    if (zneed && zoff + zneed > kZSeg && j > seg.job0) close_segment(j);
    zoffs[j] = zoff;
    zoff += zneed;
    if (qbad) {
      bad[j] = 1;
      P->status[j] = VOOM_ZSTD_ST_FORMAT;
      P->n_bad++;
      continue;
    }
    base[j] = run;
    const JobSpan& c = span[j];
    run.f += c.nf;
    run.b += c.nb;
    run.h += c.nh;
    run.s += c.ns;
    run.t += c.nt;
    run.dl += c.ndl;
    run.bl += c.nbl;
    run.lit += c.lit;
    run.seq += c.nseq;
    P->decoded += jobs[j].dst_len;
    P->n_direct += direct[j];
  }
  close_segment(n_jobs);

  // 4. image layout, then every job's entries written in parallel
  ZPlanHeader& h = P->hdr;
  memset(&h, 0, sizeof h);
  h.n_jobs = n_jobs;
  h.n_frames = run.f;
  h.n_blocks = run.b;
  h.n_huf = run.h;
  h.n_fse = run.s;
  h.n_tiles = run.t;
  h.n_dlit = run.dl;
  h.n_blist = run.bl;
  uint64_t o = align_up(sizeof(ZPlanHeader), 256);
  h.off_jobs = o; o = align_up(o + sizeof(ZJob) * uint64_t(n_jobs), 256);
  h.off_frames = o; o = align_up(o + sizeof(ZFrame) * uint64_t(run.f), 256);
  h.off_blocks = o; o = align_up(o + sizeof(ZBlock) * uint64_t(run.b), 256);
  h.off_huf = o; o = align_up(o + sizeof(ZHuf) * uint64_t(run.h), 256);
  h.off_fse = o; o = align_up(o + sizeof(ZFse) * uint64_t(run.s), 256);
  h.off_tiles = o; o = align_up(o + sizeof(ZOutTile) * uint64_t(run.t), 256);
  h.off_dlit = o; o = align_up(o + sizeof(uint32_t) * uint64_t(run.dl), 256);
  h.off_blist = o; o = align_up(o + sizeof(uint32_t) * uint64_t(run.bl), 256);
  h.off_k1list = o; o = align_up(o + sizeof(uint32_t) * uint64_t(run.bl), 256);
  P->image_bytes = o;
  h.lit_bytes = run.lit;
  h.n_seq = run.seq;
  h.zbytes = zmax;  // the largest segment: the link-word scratch is reused by every segment
  uint64_t s = 0;
  h.s_res = s; s = align_up(s + 4 * zmax, 256);
  h.s_lit = s; s = align_up(s + run.lit + 64, 256);
  h.s_seq = s; s = align_up(s + sizeof(ZSeq) * run.seq, 256);
  h.s_blk = s; s = align_up(s + sizeof(ZBlockRt) * uint64_t(run.b), 256);
  h.s_ctr = s; s = align_up(s + 4 * uint64_t(run.t) + 256, 256);
  // three worklists of Z positions still unresolved: list 0 from the output
  // pass (kept for the patch pass), lists 1 and 2 alternating between the
  // resolve passes
  h.list_cap = std::max<uint64_t>(65536, zmax / 64);
  h.s_list = s; s = align_up(s + 3 * 8 * h.list_cap, 256);
  h.s_total = s;

  P->image.reset(new (std::nothrow) uint8_t[P->image_bytes]);
  if (!P->image) {
    delete P;
    return nullptr;
  }
  uint8_t* img = P->image.get();
  // the alignment gaps between the arrays are zero
  const uint64_t ends[10][2] = {{sizeof(ZPlanHeader), h.off_jobs},
                               {h.off_jobs + sizeof(ZJob) * uint64_t(n_jobs), h.off_frames},
                               {h.off_frames + sizeof(ZFrame) * uint64_t(run.f), h.off_blocks},
                               {h.off_blocks + sizeof(ZBlock) * uint64_t(run.b), h.off_huf},
                               {h.off_huf + sizeof(ZHuf) * uint64_t(run.h), h.off_fse},
                               {h.off_fse + sizeof(ZFse) * uint64_t(run.s), h.off_tiles},
                               {h.off_tiles + sizeof(ZOutTile) * uint64_t(run.t), h.off_dlit},
                               {h.off_dlit + sizeof(uint32_t) * uint64_t(run.dl), h.off_blist},
                               {h.off_blist + sizeof(uint32_t) * uint64_t(run.bl), h.off_k1list},
                               {h.off_k1list + sizeof(uint32_t) * uint64_t(run.bl), P->image_bytes}};
  for (const auto& g : ends) memset(img + g[0], 0, g[1] - g[0]);
  memcpy(img, &h, sizeof h);
  ZJob* J = reinterpret_cast<ZJob*>(img + h.off_jobs);
  ZFrame* F = reinterpret_cast<ZFrame*>(img + h.off_frames);
  ZBlock* B = reinterpret_cast<ZBlock*>(img + h.off_blocks);
  ZHuf* H = reinterpret_cast<ZHuf*>(img + h.off_huf);
  ZFse* S = reinterpret_cast<ZFse*>(img + h.off_fse);
  ZOutTile* TL = reinterpret_cast<ZOutTile*>(img + h.off_tiles);
  uint32_t* DL = reinterpret_cast<uint32_t*>(img + h.off_dlit);
  uint32_t* BL = reinterpret_cast<uint32_t*>(img + h.off_blist);
  for (int k = 0; k < 3; k++) {
    ZFse f;
    memset(&f, 0, sizeof f);
    const int16_t* d = k == 0 ? kLLDef : (k == 1 ? kOFDef : kMLDef);
    const int n = k == 0 ? 36 : (k == 1 ? 29 : 53);
    for (int i = 0; i < n; i++) f.norm[i] = d[i];
    f.nsym = uint16_t(n);
    f.al = uint8_t(k == 1 ? 5 : 6);
    S[k] = f;
  }
  parallel(n_jobs, 256, [&](uint64_t jj) {
    const uint32_t j = uint32_t(jj);
    ZJob zj;
    memset(&zj, 0, sizeof zj);
    zj.src = jobs[j].src;
    zj.src_len = jobs[j].src_len;
    zj.dst = jobs[j].dst;
    zj.dst_len = jobs[j].dst_len;
    zj.lo_src = jobs[j].lo_src;
    zj.flags = jobs[j].flags;
    zj.zoff = zoffs[j];
    if (bad[j]) {
      zj.bad = 1;
      zj.direct = (P->status[j] == VOOM_ZSTD_ST_TOO_LARGE) ? 0u : direct[j];
      J[j] = zj;
      return;
    }
    zj.direct = direct[j];
    const JobPlan& q = jp[j];
    const JobBase& bs = base[j];
    zj.frame_first = bs.f;
    zj.n_frames = uint32_t(q.frames.size());
    for (size_t k = 0; k < q.frames.size(); k++) {
      ZFrame f = q.frames[k];
      f.block_first += bs.b;
      f.job = j;
      F[bs.f + k] = f;
    }
    uint64_t lit = bs.lit, nseq = bs.seq;
    uint32_t ndl = 0, nbl = 0;
    for (size_t i = 0; i < q.blocks.size(); i++) {
      ZBlock b = q.blocks[i];
      b.frame += bs.f;
      b.job = j;
      if (b.huf != kNone) b.huf += bs.h;
      for (int k = 0; k < 3; k++) {
        if (b.fse[k] == kNone) continue;
        b.fse[k] = (b.fse[k] & kPredef) ? (b.fse[k] & 3u) : b.fse[k] + bs.s;
      }
      b.lit_off = lit;
      b.seq_off = nseq;
      const uint32_t gi = bs.b + uint32_t(i);
      if (b.type == 2 && zj.direct && b.lit_type == 2)
        DL[bs.dl + ndl++] = gi;
      else
        BL[bs.bl + nbl++] = gi;
      if (b.type == 2 && !zj.direct) {
        lit += align_up(b.lit_regen, 16);
        nseq += b.nseq;
      }
      B[gi] = b;
    }
    for (size_t k = 0; k < q.huf.size(); k++) H[bs.h + k] = q.huf[k];
    for (size_t k = 0; k < q.fse.size(); k++) S[bs.s + k] = q.fse[k];
    uint32_t nt = 0;
    for (uint64_t s0 = 0; !zj.direct && s0 < jobs[j].dst_len; s0 += kOutTile) {
      ZOutTile t;
      memset(&t, 0, sizeof t);
      t.job = j;
      t.begin = s0;
      t.len = std::min<uint64_t>(kOutTile, jobs[j].dst_len - s0);
      TL[bs.t + nt++] = t;
    }
    J[j] = zj;
  });
  // the per-job lists are released by the workers too (one thread freeing
  // four small vectors per job took milliseconds on KV page batches)
  parallel(n_jobs, 256, [&](uint64_t j) { jp[j] = JobPlan(); });
  // each segment's block list ordered by sequence count, most first (stable)
  uint32_t* K1 = reinterpret_cast<uint32_t*>(img + h.off_k1list);
  for (const ZSegment& g : P->segs) {
    std::copy(BL + g.bl0, BL + g.bl0 + g.n_bl, K1 + g.bl0);
    std::stable_sort(K1 + g.bl0, K1 + g.bl0 + g.n_bl, [&](uint32_t a, uint32_t b) {
      const uint32_t na = B[a].type == 2 ? B[a].nseq : 0u, nb = B[b].type == 2 ? B[b].nseq : 0u;
      return na > nb;
    });
  }
  return P;
}

VOOM_API int voom_zstd_plan_info_get(const void* plan, voom_zstd_plan_info* info) {
  if (!plan || !info) return VOOM_E_INVALID_ARG;
  const Plan* P = static_cast<const Plan*>(plan);
  memset(info, 0, sizeof(*info));
  info->n_jobs = P->hdr.n_jobs;
  info->n_frames = P->hdr.n_frames;
  info->n_blocks = P->hdr.n_blocks;
  info->n_huf = P->hdr.n_huf;
  info->n_fse = P->hdr.n_fse;
  info->n_bad_jobs = P->n_bad;
  info->lit_bytes = P->hdr.lit_bytes;
  info->n_seq = P->hdr.n_seq;
  info->decoded_bytes = P->decoded;
  info->scratch_bytes = P->hdr.s_total;
  info->plan_bytes = P->image_bytes;
  info->n_segments = uint32_t(P->segs.size());
  info->n_direct_jobs = P->n_direct;
  return VOOM_OK;
}

VOOM_API int voom_zstd_plan_image(const void* plan, void* h_image, uint64_t cap) {
  if (!plan || !h_image) return VOOM_E_INVALID_ARG;
  const Plan* P = static_cast<const Plan*>(plan);
  if (cap < P->image_bytes) return VOOM_E_CAPACITY;
  memcpy(h_image, P->image.get(), P->image_bytes);
  return VOOM_OK;
}

VOOM_API int voom_zstd_plan_job_status(const void* plan, uint32_t* h_status) {
  if (!plan || !h_status) return VOOM_E_INVALID_ARG;
  const Plan* P = static_cast<const Plan*>(plan);
  for (size_t j = 0; j < P->status.size(); j++) h_status[j] = P->status[j];
  return VOOM_OK;
}

VOOM_API void voom_zstd_plan_destroy(void* plan) { delete static_cast<Plan*>(plan); }

namespace voom {
namespace zstd {
// Launch sizes for voom_zstd_decode, read from the host plan handle.
bool plan_counts(const void* plan, ZPlanHeader* out, std::vector<ZSegment>* segs) {
  if (!plan) return false;
  *out = static_cast<const Plan*>(plan)->hdr;
  *segs = static_cast<const Plan*>(plan)->segs;
  return true;
}
}  // namespace zstd
}  // namespace voom
