/*
 * CPU ORACLE - test infrastructure only (see oracle/__init__.py).
 *
 * Serial restatement of the Zstandard frame decoder, written from the public
 * format specification (RFC 8878).  The reference decodes vpack hi planes and
 * kv_paged spill pages with `compression.zstd.decompress`
 * (formats/packed.py:20,376-378; formats/packed2.py:31-34,178-191;
 * runtime/kv_paged.py:98-113), i.e. libzstd; that library is not part of the
 * reference checkout, so its algorithm is restated here and pinned against the
 * system libzstd (1.5.5) on frames produced by the reference's own calls
 * (zstd.compress(level=1) and the streamed ZstdCompressor).
 *
 * Supports: concatenated and skippable frames, Raw/RLE/Compressed blocks,
 * Raw/RLE/Huffman/Treeless literals (1 and 4 streams), predefined/RLE/FSE/
 * repeat sequence tables, repeat offsets, content size and XXH64 checksum.
 * Dictionaries are not used by the reference and are rejected.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BLOCK_MAX (128 * 1024)

typedef struct { uint8_t sym, nb; uint16_t base; } fse_e;
typedef struct { uint8_t sym, nb; } huf_e;

static int hb32(uint32_t v) { return 31 - __builtin_clz(v); }

static uint64_t le_bounded(const uint8_t* p, size_t n, size_t at, int bytes) {
  uint64_t v = 0;
  for (int i = 0; i < bytes; i++)
    if (at + (size_t)i < n) v |= (uint64_t)p[at + i] << (8 * i);
  return v;
}

/* ---------------------------------------------------- forward bit reader */
typedef struct { const uint8_t* p; size_t n; uint64_t pos; } fbr_t;

static uint32_t fbr_peek(const fbr_t* r, int nb) {
  uint32_t v = 0;
  for (int i = 0; i < nb; i++) {
    uint64_t q = r->pos + (uint64_t)i;
    uint32_t bit = (q / 8 < r->n) ? (r->p[q / 8] >> (q % 8)) & 1u : 0u;
    v |= bit << i;
  }
  return v;
}

static uint32_t fbr_get(fbr_t* r, int nb) {
  uint32_t v = fbr_peek(r, nb);
  r->pos += (uint64_t)nb;
  return v;
}

/* --------------------------------------------------- backward bit reader */
typedef struct { const uint8_t* p; size_t n; int64_t pos; } bbr_t;

static int bbr_init(bbr_t* r, const uint8_t* p, size_t n) {
  if (n == 0 || p[n - 1] == 0) return -1;
  r->p = p;
  r->n = n;
  r->pos = (int64_t)(8 * (n - 1)) + hb32(p[n - 1]);
  return 0;
}

/* Bits [pos-nb, pos) as a number (bits below the stream start read as 0). */
static uint64_t bbr_peek(const bbr_t* r, int nb) {
  if (nb == 0) return 0;
  int64_t q = r->pos - nb;
  uint64_t v;
  if (q >= 0) {
    v = le_bounded(r->p, r->n, (size_t)(q >> 3), 8) >> (q & 7);
  } else {
    int64_t top = q + nb;
    v = top > 0 ? (le_bounded(r->p, r->n, 0, 8) & ((1ull << top) - 1)) << (-q) : 0;
  }
  return v & ((nb == 64) ? ~0ull : ((1ull << nb) - 1));
}

static uint64_t bbr_read(bbr_t* r, int nb) {
  uint64_t v = bbr_peek(r, nb);
  r->pos -= nb;
  return v;
}

/* ------------------------------------------------------------------ FSE */
/* Normalized-count header (RFC 8878 4.1.1).  Returns the symbol count or -1. */
static int read_ncount(const uint8_t* p, size_t n, int max_al, int max_sym, int16_t* norm, int* al_out,
                       size_t* used) {
  if (n == 0) return -1;
  fbr_t r = {p, n, 0};
  int al = (int)fbr_get(&r, 4) + 5;
  if (al > max_al) return -1;
  int remaining = (1 << al) + 1, threshold = 1 << al, nb = al + 1, sym = 0;
  for (int i = 0; i <= max_sym; i++) norm[i] = 0;
  while (remaining > 1) {
    if (sym > max_sym) return -1;
    int mx = (2 * threshold - 1) - remaining;
    int count;
    uint32_t low = fbr_peek(&r, nb - 1);
    if ((int)low < mx) {
      count = (int)low;
      r.pos += (uint64_t)(nb - 1);
    } else {
      uint32_t v = fbr_peek(&r, nb);
      if ((int)v >= threshold) v -= (uint32_t)mx;
      count = (int)v;
      r.pos += (uint64_t)nb;
    }
    count -= 1;
    remaining -= count < 0 ? -count : count;
    norm[sym++] = (int16_t)count;
    if (count == 0) {
      for (;;) {
        uint32_t rep = fbr_get(&r, 2);
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
  if (remaining != 1 || r.pos > 8 * (uint64_t)n) return -1;
  *used = (size_t)((r.pos + 7) / 8);
  *al_out = al;
  return sym;
}

static int fse_build(const int16_t* norm, int nsym, int al, fse_e* t) {
  int size = 1 << al, high = size - 1;
  uint32_t next[256];
  uint8_t symtab[512];
  for (int s = 0; s < nsym; s++) {
    if (norm[s] == -1) {
      symtab[high--] = (uint8_t)s;
      next[s] = 1;
    } else {
      next[s] = (uint32_t)(norm[s] > 0 ? norm[s] : 0);
    }
  }
  int pos = 0, step = (size >> 1) + (size >> 3) + 3, mask = size - 1;
  for (int s = 0; s < nsym; s++) {
    for (int i = 0; i < norm[s]; i++) {
      symtab[pos] = (uint8_t)s;
      do pos = (pos + step) & mask; while (pos > high);
    }
  }
  if (pos != 0) return -1;
  for (int u = 0; u < size; u++) {
    int s = symtab[u];
    uint32_t x = next[s]++;
    int nbits = al - hb32(x);
    t[u].sym = (uint8_t)s;
    t[u].nb = (uint8_t)nbits;
    t[u].base = (uint16_t)((x << nbits) - (uint32_t)size);
  }
  return 0;
}

/* -------------------------------------------------------------- Huffman */
typedef struct { huf_e t[1 << 11]; int maxbits; int valid; } huf_t;

static int huf_read_table(const uint8_t* p, size_t n, huf_t* h, size_t* used) {
  uint8_t w[256];
  int nw = 0;
  if (n < 1) return -1;
  int hbyte = p[0];
  if (hbyte >= 128) {
    nw = hbyte - 127;
    size_t bytes = (size_t)(nw + 1) / 2;
    if (1 + bytes > n) return -1;
    for (int i = 0; i < nw; i++) w[i] = (i % 2 == 0) ? p[1 + i / 2] >> 4 : p[1 + i / 2] & 15;
    *used = 1 + bytes;
  } else {
    if ((size_t)(1 + hbyte) > n || hbyte == 0) return -1;
    const uint8_t* q = p + 1;
    int16_t norm[256];
    int al;
    size_t hdr;
    int ns = read_ncount(q, (size_t)hbyte, 6, 255, norm, &al, &hdr);
    if (ns < 0 || hdr >= (size_t)hbyte) return -1;
    fse_e ft[64];
    if (fse_build(norm, ns, al, ft)) return -1;
    bbr_t r;
    if (bbr_init(&r, q + hdr, (size_t)hbyte - hdr)) return -1;
    uint32_t s1 = (uint32_t)bbr_read(&r, al), s2 = (uint32_t)bbr_read(&r, al);
    for (;;) {
      if (nw > 253) return -1;
      w[nw++] = ft[s1].sym;
      s1 = ft[s1].base + (uint32_t)bbr_read(&r, ft[s1].nb);
      if (r.pos < 0) { w[nw++] = ft[s2].sym; break; }
      w[nw++] = ft[s2].sym;
      s2 = ft[s2].base + (uint32_t)bbr_read(&r, ft[s2].nb);
      if (r.pos < 0) { w[nw++] = ft[s1].sym; break; }
    }
    *used = 1 + (size_t)hbyte;
  }
  uint32_t total = 0;
  for (int i = 0; i < nw; i++) {
    if (w[i] > 11) return -1;
    if (w[i]) total += 1u << (w[i] - 1);
  }
  if (total == 0) return -1;
  int maxbits = hb32(total) + 1;
  if (maxbits > 11) return -1;
  uint32_t rest = (1u << maxbits) - total;
  if (rest & (rest - 1)) return -1;
  w[nw++] = (uint8_t)(hb32(rest) + 1);
  uint32_t count[13] = {0}, start[13] = {0};
  for (int i = 0; i < nw; i++) count[w[i]]++;
  uint32_t pos = 0;
  for (int k = 1; k <= maxbits; k++) { start[k] = pos; pos += count[k] << (k - 1); }
  if (pos != (1u << maxbits)) return -1;
  for (int s = 0; s < nw; s++) {
    if (!w[s]) continue;
    uint32_t len = 1u << (w[s] - 1);
    for (uint32_t i = 0; i < len; i++) {
      h->t[start[w[s]] + i].sym = (uint8_t)s;
      h->t[start[w[s]] + i].nb = (uint8_t)(maxbits + 1 - w[s]);
    }
    start[w[s]] += len;
  }
  h->maxbits = maxbits;
  h->valid = 1;
  return 0;
}

static int huf_stream(const uint8_t* p, size_t n, const huf_t* h, uint8_t* out, size_t count) {
  bbr_t r;
  if (bbr_init(&r, p, n)) return -1;
  for (size_t i = 0; i < count; i++) {
    uint32_t v = (uint32_t)bbr_peek(&r, h->maxbits);
    out[i] = h->t[v].sym;
    r.pos -= h->t[v].nb;
  }
  return r.pos == 0 ? 0 : -1;
}

static int decode_literals(const uint8_t* p, size_t n, huf_t* h, uint8_t* lit, size_t* lit_len,
                           size_t* used) {
  if (n < 1) return -1;
  int type = p[0] & 3, sf = (p[0] >> 2) & 3;
  if (type <= 1) {
    size_t regen, hsz;
    if (sf == 0 || sf == 2) { regen = p[0] >> 3; hsz = 1; }
    else if (sf == 1) { if (n < 2) return -1; regen = (p[0] >> 4) + ((size_t)p[1] << 4); hsz = 2; }
    else { if (n < 3) return -1; regen = (p[0] >> 4) + ((size_t)p[1] << 4) + ((size_t)p[2] << 12); hsz = 3; }
    if (regen > BLOCK_MAX) return -1;
    if (type == 0) {
      if (hsz + regen > n) return -1;
      memcpy(lit, p + hsz, regen);
      *used = hsz + regen;
    } else {
      if (hsz + 1 > n) return -1;
      memset(lit, p[hsz], regen);
      *used = hsz + 1;
    }
    *lit_len = regen;
    return 0;
  }
  int streams = sf == 0 ? 1 : 4;
  int hsz = sf <= 1 ? 3 : (sf == 2 ? 4 : 5);
  int bits = sf <= 1 ? 10 : (sf == 2 ? 14 : 18);
  if ((size_t)hsz > n) return -1;
  uint64_t hv = le_bounded(p, n, 0, hsz);
  size_t regen = (size_t)((hv >> 4) & ((1u << bits) - 1));
  size_t csize = (size_t)((hv >> (4 + bits)) & ((1u << bits) - 1));
  if (regen > BLOCK_MAX || (size_t)hsz + csize > n) return -1;
  const uint8_t* q = p + hsz;
  size_t avail = csize;
  if (type == 2) {
    size_t wu;
    if (huf_read_table(q, avail, h, &wu)) return -1;
    q += wu;
    avail -= wu;
  } else if (!h->valid) {
    return -1;
  }
  if (streams == 1) {
    if (huf_stream(q, avail, h, lit, regen)) return -1;
  } else {
    if (avail < 10) return -1;
    size_t s1 = q[0] | (q[1] << 8), s2 = q[2] | (q[3] << 8), s3 = q[4] | (q[5] << 8);
    if (6 + s1 + s2 + s3 > avail) return -1;
    size_t s4 = avail - 6 - s1 - s2 - s3;
    size_t seg = (regen + 3) / 4;
    if (3 * seg > regen) return -1;
    const uint8_t* d = q + 6;
    if (huf_stream(d, s1, h, lit, seg) || huf_stream(d + s1, s2, h, lit + seg, seg) ||
        huf_stream(d + s1 + s2, s3, h, lit + 2 * seg, seg) ||
        huf_stream(d + s1 + s2 + s3, s4, h, lit + 3 * seg, regen - 3 * seg))
      return -1;
  }
  *lit_len = regen;
  *used = (size_t)hsz + csize;
  return 0;
}

/* ------------------------------------------------------------ sequences */
static const int16_t LL_DEF[36] = {4, 3, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 1, 1, 1, 2, 2,
                                   2, 2, 2, 2, 2, 2, 2, 3, 2, 1, 1, 1, 1, 1, -1, -1, -1, -1};
static const int16_t ML_DEF[53] = {1, 4, 3, 2, 2, 2, 2, 2, 2, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                                   1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                                   1, 1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1, -1, -1};
static const int16_t OF_DEF[29] = {1, 1, 1, 1, 1, 1, 2, 2, 2, 1, 1, 1, 1, 1, 1,
                                   1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1};
static const uint32_t LL_BASE[36] = {0,  1,  2,  3,  4,  5,  6,  7,  8,  9,    10,   11,
                                     12, 13, 14, 15, 16, 18, 20, 22, 24, 28,   32,   40,
                                     48, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768, 65536};
static const uint8_t LL_BITS[36] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1,
                                    1, 1, 2, 2, 3, 3, 4, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16};
static const uint32_t ML_BASE[53] = {3,  4,  5,  6,  7,  8,  9,  10, 11, 12, 13, 14, 15, 16,
                                     17, 18, 19, 20, 21, 22, 23, 24, 25, 26, 27, 28, 29, 30,
                                     31, 32, 33, 34, 35, 37, 39, 41, 43, 47, 51, 59, 67, 83,
                                     99, 131, 259, 515, 1027, 2051, 4099, 8195, 16387, 32771, 65539};
static const uint8_t ML_BITS[53] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                                    0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1,
                                    2, 2, 3, 3, 4, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16};

typedef struct {
  fse_e t[512];
  int al;
  int valid;
} seqtab_t;

typedef struct {
  huf_t huf;
  seqtab_t ll, of, ml;
  uint64_t rep[3];
} fstate_t;

static int seq_table(const uint8_t* p, size_t n, int mode, seqtab_t* st, const int16_t* def, int def_n,
                     int def_al, int max_al, int max_sym, size_t* used) {
  int16_t norm[64];
  switch (mode) {
    case 0:
      if (fse_build(def, def_n, def_al, st->t)) return -1;
      st->al = def_al;
      st->valid = 1;
      *used = 0;
      return 0;
    case 1:
      if (n < 1 || p[0] > max_sym) return -1;
      st->t[0].sym = p[0];
      st->t[0].nb = 0;
      st->t[0].base = 0;
      st->al = 0;
      st->valid = 1;
      *used = 1;
      return 0;
    case 2: {
      int al;
      int ns = read_ncount(p, n, max_al, max_sym, norm, &al, used);
      if (ns < 0 || fse_build(norm, ns, al, st->t)) return -1;
      st->al = al;
      st->valid = 1;
      return 0;
    }
    default:
      *used = 0;
      return st->valid ? 0 : -1;
  }
}

static int decode_block(const uint8_t* p, size_t n, fstate_t* fs, uint8_t* out, size_t* opos, size_t cap,
                        size_t frame_start, uint8_t* lit) {
  size_t lit_len, used;
  if (decode_literals(p, n, &fs->huf, lit, &lit_len, &used)) return -1;
  p += used;
  n -= used;
  if (n < 1) return -1;
  size_t nseq, hsz;
  if (p[0] == 0) {
    if (n != 1) return -1;
    nseq = 0;
    hsz = 1;
  } else if (p[0] < 128) {
    nseq = p[0];
    hsz = 1;
  } else if (p[0] < 255) {
    if (n < 2) return -1;
    nseq = ((size_t)(p[0] - 128) << 8) + p[1];
    hsz = 2;
  } else {
    if (n < 3) return -1;
    nseq = p[1] + ((size_t)p[2] << 8) + 0x7F00;
    hsz = 3;
  }
  size_t lp = 0, o = *opos;
  if (nseq) {
    if (hsz >= n) return -1;
    uint8_t modes = p[hsz++];
    if (modes & 3) return -1;
    size_t u;
    if (seq_table(p + hsz, n - hsz, modes >> 6, &fs->ll, LL_DEF, 36, 6, 9, 35, &u)) return -1;
    hsz += u;
    if (seq_table(p + hsz, n - hsz, (modes >> 4) & 3, &fs->of, OF_DEF, 29, 5, 8, 31, &u)) return -1;
    hsz += u;
    if (seq_table(p + hsz, n - hsz, (modes >> 2) & 3, &fs->ml, ML_DEF, 53, 6, 9, 52, &u)) return -1;
    hsz += u;
    bbr_t r;
    if (hsz > n || bbr_init(&r, p + hsz, n - hsz)) return -1;
    uint32_t sll = (uint32_t)bbr_read(&r, fs->ll.al);
    uint32_t sof = (uint32_t)bbr_read(&r, fs->of.al);
    uint32_t sml = (uint32_t)bbr_read(&r, fs->ml.al);
    for (size_t i = 0; i < nseq; i++) {
      int ofc = fs->of.t[sof].sym, llc = fs->ll.t[sll].sym, mlc = fs->ml.t[sml].sym;
      if (ofc > 31) return -1;
      uint64_t ofv = (1ull << ofc) + bbr_read(&r, ofc);
      uint64_t ml = ML_BASE[mlc] + bbr_read(&r, ML_BITS[mlc]);
      uint64_t ll = LL_BASE[llc] + bbr_read(&r, LL_BITS[llc]);
      uint64_t off;
      if (ofv > 3) {
        off = ofv - 3;
        fs->rep[2] = fs->rep[1];
        fs->rep[1] = fs->rep[0];
        fs->rep[0] = off;
      } else {
        int idx = (int)ofv - 1 + (ll == 0);
        if (idx == 0) {
          off = fs->rep[0];
        } else {
          off = idx == 3 ? fs->rep[0] - 1 : fs->rep[idx];
          if (idx != 1) fs->rep[2] = fs->rep[1];
          fs->rep[1] = fs->rep[0];
          fs->rep[0] = off;
        }
      }
      if (i + 1 < nseq) {
        sll = fs->ll.t[sll].base + (uint32_t)bbr_read(&r, fs->ll.t[sll].nb);
        sml = fs->ml.t[sml].base + (uint32_t)bbr_read(&r, fs->ml.t[sml].nb);
        sof = fs->of.t[sof].base + (uint32_t)bbr_read(&r, fs->of.t[sof].nb);
      }
      if (lp + ll > lit_len || o + ll + ml > cap) return -1;
      memcpy(out + o, lit + lp, ll);
      o += ll;
      lp += ll;
      if (off == 0 || off > o - frame_start) return -1;
      for (uint64_t k = 0; k < ml; k++, o++) out[o] = out[o - off];
    }
    if (r.pos != 0) return -1;
  }
  if (o + (lit_len - lp) > cap) return -1;
  memcpy(out + o, lit + lp, lit_len - lp);
  o += lit_len - lp;
  if (o - *opos > BLOCK_MAX) return -1;
  *opos = o;
  return 0;
}

/* ---------------------------------------------------------------- XXH64 */
static const uint64_t P1 = 0x9E3779B185EBCA87ull, P2 = 0xC2B2AE3D27D4EB4Full, P3 = 0x165667B19E3779F9ull,
                      P4 = 0x85EBCA77C2B2AE63ull, P5 = 0x27D4EB2F165667C5ull;
static uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t xround(uint64_t acc, uint64_t in) { return rotl64(acc + in * P2, 31) * P1; }
static uint64_t xmerge(uint64_t acc, uint64_t v) { return (acc ^ xround(0, v)) * P1 + P4; }

uint64_t oracle_xxh64(const uint8_t* p, size_t n, uint64_t seed) {
  const uint8_t* e = p + n;
  uint64_t h;
  if (n >= 32) {
    uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
    while (e - p >= 32) {
      v1 = xround(v1, le_bounded(p, 8, 0, 8));
      v2 = xround(v2, le_bounded(p + 8, 8, 0, 8));
      v3 = xround(v3, le_bounded(p + 16, 8, 0, 8));
      v4 = xround(v4, le_bounded(p + 24, 8, 0, 8));
      p += 32;
    }
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = xmerge(h, v1);
    h = xmerge(h, v2);
    h = xmerge(h, v3);
    h = xmerge(h, v4);
  } else {
    h = seed + P5;
  }
  h += (uint64_t)n;
  while (e - p >= 8) {
    h ^= xround(0, le_bounded(p, 8, 0, 8));
    h = rotl64(h, 27) * P1 + P4;
    p += 8;
  }
  if (e - p >= 4) {
    h ^= le_bounded(p, 4, 0, 4) * P1;
    h = rotl64(h, 23) * P2 + P3;
    p += 4;
  }
  while (p < e) {
    h ^= (*p++) * P5;
    h = rotl64(h, 11) * P1;
  }
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}

/* ---------------------------------------------------------------- frames */
/* Decompresses every frame in src (like ZSTD_decompress).  Returns 0 and the
 * output length, or -1 on any malformed input / insufficient capacity. */
int oracle_zstd_decompress(const uint8_t* src, size_t n, uint8_t* out, size_t cap, size_t* out_len) {
  size_t pos = 0, o = 0;
  fstate_t* fs = (fstate_t*)malloc(sizeof(fstate_t));
  uint8_t* lit = (uint8_t*)malloc(BLOCK_MAX + 64);
  int rc = -1;
  if (!fs || !lit) goto done;
  if (n == 0) goto done; /* libzstd: an empty input is not a frame */
  while (pos < n) {
    if (n - pos < 4) goto done;
    uint32_t magic = (uint32_t)le_bounded(src, n, pos, 4);
    if ((magic & 0xFFFFFFF0u) == 0x184D2A50u) {
      if (n - pos < 8) goto done;
      uint64_t sz = le_bounded(src, n, pos + 4, 4);
      if (pos + 8 + sz > n) goto done;
      pos += 8 + sz;
      continue;
    }
    if (magic != 0xFD2FB528u) goto done;
    pos += 4;
    if (pos >= n) goto done;
    uint8_t fhd = src[pos++];
    int fcs_flag = fhd >> 6, single = (fhd >> 5) & 1, csum = (fhd >> 2) & 1, did = fhd & 3;
    if (fhd & 8) goto done;
    uint64_t wsize = 0;
    if (!single) {
      if (pos >= n) goto done;
      uint8_t wd = src[pos++];
      uint64_t wbase = 1ull << (10 + (wd >> 3));
      wsize = wbase + (wbase / 8) * (wd & 7);
    }
    static const int DID_SZ[4] = {0, 1, 2, 4};
    if (pos + DID_SZ[did] > n) goto done;
    if (DID_SZ[did] && le_bounded(src, n, pos, DID_SZ[did]) != 0) goto done; /* dictionaries unsupported */
    pos += (size_t)DID_SZ[did];
    int fcs_sz = fcs_flag == 0 ? (single ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
    int has_fcs = fcs_sz > 0;
    uint64_t fcs = 0;
    if (pos + (size_t)fcs_sz > n) goto done;
    if (fcs_sz) fcs = le_bounded(src, n, pos, fcs_sz) + (fcs_sz == 2 ? 256 : 0);
    pos += (size_t)fcs_sz;
    if (single) wsize = fcs;
    size_t block_max = wsize < BLOCK_MAX ? (size_t)wsize : BLOCK_MAX;
    size_t frame_start = o;
    memset(fs, 0, sizeof(*fs));
    fs->rep[0] = 1;
    fs->rep[1] = 4;
    fs->rep[2] = 8;
    for (;;) {
      if (pos + 3 > n) goto done;
      uint32_t bh = (uint32_t)le_bounded(src, n, pos, 3);
      pos += 3;
      int last = bh & 1, type = (bh >> 1) & 3;
      size_t bs = bh >> 3;
      if (type == 3) goto done;
      if (type == 0) {
        if (bs > block_max || pos + bs > n || o + bs > cap) goto done;
        memcpy(out + o, src + pos, bs);
        o += bs;
        pos += bs;
      } else if (type == 1) {
        if (bs > block_max || pos + 1 > n || o + bs > cap) goto done;
        memset(out + o, src[pos], bs);
        o += bs;
        pos += 1;
      } else {
        if (bs > block_max || pos + bs > n) goto done;
        size_t before = o;
        if (decode_block(src + pos, bs, fs, out, &o, cap, frame_start, lit)) goto done;
        if (o - before > block_max) goto done;
        pos += bs;
      }
      if (last) break;
    }
    if (has_fcs && o - frame_start != fcs) goto done;
    if (csum) {
      if (pos + 4 > n) goto done;
      uint32_t want = (uint32_t)le_bounded(src, n, pos, 4);
      if ((uint32_t)oracle_xxh64(out + frame_start, o - frame_start, 0) != want) goto done;
      pos += 4;
    }
  }
  *out_len = o;
  rc = 0;
done:
  free(fs);
  free(lit);
  return rc;
}
