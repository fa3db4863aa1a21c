/*
 * CPU ORACLE - test infrastructure only.  Nothing in the product path links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs use it, as the checker.
 *
 * Plain-C restatement of the vOOM "VRN1" BF16 rANS codec,
 * formats/bf16_rans.py (the reference is pure Python, stdlib only):
 *   oracle_rans_normalize : _normalize_frequencies  bf16_rans.py:36-58
 *   oracle_rans_encode    : _encode_plane + encode   bf16_rans.py:72-94, 148-177
 *   oracle_rans_decode    : _decode_plane + decode   bf16_rans.py:97-130, 180-222
 *   oracle_crc32          : zlib.crc32 (reflected polynomial 0xEDB88320)
 * Error codes are the VOOM_RANS_* values of include/voom_b200.h, one per
 * ValueError message the reference raises, checked in the reference's order.
 * Parity is pinned by tests/golden (frames produced by the reference encode)
 * and by tests/test_oracle_rans.py.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/voom_b200.h"

#define SCALE_BITS 12
#define TOTAL (1u << SCALE_BITS)
#define RANS_L (1u << 23)
#define FRAME_HDR 16 /* <4sIII> */
#define TILE_HDR 13  /* <BIII>  */
#define PLANE_HDR (4 + 512)

static uint32_t crc_table[256];
static int crc_ready = 0;

static void crc_init(void) {
  for (uint32_t n = 0; n < 256; n++) {
    uint32_t c = n;
    for (int k = 0; k < 8; k++) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
    crc_table[n] = c;
  }
  crc_ready = 1;
}

uint32_t oracle_crc32(const uint8_t* p, uint64_t n) {
  if (!crc_ready) crc_init();
  uint32_t c = 0xFFFFFFFFu;
  for (uint64_t i = 0; i < n; i++) c = crc_table[(c ^ p[i]) & 0xFF] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

static uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static void wr32(uint8_t* p, uint32_t v) {
  p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}

/* ---------------------------------------------------------------- encode */

typedef struct { uint64_t rem; uint64_t count; int sym; } frac_t;

/* Sort key of bf16_rans.py:50-55: descending (remainder, count, -symbol). */
static int frac_cmp(const void* a, const void* b) {
  const frac_t* x = (const frac_t*)a;
  const frac_t* y = (const frac_t*)b;
  if (x->rem != y->rem) return x->rem > y->rem ? -1 : 1;
  if (x->count != y->count) return x->count > y->count ? -1 : 1;
  return x->sym < y->sym ? -1 : (x->sym > y->sym ? 1 : 0);
}

/* _normalize_frequencies (bf16_rans.py:36-58), data read with a stride. */
void oracle_rans_normalize(const uint8_t* data, uint64_t n, uint64_t stride, uint16_t freq[256]) {
  uint64_t counts[256];
  memset(counts, 0, sizeof counts);
  for (uint64_t i = 0; i < n; i++) counts[data[i * stride]]++;
  memset(freq, 0, 256 * sizeof(uint16_t));
  int n_active = 0;
  for (int s = 0; s < 256; s++) n_active += counts[s] != 0;
  if (!n_active) return;
  uint64_t remaining = TOTAL - (uint64_t)n_active;
  uint64_t assigned = 0;
  frac_t fr[256];
  int nf = 0;
  for (int s = 0; s < 256; s++) {
    if (!counts[s]) continue;
    uint64_t scaled = counts[s] * remaining;
    uint64_t extra = scaled / n;
    freq[s] = (uint16_t)(1 + extra);
    assigned += extra;
    fr[nf].rem = scaled % n;
    fr[nf].count = counts[s];
    fr[nf].sym = s;
    nf++;
  }
  uint64_t left = remaining - assigned;
  qsort(fr, (size_t)nf, sizeof(frac_t), frac_cmp);
  for (uint64_t i = 0; i < left && i < (uint64_t)nf; i++) freq[fr[i].sym]++;
}

/* _encode_plane (bf16_rans.py:72-94).  Writes <I payload_len><256H freq><payload>
 * into out (capacity cap); returns bytes written or 0 if cap is too small.
 * scratch must hold n + 8 bytes. */
static uint64_t encode_plane(const uint8_t* data, uint64_t n, uint64_t stride, uint8_t* out,
                             uint64_t cap, uint8_t* scratch) {
  uint16_t freq[256];
  uint32_t cum[256];
  if (cap < PLANE_HDR + 4) return 0;
  if (n == 0) {
    wr32(out, 4);
    memset(out + 4, 0, 512);
    wr32(out + PLANE_HDR, RANS_L);
    return PLANE_HDR + 4;
  }
  oracle_rans_normalize(data, n, stride, freq);
  uint32_t t = 0;
  for (int s = 0; s < 256; s++) { cum[s] = t; t += freq[s]; }
  uint64_t state = RANS_L;
  uint64_t emitted = 0; /* bytes written to scratch, in emission order */
  for (uint64_t i = n; i-- > 0;) {
    uint8_t s = data[i * stride];
    uint64_t f = freq[s];
    uint64_t threshold = ((uint64_t)(RANS_L >> SCALE_BITS) << 8) * f;
    while (state >= threshold) {
      scratch[emitted++] = (uint8_t)(state & 0xFF);
      state >>= 8;
    }
    state = ((state / f) << SCALE_BITS) + (state % f) + cum[s];
  }
  uint64_t payload = 4 + emitted;
  if (cap < PLANE_HDR + payload) return 0;
  wr32(out, (uint32_t)payload);
  for (int s = 0; s < 256; s++) { out[4 + 2 * s] = (uint8_t)freq[s]; out[5 + 2 * s] = (uint8_t)(freq[s] >> 8); }
  wr32(out + PLANE_HDR, (uint32_t)state);
  for (uint64_t i = 0; i < emitted; i++) out[PLANE_HDR + 4 + i] = scratch[emitted - 1 - i];
  return PLANE_HDR + payload;
}

/* encode (bf16_rans.py:148-177).  Returns the frame length, or 0 on a bad
 * argument / insufficient capacity.  stats[0] = tiles, stats[1] = compressed tiles. */
uint64_t oracle_rans_encode(const uint8_t* data, uint64_t n, uint32_t tile_bytes, uint8_t* out,
                            uint64_t cap, uint64_t stats[2]) {
  if (tile_bytes == 0 || cap < FRAME_HDR) return 0;
  uint64_t tiles = (n + tile_bytes - 1) / tile_bytes;
  memcpy(out, "VRN1", 4);
  wr32(out + 4, (uint32_t)n);
  wr32(out + 8, tile_bytes);
  wr32(out + 12, (uint32_t)tiles);
  uint64_t pos = FRAME_HDR, ctiles = 0;
  uint8_t* scratch = (uint8_t*)malloc(tile_bytes + 16);
  uint8_t* coded = (uint8_t*)malloc(2 * (uint64_t)tile_bytes + 4 * PLANE_HDR + 64);
  if (!scratch || !coded) { free(scratch); free(coded); return 0; }
  for (uint64_t t = 0; t < tiles; t++) {
    const uint8_t* raw = data + t * tile_bytes;
    uint64_t len = n - t * tile_bytes < tile_bytes ? n - t * tile_bytes : tile_bytes;
    uint64_t ccap = 2 * (uint64_t)tile_bytes + 4 * PLANE_HDR + 64;
    uint64_t a = encode_plane(raw, (len + 1) / 2, 2, coded, ccap, scratch);
    uint64_t b = a ? encode_plane(raw + 1, len / 2, 2, coded + a, ccap - a, scratch) : 0;
    uint32_t crc = oracle_crc32(raw, len);
    int compressed = a && b && (a + b) < len;
    uint64_t body = compressed ? a + b : len;
    if (pos + TILE_HDR + body > cap) { free(scratch); free(coded); return 0; }
    out[pos] = compressed ? 1 : 0;
    wr32(out + pos + 1, (uint32_t)len);
    wr32(out + pos + 5, (uint32_t)body);
    wr32(out + pos + 9, crc);
    pos += TILE_HDR;
    memcpy(out + pos, compressed ? coded : raw, body);
    pos += body;
    ctiles += compressed;
  }
  free(scratch);
  free(coded);
  if (stats) { stats[0] = tiles; stats[1] = ctiles; }
  return pos;
}

/* ---------------------------------------------------------------- decode */

/* _decode_plane (bf16_rans.py:97-130): decodes `length` symbols of the plane
 * whose header starts at enc (avail bytes readable) into out[i*stride].
 * *used = bytes consumed (header + payload). */
static int decode_plane(const uint8_t* enc, uint64_t avail, uint64_t length, uint8_t* out,
                        uint64_t stride, uint64_t* used) {
  if (avail < PLANE_HDR) return VOOM_RANS_TRUNC_PLANE_HEADER;
  uint64_t payload_size = rd32(enc);
  uint32_t freq[256], cum[256];
  for (int s = 0; s < 256; s++) freq[s] = (uint32_t)enc[4 + 2 * s] | ((uint32_t)enc[5 + 2 * s] << 8);
  uint64_t end = PLANE_HDR + payload_size;
  if (payload_size < 4 || end > avail) return VOOM_RANS_TRUNC_PLANE_PAYLOAD;
  const uint8_t* payload = enc + PLANE_HDR;
  uint64_t state = rd32(payload);
  uint64_t cursor = 4;
  uint64_t total = 0;
  for (int s = 0; s < 256; s++) { cum[s] = (uint32_t)total; total += freq[s]; }
  if (total != 0 && total != TOTAL) return VOOM_RANS_BAD_FREQ_TOTAL;
  uint8_t lookup[TOTAL];
  memset(lookup, 0, sizeof lookup);
  for (int s = 0; s < 256; s++)
    for (uint32_t k = 0; k < freq[s]; k++) lookup[cum[s] + k] = (uint8_t)s;
  for (uint64_t i = 0; i < length; i++) {
    uint64_t slot = state & (TOTAL - 1);
    uint8_t sym = lookup[slot];
    out[i * stride] = sym;
    state = (uint64_t)freq[sym] * (state >> SCALE_BITS) + slot - cum[sym];
    while (state < RANS_L && cursor < payload_size) {
      state = (state << 8) | payload[cursor];
      cursor++;
    }
  }
  if (cursor != payload_size) return VOOM_RANS_TRAILING_RENORM;
  *used = end;
  return VOOM_OK;
}

/* Output capacity decode() needs for this frame: the sum of tile raw sizes
 * the walk can reach (an upper bound when the frame is malformed). */
uint64_t oracle_rans_capacity(const uint8_t* f, uint64_t n) {
  if (n < FRAME_HDR) return 0;
  uint64_t tile_count = rd32(f + 12), pos = FRAME_HDR, total = 0;
  for (uint64_t t = 0; t < tile_count; t++) {
    if (pos + TILE_HDR > n) break;
    uint64_t raw = rd32(f + pos + 1), pay = rd32(f + pos + 5);
    pos += TILE_HDR;
    if (pos + pay > n) break;
    total += raw;
    pos += pay;
  }
  return total;
}

/* decode (bf16_rans.py:180-222).  out must hold oracle_rans_capacity() bytes.
 * Returns VOOM_OK or the VOOM_RANS_* code of the first ValueError; *err_tile is
 * the failing tile (tile_count for frame-level errors), *bad_mode the mode
 * byte of an unknown-mode tile. */
int oracle_rans_decode(const uint8_t* f, uint64_t n, uint8_t* out, uint64_t cap, uint64_t* out_len,
                       uint32_t* err_tile, uint32_t* bad_mode) {
  *out_len = 0;
  *err_tile = 0;
  if (n < FRAME_HDR) return VOOM_RANS_TRUNC_FRAME;
  if (memcmp(f, "VRN1", 4) != 0) return VOOM_RANS_NOT_FRAME;
  uint64_t raw_size = rd32(f + 4), tile_count = rd32(f + 12);
  uint64_t pos = FRAME_HDR, olen = 0;
  for (uint64_t t = 0; t < tile_count; t++) {
    *err_tile = (uint32_t)t;
    if (pos + TILE_HDR > n) return VOOM_RANS_TRUNC_TILE_HEADER;
    uint32_t mode = f[pos];
    uint64_t raw = rd32(f + pos + 1), pay = rd32(f + pos + 5);
    uint32_t crc = rd32(f + pos + 9);
    pos += TILE_HDR;
    uint64_t end = pos + pay;
    if (end > n) return VOOM_RANS_TRUNC_TILE_PAYLOAD;
    const uint8_t* payload = f + pos;
    pos = end;
    if (olen + raw > cap) return VOOM_E_CAPACITY;
    uint8_t* tile = out + olen;
    if (mode == 0) {
      if (pay != raw) return VOOM_RANS_RAW_SIZE_MISMATCH;
      memcpy(tile, payload, raw);
    } else if (mode == 1) {
      uint64_t used = 0, used_high = 0;
      int rc = decode_plane(payload, pay, (raw + 1) / 2, tile, 2, &used);
      if (rc) return rc;
      rc = decode_plane(payload + used, pay - used, raw / 2, tile + 1, 2, &used_high);
      if (rc) return rc;
      if (used + used_high != pay) return VOOM_RANS_TILE_TRAILING;
    } else {
      *bad_mode = mode;
      return VOOM_RANS_UNKNOWN_MODE;
    }
    if (oracle_crc32(tile, raw) != crc) return VOOM_RANS_CHECKSUM;
    olen += raw;
  }
  *err_tile = (uint32_t)tile_count;
  if (pos != n || olen != raw_size) return VOOM_RANS_LENGTH_MISMATCH;
  *out_len = olen;
  return VOOM_OK;
}
