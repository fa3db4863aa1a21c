// Pieces of the zstd block encoder (RFC 8878) shared by the GPU kernel and a
// host build of the same code (tests compile this header with a plain C++
// compiler to check the encoder's decisions against libzstd on the CPU).
//
// A block is at most kEncBlock bytes of input and becomes one of:
//  - a Compressed block whose literals section is Huffman coded in four
//    streams (4.2), with the Huffman weights FSE compressed (4.2.1.2) or, for
//    at most 128 weights, stored as 4-bit values (4.2.1.1), and no sequences;
//  - a Compressed block of RLE literals, when one byte value fills the block;
//  - a Raw block, when Huffman coding would not make the block smaller.
// Everything here is integer arithmetic on byte counts; given the same
// histogram every build makes the same choices and writes the same bytes.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define VOOM_HD __host__ __device__ __forceinline__
#else
#define VOOM_HD inline
#endif

namespace voom {
namespace zenc {

constexpr uint32_t kEncBlock = 32768;   // input bytes per block
constexpr uint32_t kMaxBits = 11;       // Huffman code length limit (4.2.1)
constexpr uint32_t kFseLog = 6;         // accuracy log of the weight FSE table
constexpr uint32_t kHdrRoom = 16;       // bytes reserved before a block for the frame header
constexpr uint32_t kDescMax = 129;      // Huffman tree description: header byte + up to 128 bytes
constexpr uint32_t kSlotBytes = kHdrRoom + 3 + 5 + kDescMax + 6 + kEncBlock + 64;

VOOM_HD uint32_t hibit(uint32_t v) {  // index of the highest set bit (v > 0)
  uint32_t r = 0;
  while (v >>= 1) r++;
  return r;
}

// Forward bit writer over a byte buffer (bits fill each byte from its lowest bit).
struct BitOut {
  uint8_t* p;
  uint32_t cap;
  uint32_t pos;  // bits written
  VOOM_HD void put(uint32_t v, uint32_t nb) {
    for (uint32_t i = 0; i < nb; i++) {
      const uint32_t b = pos + i;
      if ((b >> 3) < cap) {
        if ((b & 7u) == 0) p[b >> 3] = 0;
        p[b >> 3] |= uint8_t(((v >> i) & 1u) << (b & 7u));
      }
    }
    pos += nb;
  }
  VOOM_HD uint32_t bytes() const { return (pos + 7) / 8; }
};

// Huffman code lengths (<= kMaxBits) of the present symbols, from the
// symbols sorted by (count ascending, symbol ascending): the two-queue
// construction (leaves in that order, internal nodes in creation order; on
// equal weights a leaf is taken first).  Returns the longest length; 0 for
// fewer than two present symbols.
VOOM_HD uint32_t huf_lengths(const uint16_t* sorted_sym, const uint32_t* count, uint32_t n, uint8_t* len,
                             uint16_t* parent /* 2n */, uint32_t* iw /* n */) {
  if (n < 2) return 0;
  uint32_t li = 0, qi = 0;
  for (uint32_t k = 0; k + 1 < n; k++) {
    uint32_t pick[2];
    uint32_t wsum = 0;
    for (int t = 0; t < 2; t++) {
      const bool leaf = li < n && (qi >= k || count[sorted_sym[li]] <= iw[qi]);
      if (leaf) {
        pick[t] = li;
        wsum += count[sorted_sym[li]];
        li++;
      } else {
        pick[t] = n + qi;
        wsum += iw[qi];
        qi++;
      }
    }
    iw[k] = wsum;
    parent[pick[0]] = uint16_t(n + k);
    parent[pick[1]] = uint16_t(n + k);
  }
  // depths: the root is internal node n - 2; parents come after their children
  uint8_t* depth = reinterpret_cast<uint8_t*>(iw);  // internal-node depths (reuses iw; weights are done)
  depth[n - 2] = 0;
  for (int k = int(n) - 3; k >= 0; k--) depth[k] = uint8_t(depth[parent[n + k] - n] + 1);
  uint32_t mx = 0;
  for (uint32_t i = 0; i < n; i++) {
    const uint32_t d = uint32_t(depth[parent[i] - n]) + 1u;
    len[sorted_sym[i]] = uint8_t(d > 255 ? 255 : d);
    mx = d > mx ? d : mx;
  }
  return mx;
}

// FSE normalized counts of the weight symbols 0..maxw (sum 2^kFseLog, every
// present symbol at least 1): rounded shares, then the excess taken from (or
// the deficit given to) the largest entries.
VOOM_HD void fse_normalize(const uint32_t* cnt, uint32_t maxw, uint32_t total, int16_t* norm) {
  const int32_t size = 1 << kFseLog;
  int32_t sum = 0;
  for (uint32_t s = 0; s <= maxw; s++) {
    int32_t v = 0;
    if (cnt[s]) {
      v = int32_t((uint64_t(cnt[s]) * uint32_t(size) * 2 + total) / (2ull * total));
      if (v < 1) v = 1;
    }
    norm[s] = int16_t(v);
    sum += v;
  }
  while (sum != size) {
    uint32_t best = 0;
    int32_t bv = -1;
    for (uint32_t s = 0; s <= maxw; s++) {
      const bool ok = sum > size ? norm[s] > 1 : cnt[s] > 0;
      if (ok && norm[s] > bv) {
        bv = norm[s];
        best = s;
      }
    }
    norm[best] = int16_t(norm[best] + (sum > size ? -1 : 1));
    sum += sum > size ? -1 : 1;
  }
}

// FSE table description (4.1.1) of norm[0..maxw] at accuracy log kFseLog.
VOOM_HD void fse_write_ncount(BitOut& b, const int16_t* norm, uint32_t maxw) {
  b.put(kFseLog - 5, 4);
  int32_t remaining = (1 << kFseLog) + 1, threshold = 1 << kFseLog;
  uint32_t nb = kFseLog + 1, s = 0;
  while (remaining > 1 && s <= maxw) {
    const int32_t count = norm[s];
    const int32_t mx = (2 * threshold - 1) - remaining;
    int32_t v = count + 1;
    if (v < mx) {
      b.put(uint32_t(v), nb - 1);
    } else {
      if (v >= threshold) v += mx;
      b.put(uint32_t(v), nb);
    }
    remaining -= count < 0 ? -count : count;
    s++;
    if (count == 0) {  // run of zero-probability symbols: 2-bit repeat flags
      uint32_t z = 0;
      while (s + z <= maxw && norm[s + z] == 0) z++;
      s += z;
      while (z >= 3) {
        b.put(3, 2);
        z -= 3;
      }
      b.put(z, 2);
    }
    while (remaining < threshold) {
      nb--;
      threshold >>= 1;
    }
  }
}

// FSE compression of the weight sequence w[0..nw-1] with two interleaved
// states (4.2.1.2: the decoder reads two initial states, then emits symbols
// alternately from them, updating each after its symbol, until a state
// update reads past the stream start).  Encoded from the last symbol back,
// states initialised from the last two symbols, as the format's reference
// encoder does.  Returns the stream bytes, or 0 if they exceed `cap`.
VOOM_HD uint32_t fse_encode_weights(const uint8_t* w, uint32_t nw, const int16_t* norm, uint32_t maxw, uint8_t* out,
                                    uint32_t cap) {
  const uint32_t size = 1u << kFseLog, mask = size - 1;
  uint8_t sym_at[1 << kFseLog];
  uint16_t state_tab[1 << kFseLog];
  uint32_t cumul[16];
  int32_t dnb[16];
  int32_t dfs[16];
  // symbol spread: the decoder's order
  uint32_t pos = 0;
  const uint32_t step = (size >> 1) + (size >> 3) + 3;
  for (uint32_t s = 0; s <= maxw; s++)
    for (int32_t i = 0; i < norm[s]; i++) {
      sym_at[pos] = uint8_t(s);
      pos = (pos + step) & mask;
    }
  uint32_t c = 0;
  for (uint32_t s = 0; s <= maxw; s++) {
    cumul[s] = c;
    c += uint32_t(norm[s] > 0 ? norm[s] : 0);
  }
  uint32_t next[16];
  for (uint32_t s = 0; s <= maxw; s++) next[s] = cumul[s];
  for (uint32_t u = 0; u < size; u++) state_tab[next[sym_at[u]]++] = uint16_t(size + u);
  for (uint32_t s = 0; s <= maxw; s++) {
    const int32_t nrm = norm[s];
    if (nrm <= 0) {
      dnb[s] = int32_t(((kFseLog + 1) << 16) - size);
      dfs[s] = 0;
    } else if (nrm == 1) {
      dnb[s] = int32_t((kFseLog << 16) - size);
      dfs[s] = int32_t(cumul[s]) - 1;
    } else {
      const uint32_t max_out = kFseLog - hibit(uint32_t(nrm - 1));
      dnb[s] = int32_t((max_out << 16) - (uint32_t(nrm) << max_out));
      dfs[s] = int32_t(cumul[s]) - nrm;
    }
  }
  BitOut b{out, cap, 0};
  auto init_state = [&](uint32_t s) -> uint32_t {
    const uint32_t nbo = uint32_t((dnb[s] + (1 << 15)) >> 16);
    const uint32_t v = (nbo << 16) - uint32_t(dnb[s]);
    return state_tab[int32_t(v >> nbo) + dfs[s]];
  };
  auto encode = [&](uint32_t& st, uint32_t s) {
    const uint32_t nbo = uint32_t((int32_t(st) + dnb[s]) >> 16);
    b.put(st & ((1u << nbo) - 1u), nbo);
    st = state_tab[int32_t(st >> nbo) + dfs[s]];
  };
  int32_t i = int32_t(nw);
  uint32_t s1, s2;
  if (nw & 1u) {
    s1 = init_state(w[--i]);
    s2 = init_state(w[--i]);
    encode(s1, w[--i]);
  } else {
    s2 = init_state(w[--i]);
    s1 = init_state(w[--i]);
  }
  while (i > 0) {
    encode(s2, w[--i]);
    encode(s1, w[--i]);
  }
  b.put(s2 & mask, kFseLog);
  b.put(s1 & mask, kFseLog);
  b.put(1, 1);  // end mark
  return b.bytes() <= cap ? b.bytes() : 0u;
}

// Huffman tree description (4.2.1) of weight[0..last-1] (the last present
// symbol's weight is implied): FSE compressed when that is possible and
// smaller, else 4-bit weights when there are at most 128.  Returns the bytes
// written to `out` (kDescMax room), or 0 when the weights cannot be described.
VOOM_HD uint32_t huf_write_desc(const uint8_t* weight, uint32_t last, uint8_t* out) {
  const uint32_t nw = last;
  uint32_t cnt[16] = {0};
  uint32_t maxw = 0, distinct = 0;
  for (uint32_t s = 0; s < nw; s++) {
    cnt[weight[s]]++;
    maxw = weight[s] > maxw ? weight[s] : maxw;
  }
  for (uint32_t v = 0; v <= maxw; v++) distinct += cnt[v] ? 1u : 0u;
  uint32_t fse_bytes = 0;
  if (nw >= 2 && distinct >= 2) {
    int16_t norm[16];
    fse_normalize(cnt, maxw, nw, norm);
    BitOut hb{out + 1, kDescMax - 1, 0};
    fse_write_ncount(hb, norm, maxw);
    const uint32_t hdr = hb.bytes();
    if (hdr < kDescMax - 1) {
      const uint32_t sb = fse_encode_weights(weight, nw, norm, maxw, out + 1 + hdr, kDescMax - 1 - hdr);
      if (sb && hdr + sb < 128) fse_bytes = hdr + sb;
    }
  }
  const uint32_t direct = nw <= 128 ? 1 + (nw + 1) / 2 : 0;
  if (fse_bytes && (!direct || fse_bytes + 1 <= direct)) {
    out[0] = uint8_t(fse_bytes);
    return 1 + fse_bytes;
  }
  if (direct && nw >= 1) {
    out[0] = uint8_t(127 + nw);
    for (uint32_t s = 0; s < nw; s += 2)
      out[1 + s / 2] = uint8_t((weight[s] << 4) | (s + 1 < nw ? weight[s + 1] : 0u));
    return direct;
  }
  return 0;
}

// Frame header: magic, single segment, content size, no checksum or
// dictionary (3.1.1.1).  Returns its length (<= 13).
VOOM_HD uint32_t frame_header(uint64_t content, uint8_t* p) {
  p[0] = 0x28;
  p[1] = 0xB5;
  p[2] = 0x2F;
  p[3] = 0xFD;
  uint32_t flag, nb;
  uint64_t v = content;
  if (content < 256) {
    flag = 0;
    nb = 1;
  } else if (content < 65536 + 256) {
    flag = 1;
    nb = 2;
    v -= 256;
  } else if (content <= 0xFFFFFFFFull) {
    flag = 2;
    nb = 4;
  } else {
    flag = 3;
    nb = 8;
  }
  p[4] = uint8_t((flag << 6) | (1u << 5));
  for (uint32_t i = 0; i < nb; i++) p[5 + i] = uint8_t(v >> (8 * i));
  return 5 + nb;
}

// Block header (3.1.1.2): last flag, type (0 raw, 2 compressed), size.
VOOM_HD void block_header(uint8_t* p, bool last, uint32_t type, uint32_t size) {
  const uint32_t h = (last ? 1u : 0u) | (type << 1) | (size << 3);
  p[0] = uint8_t(h);
  p[1] = uint8_t(h >> 8);
  p[2] = uint8_t(h >> 16);
}

// Literals section header of Huffman-coded four-stream literals
// (3.1.1.3.1.1): the smallest size format holding both sizes.
VOOM_HD uint32_t lit_header_bytes(uint32_t regen, uint32_t comp) {
  const uint32_t m = regen > comp ? regen : comp;
  return m < 1024 ? 3u : (m < 16384 ? 4u : 5u);
}

VOOM_HD void lit_header(uint8_t* p, uint32_t regen, uint32_t comp) {
  const uint32_t n = lit_header_bytes(regen, comp);
  const uint32_t sf = n == 3 ? 1u : (n == 4 ? 2u : 3u);
  const uint32_t bits = n == 3 ? 10u : (n == 4 ? 14u : 18u);
  const uint64_t h = 2ull | (uint64_t(sf) << 2) | (uint64_t(regen) << 4) | (uint64_t(comp) << (4 + bits));
  for (uint32_t i = 0; i < n; i++) p[i] = uint8_t(h >> (8 * i));
}

// RLE literals header (one repeated byte), 3 bytes (20-bit size).
VOOM_HD void rle_header(uint8_t* p, uint32_t regen) {
  const uint32_t h = 1u | (3u << 2) | (regen << 4);
  p[0] = uint8_t(h);
  p[1] = uint8_t(h >> 8);
  p[2] = uint8_t(h >> 16);
}

// Canonical prefix code of every symbol from the weights (4.2.1.3: codes
// ascend with weight, symbols ascending within a weight, the first code of a
// weight being (first + count of the previous weight) >> 1).
VOOM_HD uint32_t huf_code(const uint8_t* weight, const uint32_t* first_code, uint32_t s) {
  const uint32_t w = weight[s];
  uint32_t rank = 0;
  for (uint32_t t = 0; t < s; t++) rank += weight[t] == w ? 1u : 0u;
  return first_code[w] + rank;
}

VOOM_HD void huf_first_codes(const uint8_t* weight, uint32_t maxbits, uint32_t* first_code) {
  uint32_t per_w[kMaxBits + 2] = {0};
  for (uint32_t s = 0; s < 256; s++)
    if (weight[s]) per_w[weight[s]]++;
  first_code[1] = 0;
  for (uint32_t w = 2; w <= maxbits; w++) first_code[w] = (first_code[w - 1] + per_w[w - 1]) >> 1;
}

}  // namespace zenc
}  // namespace voom
