// Host build of the GPU zstd block encoder (voom_b200/csrc/zstd_enc.cu) --
// TEST INFRASTRUCTURE ONLY.  The planning code is the kernel's own
// (zstd_enc.cuh, compiled here for the CPU); the kernel's parallel steps
// (histogram, bitonic sort, per-symbol codes, the stream scan) are done
// serially with the same results, so the bytes must equal the GPU's.  The
// CPU tests hand its frames to libzstd; the GPU tests compare the kernel's
// frames with these.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../voom_b200/csrc/zstd_enc.cuh"

using namespace voom::zenc;

extern "C" uint32_t zenc_slot_bytes(void) { return kSlotBytes; }

// Encodes one block (n <= kEncBlock) into `slot` (kSlotBytes); returns the
// byte count and stores the first byte's offset in *start.
extern "C" uint32_t zenc_encode_block(const uint8_t* in, uint32_t n, uint64_t frame_len, uint32_t first,
                                      uint32_t last_block, uint8_t* slot, uint32_t* start) {
  memset(slot, 0, kSlotBytes);
  uint32_t hist[256] = {0};
  for (uint32_t i = 0; i < n; i++) hist[in[i]]++;
  uint32_t present = 0, last = 0;
  for (uint32_t s = 0; s < 256; s++)
    if (hist[s]) {
      present++;
      last = s;
    }
  const uint32_t block_at = kHdrRoom;
  enum { HUF, RLE, RAW } mode = n < 64 ? RAW : (present == 1 ? RLE : HUF);
  uint32_t body = 0;
  if (mode == HUF) {
    uint8_t len[256] = {0}, weight[256] = {0};
    uint16_t parent[512], sorted[256];
    uint32_t iw[256], maxbits = 0;
    for (int iter = 0; iter < 32; iter++) {
      std::vector<uint32_t> key;
      for (uint32_t s = 0; s < 256; s++) key.push_back(hist[s] ? ((hist[s] << 8) | s) : 0xFFFFFFFFu);
      std::sort(key.begin(), key.end());
      for (uint32_t i = 0; i < 256; i++) sorted[i] = uint16_t(key[i] & 0xFFu);
      maxbits = huf_lengths(sorted, hist, present, len, parent, iw);
      if (maxbits <= kMaxBits) break;
      for (uint32_t s = 0; s < 256; s++)
        if (hist[s]) hist[s] = std::max(1u, hist[s] >> 1);
    }
    for (uint32_t s = 0; s < 256; s++) weight[s] = len[s] ? uint8_t(maxbits + 1 - len[s]) : 0;
    uint8_t desc[kDescMax + 3];
    const uint32_t desc_len = maxbits <= kMaxBits ? huf_write_desc(weight, last, desc) : 0;
    uint32_t first_code[kMaxBits + 2];
    huf_first_codes(weight, maxbits, first_code);
    if (desc_len == 0) {
      mode = RAW;
    } else {
      uint16_t code[256];
      for (uint32_t s = 0; s < 256; s++) code[s] = weight[s] ? uint16_t(huf_code(weight, first_code, s)) : 0;
      const uint32_t seg = (n + 3) / 4;
      uint32_t bits[4], sbytes[4], comp = desc_len + 6;
      for (int q = 0; q < 4; q++) {
        const uint32_t a = std::min(n, q * seg), b = std::min(n, a + seg);
        bits[q] = 0;
        for (uint32_t i = a; i < b; i++) bits[q] += len[in[i]];
        sbytes[q] = (bits[q] + 1 + 7) / 8;
        comp += sbytes[q];
      }
      const uint32_t lh = lit_header_bytes(n, comp);
      body = lh + comp + 1;
      if (body >= n) {
        mode = RAW;
      } else {
        uint32_t sb = block_at + 3 + lh + desc_len + 6;
        for (int q = 0; q < 4; q++) {
          const uint32_t a = std::min(n, q * seg), b = std::min(n, a + seg);
          BitOut w{slot + sb, sbytes[q], 0};
          for (uint32_t i = b; i > a; i--) w.put(code[in[i - 1]], len[in[i - 1]]);
          w.put(1, 1);
          sb += sbytes[q];
        }
        uint8_t* p = slot + block_at + 3;
        lit_header(p, n, comp);
        p += lh;
        memcpy(p, desc, desc_len);
        p += desc_len;
        for (int k = 0; k < 3; k++) {
          p[2 * k] = uint8_t(sbytes[k]);
          p[2 * k + 1] = uint8_t(sbytes[k] >> 8);
        }
      }
    }
  }
  if (mode == RLE) {
    body = 5;
    rle_header(slot + block_at + 3, n);
    slot[block_at + 6] = uint8_t(last);
    slot[block_at + 7] = 0;
  } else if (mode == RAW) {
    body = n;
    memcpy(slot + block_at + 3, in, n);
  }
  block_header(slot + block_at, last_block != 0, mode == RAW ? 0u : 2u, body);
  uint32_t st = block_at;
  if (first) {
    uint8_t fh[16];
    const uint32_t fl = frame_header(frame_len, fh);
    memcpy(slot + block_at - fl, fh, fl);
    st = block_at - fl;
  }
  *start = st;
  return block_at + 3 + body - st;
}
