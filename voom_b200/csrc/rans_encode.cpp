// Pack-side VRN1 encoder (host, multi-threaded over tiles).
//
// Produces frames byte-identical to formats/bf16_rans.py encode() (:148-177):
// per tile, each byte plane gets a 12-bit static model normalised as in
// _normalize_frequencies (:36-58) and is rANS-coded in reverse symbol order
// (_encode_plane, :72-94); a tile whose coded form is not smaller than its raw
// bytes is stored verbatim (mode 0).  Tiles are independent, so worker
// threads encode disjoint tile ranges into private buffers that are then
// concatenated in tile order.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/voom_b200.h"

#define VOOM_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr uint32_t kScaleBits = 12;
constexpr uint32_t kTotal = 1u << kScaleBits;
constexpr uint32_t kRansL = 1u << 23;
constexpr size_t kPlaneHdr = 4 + 512;

uint32_t crc_tab[256];
struct CrcInit {
  CrcInit() {
    for (uint32_t n = 0; n < 256; n++) {
      uint32_t c = n;
      for (int k = 0; k < 8; k++) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      crc_tab[n] = c;
    }
  }
} crc_init_once;

uint32_t crc32_host(const uint8_t* p, size_t n) {
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; i++) c = crc_tab[(c ^ p[i]) & 0xFF] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

void put32(std::vector<uint8_t>& v, uint32_t x) {
  for (int i = 0; i < 4; i++) v.push_back(uint8_t(x >> (8 * i)));
}

// Frequencies of the plane data[0], data[stride], ... (n symbols).
void normalize(const uint8_t* data, size_t n, size_t stride, uint32_t freq[256]) {
  uint64_t counts[256] = {0};
  for (size_t i = 0; i < n; i++) counts[data[i * stride]]++;
  memset(freq, 0, 256 * sizeof(uint32_t));
  int active = 0;
  for (int s = 0; s < 256; s++) active += counts[s] != 0;
  if (!active) return;
  const uint64_t remaining = kTotal - uint64_t(active);
  uint64_t assigned = 0;
  struct Frac { uint64_t rem, count; int sym; };
  Frac fr[256];
  int nf = 0;
  for (int s = 0; s < 256; s++) {
    if (!counts[s]) continue;
    uint64_t scaled = counts[s] * remaining;
    uint64_t extra = scaled / n;
    freq[s] = uint32_t(1 + extra);
    assigned += extra;
    fr[nf++] = Frac{scaled % n, counts[s], s};
  }
  // largest remainder first; ties: larger count, then smaller symbol
  std::sort(fr, fr + nf, [](const Frac& a, const Frac& b) {
    if (a.rem != b.rem) return a.rem > b.rem;
    if (a.count != b.count) return a.count > b.count;
    return a.sym < b.sym;
  });
  uint64_t left = remaining - assigned;
  for (uint64_t i = 0; i < left && i < uint64_t(nf); i++) freq[fr[i].sym]++;
}

void encode_plane(const uint8_t* data, size_t n, size_t stride, std::vector<uint8_t>& out,
                  std::vector<uint8_t>& scratch) {
  uint32_t freq[256], cum[256];
  if (n == 0) {
    put32(out, 4);
    out.insert(out.end(), 512, 0);
    put32(out, kRansL);
    return;
  }
  normalize(data, n, stride, freq);
  uint32_t t = 0;
  for (int s = 0; s < 256; s++) { cum[s] = t; t += freq[s]; }
  scratch.clear();
  uint64_t state = kRansL;
  for (size_t i = n; i-- > 0;) {
    const uint8_t s = data[i * stride];
    const uint64_t f = freq[s];
    const uint64_t threshold = (uint64_t(kRansL >> kScaleBits) << 8) * f;
    while (state >= threshold) {
      scratch.push_back(uint8_t(state & 0xFF));
      state >>= 8;
    }
    state = ((state / f) << kScaleBits) + (state % f) + cum[s];
  }
  put32(out, uint32_t(4 + scratch.size()));
  for (int s = 0; s < 256; s++) { out.push_back(uint8_t(freq[s])); out.push_back(uint8_t(freq[s] >> 8)); }
  put32(out, uint32_t(state));
  out.insert(out.end(), scratch.rbegin(), scratch.rend());
}

void encode_tile(const uint8_t* raw, size_t len, std::vector<uint8_t>& out,
                 std::vector<uint8_t>& coded, std::vector<uint8_t>& scratch, bool& compressed) {
  coded.clear();
  encode_plane(raw, (len + 1) / 2, 2, coded, scratch);
  encode_plane(raw + 1, len / 2, 2, coded, scratch);
  const uint32_t crc = crc32_host(raw, len);
  compressed = coded.size() < len;
  out.push_back(compressed ? 1 : 0);
  put32(out, uint32_t(len));
  put32(out, uint32_t(compressed ? coded.size() : len));
  put32(out, crc);
  if (compressed) out.insert(out.end(), coded.begin(), coded.end());
  else out.insert(out.end(), raw, raw + len);
}

}  // namespace

// Encodes `n` bytes into a VRN1 frame (formats/bf16_rans.py:148-177).
// Call with h_out == NULL to get the worst-case capacity in *out_len; then
// with a buffer of that capacity.  threads <= 0 uses the hardware count.
// stats (may be NULL): [0] tiles, [1] compressed tiles.
VOOM_API int voom_rans_encode(const uint8_t* h_data, uint64_t n, uint32_t tile_bytes, uint8_t* h_out,
                              uint64_t out_cap, uint64_t* out_len, uint64_t* stats, int threads) {
  if (!out_len || tile_bytes == 0 || (n && !h_data)) return VOOM_E_INVALID_ARG;
  if (n > 0xFFFFFFFFull) return VOOM_E_UNSUPPORTED;  // raw_size is a u32 field
  const uint64_t tiles = (n + tile_bytes - 1) / tile_bytes;
  const uint64_t worst = 16 + tiles * 13 + n;  // every tile stored verbatim at worst
  if (!h_out) {
    *out_len = worst;
    return VOOM_OK;
  }
  if (out_cap < 16) return VOOM_E_CAPACITY;
  int nt = threads > 0 ? threads : int(std::max(1u, std::thread::hardware_concurrency()));
  nt = int(std::min<uint64_t>(uint64_t(nt), std::max<uint64_t>(tiles, 1)));
  std::vector<std::vector<uint8_t>> parts(static_cast<size_t>(nt));
  std::vector<uint64_t> ncomp(static_cast<size_t>(nt), 0);
  auto work = [&](int w) {
    std::vector<uint8_t> coded, scratch;
    const uint64_t t0 = tiles * uint64_t(w) / uint64_t(nt), t1 = tiles * uint64_t(w + 1) / uint64_t(nt);
    for (uint64_t t = t0; t < t1; t++) {
      const uint64_t off = t * tile_bytes;
      const size_t len = size_t(std::min<uint64_t>(tile_bytes, n - off));
      bool comp = false;
      encode_tile(h_data + off, len, parts[size_t(w)], coded, scratch, comp);
      ncomp[size_t(w)] += comp;
    }
  };
  std::vector<std::thread> pool;
  for (int w = 1; w < nt; w++) pool.emplace_back(work, w);
  work(0);
  for (auto& th : pool) th.join();
  uint64_t total = 16;
  for (auto& p : parts) total += p.size();
  if (total > out_cap) return VOOM_E_CAPACITY;
  memcpy(h_out, "VRN1", 4);
  uint32_t hdr[3] = {uint32_t(n), tile_bytes, uint32_t(tiles)};
  for (int i = 0; i < 3; i++)
    for (int b = 0; b < 4; b++) h_out[4 + 4 * i + b] = uint8_t(hdr[i] >> (8 * b));
  uint64_t pos = 16, comp = 0;
  for (int w = 0; w < nt; w++) {
    memcpy(h_out + pos, parts[size_t(w)].data(), parts[size_t(w)].size());
    pos += parts[size_t(w)].size();
    comp += ncomp[size_t(w)];
  }
  *out_len = pos;
  if (stats) { stats[0] = tiles; stats[1] = comp; }
  return VOOM_OK;
}
