// Host gather + parse of compressed KV spill pages (`.kvz`).
//
// A `.kvz` page is the pickle the reference writes in runtime/kv_paged.py:86-88:
// a dict {"shape": tuple of ints, "k": bytes, "v": bytes} where "k" / "v" are
// zstd level-1 frames of the raw BF16 K and V bits.  Reload (kv_paged.py:98-113)
// unpickles it and zstd-decompresses both frames.  Here many pages are copied
// into one pinned host buffer by worker threads and each page's pickle is walked
// in place to find the two frames and the shape, so one DMA and one batched GPU
// decode reload every page without a Python object per frame.
//
// The walker accepts the opcodes a pickler of protocol 3-5 emits for such a dict
// (frames, memo puts and gets, str keys, small ints, tuples, bytes); anything
// else marks the page unparsed and the caller unpickles that page itself.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

#include "../../include/voom_b200.h"

#define VOOM_API extern "C" __attribute__((visibility("default")))

namespace {

enum Kind : uint8_t { kMark, kStr, kBytes, kInt, kTuple, kDict, kOther };

struct Item {
  Kind kind;
  uint8_t ndim;   // tuple: element count (all ints, at most 8)
  uint64_t a, b;  // str / bytes: offset, length; int: value
  int64_t dims[8];
};

inline uint64_t rd(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = 0; i < n; i++) v |= uint64_t(p[i]) << (8 * i);
  return v;
}

// Walks one pickle of `n` bytes at `p` (offsets recorded relative to `base`).
bool walk(const uint8_t* p, uint64_t n, uint64_t base, voom_kvz_page& pg) {
  Item st[64];
  Item memo[64];
  for (auto& m : memo) m.kind = kOther;
  int sp = 0, nmemo = 0;
  bool have_shape = false, have_k = false, have_v = false, done = false;
  uint64_t i = 0;
  auto need = [&](uint64_t k) { return i + k <= n; };
  auto push = [&](const Item& it) {
    if (sp >= 64) return false;
    st[sp++] = it;
    return true;
  };
  auto assign = [&](const Item& key, const Item& val) {
    if (key.kind != kStr) return true;  // non-str keys are not ours: ignore
    const uint8_t* s = p + (key.a - base);
    if (key.b == 5 && memcmp(s, "shape", 5) == 0) {
      if (val.kind != kTuple) return false;
      pg.ndim = val.ndim;
      for (int d = 0; d < val.ndim; d++) pg.shape[d] = val.dims[d];
      have_shape = true;
    } else if (key.b == 1 && (s[0] == 'k' || s[0] == 'v')) {
      if (val.kind != kBytes) return false;
      if (s[0] == 'k') {
        pg.k_off = val.a;
        pg.k_len = val.b;
        have_k = true;
      } else {
        pg.v_off = val.a;
        pg.v_len = val.b;
        have_v = true;
      }
    }
    return true;
  };
  while (i < n && !done) {
    const uint8_t op = p[i++];
    Item it;
    memset(&it, 0, sizeof it);
    switch (op) {
      case 0x80:  // PROTO
        if (!need(1) || p[i] < 3) return false;
        i += 1;
        break;
      case 0x95:  // FRAME
        if (!need(8)) return false;
        i += 8;
        break;
      case '}':  // EMPTY_DICT
        it.kind = kDict;
        if (!push(it)) return false;
        break;
      case '(':  // MARK
        it.kind = kMark;
        if (!push(it)) return false;
        break;
      case 0x94:  // MEMOIZE
        if (sp == 0 || nmemo >= 64) return false;
        memo[nmemo++] = st[sp - 1];
        break;
      case 'q':  // BINPUT
      case 'r': {  // LONG_BINPUT
        const int w = op == 'q' ? 1 : 4;
        if (!need(w) || sp == 0) return false;
        const uint64_t idx = rd(p + i, w);
        i += w;
        if (idx >= 64) return false;
        memo[idx] = st[sp - 1];
        nmemo = std::max<int>(nmemo, int(idx) + 1);
        break;
      }
      case 'h':  // BINGET
      case 'j': {  // LONG_BINGET
        const int w = op == 'h' ? 1 : 4;
        if (!need(w)) return false;
        const uint64_t idx = rd(p + i, w);
        i += w;
        if (idx >= uint64_t(nmemo)) return false;
        if (!push(memo[idx])) return false;
        break;
      }
      case 0x8c:  // SHORT_BINUNICODE
      case 'X':   // BINUNICODE
      case 0x8d:  // BINUNICODE8
      case 'C':   // SHORT_BINBYTES
      case 'B':   // BINBYTES
      case 0x8e: {  // BINBYTES8
        const int w = (op == 0x8c || op == 'C') ? 1 : ((op == 'X' || op == 'B') ? 4 : 8);
        if (!need(w)) return false;
        const uint64_t len = rd(p + i, w);
        i += w;
        if (len > n - i) return false;
        it.kind = (op == 'C' || op == 'B' || op == 0x8e) ? kBytes : kStr;
        it.a = base + i;
        it.b = len;
        i += len;
        if (!push(it)) return false;
        break;
      }
      case 'K':  // BININT1
      case 'M':  // BININT2
      case 'J': {  // BININT (signed)
        const int w = op == 'K' ? 1 : (op == 'M' ? 2 : 4);
        if (!need(w)) return false;
        uint64_t v = rd(p + i, w);
        i += w;
        it.kind = kInt;
        it.a = op == 'J' ? uint64_t(int64_t(int32_t(uint32_t(v)))) : v;
        if (!push(it)) return false;
        break;
      }
      case 0x8a: {  // LONG1: little-endian two's complement, up to 8 bytes here
        if (!need(1)) return false;
        const int w = p[i++];
        if (w > 8 || !need(w)) return false;
        uint64_t v = rd(p + i, w);
        if (w > 0 && w < 8 && (p[i + w - 1] & 0x80)) v |= ~uint64_t(0) << (8 * w);
        i += w;
        it.kind = kInt;
        it.a = v;
        if (!push(it)) return false;
        break;
      }
      case ')':   // EMPTY_TUPLE
      case 0x85:  // TUPLE1
      case 0x86:  // TUPLE2
      case 0x87:  // TUPLE3
      case 't': {  // TUPLE (to the mark)
        int k;
        if (op == 't') {
          int m = sp - 1;
          while (m >= 0 && st[m].kind != kMark) m--;
          if (m < 0) return false;
          k = sp - 1 - m;
        } else {
          k = op == ')' ? 0 : op - 0x84;
        }
        if (k > 8 || k > sp) return false;
        it.kind = kTuple;
        it.ndim = uint8_t(k);
        for (int d = 0; d < k; d++) {
          const Item& e = st[sp - k + d];
          if (e.kind != kInt) return false;
          it.dims[d] = int64_t(e.a);
        }
        sp -= k;
        if (op == 't') sp--;  // the mark
        if (!push(it)) return false;
        break;
      }
      case 's': {  // SETITEM
        if (sp < 3 || st[sp - 3].kind != kDict) return false;
        if (!assign(st[sp - 2], st[sp - 1])) return false;
        sp -= 2;
        break;
      }
      case 'u': {  // SETITEMS
        int m = sp - 1;
        while (m >= 0 && st[m].kind != kMark) m--;
        if (m < 1 || st[m - 1].kind != kDict || ((sp - 1 - m) & 1)) return false;
        for (int q = m + 1; q < sp; q += 2)
          if (!assign(st[q], st[q + 1])) return false;
        sp = m;
        break;
      }
      case '.':  // STOP
        if (sp != 1 || st[0].kind != kDict) return false;
        done = true;
        break;
      default:
        return false;
    }
  }
  return done && have_shape && have_k && have_v;
}

}  // namespace

VOOM_API int voom_kvz_gather(const uint64_t* h_src_addrs, const uint64_t* lens, const uint64_t* dst_offs,
                             uint32_t n, uint8_t* h_dst, voom_kvz_page* pages, int threads) {
  if (n && (!lens || !dst_offs || !h_dst || !pages)) return VOOM_E_INVALID_ARG;
  const int nt = std::max(1, std::min<int>(threads > 0 ? threads : int(std::thread::hardware_concurrency()),
                                           int(std::max<uint32_t>(1, n / 64))));
  std::atomic<uint32_t> next{0};
  auto run = [&]() {
    for (;;) {
      const uint32_t a = next.fetch_add(64);
      if (a >= n) break;
      const uint32_t b = std::min<uint32_t>(n, a + 64);
      for (uint32_t j = a; j < b; j++) {
        uint8_t* d = h_dst + dst_offs[j];
        if (h_src_addrs) memcpy(d, reinterpret_cast<const void*>(h_src_addrs[j]), lens[j]);
        voom_kvz_page& pg = pages[j];
        memset(&pg, 0, sizeof pg);
        pg.status = walk(d, lens[j], dst_offs[j], pg) ? 0u : 1u;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int w = 1; w < nt; w++) pool.emplace_back(run);
  run();
  for (auto& t : pool) t.join();
  return VOOM_OK;
}
