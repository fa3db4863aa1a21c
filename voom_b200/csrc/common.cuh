// Shared device helpers for the voom_b200 sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/voom_b200.h"

#define VOOM_API extern "C" __attribute__((visibility("default")))

namespace voom {

// ------------------------------------------------------------------ CRC-32
// zlib CRC-32: reflected polynomial 0xEDB88320, register preset 0xFFFFFFFF,
// final inversion.  Tables are generated at compile time.
constexpr uint32_t kCrcPoly = 0xEDB88320u;

struct CrcTables {
  uint32_t t[8][256];  // slicing-by-8
};

constexpr CrcTables make_crc_tables() {
  CrcTables c{};
  for (uint32_t n = 0; n < 256; n++) {
    uint32_t v = n;
    for (int k = 0; k < 8; k++) v = (v & 1u) ? kCrcPoly ^ (v >> 1) : v >> 1;
    c.t[0][n] = v;
  }
  for (int j = 1; j < 8; j++)
    for (uint32_t n = 0; n < 256; n++) c.t[j][n] = (c.t[j - 1][n] >> 8) ^ c.t[0][c.t[j - 1][n] & 0xFFu];
  return c;
}

// x^(2^k) mod P in reflected form (bit 31 = x^0), k = 0..63.
struct CrcPow2 {
  uint32_t p[64];
};

constexpr uint32_t gf2_mulmod_c(uint32_t a, uint32_t b) {
  uint32_t m = 1u << 31, p = 0;
  for (int i = 0; i < 32; i++) {
    if (a & m) p ^= b;
    m >>= 1;
    b = (b & 1u) ? (b >> 1) ^ kCrcPoly : b >> 1;
  }
  return p;
}

constexpr CrcPow2 make_crc_pow2() {
  CrcPow2 c{};
  c.p[0] = 1u << 30;  // x^1
  for (int k = 1; k < 64; k++) c.p[k] = gf2_mulmod_c(c.p[k - 1], c.p[k - 1]);
  return c;
}

__device__ __forceinline__ uint32_t gf2_mulmod(uint32_t a, uint32_t b) {
  uint32_t p = 0;
#pragma unroll 4
  for (int i = 31; i >= 0; i--) {
    p ^= (0u - ((a >> i) & 1u)) & b;
    b = (b >> 1) ^ ((0u - (b & 1u)) & kCrcPoly);
  }
  return p;
}

// x^(8 n) mod P: the operator "append n zero bytes" on a CRC register.
__device__ __forceinline__ uint32_t crc_zeros_op(const uint32_t* pow2, uint64_t nbytes) {
  uint64_t e = nbytes << 3;
  uint32_t r = 1u << 31;  // x^0
  int k = 0;
  while (e) {
    if (e & 1u) r = gf2_mulmod(r, pow2[k]);
    e >>= 1;
    k++;
  }
  return r;
}

// Advance a CRC register over 8 bytes (little-endian u64) with slicing-by-8.
__device__ __forceinline__ uint32_t crc_step8(const uint32_t (*t)[256], uint32_t c, uint32_t lo,
                                              uint32_t hi) {
  lo ^= c;
  return t[7][lo & 0xFFu] ^ t[6][(lo >> 8) & 0xFFu] ^ t[5][(lo >> 16) & 0xFFu] ^ t[4][lo >> 24] ^
         t[3][hi & 0xFFu] ^ t[2][(hi >> 8) & 0xFFu] ^ t[1][(hi >> 16) & 0xFFu] ^ t[0][hi >> 24];
}

__device__ __forceinline__ uint32_t crc_step1(const uint32_t (*t)[256], uint32_t c, uint32_t b) {
  return t[0][(c ^ b) & 0xFFu] ^ (c >> 8);
}

// Raw CRC register over [p, p+n) starting from `c` (no pre/post inversion).
__device__ __forceinline__ uint32_t crc_run(const uint32_t (*t)[256], uint32_t c, const uint8_t* p,
                                            uint64_t n) {
  while (n && (reinterpret_cast<uintptr_t>(p) & 15u)) {
    c = crc_step1(t, c, *p++);
    n--;
  }
  while (n >= 16) {
    uint4 v = __ldcg(reinterpret_cast<const uint4*>(p));
    c = crc_step8(t, c, v.x, v.y);
    c = crc_step8(t, c, v.z, v.w);
    p += 16;
    n -= 16;
  }
  while (n) {
    c = crc_step1(t, c, *p++);
    n--;
  }
  return c;
}

// Block-wide raw CRC register of [p, p+n) starting from `init` (no final
// inversion).  Every thread of the block must call it; `t` is the slicing
// table in shared memory, `pow2` the x^(2^k) table, `red` a shared scratch of
// blockDim.x/32 words.  Each thread folds an aligned slice, shifts its
// register to the end of the range (x^(8*bytes after it) mod P) and the
// registers are XOR-reduced.  Returns the register on every thread.
__device__ __forceinline__ uint32_t block_crc_reg(const uint32_t (*t)[256], const uint32_t* pow2,
                                                  const uint8_t* p, uint64_t n, uint32_t init,
                                                  uint32_t* red) {
  const uint32_t nt = blockDim.x, tid = threadIdx.x;
  uint64_t chunk = ((n + nt - 1) / nt + 15) & ~uint64_t(15);
  if (chunk == 0) chunk = 16;
  uint64_t b = (uint64_t)tid * chunk;
  uint64_t e = b + chunk;
  if (b > n) b = n;
  if (e > n) e = n;
  uint32_t c = crc_run(t, tid == 0 ? init : 0u, p + b, e - b);
  if (n - e) c = gf2_mulmod(crc_zeros_op(pow2, n - e), c);
  for (int o = 16; o; o >>= 1) c ^= __shfl_xor_sync(0xFFFFFFFFu, c, o);
  if ((tid & 31) == 0) red[tid >> 5] = c;
  __syncthreads();
  uint32_t r = 0;
  for (uint32_t w = 0; w < nt / 32; w++) r ^= red[w];
  __syncthreads();
  return r;
}

// Block-wide zlib CRC-32 of [p, p+n).
__device__ __forceinline__ uint32_t block_crc32(const uint32_t (*t)[256], const uint32_t* pow2,
                                                const uint8_t* p, uint64_t n, uint32_t* red) {
  return block_crc_reg(t, pow2, p, n, 0xFFFFFFFFu, red) ^ 0xFFFFFFFFu;
}

}  // namespace voom
