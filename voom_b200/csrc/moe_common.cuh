// Shared pieces of the fused MoE kernels: limits, the device route table
// and BF16 rounding helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace voom {
namespace moe {

constexpr int kThreads = 256;
constexpr int kTok = 8;          // tokens per expert pass
constexpr int kMaxTK = 512;      // T * top_k
constexpr int kMaxE = 1024;      // experts
constexpr int kMaxU = kMaxTK + 1;     // unique experts: the routed ones + the shared expert
constexpr int kMaxRows = 2 * kMaxTK;  // route rows: T * top_k routed + T shared (T <= kMaxTK)

// Families (which reference layer the math follows): VOOM_MOE_GENERIC,
// VOOM_MOE_QWEN35, VOOM_MOE_GLM (include/voom_b200.h).
constexpr uint32_t kNoShared = 0xFFFFFFFFu;

struct Routes {
  uint32_t n_unique;            // unique experts, the shared expert (if any) last
  uint32_t T, k, family;
  uint32_t expert[kMaxU];       // unique experts: first-appearance (generic) or ascending id order
  uint32_t ntok[kMaxU];         // tokens routed to unique expert u
  uint32_t uoff[kMaxU + 1];     // first route row of unique expert u
  uint32_t upair[kMaxRows];     // [uoff[u] + i] -> token of the i-th route of u
  uint32_t tok_order[kMaxTK];   // [t*k + j] -> route row, sorted by u per token
  uint16_t w_bf16[kMaxRows];    // [route row] route weight in BF16 (generic, qwen35)
  float w_row[kMaxRows];        // [route row] route weight in fp32 (glm)
  uint32_t idx[kMaxTK];         // [t*k + j] expert
  float w[kMaxTK];              // [t*k + j] route weight (fp32)
  uint16_t sgate[kMaxTK];       // qwen35: bf16(sigmoid(bf16(h_t . Wsg))) per token
  uint32_t shared_u;            // unique index of the shared expert, or kNoShared
  uint32_t n_rows;              // route rows in use
  // the unique experts this GPU computes (all of them unless expert
  // parallelism assigns owners): owned[0 .. n_owned), and mine[u] = 1 for those
  uint32_t n_owned;
  uint32_t owned[kMaxU];
  uint8_t mine[kMaxU];
  uint16_t row_u[kMaxRows];     // [route row] unique expert of the row
};

__device__ __forceinline__ float bf2f(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ uint32_t f2bf(float f) {  // round to nearest even
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u) return (u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

}  // namespace moe
}  // namespace voom
