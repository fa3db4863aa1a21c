// GPU zstd compression into valid RFC 8878 frames (the KV-page spill codec:
// runtime/kv_paged.py:77-96 compresses each page's K and V with zstd level
// 1; any frame zstd.decompress accepts gives the same page back).
//
// One CTA of 256 threads per block of at most 32 KiB:
//   histogram (shared atomics) -> symbols sorted by (count, symbol) with a
//   bitonic sort -> Huffman code lengths (two-queue construction by one
//   thread, counts halved until no code is longer than 11 bits) -> zstd
//   weights and their description (FSE or 4-bit, one thread) -> canonical
//   codes (one thread per symbol) -> the four literal streams: each thread
//   takes a run of a stream's symbols, the runs' bit offsets come from a
//   scan of their code lengths in reverse (a Huffman stream is read from its
//   end, so the first symbol's code sits at the top), and every code is OR-ed
//   into a shared-memory bit buffer -> headers -> one coalesced copy out.
// A block whose Huffman form would not be smaller becomes a Raw block; a
// block of one repeated byte becomes RLE literals.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "zstd_enc.cuh"

using namespace voom;
using namespace voom::zenc;

namespace {

constexpr int kEncThreads = 256;
constexpr int kPerStream = kEncThreads / 4;  // threads per literal stream

struct EncShared {
  uint32_t out[kSlotBytes / 4 + 1];
  uint32_t hist[256];
  uint32_t key[256];
  uint32_t iw[256];
  uint32_t bits[kEncThreads];     // code bits of each thread's run
  uint32_t first_code[kMaxBits + 2];
  uint32_t stream_bits[4];
  uint16_t parent[512];
  uint16_t sorted[256];
  uint16_t code[256];
  uint8_t len[256];
  uint8_t weight[256];
  uint8_t desc[kDescMax + 3];
  uint32_t n_present, last, maxbits, desc_len, mode;
};

enum : uint32_t { kModeHuf = 0, kModeRle = 1, kModeRaw = 2 };

__device__ __forceinline__ uint8_t* obytes(EncShared& sh) { return reinterpret_cast<uint8_t*>(sh.out); }

// ORs the low nb bits of v into the bit buffer at bit position p.
__device__ __forceinline__ void or_bits(EncShared& sh, uint32_t p, uint32_t v, uint32_t nb) {
  if (!nb) return;
  const uint64_t x = uint64_t(v & ((1u << nb) - 1u)) << (p & 31u);
  atomicOr(&sh.out[p >> 5], uint32_t(x));
  if ((p & 31u) + nb > 32u) atomicOr(&sh.out[(p >> 5) + 1], uint32_t(x >> 32));
}

__global__ void __launch_bounds__(kEncThreads) zstd_encode_block(const uint8_t* __restrict__ src,
                                                                 const voom_zenc_block* __restrict__ blocks,
                                                                 uint8_t* __restrict__ slots,
                                                                 uint32_t* __restrict__ sizes) {
  __shared__ EncShared sh;
  const uint32_t tid = threadIdx.x;
  const voom_zenc_block B = blocks[blockIdx.x];
  const uint8_t* in = src + B.src;
  const uint32_t n = min(B.len, kEncBlock);  // the host splits frames into blocks of at most kEncBlock
  uint8_t* ob = obytes(sh);
  for (uint32_t i = tid; i < kSlotBytes / 4 + 1; i += kEncThreads) sh.out[i] = 0;
  sh.hist[tid] = 0;
  sh.len[tid] = 0;
  sh.weight[tid] = 0;
  if (tid == 0) sh.last = 0;
  __syncthreads();
  for (uint32_t i = tid; i < n; i += kEncThreads) atomicAdd(&sh.hist[__ldg(in + i)], 1u);
  __syncthreads();
  const uint32_t present = __syncthreads_count(sh.hist[tid] != 0);
  if (sh.hist[tid]) atomicMax(&sh.last, tid);
  if (tid == 0) {
    sh.n_present = present;
    sh.mode = n < 64 ? kModeRaw : (present == 1 ? kModeRle : kModeHuf);
  }
  __syncthreads();
  const uint32_t block_at = kHdrRoom;  // block header position in the slot
  uint32_t body = 0;                   // block content bytes (after the block header)
  if (sh.mode == kModeHuf) {
    // code lengths; counts halved until the longest code fits 11 bits
    for (int iter = 0; iter < 32; iter++) {
      sh.key[tid] = sh.hist[tid] ? ((sh.hist[tid] << 8) | tid) : 0xFFFFFFFFu;
      __syncthreads();
      for (uint32_t k = 2; k <= 256; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
          const uint32_t o = tid ^ j;
          if (o > tid) {
            const uint32_t a = sh.key[tid], b = sh.key[o];
            if ((a > b) == ((tid & k) == 0)) {
              sh.key[tid] = b;
              sh.key[o] = a;
            }
          }
          __syncthreads();
        }
      }
      sh.sorted[tid] = uint16_t(sh.key[tid] & 0xFFu);
      __syncthreads();
      if (tid == 0) sh.maxbits = huf_lengths(sh.sorted, sh.hist, sh.n_present, sh.len, sh.parent, sh.iw);
      __syncthreads();
      if (sh.maxbits <= kMaxBits) break;
      if (sh.hist[tid]) sh.hist[tid] = max(1u, sh.hist[tid] >> 1);
      __syncthreads();
    }
    const uint32_t maxbits = sh.maxbits;
    sh.weight[tid] = sh.len[tid] ? uint8_t(maxbits + 1 - sh.len[tid]) : uint8_t(0);
    __syncthreads();
    if (tid == 0) {
      sh.desc_len = maxbits <= kMaxBits ? huf_write_desc(sh.weight, sh.last, sh.desc) : 0u;
      huf_first_codes(sh.weight, maxbits, sh.first_code);
    }
    __syncthreads();
    if (sh.desc_len == 0) {
      if (tid == 0) sh.mode = kModeRaw;
    } else {
      sh.code[tid] = sh.weight[tid] ? uint16_t(huf_code(sh.weight, sh.first_code, tid)) : uint16_t(0);
      // each stream's runs and their code bits
      const uint32_t seg = (n + 3) / 4, s = tid / kPerStream, j = tid % kPerStream;
      const uint32_t s0 = s * seg, s1 = min(n, s0 + seg);
      const uint32_t run = (seg + kPerStream - 1) / kPerStream;
      const uint32_t r0 = min(s1, s0 + j * run), r1 = min(s1, r0 + run);
      __syncthreads();
      uint32_t nbits = 0;
      for (uint32_t i = r0; i < r1; i++) nbits += sh.len[__ldg(in + i)];
      sh.bits[tid] = nbits;
      __syncthreads();
      // bit offset of the run: the code bits of the later runs of its stream
      uint32_t off = 0;
      for (uint32_t t = j + 1; t < uint32_t(kPerStream); t++) off += sh.bits[s * kPerStream + t];
      if (j == 0) sh.stream_bits[s] = off + nbits;
      __syncthreads();
      uint32_t sbytes[4], comp = sh.desc_len + 6;
      for (int q = 0; q < 4; q++) {
        sbytes[q] = (sh.stream_bits[q] + 1 + 7) / 8;  // with the end mark
        comp += sbytes[q];
      }
      const uint32_t lh = lit_header_bytes(n, comp);
      body = lh + comp + 1;  // + the sequences section (zero sequences)
      if (body >= n) {
        if (tid == 0) sh.mode = kModeRaw;
      } else {
        uint32_t sb = block_at + 3 + lh + sh.desc_len + 6;
        for (uint32_t q = 0; q < s; q++) sb += sbytes[q];
        // codes of the run, last symbol first (lowest bits)
        uint32_t p = 8 * sb + off;
        for (uint32_t i = r1; i > r0; i--) {
          const uint32_t c = __ldg(in + i - 1);
          or_bits(sh, p, sh.code[c], sh.len[c]);
          p += sh.len[c];
        }
        if (j == 0) or_bits(sh, 8 * sb + sh.stream_bits[s], 1u, 1u);  // end mark
        // headers go in after every bit is in (byte stores must not race the
        // word atomics); the zeroed buffer already holds Number_of_Sequences = 0
        __syncthreads();
        if (tid == 0) {
          uint8_t* q = ob + block_at + 3;
          lit_header(q, n, comp);
          q += lh;
          for (uint32_t i = 0; i < sh.desc_len; i++) q[i] = sh.desc[i];
          q += sh.desc_len;
          for (int k = 0; k < 3; k++) {
            q[2 * k] = uint8_t(sbytes[k]);
            q[2 * k + 1] = uint8_t(sbytes[k] >> 8);
          }
        }
      }
    }
    __syncthreads();
  }
  const uint32_t mode = sh.mode;
  if (mode == kModeRle) {
    body = 5;
    if (tid == 0) {
      rle_header(ob + block_at + 3, n);
      ob[block_at + 6] = uint8_t(sh.last);
      ob[block_at + 7] = 0;
    }
  } else if (mode == kModeRaw) {
    body = n;
  }
  uint32_t start = block_at;
  if (tid == 0) {
    block_header(ob + block_at, (B.flags & VOOM_ZENC_LAST) != 0, mode == kModeRaw ? 0u : 2u, body);
    if (B.flags & VOOM_ZENC_FIRST) {
      uint8_t fh[16];
      const uint32_t fl = frame_header(B.frame_len, fh);
      for (uint32_t i = 0; i < fl; i++) ob[block_at - fl + i] = fh[i];
    }
  }
  __syncthreads();
  if (B.flags & VOOM_ZENC_FIRST) {
    uint8_t fh[16];
    start = block_at - frame_header(B.frame_len, fh);
  }
  uint8_t* dst = slots + uint64_t(blockIdx.x) * kSlotBytes;
  const uint32_t head_end = mode == kModeRaw ? block_at + 3 : block_at + 3 + body;
  for (uint32_t i = start + tid; i < head_end; i += kEncThreads) dst[i] = ob[i];
  if (mode == kModeRaw)
    for (uint32_t i = tid; i < n; i += kEncThreads) dst[block_at + 3 + i] = __ldg(in + i);
  if (tid == 0) {
    sizes[2 * blockIdx.x] = start;
    sizes[2 * blockIdx.x + 1] = block_at + 3 + body - start;
  }
}

// Packs every block's bytes (slot offset and length from the encoder's sizes)
// to d_dst[b] in one buffer: one CTA per block, 16-byte copies where the two
// ends line up.
__global__ void __launch_bounds__(256) zstd_encode_pack(const uint8_t* __restrict__ slots,
                                                        const uint32_t* __restrict__ sizes,
                                                        const uint64_t* __restrict__ dst,
                                                        uint8_t* __restrict__ out) {
  const uint32_t b = blockIdx.x;
  const uint8_t* s = slots + uint64_t(b) * kSlotBytes + sizes[2 * b];
  const uint32_t n = sizes[2 * b + 1];
  uint8_t* d = out + dst[b];
  const uint32_t head = uint32_t((16u - (reinterpret_cast<uintptr_t>(d) & 15u)) & 15u);
  if (((reinterpret_cast<uintptr_t>(s) + head) & 15u) == 0 && n > head + 16) {
    for (uint32_t i = threadIdx.x; i < head; i += blockDim.x) d[i] = s[i];
    const uint32_t nv = (n - head) / 16;
    const uint4* sv = reinterpret_cast<const uint4*>(s + head);
    uint4* dv = reinterpret_cast<uint4*>(d + head);
    for (uint32_t i = threadIdx.x; i < nv; i += blockDim.x) dv[i] = sv[i];
    for (uint32_t i = head + 16 * nv + threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
  } else {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
  }
}

}  // namespace

VOOM_API int voom_zstd_encode_pack(const uint8_t* d_slots, const uint32_t* d_sizes, const uint64_t* d_dst,
                                   uint32_t n_blocks, uint8_t* d_out, void* stream) {
  if (!n_blocks) return VOOM_OK;
  if (!d_slots || !d_sizes || !d_dst || !d_out) return VOOM_E_INVALID_ARG;
  zstd_encode_pack<<<n_blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_slots, d_sizes, d_dst, d_out);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}

VOOM_API uint64_t voom_zstd_encode_slot_bytes(void) { return kSlotBytes; }
VOOM_API uint32_t voom_zstd_encode_block_bytes(void) { return kEncBlock; }

VOOM_API int voom_zstd_encode(const uint8_t* d_src, const voom_zenc_block* d_blocks, uint32_t n_blocks,
                              uint8_t* d_slots, uint32_t* d_sizes, void* stream) {
  if (!n_blocks) return VOOM_OK;
  if (!d_src || !d_blocks || !d_slots || !d_sizes) return VOOM_E_INVALID_ARG;
  zstd_encode_block<<<n_blocks, kEncThreads, 0, static_cast<cudaStream_t>(stream)>>>(d_src, d_blocks, d_slots,
                                                                                       d_sizes);
  return cudaGetLastError() == cudaSuccess ? VOOM_OK : VOOM_E_CUDA;
}
