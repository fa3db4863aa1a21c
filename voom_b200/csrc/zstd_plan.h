// Private layout of the zstd decode plan image and scratch, shared by the
// host planner (zstd_plan.cpp) and the GPU kernels (zstd.cu).
#pragma once

#include <stdint.h>

namespace voom {
namespace zstd {

constexpr uint32_t kBlockMax = 128 * 1024;
constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr uint32_t kOutTile = 64 * 1024;  // Z-space bytes per output-pass work unit

struct ZJob {
  uint64_t src, src_len, dst, dst_len, lo_src;
  uint64_t zoff;  // first byte of this job in its segment's decoded space (Z-space)
  uint32_t flags;
  uint32_t frame_first, n_frames;
  uint32_t bad;  // structural error found by the planner: not decoded
  // 1: no block of the job has sequences and it is not interleaved, so the
  // planner knows every block's output offset: literals and raw / RLE bytes
  // are written straight to the output (no Z-space, no link words)
  uint32_t direct;
  uint32_t pad;
};

struct ZFrame {
  uint64_t fcs;  // frame content size, or ~0 when absent
  uint32_t block_first, n_blocks;
  uint32_t job;
  uint32_t csum_flag, csum;
  uint32_t pad;
};

struct ZBlock {
  uint64_t src;      // raw: bytes; rle: the byte; compressed: first literal stream byte
  uint64_t seq_src;  // compressed: sequence bitstream
  uint64_t lit_off;  // literal scratch offset of this block
  uint64_t seq_off;  // first sequence record of this block
  uint64_t out_off;  // direct jobs: output offset of the block within the job
  uint32_t type;     // 0 raw, 1 rle, 2 compressed
  uint32_t size;     // raw/rle: decoded bytes
  uint32_t frame;    // global frame index
  uint32_t job;
  uint32_t lit_type;  // 0 raw, 1 rle, 2 huffman
  uint32_t lit_regen;
  uint32_t lit_streams;
  uint32_t lit_len[4];
  uint32_t huf;
  uint32_t nseq;
  uint32_t seq_len;
  uint32_t fse[3];  // LL, OF, ML
  uint32_t max_out;  // largest decoded size a block of this frame may have
};

struct ZHuf {
  uint8_t w[256];  // weight of every symbol (last one already deduced)
  uint16_t nsym;
  uint8_t maxbits;
  uint8_t pad;
};

struct ZFse {
  int16_t norm[64];
  uint16_t nsym;
  uint8_t al;
  uint8_t rle;  // 1: single-symbol table (RLE mode)
  uint8_t rle_sym;
  uint8_t pad[3];
};

struct ZOutTile {
  uint32_t job;
  uint32_t pad;
  uint64_t begin;  // decoded-byte index within the job
  uint64_t len;
};

// Z positions are 31-bit (bit 31 of a link word flags a resolved byte), so the
// jobs that need match resolution are decoded in segments of at most kZSeg
// Z-space bytes; a job is never split, and one whose own Z size exceeds
// kZJobMax is refused.
constexpr uint64_t kZSeg = 1ull << 30;
constexpr uint64_t kZJobMax = (1ull << 31) - (1ull << 20);

// Contiguous job / frame / block / tile ranges of one segment (host only).
struct ZSegment {
  uint32_t job0, n_jobs, frame0, n_frames, block0, n_blocks, tile0, n_tiles;
  uint32_t bl0, n_bl;  // range of the block list (the blocks zstd_block_decode etc. run on)
  uint64_t zbytes;
};

// Plan image: this header followed by the arrays at the given byte offsets.
struct ZPlanHeader {
  uint32_t n_jobs, n_frames, n_blocks, n_huf, n_fse, n_tiles;
  uint64_t off_jobs, off_frames, off_blocks, off_huf, off_fse, off_tiles;
  // direct jobs' blocks with Huffman literals (global block indices): their
  // streams are decoded one lane each by zstd_direct_literals
  uint32_t n_dlit, pad_dlit;
  uint64_t off_dlit;
  // every other block (global indices, job order): the block decode, sequence
  // scan and block execute kernels run on this list, segment by segment
  uint32_t n_blist, pad_blist;
  uint64_t off_blist;
  // the same block list, each segment's range ordered by sequence count
  // (most first): the order zstd_block_decode pairs its walkers in
  uint64_t off_k1list;
  uint64_t lit_bytes, n_seq, zbytes;
  // scratch layout (byte offsets into d_scratch)
  uint64_t s_res, s_lit, s_seq, s_blk, s_ctr, s_list, s_total;
  uint64_t list_cap;  // entries per resolve worklist
};

// Per-sequence record in scratch.  The offset is stored symbolically, as
// the block decoder knows it before the block's repeat offsets are known:
// okind 0..2 = repeat slot okind at block start minus oval, 3 = constant oval.
struct ZSeq {
  uint32_t ll, ml;
  uint32_t oval, okind;
  uint32_t dst;  // block-relative output position of the literal run
  uint32_t lit;  // block-relative literal position
};

// Per-block runtime record in scratch.
struct ZBlockRt {
  uint64_t zstart;        // Z-space position of the block's first byte
  uint64_t frame_zstart;  // Z-space position of its frame's first byte
  uint32_t out_size;
  uint32_t status;
  uint32_t rep_kind[3];  // block repeat-offset transform: kind 0..2 = input slot, 3 = constant
  uint32_t rep_val[3];   // input slot minus val, or the constant
  uint32_t init_rep[3];  // repeat offsets at the block start
  uint32_t pad;
};

}  // namespace zstd
}  // namespace voom
