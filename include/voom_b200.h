/*
 * voom_b200.h - C ABI of the B200 (sm_100a) weight-page codec library.
 *
 * The library decodes vOOM's lossless BF16 weight-page formats on the GPU:
 *   - "VRN1" rANS frames            (reference: formats/bf16_rans.py)
 *   - vpack / vpack2 byte-plane bodies, zstd hi plane + raw lo plane
 *                                   (reference: formats/packed.py, formats/packed2.py)
 *   - kv_paged compressed spill pages (reference: runtime/kv_paged.py)
 * and fuses the rANS page decode with the MoE expert SwiGLU GEMV that consumes
 * the pages (reference: runtime/layer_runner.py _swiglu / run_moe_mlp).
 *
 * Conventions for every entry point:
 *   - Plain pointers and sizes only.  "d_" pointers are device memory, "h_"
 *     pointers are host memory.  `stream` is a cudaStream_t passed as void*.
 *   - Device entry points only enqueue work on `stream`; results (outputs and
 *     per-item status words) are valid once the stream has been synchronised.
 *   - Every entry point is re-entrant: no global mutable host state, so two
 *     host threads may call concurrently on different streams.
 *   - Return value: VOOM_OK, a negative VOOM_E_* for API misuse or a CUDA
 *     launch failure, or a positive format status (the codes below), which the
 *     Python layer maps to the exception the reference raises.
 */
#ifndef VOOM_B200_H
#define VOOM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum {
  VOOM_OK = 0,
  VOOM_E_INVALID_ARG = -1, /* null pointer, bad size, misaligned buffer      */
  VOOM_E_CUDA = -2,        /* a CUDA launch or runtime call failed            */
  VOOM_E_CAPACITY = -3,    /* caller-provided array or buffer is too small    */
  VOOM_E_UNSUPPORTED = -4, /* a valid input outside what this build decodes   */

  /* formats/bf16_rans.py decode() ValueError messages, in the order the
   * reference checks them (bf16_rans.py:97-130, 180-222). */
  VOOM_RANS_TRUNC_FRAME = 101,         /* "truncated rANS frame"               */
  VOOM_RANS_NOT_FRAME = 102,           /* "not a vOOM rANS frame"              */
  VOOM_RANS_TRUNC_TILE_HEADER = 103,   /* "truncated rANS tile header"         */
  VOOM_RANS_TRUNC_TILE_PAYLOAD = 104,  /* "truncated rANS tile payload"        */
  VOOM_RANS_RAW_SIZE_MISMATCH = 105,   /* "raw rANS tile size mismatch"        */
  VOOM_RANS_TRUNC_PLANE_HEADER = 106,  /* "truncated rANS plane header"        */
  VOOM_RANS_TRUNC_PLANE_PAYLOAD = 107, /* "truncated rANS plane payload"       */
  VOOM_RANS_BAD_FREQ_TOTAL = 108,      /* "invalid rANS frequency total"       */
  VOOM_RANS_TRAILING_RENORM = 109,     /* "rANS plane has trailing renormalization bytes" */
  VOOM_RANS_TILE_TRAILING = 110,       /* "compressed rANS tile has trailing bytes" */
  VOOM_RANS_UNKNOWN_MODE = 111,        /* "unknown rANS tile mode {mode}"      */
  VOOM_RANS_CHECKSUM = 112,            /* "rANS tile checksum mismatch"        */
  VOOM_RANS_LENGTH_MISMATCH = 113      /* "rANS frame length mismatch"         */
};

/* ------------------------------------------------------------ bf16_rans */

/* Per-tile decode plan.  Offsets are absolute byte offsets into the device
 * source buffer (src) and the device output buffer (dst), so one plan array
 * can describe tiles of many frames packed into one buffer. */
typedef struct voom_rans_tile {
  uint64_t src;         /* mode 0: first payload byte; mode 1: unused        */
  uint64_t dst;         /* output offset of the tile's first decoded byte    */
  uint64_t low_freq;    /* mode 1: offset of the low plane's 256 x u16 table */
  uint64_t high_freq;   /* mode 1: offset of the high plane's table          */
  uint32_t low_payload; /* mode 1: low plane payload bytes (>= 4)            */
  uint32_t high_payload;/* mode 1: high plane payload bytes (>= 4)           */
  uint32_t raw_len;     /* decoded bytes of this tile                         */
  uint32_t crc32;       /* expected zlib CRC-32 of the decoded tile          */
  uint32_t mode;        /* 0 = stored verbatim, 1 = two rANS byte planes     */
  uint32_t flags;       /* VOOM_RANS_DO_* bits                               */
} voom_rans_tile;

enum {
  VOOM_RANS_DO_LOW = 1u,  /* decode the low plane                           */
  VOOM_RANS_DO_HIGH = 2u, /* decode the high plane                          */
  VOOM_RANS_DO_CRC = 4u,  /* verify the tile CRC-32 (or copy a mode 0 tile) */
  VOOM_RANS_DO_COPY = 8u  /* mode 0: copy the stored bytes                  */
};

/* Bits of the per-tile status word written by voom_rans_decode. */
enum {
  VOOM_RANS_ST_LOW_TRAILING = 1u,  /* low plane left renormalisation bytes  */
  VOOM_RANS_ST_HIGH_TRAILING = 2u, /* high plane left renormalisation bytes */
  VOOM_RANS_ST_CRC_MISMATCH = 4u   /* decoded tile fails its CRC-32          */
};

typedef struct voom_rans_plan_info {
  uint64_t raw_size;      /* frame header raw size                          */
  uint64_t out_bytes;     /* sum of raw_len over planned tiles              */
  uint32_t tile_bytes;    /* frame header tile size                          */
  uint32_t tile_count;    /* frame header tile count                         */
  uint32_t n_tiles;       /* planned tiles (descriptors needed)             */
  int32_t struct_error;   /* first structural error (0 = none)             */
  uint32_t struct_tile;   /* tile index of struct_error                     */
  uint32_t struct_ordinal;/* position of struct_error within the tile       */
  uint32_t bad_mode;      /* mode byte for VOOM_RANS_UNKNOWN_MODE           */
  uint32_t frame_end;     /* 1 if the walk reached the end-of-frame checks  */
} voom_rans_plan_info;

/* Walks one VRN1 frame held in host memory the way formats/bf16_rans.py:180-222
 * and _decode_plane (:97-130) walk it, without decoding any symbol: frame and
 * tile headers, plane headers, payload bounds and frequency totals.  Stops at
 * the first structural error; every tile before it (and the planes of the
 * failing tile that the reference decodes before failing) is planned.
 * `src_base`/`dst_base` are added to every offset written.  With
 * max_tiles == 0 only `info` is filled (sizing pass).
 * Returns VOOM_OK, or VOOM_E_CAPACITY if max_tiles < info->n_tiles.
 * Replaces: formats/bf16_rans.py:180-222 (header walk of decode()). */
int voom_rans_plan(const uint8_t* h_frame, uint64_t frame_len, uint64_t src_base,
                   uint64_t dst_base, voom_rans_tile* h_tiles, uint32_t max_tiles,
                   voom_rans_plan_info* info);

/* Decodes planned tiles on the GPU: per-plane rANS decode (bf16_rans.py:97-130),
 * byte-plane interleave into the output (:211-213), CRC-32 check (:217).
 * d_src holds the frame bytes, padded to a multiple of 16 bytes with at least
 * 16 readable bytes after the last frame byte.  d_out receives decoded bytes at
 * each tile's dst.  d_status (n_tiles words) receives VOOM_RANS_ST_* bits.
 * If d_ckpt is non-null, the low/high plane decoders record a checkpoint
 * (state, cursor) every `ckpt_every` symbols (a power of two >= 64) at
 * d_ckpt[ckpt_base[t] + 2*k + plane] as two u32 words; ckpt_base is a device
 * array of n_tiles u32 (pass NULL when d_ckpt is NULL).
 * Replaces: formats/bf16_rans.py:180-222 decode() (symbol work). */
int voom_rans_decode(const uint8_t* d_src, const voom_rans_tile* d_tiles, uint32_t n_tiles,
                     uint8_t* d_out, uint32_t* d_status, uint32_t* d_ckpt,
                     const uint32_t* d_ckpt_base, uint32_t ckpt_every, void* stream);

/* Work unit of the indexed decoder: up to 128 checkpoint segments of one tile
 * (a stored tile is one unit).  Built by voom_rans_chunks. */
typedef struct voom_rans_chunk {
  uint32_t tile;       /* tile index                                */
  uint32_t seg_begin;  /* first checkpoint segment                   */
  uint32_t seg_end;    /* one past the last segment                  */
  uint32_t n_in_tile;  /* units of this tile (for the CRC assembly)  */
} voom_rans_chunk;

/* Host helper: splits planned tiles into indexed-decode units.  With
 * chunks == NULL only *n_chunks is set. */
int voom_rans_chunks(const voom_rans_tile* h_tiles, uint32_t n_tiles, uint32_t ckpt_every,
                     voom_rans_chunk* h_chunks, uint32_t max_chunks, uint32_t* n_chunks);

/* Decodes planned tiles from a checkpoint index built by voom_rans_decode:
 * every (tile, plane, segment of ckpt_every symbols) is decoded independently
 * and must land exactly on the next checkpoint (else the *_TRAILING bit);
 * the CRC-32 of each tile is assembled from its units and verified when the
 * tile has VOOM_RANS_DO_CRC.  d_tile_scratch: 4 u32 per tile, zero before the
 * first call; every call leaves it zero again.  d_status gets one word per tile.
 * Replaces: formats/bf16_rans.py:180-222 decode() for pages kept resident
 * in HBM and decoded on every use. */
int voom_rans_decode_indexed(const uint8_t* d_src, const voom_rans_tile* d_tiles,
                             const voom_rans_chunk* d_chunks, uint32_t n_chunks, uint8_t* d_out,
                             uint32_t* d_status, const uint32_t* d_ckpt, const uint32_t* d_ckpt_base,
                             uint32_t ckpt_every, uint32_t* d_tile_scratch, void* stream);

/* Checkpoint words a tile needs for a given interval (2 per plane-segment
 * boundary, both planes).  Host helper. */
uint64_t voom_rans_ckpt_words(uint32_t raw_len, uint32_t ckpt_every);

/* Pack side: encodes n bytes into a VRN1 frame byte-identical to
 * formats/bf16_rans.py encode() (:148-177), tiles encoded on `threads` host
 * threads (<= 0: all cores).  With h_out == NULL, *out_len receives the
 * worst-case frame size (size the buffer with it).  stats (may be NULL):
 * [0] tiles, [1] tiles stored compressed.
 * Replaces: formats/bf16_rans.py:148-177 (encode, _encode_plane,
 * _normalize_frequencies). */
int voom_rans_encode(const uint8_t* h_data, uint64_t n, uint32_t tile_bytes, uint8_t* h_out,
                     uint64_t out_cap, uint64_t* out_len, uint64_t* stats, int threads);

/* Combines the plan's structural error with the per-tile GPU status (host
 * copies) into the error formats/bf16_rans.py decode() raises first.
 * Returns VOOM_OK or a VOOM_RANS_* code; *err_tile receives the tile index. */
int voom_rans_resolve(const voom_rans_plan_info* info, const uint32_t* h_status,
                      uint32_t n_tiles, uint32_t* err_tile);

/* ------------------------------------------------------------------ zstd */
/* One decompression job = one `compression.zstd.decompress(data)` call of the
 * reference (one or more concatenated frames, skippable frames allowed),
 * optionally interleaved with a raw byte plane as vpack bodies are
 * (formats/packed2.py:178-191: out[0::2] = lo, out[1::2] = hi). */
typedef struct voom_zstd_job {
  uint64_t src;     /* offset of the compressed bytes in the source buffer    */
  uint64_t src_len; /* compressed bytes                                       */
  uint64_t dst;     /* output offset of the first decoded byte                */
  uint64_t dst_len; /* decoded zstd bytes the job must produce                */
  uint64_t lo_src;  /* VOOM_ZSTD_INTERLEAVE: offset of the raw lo plane       */
  uint32_t flags;   /* VOOM_ZSTD_* bits                                       */
  uint32_t pad;
} voom_zstd_job;

enum {
  VOOM_ZSTD_INTERLEAVE = 1u /* out[dst+2k] = lo[k], out[dst+2k+1] = decoded[k] */
};

/* Per-job status bits written by the decoder (0 = exact). */
enum {
  VOOM_ZSTD_ST_FORMAT = 1u,    /* malformed frame/block header or table (host plan) */
  VOOM_ZSTD_ST_LITERALS = 2u,  /* Huffman stream not consumed exactly / overrun */
  VOOM_ZSTD_ST_SEQUENCES = 4u, /* FSE bitstream not consumed exactly / bad code */
  VOOM_ZSTD_ST_OFFSET = 8u,    /* match reaches before the frame start / zero   */
  VOOM_ZSTD_ST_SIZE = 16u,     /* content size / block size / job length mismatch */
  VOOM_ZSTD_ST_CHECKSUM = 32u, /* XXH64 content checksum mismatch */
  VOOM_ZSTD_ST_UNRESOLVED = 64u, /* match chains not resolved (internal limit) */
  VOOM_ZSTD_ST_TOO_LARGE = 128u  /* a job with matches decoding to more than
                                    2 GiB - 1 MiB (split it into several jobs) */
};

typedef struct voom_zstd_plan_info {
  uint32_t n_jobs, n_frames, n_blocks, n_huf, n_fse;
  uint32_t n_bad_jobs;      /* jobs with a structural error (not planned)   */
  uint64_t lit_bytes;       /* literal scratch bytes                         */
  uint64_t n_seq;           /* sequences over all blocks                     */
  uint64_t decoded_bytes;   /* sum of dst_len over planned jobs              */
  uint64_t scratch_bytes;   /* device scratch voom_zstd_decode needs         */
  uint64_t plan_bytes;      /* bytes of the device plan image                */
  uint32_t n_segments;      /* decode passes (each at most 1 GiB of jobs that
                               need match resolution)                         */
  uint32_t n_direct_jobs;   /* jobs without sequences, decoded straight to the
                               output                                         */
} voom_zstd_plan_info;

/* Host plan of a batch of jobs whose bytes are in host memory h_src: walks
 * frame headers (RFC 8878 3.1.1), block headers, literal and sequence section
 * headers, decodes Huffman tree descriptions and FSE table descriptions; the
 * entropy-coded payloads are left to the GPU.  Returns an opaque handle (NULL
 * on bad arguments).  Jobs with a structural error are marked in the plan and
 * skipped by the decoder.  `threads` <= 0 uses up to 8 host threads, fewer
 * for small batches (each thread takes at least 64 blocks or 32 jobs).
 * Replaces: the frame/block header walk inside libzstd ZSTD_decompress as
 * reached from formats/packed2.py:178-191 and runtime/kv_paged.py:98-113. */
void* voom_zstd_plan_create(const uint8_t* h_src, uint64_t src_len, const voom_zstd_job* jobs,
                            uint32_t n_jobs, int threads);
int voom_zstd_plan_info_get(const void* plan, voom_zstd_plan_info* info);
/* Writes the device plan image (info.plan_bytes) to host memory h_image; copy
 * it to device memory unchanged and pass it to voom_zstd_decode. */
int voom_zstd_plan_image(const void* plan, void* h_image, uint64_t cap);
/* Per-job structural status (VOOM_ZSTD_ST_FORMAT or 0), n_jobs words. */
int voom_zstd_plan_job_status(const void* plan, uint32_t* h_status);
void voom_zstd_plan_destroy(void* plan);

/* GPU decode of a planned batch: d_src = the same bytes as h_src, 16-byte
 * aligned, with 16 bytes of readable padding after the end; d_plan = the plan image in device memory,
 * d_scratch = info.scratch_bytes of device memory (contents ignored),
 * d_out = output, d_status = n_jobs u32 status words (VOOM_ZSTD_ST_* bits,
 * accumulated: clear before the call).  Enqueues every pass on `stream`
 * without host synchronisation (the resolve passes read their worklist
 * counts on the device).
 * Replaces: compression.zstd.decompress + the lo/hi interleave of
 * formats/packed2.py:178-191 (decode_body) and runtime/kv_paged.py:98-113. */
int voom_zstd_decode(const uint8_t* d_src, const void* d_plan, const void* h_plan, void* d_scratch,
                     uint8_t* d_out, uint32_t* d_status, void* stream);

/* GPU zstd compression into valid RFC 8878 frames, the KV-page spill codec
 * (and the warm tier's admission): any frame zstd.decompress accepts gives
 * the page back, so the frames need not be libzstd's.  A frame is split into
 * blocks of at most voom_zstd_encode_block_bytes() input bytes; each becomes a
 * Compressed block of Huffman-coded literals (four streams, FSE-compressed or
 * 4-bit weights, no sequences), RLE literals when one byte value fills it, or
 * a Raw block when Huffman coding would not shrink it.  Frames are single
 * segment with the content size and no checksum.  Block b is written into
 * slot b (voom_zstd_encode_slot_bytes() bytes each) of d_slots; d_sizes[2b] /
 * d_sizes[2b+1] give the offset and length of its bytes in the slot (the
 * first block of a frame carries the frame header), so a frame is the
 * concatenation of its blocks' byte ranges.
 * Replaces: zstd.compress(raw, level=1) in runtime/kv_paged.py:79-91 and
 * runtime/warm_tier.py:74-83. */
typedef struct voom_zenc_block {
  uint64_t src;       /* offset of the block's first input byte in d_src */
  uint64_t frame_len; /* content size of the frame the block belongs to */
  uint32_t len;       /* input bytes of the block (<= voom_zstd_encode_block_bytes()) */
  uint32_t flags;     /* VOOM_ZENC_FIRST | VOOM_ZENC_LAST */
} voom_zenc_block;

#define VOOM_ZENC_FIRST 1u /* first block of its frame: the frame header precedes it */
#define VOOM_ZENC_LAST 2u  /* last block of its frame */

uint64_t voom_zstd_encode_slot_bytes(void);
uint32_t voom_zstd_encode_block_bytes(void);
int voom_zstd_encode(const uint8_t* d_src, const voom_zenc_block* d_blocks, uint32_t n_blocks, uint8_t* d_slots,
                     uint32_t* d_sizes, void* stream);
/* Packs the encoded blocks into one buffer: block b's bytes (its range in
 * slot b, from d_sizes) go to d_out + d_dst[b].  No counterpart in the
 * reference (it writes frames from host memory). */
int voom_zstd_encode_pack(const uint8_t* d_slots, const uint32_t* d_sizes, const uint64_t* d_dst, uint32_t n_blocks,
                          uint8_t* d_out, void* stream);

/* Copies n bytes of pinned host memory (allocated or registered with the CUDA
 * runtime, so mapped into the device's address space) to device memory with a
 * kernel on `stream`: the SMs read the host memory directly, so the copy does
 * not wait on a copy engine behind transfers enqueued before it (used for
 * plan images while body uploads are in flight).  [h_src, h_src + n) must lie
 * in ONE such allocation, as for cudaMemcpyAsync.  VOOM_E_INVALID_ARG when it
 * is not mapped pinned memory (nothing is launched; use cudaMemcpyAsync).  No
 * counterpart in the reference. */
int voom_copy_from_host(void* d_dst, const void* h_src, uint64_t n, void* stream);

/* Per-kernel timing of voom_zstd_decode (diagnostics; no counterpart in the
 * reference).  voom_zstd_set_timing(1) makes every later voom_zstd_decode
 * record a CUDA event after each of its launches (on the device current when
 * timing was switched on); voom_zstd_kernel_times(ms, ids, cap) waits for the
 * last decode and returns how many (interval ms, kernel id) pairs it wrote, in
 * launch order.  A profiling aid: one process-wide event set, so time one
 * decode at a time (not thread-safe).  Kernel ids: */
enum {
  VOOM_ZSTD_K_DIRECT_LITERALS = 1, VOOM_ZSTD_K_BLOCK_DECODE = 2, VOOM_ZSTD_K_SEQ_SCAN = 3,
  VOOM_ZSTD_K_JOB_SCAN = 4, VOOM_ZSTD_K_BLOCK_EXECUTE = 5, VOOM_ZSTD_K_OUTPUT = 6,
  VOOM_ZSTD_K_RESOLVE = 7, /* all resolve passes of one segment */
  VOOM_ZSTD_K_PATCH = 8, VOOM_ZSTD_K_CHECKSUM = 9, VOOM_ZSTD_K_BLOCK_LITERALS = 10
};
int voom_zstd_set_timing(int on);
int voom_zstd_kernel_times(float* ms, uint32_t* ids, int cap);

/* ------------------------------------------------- KV spill pages (.kvz) */
/* One compressed KV page as runtime/kv_paged.py:86-88 writes it: the pickle
 * of {"shape": tuple, "k": zstd(K bits, 1), "v": zstd(V bits, 1)}. */
typedef struct voom_kvz_page {
  uint64_t k_off, k_len; /* the K frame: offset in the gather buffer, bytes */
  uint64_t v_off, v_len; /* the V frame                                     */
  int64_t shape[8];      /* the "shape" tuple                               */
  uint32_t ndim;
  uint32_t status;       /* 0 = parsed; 1 = not a pickle this walker reads
                            (the caller unpickles that page itself)          */
} voom_kvz_page;

/* Copies n pages (h_src_addrs[j], lens[j] bytes; h_src_addrs NULL = the pages
 * are already at h_dst + dst_offs[j]) into h_dst at dst_offs[j] on `threads`
 * host threads (<= 0: all cores) and walks each page's pickle in place,
 * filling pages[j] with the offsets of its two zstd frames in h_dst.
 * Replaces: the pickle.load of runtime/kv_paged.py:104-105. */
int voom_kvz_gather(const uint64_t* h_src_addrs, const uint64_t* lens, const uint64_t* dst_offs, uint32_t n,
                    uint8_t* h_dst, voom_kvz_page* pages, int threads);

/* ------------------------------------------------------- BF16 NF12 sidecar */
/* One NF12 layer stream in device memory (16-byte aligned): header_bytes of
 * 16-byte block headers, 384 code bytes per block, then the 3-byte patches
 * (formats/bf16_nf12_sidecar.py:318-420 of the reference).
 *
 * voom_nf12_decode: blocks [first_block, first_block + n_blocks) to BF16 bits,
 * each at its header's output offset minus output_base in d_out (out_values
 * entries).  A block whose header points outside the stream or the output is
 * skipped and sets bit 0 of *d_status.
 * Replaces: runtime/bf16_nf12_sidecar.py:21-98 (voom_bf16_nf12_decode_v1 and
 * _decode_span), used by decode_layer / decode_names :126-248. */
int voom_nf12_decode(const uint8_t* d_enc, uint64_t enc_bytes, uint64_t header_bytes, uint32_t first_block,
                     uint32_t n_blocks, uint64_t output_base, uint16_t* d_out, uint64_t out_values,
                     uint32_t* d_status, void* stream);

/* Fused NF12 decode + small-M linear: d_out[p, n] = sum_k d_x[p, k] * W[n, k]
 * (BF16 in and out, fp32 accumulation) for 1 <= M <= 8 activation rows, W the
 * N x K tensor whose blocks start at first_block (K % 512 == 0, N % 8 == 0:
 * the reference's direct_linear_eligible shapes).  d_scratch must hold
 * voom_nf12_linear_scratch_bytes(M, K, N) bytes (0: may be NULL).  A block
 * that is not full or whose patches leave the stream sets bit 1 of
 * *d_status.
 * Replaces: runtime/bf16_nf12_linear.py:19-135 (voom_nf12_small_gemm_k{K}_n{N}_p{P}
 * and NF12Tensor.matmul). */
uint64_t voom_nf12_linear_scratch_bytes(uint32_t M, uint32_t K, uint32_t N);
int voom_nf12_linear(const uint16_t* d_x, uint32_t M, uint32_t K, uint32_t N, const uint8_t* d_enc,
                     uint64_t enc_bytes, uint64_t header_bytes, uint32_t first_block, void* d_scratch,
                     uint64_t scratch_bytes, uint16_t* d_out, uint32_t* d_status, void* stream);

/* Several NF12 linears of one layer stream and one M in a single launch (up
 * to 16, e.g. the q/k/v/o and gate/up/down projections of a decoder layer),
 * so small matrices share the GPU instead of each filling it alone.  Each
 * task: d_x (M x K BF16), d_out (M x N BF16), K, N, first_block, with the
 * same shape rules as voom_nf12_linear.  Same results as one call per task.
 * Replaces: the per-projection NF12Tensor.matmul calls of one layer
 * (runtime/bf16_nf12_linear.py:223-244). */
typedef struct voom_nf12_linear_task {
  const uint16_t* d_x;
  uint16_t* d_out;
  uint32_t K;
  uint32_t N;
  uint32_t first_block;
  uint32_t pad;
} voom_nf12_linear_task;

uint64_t voom_nf12_linear_batch_scratch_bytes(const voom_nf12_linear_task* tasks, uint32_t n, uint32_t M);
int voom_nf12_linear_batch(const voom_nf12_linear_task* tasks, uint32_t n, uint32_t M, const uint8_t* d_enc,
                           uint64_t enc_bytes, uint64_t header_bytes, void* d_scratch, uint64_t scratch_bytes,
                           uint32_t* d_status, void* stream);

/* ---------------------------------------------------- fused MoE experts */
/* One projection (rows x cols BF16, row-major, HF layout) of one expert kept
 * compressed in HBM as a VRN1 frame with its tile plan and checkpoint index
 * (device pointers; tile src/dst offsets relative to `src` / the matrix).
 * The fused kernels need: every tile holding whole rows, `cols` a multiple of
 * `every`, at most 128 segments of `every` symbols per tile. */
typedef struct voom_expert_proj {
  const uint8_t* src;
  const voom_rans_tile* tiles;
  const uint32_t* ckpt;
  const uint32_t* ckpt_base;
  uint32_t n_tiles;
  uint32_t every;
  uint32_t rows;
  uint32_t cols;
} voom_expert_proj;

typedef struct voom_expert_pages {
  voom_expert_proj gate; /* I x H */
  voom_expert_proj up;   /* I x H */
  voom_expert_proj down; /* H x I */
} voom_expert_pages;

/* Scratch bytes voom_moe_layer needs. */
uint64_t voom_moe_scratch_bytes(uint32_t T, uint32_t H, uint32_t I, uint32_t top_k);

/* MoE families: which reference layer the routing and accumulation follow.
 *   VOOM_MOE_GENERIC  runtime/layer_runner.py:347-394 (run_moe_mlp): BF16
 *                     logits, fp32 softmax, top-k, optional renormalisation,
 *                     BF16 route weights, experts accumulated in first-
 *                     appearance order over (position, slot).
 *   VOOM_MOE_QWEN35   runtime/qwen35.py:584-638 (_route_experts, _moe): as
 *                     generic but always renormalised (norm_topk must be 1),
 *                     ascending expert order, zero-centred RMSNorm weight
 *                     (1 + w, qwen35.py:133-150), and a shared expert gated
 *                     by bf16(sigmoid(bf16(h . shared_gate_w))).
 *   VOOM_MOE_GLM      runtime/glm.py:364-392, 429-486: fp32 router logits,
 *                     sigmoid scores, choice by score + d_router_bias (the
 *                     e_score_correction_bias, fp32), weights = the chosen
 *                     scores (/ (sum + 1e-20) when norm_topk) x routed_scale,
 *                     kept in fp32, ascending expert order, then + the
 *                     shared expert. */
#define VOOM_MOE_GENERIC 0u
#define VOOM_MOE_QWEN35 1u
#define VOOM_MOE_GLM 2u

typedef struct voom_moe_variant {
  uint32_t family;                 /* VOOM_MOE_* */
  uint32_t norm_topk;              /* renormalise the chosen route weights */
  float routed_scale;              /* GLM routed_scaling_factor (1 for the others) */
  int32_t shared_expert;           /* page-table index of the shared expert (>= n_experts), or -1 */
  const uint16_t* d_shared_gate_w; /* qwen35 shared_expert_gate weight, H BF16; NULL otherwise */
  const float* d_router_bias;      /* GLM: correction bias (E fp32); generic: added to the logits; or NULL */
} voom_moe_variant;

/* Scratch bytes voom_moe_layer_v / voom_moe_experts_v need (a shared expert
 * adds one route row per token). */
uint64_t voom_moe_scratch_bytes_v(const voom_moe_variant* v, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k);

/* One MoE layer for T tokens, entirely on the device: RMSNorm (d_norm_w may
 * be NULL), router GEMV, fp32 softmax, top-k, optional renormalisation,
 * fused rANS-decode + SwiGLU GEMV of every routed expert straight from its
 * compressed pages, route-weighted BF16 accumulation in the reference's order
 * and the residual add: d_x_out = x + moe(x) (residual = 1) or moe(x)
 * (residual = 0).  gate_tiles / down_tiles: the
 * largest tile count of any expert's gate / down frame (grid size).  Bit 0 of
 * *d_status is set if a page segment misses its checkpoint.
 * Replaces: runtime/layer_runner.py:347-394 (run_moe_mlp) with
 * :185-190 (_swiglu) over pages fetched by weight_cache.py:191 get_many. */
int voom_moe_layer(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                   const uint16_t* d_norm_w, float eps, const uint16_t* d_x, uint16_t* d_x_out, uint32_t T,
                   uint32_t H, uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles,
                   uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                   uint32_t* d_status, void* stream);

/* Expert-parallel form of voom_moe_layer, split at the collective.
 * voom_moe_experts: RMSNorm, router and top-k for all T tokens (replicated on
 * every rank), then the fused decode + SwiGLU only for experts whose pages
 * are present in d_pages (n_tiles > 0; other experts' entries have zero
 * tiles).  d_y (T*top_k rows of H BF16, zeroed here) receives the unweighted
 * output of each route row; rows of absent experts stay zero, so summing d_y
 * over ranks (NCCL all-reduce) reproduces the single-GPU rows exactly.  The
 * routes stay in d_scratch for voom_moe_combine, which applies the route
 * weights in the reference's accumulation order and the residual.
 * d_router_bias (E floats, may be NULL) is added to the BF16 router logits
 * before the softmax.
 * Replaces: runtime/layer_runner.py:347-394 across experts spread over GPUs
 * (the reference has no multi-device path). */
int voom_moe_experts(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                     const float* d_router_bias, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                     uint32_t T, uint32_t H,
                     uint32_t I, uint32_t top_k, uint32_t norm_topk, uint32_t gate_tiles, uint32_t down_tiles,
                     uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status, void* stream);
int voom_moe_combine(const void* d_scratch, const uint16_t* d_y, const uint16_t* d_x, uint16_t* d_x_out,
                     uint32_t T, uint32_t H, uint32_t residual, void* stream);

/* voom_moe_layer / voom_moe_experts for any family (voom_moe_variant).  The
 * page table holds the n_experts routed experts and, at index
 * v->shared_expert, the shared expert (same intermediate size I), which every
 * token uses.  voom_moe_experts_v's d_y has T * (top_k + 1) rows with a shared
 * expert (its rows last, in token order), else T * top_k; in expert-parallel
 * use the shared expert's pages are present on one rank only.
 * voom_moe_combine applies the family's accumulation (the routes carry it).
 * Replaces: runtime/layer_runner.py:347-394, runtime/qwen35.py:584-638 and
 * runtime/glm.py:364-406, 429-486 over pages fetched by WeightCache. */
int voom_moe_layer_v(const voom_moe_variant* v, const voom_expert_pages* d_pages, uint32_t n_experts,
                     const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                     uint16_t* d_x_out, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k, uint32_t gate_tiles,
                     uint32_t down_tiles, uint32_t residual, void* d_scratch, uint64_t scratch_bytes,
                     uint32_t* d_status, void* stream);
int voom_moe_experts_v(const voom_moe_variant* v, const voom_expert_pages* d_pages, uint32_t n_experts,
                       const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps, const uint16_t* d_x,
                       uint32_t T, uint32_t H, uint32_t I, uint32_t top_k, uint32_t gate_tiles, uint32_t down_tiles,
                       uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status, void* stream);

/* Expert parallelism over `world` GPUs (one process each) with an exchange
 * that scales: every rank routes all T tokens (the same routes on every
 * rank), each routed expert is computed by exactly one rank -- the one that
 * holds its pages, or, for an expert several ranks hold (replicated hot
 * experts), the least loaded of them by a rule every rank evaluates alike --
 * and only the owned experts' work is launched.  d_y_tm (t_pad * rows_per_token
 * rows of H BF16, rows_per_token = top_k + 1 with a shared expert) receives the
 * route rows in token-major order (row t * rows_per_token + j = token t's j-th
 * route in the combine's order, the shared expert last), zero where another
 * rank computes the row and for padding tokens t >= T.  A reduce-scatter of
 * d_y_tm over ranks (sum; every row has one nonzero contributor, so the sum
 * is exact) leaves rank r the rows of tokens [r * t_pad / world, (r + 1) *
 * t_pad / world); voom_moe_combine_tm combines those, and an all-gather of the
 * combined rows gives every rank the layer output, bit-identical to
 * voom_moe_layer_v on one GPU.  d_holders: n_experts words (n_experts + 1 with
 * a shared expert, its entry last), bit r = rank r holds the expert's pages
 * (world <= 32); t_pad >= T, a multiple of world.  Status bit 16: a routed
 * expert no rank holds (its rows stay zero).
 * Replaces: runtime/layer_runner.py:347-394 across GPUs (the reference has no
 * multi-device path). */
typedef struct voom_moe_ep {
  const uint32_t* d_holders;
  uint32_t rank, world;
  uint32_t t_pad;
} voom_moe_ep;
int voom_moe_experts_ep(const voom_moe_variant* v, const voom_moe_ep* ep, const voom_expert_pages* d_pages,
                        uint32_t n_experts, const uint16_t* d_router_w, const uint16_t* d_norm_w, float eps,
                        const uint16_t* d_x, uint32_t T, uint32_t H, uint32_t I, uint32_t top_k,
                        uint32_t gate_tiles, uint32_t down_tiles, uint16_t* d_y_tm, void* d_scratch,
                        uint64_t scratch_bytes, uint32_t* d_status, void* stream);
/* The combine of voom_moe_layer_v for tokens [t0, t0 + t_count) from their
 * token-major rows d_y_shard (t_count * rows_per_token rows), with the routes
 * voom_moe_experts_ep left in d_scratch; d_out_shard receives t_count rows of
 * H (tokens t >= T: zeros).  d_x holds all T input rows (the residual). */
int voom_moe_combine_tm(const void* d_scratch, const uint16_t* d_y_shard, const uint16_t* d_x,
                        uint16_t* d_out_shard, uint32_t t0, uint32_t t_count, uint32_t H, uint32_t residual,
                        void* stream);

/* voom_moe_layer without any device allocation, for callers that cannot
 * allocate device memory themselves: runtimes that own every byte of the GPU
 * through their own pool, serving loops that must not hit the allocator (and
 * its device-wide synchronisation) between decode steps, and foreign hosts
 * that reach this library only through the C ABI and have no CUDA allocator.
 * It has no counterpart in the reference.
 * Same arguments and results as voom_moe_layer minus d_scratch /
 * scratch_bytes: the scratch is one fixed device array (about 8.5 MiB) per GPU,
 * loaded with the library and held until the process exits.  Limits:
 * T <= 64, T * top_k <= 256, H <= 8192, I <= 4096; larger calls return
 * VOOM_E_CAPACITY without launching anything.  Nothing in the array needs
 * clearing between calls (every call writes what it reads).  Calls share the
 * array: two calls that overlap on the GPU (different streams, or different
 * host threads on one device) race and corrupt each other's results, so
 * serialise them.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture.  Pass a stream of the current device. */
int voom_moe_layer_noalloc(const voom_expert_pages* d_pages, uint32_t n_experts, const uint16_t* d_router_w,
                           const uint16_t* d_norm_w, float eps, const uint16_t* d_x, uint16_t* d_x_out,
                           uint32_t T, uint32_t H, uint32_t I, uint32_t top_k, uint32_t norm_topk,
                           uint32_t gate_tiles, uint32_t down_tiles, uint32_t residual, uint32_t* d_status,
                           void* stream);

/* Fused decode + SwiGLU for experts routed on the host (the
 * consume_expert_batches path): unique expert u = d_expert_ids[u] (index into
 * d_pages) takes the tokens d_upair[off_u .. off_u + d_ntok[u]), off_u the sum
 * of earlier counts (n_rows in total); y row off_u + i (H BF16) receives
 * expert u's output for its i-th token, unweighted.  d_h: T x H BF16.
 * Scratch: voom_moe_scratch_bytes(n_rows, H, I, 1) suffices.
 * Replaces: runtime/expert_batching.py:13-41 consume callback body
 * (qwen35.py:617-633 / glm.py:466-480 / layer_runner.py:387-393 _swiglu). */
int voom_expert_swiglu(const voom_expert_pages* d_pages, const uint32_t* d_expert_ids, uint32_t n_unique,
                       const uint32_t* d_ntok, const uint32_t* d_upair, uint32_t n_rows, uint32_t T,
                       const uint16_t* d_h, uint32_t H, uint32_t I, uint32_t gate_tiles, uint32_t down_tiles,
                       uint16_t* d_y, void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VOOM_B200_H */
