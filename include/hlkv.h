/*
 * hlkv.h -- C ABI of the HL-KV quantized KV-block path on NVIDIA B200 (sm_100a).
 *
 * One shared library, libhlkv.so, behind plain C types: pointers, sizes and a
 * CUDA stream handle.  It binds from any FFI (ctypes, cgo, JNI, N-API).  The
 * C++20 API that the reference exposes (hl::alloc::HeteroBlockTable,
 * hl::alloc::IdArena, hl::quant::cuda::dequantize_fp8_to_fp16) is in
 * include/hl_allocator/ and include/hl_quant/; this header is the flat view
 * of the same objects, and the only way into the CUDA kernels.
 *
 * Conventions
 *  - Device entry points are asynchronous on `stream`, launch nothing on an
 *    argument error (outputs untouched), and treat n == 0 as a no-op.
 *    They return an HLKV_* status; HLKV_CUDA_ERROR carries the cudaError_t in
 *    hlkv_last_cuda_error() (per thread).
 *  - Per-block problems found on the device (a non-executable descriptor, an
 *    index out of range, ...) never fault: the block is skipped and its
 *    HLKV_ERR_* bit is OR-ed into *d_err (device memory, one uint32_t the
 *    caller owns and clears).
 *  - Table entry points return an hl::alloc::Status value (HLKV_STATUS_*).
 *  - The caller owns every device buffer; no entry point allocates device
 *    memory except hlkv_device_tables_* (the persistent table mirror).
 */
#ifndef HLKV_H_
#define HLKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HLKV_ABI_VERSION 1 /* == hl::alloc::kAbiVersion */

/* A CUDA stream (the same type as cudaStream_t / CUstream). NULL = legacy default stream. */
typedef struct CUstream_st* hlkv_stream_t;

/* ---- device status (== hl::quant::QuantStatus, quant_types.hpp:54-60) ------------------- */
enum {
  HLKV_OK = 0,
  HLKV_INVALID_ARGUMENT = 1,
  HLKV_BUFFER_TOO_SMALL = 2,
  HLKV_UNSUPPORTED_FORMAT = 3,
  HLKV_CUDA_ERROR = 4
};

/* ---- table status (== hl::alloc::Status, status.hpp:17-30) ---------------------------- */
enum {
  HLKV_STATUS_OK = 0,
  HLKV_STATUS_OUT_OF_BLOCKS = 1,
  HLKV_STATUS_OUT_OF_SLOTS = 2,
  HLKV_STATUS_INVALID_HANDLE = 3,
  HLKV_STATUS_STALE_HANDLE = 4,
  HLKV_STATUS_INVALID_STATE = 5,
  HLKV_STATUS_INVALID_ARGUMENT = 6,
  HLKV_STATUS_UNKNOWN_FORMAT = 7,
  HLKV_STATUS_NOT_DEVICE_RESIDENT = 8,
  HLKV_STATUS_REFCOUNT_OVERFLOW = 9,
  HLKV_STATUS_CORRUPT = 10,
  HLKV_STATUS_CAPACITY_EXCEEDED = 11
};

/* ---- formats (== hl::quant::QuantFormat, quant_types.hpp:40-46) --------------------- */
enum { HLKV_FP16 = 0, HLKV_FP8_E4M3 = 1, HLKV_FP8_E5M2 = 2, HLKV_INT4 = 3, HLKV_INVALID_FORMAT = 15 };

/* ---- per-block error bits written to *d_err ------------------------------------------ */
enum {
  HLKV_ERR_NOT_EXECUTABLE = 1u << 0,  /* descriptor format 15 (free / not resident)    */
  HLKV_ERR_BAD_FORMAT = 1u << 1,      /* no pool for the format, or not decodable     */
  HLKV_ERR_SLOT_RANGE = 1u << 2,      /* slot >= num_slots of its pool                */
  HLKV_ERR_ARENA_RANGE = 1u << 3,     /* segment offset + j >= arena_size             */
  HLKV_ERR_BLOCK_ID_RANGE = 1u << 4,  /* arena entry / target id >= table_size        */
  HLKV_ERR_VALID_TOKENS = 1u << 5,    /* valid_tokens > block_tokens                  */
  HLKV_ERR_LAYOUT = 1u << 6,          /* descriptor layout tag != layout->layout_id   */
  HLKV_ERR_SCALE_MODE = 1u << 7,      /* quantized block with scale mode 3 (external)
                                         or block-wide parameters that are non-finite
                                         or give FP8 a nonzero bias                  */
  HLKV_ERR_DESC_MISMATCH = 1u << 8,   /* table[id].block_id != id                     */
  HLKV_ERR_NONFINITE = 1u << 9,       /* a group with a non-finite value was skipped  */
  HLKV_ERR_TOKEN_RANGE = 1u << 10,    /* append target token >= block_tokens          */
  HLKV_ERR_PATCH_RANGE = 1u << 11,    /* delta patch target out of range              */
  HLKV_ERR_OUT_ALIGN = 1u << 12       /* output offset not a multiple of 8 elements   */
};

/* ---- ABI records (byte-identical to hl::alloc, block_descriptor.hpp:137-150 and
 *      id_arena.hpp:32-43) -------------------------------------------------------------- */
typedef struct {
  uint32_t slot;
  uint32_t info; /* format:4 | scale_mode:2 | layout:4 | valid_tokens:10 | 0:12 */
  uint32_t scale_ref;
  uint32_t block_id;
} HlkvExecDescriptor;

typedef struct {
  uint32_t offset;
  uint32_t block_id;
} HlkvIdPatch;

typedef struct {
  uint32_t offset;
  uint32_t length;
} HlkvSegment;

/* ---- payload pools and layout -------------------------------------------------------- */
/* Pool of one format: slot s starts at base + s * slot_bytes (block_descriptor.hpp:144).  */
typedef struct {
  void* base;          /* device pointer, 16-byte aligned; NULL = no pool for this format */
  uint64_t slot_bytes; /* multiple of 16, >= hlkv_layout_slot_bytes(format, layout)      */
  uint32_t num_slots;
  uint32_t reserved;   /* 0 */
} HlkvPool;

typedef struct {
  HlkvPool pool[15]; /* indexed by format code */
} HlkvPools;

/*
 * Payload layout of a block (the "layout" tag of the descriptor):
 * 2 (K, V) x block_tokens x kv_heads rows of head_dim elements, row-major in
 * that order, one parameter group per row.  A slot holds the codes of all rows
 * (packed_bytes(format, rows * head_dim)) followed by the row parameters:
 * nothing for FP16, one binary32 scale per row for FP8, one {scale, bias}
 * binary32 pair per row for INT4.  head_dim is 64, 128 or 256.
 */
typedef struct {
  uint32_t block_tokens; /* 1 .. 512 */
  uint32_t kv_heads;     /* >= 1 */
  uint32_t head_dim;     /* 64, 128 or 256 */
  uint32_t layout_id;    /* descriptors must carry this tag (0 .. 15) */
} HlkvLayout;

/* Bytes one slot of `format` needs under `layout` (0 for an unsupported format/layout). */
uint64_t hlkv_layout_slot_bytes(int format, const HlkvLayout* layout);

/* The cudaError_t of this thread's last HLKV_CUDA_ERROR (cudaSuccess otherwise). */
int hlkv_last_cuda_error(void);

/* ---- kernel (1): heterogeneous gather-dequant ------------------------------------------ */
/*
 * For every sequence i < nseq and block j < d_segs[i].length:
 *   d = d_table[d_arena[d_segs[i].offset + j]]          (hetero_block_table.hpp:22-25)
 *   payload = pools->pool[d.format].base + d.slot * slot_bytes
 *   out block = d_out + off_i + j * block_elems,  block_elems = 2*T*H*D,
 *   off_i = d_out_offsets[i] (elements, multiple of 8), or the packed prefix
 *           sum of the lengths * block_elems when d_out_offsets is NULL.
 * Rows of tokens < valid_tokens are decoded per hl::quant's
 * dequantize_reference_to_fp16 (cpu_dequant.cpp:127-141), bit for bit; rows of
 * later tokens are written as +0.  A quantized block's parameters are per row
 * (after its codes) for scale mode 0, or block-wide from the descriptor
 * (block_descriptor.hpp:61-72): mode 1 scale = the binary32 bits of scale_ref, bias
 * 0; mode 2 scale and bias = the binary16 halves of scale_ref (bits 0..15, 16..31).
 * A block failing a check is skipped and its bit set in *d_err.  The reference has
 * no gather; its per-block semantics are the reference's CPU decoder.
 */
int hlkv_gather_dequant(const HlkvPools* pools, const HlkvLayout* layout,
                        const HlkvExecDescriptor* d_table, uint32_t table_size,
                        const uint32_t* d_arena, uint32_t arena_size, const HlkvSegment* d_segs,
                        uint32_t nseq, uint16_t* d_out, const uint64_t* d_out_offsets,
                        uint32_t* d_err, hlkv_stream_t stream);

/*
 * hlkv_gather_dequant with launch flags.  HLKV_LAUNCH_OVERLAP_PREVIOUS launches the gather
 * with programmatic dependent launch: its CTAs may start while the kernel queued before it
 * on `stream` is still running, and do the segment scan and block resolution (reads of
 * d_segs, d_out_offsets, d_arena and d_table only) before waiting for that kernel to
 * complete; the pools, d_out and *d_err are touched only after it.  Set the flag only when
 * the kernel before it on the stream writes none of d_segs, d_out_offsets, d_arena and
 * d_table -- typically the gather of the previous layer of the same cache (writing the
 * same or another d_out is fine).  Not when it follows kernel (3) or any kernel that
 * changes the tables.  flags == 0 is hlkv_gather_dequant.  No counterpart in the reference.
 */
#define HLKV_LAUNCH_OVERLAP_PREVIOUS 1u
int hlkv_gather_dequant_ex(const HlkvPools* pools, const HlkvLayout* layout,
                           const HlkvExecDescriptor* d_table, uint32_t table_size,
                           const uint32_t* d_arena, uint32_t arena_size, const HlkvSegment* d_segs,
                           uint32_t nseq, uint16_t* d_out, const uint64_t* d_out_offsets,
                           uint32_t* d_err, uint32_t flags, hlkv_stream_t stream);

/* ---- kernel (2): append-encode ---------------------------------------------------------- */
typedef struct {
  uint32_t block_id; /* resolved through d_table */
  uint32_t token;    /* token slot inside the block, < block_tokens */
} HlkvAppendTarget;

/*
 * Encodes d_tokens[k] (binary16, [2][kv_heads][head_dim]) into token slot
 * d_targets[k].token of block d_targets[k].block_id, in the block's format:
 * each row is one group of quantize_reference (cpu_quant.cpp:97-170) on the
 * binary32 values of the inputs -- FP8 scale = max(amax/max_finite, FLT_MIN)
 * (1 when amax == 0), INT4 {scale = (max-min)/15, bias = min} -- codes and
 * parameters bit-exact.  A row with a non-finite input is skipped
 * (HLKV_ERR_NONFINITE), as quantize_reference rejects it.  Targets must be
 * distinct (block, token) pairs.  valid_tokens is not changed here: the host
 * table's set_valid_tokens + delta (kernel 3) does that.
 */
int hlkv_append_encode(const HlkvPools* pools, const HlkvLayout* layout,
                       const HlkvExecDescriptor* d_table, uint32_t table_size,
                       const HlkvAppendTarget* d_targets, uint32_t n, const uint16_t* d_tokens,
                       uint32_t* d_err, hlkv_stream_t stream);

/* ---- kernel (3): delta apply ------------------------------------------------------------ */
/*
 * Applies one hl::alloc::ExecDelta (hetero_block_table.hpp:100-114) to device
 * tables that already have room for it:
 *   d_table[p.block_id] = p  for each descriptor patch,
 *   d_arena[p.offset] = p.block_id  for each id patch.
 * Targets are unique per list, so all patches go in parallel.  Out-of-range
 * targets are skipped with HLKV_ERR_PATCH_RANGE.  The device restatement of
 * the reference's ExecMirror::apply (tests/project1/exec_mirror.hpp:23-49).
 * The kernel allows a kernel queued after it with programmatic dependent launch to start
 * before it completes; such a kernel must wait for it (griddepcontrol.wait) before reading
 * d_table or d_arena.  An ordinarily launched kernel is not affected.
 */
int hlkv_apply_delta(HlkvExecDescriptor* d_table, uint32_t table_size, uint32_t* d_arena,
                     uint32_t arena_size, const HlkvExecDescriptor* d_desc_patches,
                     uint32_t n_desc, const HlkvIdPatch* d_id_patches, uint32_t n_id,
                     uint32_t* d_err, hlkv_stream_t stream);

/* ---- arena relocation ------------------------------------------------------------------- */
/* A live segment's move in an arena compaction (hl::alloc::SegmentMove): entries
 * [from, from + length) go to [to, to + length) through scratch[scratch ...].  from, to and
 * scratch are multiples of 8 entries. */
typedef struct {
  uint32_t from;
  uint32_t to;
  uint32_t length;
  uint32_t scratch;
} HlkvSegmentMove;

/* Scratch entries (uint32) that a compaction's moves need: the last move's scratch offset
 * plus its length rounded up to 8 (0 for no moves). */
uint64_t hlkv_segment_moves_scratch_entries(const HlkvSegmentMove* moves, size_t n);

/*
 * Makes the moves of hlkv_table_compact_arena on a device copy of the arena, in stream
 * order: a first launch gathers every moved segment into d_scratch (at least
 * hlkv_segment_moves_scratch_entries entries), a second scatters it to its new offset, so
 * overlapping moves are safe.  arena_size is the device arena's current (pre-compaction)
 * size.  `moves` must be device-readable (device or page-locked host memory) and 16-byte
 * aligned, as must d_arena and d_scratch.  Apply it before any delta collected after the
 * compaction.  A move outside the arena or the scratch is skipped with
 * HLKV_ERR_PATCH_RANGE.  No counterpart in the reference, whose arena never compacts.
 */
int hlkv_arena_relocate(uint32_t* d_arena, uint32_t arena_size, const HlkvSegmentMove* moves,
                        uint32_t n, uint32_t* d_scratch, uint64_t scratch_entries, uint32_t* d_err,
                        hlkv_stream_t stream);

/* ---- decode attention over the quantized blocks ------------------------------------------ */
/*
 * One query token per sequence attends to the sequence's cached K and V, read from the
 * quantized blocks through the descriptor table (no FP16 K/V written to HBM).  K and V are
 * exactly the binary16 values hlkv_gather_dequant would write (the reference's
 * dequantize_reference_to_fp16), for the valid tokens of each block in sequence order.
 * For query head qh and KV head h = qh / (q_heads / kv_heads):
 *   out[i][qh] = softmax_t(softmax_scale * <q[i][qh], k_t>) . v_t
 * in binary32 arithmetic, rounded to binary16; zeros for a sequence without valid tokens.
 * d_q and d_out are binary16 [nseq][q_heads][head_dim].  head_dim 64 or 128; q_heads /
 * kv_heads in {1, 2, 4, 8}; softmax_scale finite and > 0.  Blocks failing kernel (1)'s checks
 * are left out with their HLKV_ERR_* bits.  The reference has no attention kernel; this is
 * the fused dequant + attention step its plan names (ADR-0004).
 */
int hlkv_decode_attention(const HlkvPools* pools, const HlkvLayout* layout,
                          const HlkvExecDescriptor* d_table, uint32_t table_size,
                          const uint32_t* d_arena, uint32_t arena_size, const HlkvSegment* d_segs,
                          uint32_t nseq, const uint16_t* d_q, uint32_t q_heads, float softmax_scale,
                          uint16_t* d_out, uint32_t* d_err, hlkv_stream_t stream);

/*
 * The same attention with each (sequence, KV head) split over `splits` CTAs, each taking a
 * contiguous share of the sequence's blocks: for few or long sequences, where one CTA per
 * (sequence, KV head) leaves SMs idle.  Each CTA writes its partial max, sum and outputs to
 * d_workspace (caller-owned, 16-byte aligned, at least
 * hlkv_decode_attention_workspace_bytes(nseq, kv_heads, head_dim, splits) bytes); a second
 * launch merges them.  splits == 1 needs no workspace and equals hlkv_decode_attention.
 * Calls that overlap on the GPU must not share a workspace.
 */
size_t hlkv_decode_attention_workspace_bytes(uint32_t nseq, uint32_t kv_heads, uint32_t head_dim,
                                             uint32_t splits);
int hlkv_decode_attention_split(const HlkvPools* pools, const HlkvLayout* layout,
                                const HlkvExecDescriptor* d_table, uint32_t table_size,
                                const uint32_t* d_arena, uint32_t arena_size, const HlkvSegment* d_segs,
                                uint32_t nseq, const uint16_t* d_q, uint32_t q_heads, float softmax_scale,
                                uint32_t splits, void* d_workspace, size_t workspace_bytes,
                                uint16_t* d_out, uint32_t* d_err, hlkv_stream_t stream);

/*
 * The same attention with the work balanced over exactly `ctas` CTAs (1 .. 2^20): the
 * (sequence, KV head) units' blocks, laid end to end, are cut into `ctas` equal ranges, so
 * sequences of any mix of lengths keep every SM equally busy.  A range can end inside a unit
 * and span several units; each part writes partial (max, sum, outputs) to the workspace
 * (16-byte aligned, at least hlkv_decode_attention_balanced_workspace_bytes(nseq, kv_heads,
 * head_dim, ctas) bytes), and a last launch merges them.  A first one-CTA launch writes the
 * units' prefix sums there.  No counterpart in the reference.  Calls that overlap on the GPU
 * must not share a workspace.
 */
size_t hlkv_decode_attention_balanced_workspace_bytes(uint32_t nseq, uint32_t kv_heads, uint32_t head_dim,
                                                      uint32_t ctas);
int hlkv_decode_attention_balanced(const HlkvPools* pools, const HlkvLayout* layout,
                                   const HlkvExecDescriptor* d_table, uint32_t table_size,
                                   const uint32_t* d_arena, uint32_t arena_size, const HlkvSegment* d_segs,
                                   uint32_t nseq, const uint16_t* d_q, uint32_t q_heads, float softmax_scale,
                                   uint32_t ctas, void* d_workspace, size_t workspace_bytes,
                                   uint16_t* d_out, uint32_t* d_err, hlkv_stream_t stream);

/*
 * hlkv_decode_attention_split with its partials in a fixed scratch array of this library
 * (HLKV_NOALLOC_SCRATCH_BYTES per device, part of its device image) instead of a caller
 * workspace: for callers that cannot allocate device memory when they call (a host binding
 * this ABI with no device allocator of its own; an engine that gave all free HBM to its KV
 * pools).  No counterpart in the reference.  The call allocates nothing.
 * - A split whose workspace (hlkv_decode_attention_workspace_bytes) exceeds
 *   HLKV_NOALLOC_SCRATCH_BYTES is rejected with HLKV_BUFFER_TOO_SMALL; nothing is launched.
 * - The scratch of the current device is used (the stream must belong to it).  The first call
 *   on each device looks up the scratch's address (cudaGetSymbolAddress) and caches it; make
 *   that first call before any stream capture.  The cached address belongs to the CUDA
 *   runtime's primary context of that device: do not call cudaDeviceReset on a device after
 *   its first call here, and do not call this entry point with another (driver-API) context
 *   current -- the cache would then point into a destroyed or foreign context.
 * - A grid of 2^31 CTAs or more (nseq * kv_heads * splits) returns HLKV_INVALID_ARGUMENT,
 *   not HLKV_BUFFER_TOO_SMALL, as hlkv_decode_attention_split rejects it; nothing is launched.
 * - All calls on a device share the scratch: calls that overlap on the GPU race.  Order them
 *   (one stream, or events).
 */
#define HLKV_NOALLOC_SCRATCH_BYTES (16u << 20)
int hlkv_decode_attention_split_noalloc(const HlkvPools* pools, const HlkvLayout* layout,
                                        const HlkvExecDescriptor* d_table, uint32_t table_size,
                                        const uint32_t* d_arena, uint32_t arena_size,
                                        const HlkvSegment* d_segs, uint32_t nseq, const uint16_t* d_q,
                                        uint32_t q_heads, float softmax_scale, uint32_t splits,
                                        uint16_t* d_out, uint32_t* d_err, hlkv_stream_t stream);

/* ---- format-change transcode ------------------------------------------------------------ */
typedef struct {
  uint32_t from_format; /* the block's current format and slot ...                  */
  uint32_t from_slot;
  uint32_t to_format;   /* ... and the target pool and slot (begin_format_change)     */
  uint32_t to_slot;
  uint32_t valid_tokens; /* rows of later tokens are encoded from zeros              */
  uint32_t from_scale_mode; /* the source descriptor's scale mode (0, 1 or 2) ...      */
  uint32_t from_scale_ref;  /* ... and scale_ref: block-wide source parameters          */
  uint32_t reserved;        /* 0 */
} HlkvTranscodeJob;

/*
 * Device half of a format change (hetero_block_table.cpp:251-287; no kernel in the
 * reference): for each job, re-encodes the block in (from_format, from_slot) into
 * (to_format, to_slot) -- each row of a valid token decoded as kernel (1) decodes it
 * (dequantize_reference_to_fp16) and encoded as kernel (2) encodes an appended row
 * (quantize_reference on those binary16 values); rows of later tokens encoded from +0.
 * Jobs come from hlkv_table_begin_format_change; commit the changes (and flush the
 * delta) after this call on the same stream, with scale mode kNone: the destination
 * carries per-row parameters.  A source block with block-wide parameters (its
 * descriptor's scale mode 1 or 2) passes that mode and scale_ref in the job.  Source and
 * destination slots must not overlap.  d_jobs 16-byte aligned.  Bad jobs and non-finite
 * rows are skipped with their HLKV_ERR_* bits.
 */
int hlkv_transcode(const HlkvPools* pools, const HlkvLayout* layout, const HlkvTranscodeJob* d_jobs,
                   uint32_t n, uint32_t* d_err, hlkv_stream_t stream);

/* ---- flat codecs ------------------------------------------------------------------------ */
/*
 * Drop-in for hl::quant::cuda::dequantize_fp8_to_fp16 (cuda_dequant.hpp:47-50,
 * dequant_kernel.cu:171-191): out[i] = fp16_rn(decode_fp8(in[i]) * params[i/group].scale),
 * any alignment, any group size >= 1.  d_params holds {scale, bias} binary32
 * pairs (AffineParams); only scale is read.
 */
int hlkv_dequantize_fp8_to_fp16(int format, const void* d_in, size_t n, const float* d_params,
                                size_t group_size, uint16_t* d_out, hlkv_stream_t stream);

/*
 * Device counterpart of hl::quant::dequantize_reference_to_fp16
 * (cpu_dequant.hpp:44-54) for every format, with the same argument rules
 * checked on the host (format, group size, parameter count, buffer sizes).
 * Parameter values are checked per group on the device: a group with a
 * non-finite parameter (or a non-zero FP8 bias) is skipped, its outputs left
 * untouched, and HLKV_ERR_NONFINITE is set in *d_err.
 */
int hlkv_dequantize_to_fp16(int format, const void* d_packed, size_t packed_size, size_t n,
                            const float* d_params, size_t n_params, size_t group_size,
                            uint16_t* d_out, size_t out_size, uint32_t* d_err,
                            hlkv_stream_t stream);

/*
 * Device counterpart of hl::quant::quantize_reference (cpu_quant.hpp:33-47):
 * same argument rules on the host; codes and parameters bit-exact.  A group
 * with a non-finite input (or an INT4 range that overflows) is skipped, its
 * codes and parameters left untouched, and HLKV_ERR_NONFINITE is set.
 */
int hlkv_quantize(int format, const float* d_in, size_t n, size_t group_size, float* d_params,
                  size_t n_params, void* d_packed, size_t packed_size, uint32_t* d_err,
                  hlkv_stream_t stream);

/* ---- host table (hl::alloc::HeteroBlockTable, hetero_block_table.hpp:141-245) ----------- */
/* The table (and device-table) calls take a handle from hlkv_table_create / _restore
 * (hlkv_device_tables_create); like the C++ object references they stand for, a NULL or
 * destroyed handle is not checked. */
typedef struct hlkv_table hlkv_table;

typedef struct {
  uint32_t format;
  uint32_t slot_bytes;
  uint32_t num_slots;
} HlkvPoolConfig;

typedef struct {
  uint32_t max_blocks;
  uint32_t block_tokens;
  uint32_t num_pools;
  const HlkvPoolConfig* pools;
} HlkvTableConfig;

typedef struct {
  uint32_t format;
  uint32_t valid_tokens;
  uint32_t layout;
  uint32_t scale_mode;
  uint32_t scale_ref;
} HlkvAllocRequest;

typedef struct {
  uint32_t id;
  uint32_t generation;
} HlkvHandle; /* BlockHandle and SequenceHandle; {0xFFFFFFFF, 0} is invalid */

int hlkv_table_validate_config(const HlkvTableConfig* config);
int hlkv_table_create(const HlkvTableConfig* config, hlkv_table** out);
void hlkv_table_destroy(hlkv_table* table);
/*
 * Versioned binary image of the whole table (HeteroBlockTable::snapshot: configuration,
 * records, free lists, pool stacks, sequences, id arena, checksum).  *size receives its
 * length; the image is written when buf holds cap >= *size bytes (buf NULL: size only;
 * cap too small: HLKV_STATUS_INVALID_ARGUMENT, nothing written).  No counterpart in the
 * reference: its ABI v1 lists the missing snapshot API among its limitations
 * (hl_allocator_abi.md, section 9).
 */
int hlkv_table_snapshot(const hlkv_table* t, void* buf, size_t cap, size_t* size);
/*
 * A new table rebuilt from a snapshot image (HeteroBlockTable::restore); destroy it with
 * hlkv_table_destroy.  HLKV_STATUS_CORRUPT for a short, damaged, foreign or inconsistent
 * image.  Every descriptor and arena entry of the restored table is pending, so the first
 * sync of a fresh hlkv_device_tables uploads the whole device image.
 */
int hlkv_table_restore(const void* buf, size_t size, hlkv_table** out);

int hlkv_table_allocate(hlkv_table* t, const HlkvAllocRequest* req, HlkvHandle* out);
int hlkv_table_retain(hlkv_table* t, HlkvHandle block);
int hlkv_table_release(hlkv_table* t, HlkvHandle block);
int hlkv_table_set_valid_tokens(hlkv_table* t, HlkvHandle block, uint32_t valid_tokens);
int hlkv_table_seal(hlkv_table* t, HlkvHandle block);
int hlkv_table_set_residency(hlkv_table* t, HlkvHandle block, uint32_t residency);
int hlkv_table_set_scale(hlkv_table* t, HlkvHandle block, uint32_t scale_mode, uint32_t scale_ref);
/* out[4] = {from_format, from_slot, to_format, to_slot} */
int hlkv_table_begin_format_change(hlkv_table* t, HlkvHandle block, uint32_t target, uint32_t out[4]);
int hlkv_table_commit_format_change(hlkv_table* t, HlkvHandle block, uint32_t scale_mode,
                                    uint32_t scale_ref);
int hlkv_table_abort_format_change(hlkv_table* t, HlkvHandle block);
/* out = the 32-byte host record (hl::alloc::BlockDescriptor) */
int hlkv_table_lookup(const hlkv_table* t, HlkvHandle block, void* out32);
int hlkv_table_lookup_batch(const hlkv_table* t, const HlkvHandle* blocks, size_t n,
                            HlkvExecDescriptor* out, size_t out_n);
HlkvHandle hlkv_table_handle_of(const hlkv_table* t, uint32_t block_id);

int hlkv_table_create_sequence(hlkv_table* t, HlkvHandle* out);
int hlkv_table_append_block(hlkv_table* t, HlkvHandle seq, const HlkvAllocRequest* req,
                            HlkvHandle* out);
int hlkv_table_append_shared_block(hlkv_table* t, HlkvHandle seq, HlkvHandle block);
int hlkv_table_release_sequence(hlkv_table* t, HlkvHandle seq);
/* Copies up to cap ids; *len = the sequence length (HLKV_STATUS_INVALID_ARGUMENT if cap < len). */
int hlkv_table_sequence_block_ids(const hlkv_table* t, HlkvHandle seq, uint32_t* out, size_t cap,
                                  size_t* len);
int hlkv_table_batch_segments(const hlkv_table* t, const HlkvHandle* seqs, size_t n,
                              HlkvSegment* out);
/*
 * Decode-step driver (no counterpart in the reference; built only from the public table
 * operations above): for each sequence seqs[i], makes room for one more token -- in its
 * tail block when that holds fewer than block_tokens valid tokens (set_valid_tokens + 1),
 * else in a new block appended with req {new_formats[i], valid_tokens 1, layout} -- and
 * writes the new token's kernel (2) target to out[i].  Stops at the first failing
 * operation and returns its status; *n_done = sequences completed.
 */
int hlkv_table_append_tokens(hlkv_table* t, const HlkvHandle* seqs, size_t n,
                             const uint32_t* new_formats, uint32_t layout,
                             HlkvAppendTarget* out, size_t* n_done);
/*
 * HeteroBlockTable::compact_arena: packs the id arena (live segments to the front, in offset
 * order, free storage given back) and writes the segment moves the device copy must make to
 * out (at most one per live sequence: cap must be at least the number of live sequences,
 * else HLKV_STATUS_INVALID_ARGUMENT and nothing changes).  HLKV_STATUS_INVALID_STATE while
 * id patches are pending (collect the delta first).  Follow it with
 * hlkv_device_tables_relocate (or hlkv_arena_relocate) before the next delta is applied.
 * No counterpart in the reference.
 */
int hlkv_table_compact_arena(hlkv_table* t, HlkvSegmentMove* out, size_t cap, size_t* n_moves);
/* CSR reference path: indptr[n+1], blocks[cap]; *total = number of blocks. */
int hlkv_table_build_exec_table(const hlkv_table* t, const HlkvHandle* seqs, size_t n,
                                uint32_t* indptr, HlkvExecDescriptor* blocks, size_t cap,
                                size_t* total);
void hlkv_table_pending(const hlkv_table* t, size_t* n_desc, size_t* n_id);
/* Moves the pending delta out (HLKV_STATUS_INVALID_ARGUMENT, nothing moved, if a cap is short). */
int hlkv_table_collect_delta(hlkv_table* t, HlkvExecDescriptor* desc, size_t desc_cap,
                             HlkvIdPatch* ids, size_t id_cap, size_t* n_desc, size_t* n_id,
                             uint32_t* table_size, uint32_t* arena_size);
HlkvExecDescriptor hlkv_table_device_descriptor(const hlkv_table* t, uint32_t block_id);
uint32_t hlkv_table_block_tokens(const hlkv_table* t);
uint32_t hlkv_table_max_blocks(const hlkv_table* t);
uint32_t hlkv_table_blocks_in_use(const hlkv_table* t);
int hlkv_table_has_pool(const hlkv_table* t, uint32_t format);
uint32_t hlkv_table_free_slots(const hlkv_table* t, uint32_t format);
uint32_t hlkv_table_pool_slots(const hlkv_table* t, uint32_t format);
uint32_t hlkv_table_slot_bytes(const hlkv_table* t, uint32_t format);
/* TableStats flattened: 3 + 15 + 4 + 4 counters, then 10 uint64 totals (36 values). */
void hlkv_table_stats(const hlkv_table* t, uint64_t out[36]);
/* Returns the status of validate(); the message (NUL-terminated, truncated) goes to msg. */
int hlkv_table_validate(const hlkv_table* t, char* msg, size_t cap);

/* ---- persistent device tables (the mirror of the table's device-facing state) ---------- */
typedef struct hlkv_device_tables hlkv_device_tables;

/* Binds to the current CUDA device; allocates lazily on the first sync. */
int hlkv_device_tables_create(hlkv_device_tables** out);
void hlkv_device_tables_destroy(hlkv_device_tables* dt);
/*
 * collect_delta() on the host table, then on `stream`: grow the device arena
 * (keeping contents), upload the patches (pinned staging) and run kernel (3).
 * Returns an HLKV_* device status.
 */
int hlkv_device_tables_sync(hlkv_device_tables* dt, hlkv_table* t, hlkv_stream_t stream);
/*
 * The two halves of hlkv_device_tables_sync, so that host table work can run ahead of
 * the stream: collect moves the table's pending changes into dt (merged with changes
 * collected earlier, later patches winning) and into pinned staging, queueing nothing;
 * flush queues their upload and kernel (3) on `stream`.  No counterpart in the reference.
 */
int hlkv_device_tables_collect(hlkv_device_tables* dt, hlkv_table* t);
int hlkv_device_tables_flush(hlkv_device_tables* dt, hlkv_stream_t stream);
/*
 * Applies a compaction to the device arena (after flushing what collect gathered): the moves
 * of hlkv_table_compact_arena (host memory) through the mirror's own staging and scratch,
 * then the arena's size becomes new_arena_size (the table's arena size after compacting),
 * and device memory beyond a quarter of headroom above it is returned.  Returning memory
 * waits for the device to go idle (cudaDeviceSynchronize): compaction is maintenance, not
 * a per-step call.  No counterpart in the reference.
 */
int hlkv_device_tables_relocate(hlkv_device_tables* dt, const HlkvSegmentMove* moves, size_t n,
                                uint32_t new_arena_size, hlkv_stream_t stream);
/* Device memory behind the arena, in bytes (the capacity it can grow into without mapping
 * more). */
uint64_t hlkv_device_tables_arena_capacity_bytes(const hlkv_device_tables* dt);
const HlkvExecDescriptor* hlkv_device_tables_table(const hlkv_device_tables* dt);
uint32_t hlkv_device_tables_table_size(const hlkv_device_tables* dt);
/* The device arena.  Where the driver supports virtual memory management, the arena lives in
 * a reserved address range and growth maps more memory behind it: the address never changes
 * (kernels already queued, or a captured CUDA graph, keep a valid pointer).  Otherwise growth
 * reallocates and copies, and the address changes at growth. */
const uint32_t* hlkv_device_tables_arena(const hlkv_device_tables* dt);
uint32_t hlkv_device_tables_arena_size(const hlkv_device_tables* dt);
/* Device word the sync's kernel (3) reports into (zeroed at creation). */
uint32_t* hlkv_device_tables_error_word(const hlkv_device_tables* dt);

/*
 * The device half of one decode step, two launches queued on `stream` from native code:
 * kernel (3) applies the delta staged by hlkv_device_tables_collect (as
 * hlkv_device_tables_flush) and, in the same launch, copies the n append targets that
 * hlkv_table_append_tokens wrote to h_targets into d_targets; then encode_event (a
 * cudaEvent_t, or NULL) is recorded and d_tokens[k] is encoded into target k through the
 * device tables (hlkv_append_encode).  start_event (a cudaEvent_t, or NULL) is recorded
 * just before kernel (3) is queued, after the call's host-side checks, so that the two
 * events and one recorded after the call bracket the step's device work.
 * h_targets must be page-locked host memory (or device memory), which the kernel reads in
 * place (HLKV_INVALID_ARGUMENT for pageable memory), and must stay untouched until the
 * stream has passed kernel (3).
 * Kernel (2) is launched with programmatic dependent launch: while kernel (3) runs, it
 * prefetches d_tokens into L2 and issues its first token loads, and it waits for kernel
 * (3) before reading d_targets and the descriptor table (d_tokens must be complete when
 * the call is made, as for any work queued before kernel (3)).  With encode_event the
 * event sits between the two kernels, and kernel (2) is launched plainly after it.
 * Returns the first failing status; what was queued before it stays queued.  No
 * counterpart in the reference: the device side of the decode loop its plan describes.
 */
int hlkv_decode_step_queue(hlkv_device_tables* dt, const HlkvPools* pools, const HlkvLayout* layout,
                           const HlkvAppendTarget* h_targets, HlkvAppendTarget* d_targets, uint32_t n,
                           const uint16_t* d_tokens, uint32_t* d_err, void* start_event,
                           void* encode_event, hlkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HLKV_H_ */
