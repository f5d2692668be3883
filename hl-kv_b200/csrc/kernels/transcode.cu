// Format-change transcode: re-encodes whole blocks from one pool format into another in
// one pass -- the device half of the table's begin_format_change -> commit_format_change
// protocol (project1_allocator/src/hetero_block_table.cpp:251-287), used to age KV
// blocks FP16 -> FP8 -> INT4.
//
// Job k moves the block in slot from_slot of pool from_format into slot to_slot of pool
// to_format.  The source block's parameters are per row, or block-wide when the job carries
// its descriptor's scale mode 1 or 2 and scale_ref (as kernel (1) reads them; mode 3 and
// parameters the reference's dequantizer rejects skip the job with HLKV_ERR_SCALE_MODE).
// The destination is written with per-row parameters (commit it with scale mode kNone).
// Per row (one parameter group of D values, layout as in kernel (1)):
//   rows of tokens < valid_tokens: decoded exactly as kernel (1) decodes them (the
//     reference's dequantize_reference_to_fp16, cpu_dequant.cpp:127-141), then encoded
//     as kernel (2) encodes an appended FP16 row (quantize_reference on those values);
//   rows of later tokens: encoded from +0 values (FP8 codes 0 with scale 1, INT4 codes 0
//     with {0, 0}, FP16 zeros), so the whole destination slot is defined.
// A transcoded block therefore equals the block that appending its gathered FP16 tokens
// in the new format would produce.  A row with a non-finite decoded value is rejected as
// quantize_reference rejects it (nothing written, HLKV_ERR_NONFINITE); a job with a bad
// format, slot or valid_tokens is skipped with its bit.
//
// One row per D/16 lanes, two chunks of 8 values per lane (chunks l and l + D/16 of the
// row, so each warp-wide load is contiguous): per chunk a 16/8/4-byte load of source codes,
// plus the row parameters, register decode, then dev::encode_row.  Two chunks per lane
// halve the per-row work (job load and checks, index arithmetic) per value.
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"
#include "row_encode.cuh"

namespace hlkv {
namespace {

constexpr int kThreads = 256;

struct DevPool {
  uint8_t* base;
  uint64_t slot_bytes;
  uint32_t num_slots;
};

struct Params {
  DevPool pool[4];
  uint64_t code_bytes[4];
  const uint4* jobs;  // HlkvTranscodeJob: {from_format, from_slot, to_format, to_slot}, {valid_tokens, 0, 0, 0}
  uint32_t* err;
  uint32_t rows_total;  // n * rows_per_block < 2^31
  uint32_t rows_per_block, T, H;
  FastDiv div_rows, div_h, div_t;
};

constexpr int kChunks = 2;  // 8-value chunks per lane

template <int kD>
__global__ void __launch_bounds__(kThreads) transcode_kernel(const Params p) {
  constexpr int kLanes = kD / (8 * kChunks);
  constexpr int kRowsPerIter = kThreads / kLanes;
  const uint32_t lane = threadIdx.x % kLanes;
  const uint32_t mask = dev::row_mask<kD, kChunks>();
  for (uint32_t g = blockIdx.x * kRowsPerIter + threadIdx.x / kLanes; g < p.rows_total;
       g += gridDim.x * kRowsPerIter) {
    // Uniform over the lanes of row g.
    const uint32_t k = p.div_rows.div(g);
    const uint32_t r = g - k * p.rows_per_block;
    const uint4 j0 = __ldg(p.jobs + 2 * uint64_t{k});
    const uint4 j1 = __ldg(p.jobs + 2 * uint64_t{k} + 1);  // {valid_tokens, from_scale_mode, from_scale_ref, 0}
    const uint32_t vt = j1.x;
    const uint32_t ff = j0.x, fs = j0.y, tf = j0.z, ts = j0.w;
    const uint32_t fmode = ff == dev::kFp16 ? 0u : j1.y;
    float2 wprm = make_float2(0.0f, 0.0f);
    uint32_t bad = 0;
    if (ff > 3 || tf > 3 || p.pool[ff].base == nullptr || p.pool[tf].base == nullptr) {
      bad = dev::kErrBadFormat;
    } else if (fmode > 2 || (fmode != 0 && !dev::block_params(ff, fmode, j1.z, &wprm))) {
      bad = dev::kErrScaleMode;
    } else if (fs >= p.pool[ff].num_slots || ts >= p.pool[tf].num_slots) {
      bad = dev::kErrSlotRange;
    } else if (vt > p.T) {
      bad = dev::kErrValidTokens;
    }
    if (bad) {
      if (r == 0 && lane == 0) atomicOr(p.err, bad);  // once per job
      continue;
    }
    const uint32_t rh = p.div_h.div(r);             // r / H
    const uint32_t tok = rh - p.div_t.div(rh) * p.T;  // (r / H) % T
    const uint8_t* src = p.pool[ff].base + uint64_t{fs} * p.pool[ff].slot_bytes;
    uint4 raw[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) raw[c] = make_uint4(0u, 0u, 0u, 0u);
    if (tok < vt) {
      const uint8_t* prm = src + p.code_bytes[ff];
      switch (ff) {
        case dev::kFp16: {
          const uint4* row = reinterpret_cast<const uint4*>(src + uint64_t{r} * kD * 2);
          uint4 v[kChunks];
#pragma unroll
          for (int c = 0; c < kChunks; ++c) v[c] = dev::ld_stream(row + c * kLanes + lane);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) raw[c] = dev::canon_f16x8(v[c]);
          break;
        }
        case dev::kE4M3:
        case dev::kE5M2: {
          const uint2* row = reinterpret_cast<const uint2*>(src + uint64_t{r} * kD);
          uint2 v[kChunks];
#pragma unroll
          for (int c = 0; c < kChunks; ++c) v[c] = dev::ld_stream(row + c * kLanes + lane);
          const float s = fmode != 0 ? wprm.x : __ldg(reinterpret_cast<const float*>(prm) + r);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            raw[c] = ff == dev::kE4M3 ? dev::fp8x8_to_f16<dev::kE4M3>(v[c], s) : dev::fp8x8_to_f16<dev::kE5M2>(v[c], s);
          }
          break;
        }
        default: {
          const uint32_t* row = reinterpret_cast<const uint32_t*>(src + uint64_t{r} * (kD / 2));
          uint32_t v[kChunks];
#pragma unroll
          for (int c = 0; c < kChunks; ++c) v[c] = dev::ld_stream(row + c * kLanes + lane);
          const float2 sb = fmode != 0 ? wprm : __ldg(reinterpret_cast<const float2*>(prm) + r);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) raw[c] = dev::int4x8_to_f16(v[c], sb.x, sb.y);
          break;
        }
      }
    }
    uint8_t* dst = p.pool[tf].base + uint64_t{ts} * p.pool[tf].slot_bytes;
    const uint32_t e = dev::encode_row<kD, kChunks>(tf, raw, lane, mask, dst, r, p.code_bytes[tf]);
    if (e != 0 && lane == 0) atomicOr(p.err, e);
  }
}

}  // namespace
}  // namespace hlkv

extern "C" int hlkv_transcode(const HlkvPools* pools, const HlkvLayout* layout,
                              const HlkvTranscodeJob* d_jobs, uint32_t n, uint32_t* d_err,
                              hlkv_stream_t stream) {
  using namespace hlkv;
  if (pools == nullptr || !layout_ok(layout) || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n == 0) return HLKV_OK;
  if (d_jobs == nullptr || (reinterpret_cast<uintptr_t>(d_jobs) & 15u) != 0) return HLKV_INVALID_ARGUMENT;
  Params p{};
  p.rows_per_block = 2 * layout->block_tokens * layout->kv_heads;
  const uint64_t elems = uint64_t{p.rows_per_block} * layout->head_dim;
  for (int f = 0; f < 4; ++f) {
    const HlkvPool& q = pools->pool[f];
    p.code_bytes[f] = layout_code_bytes(f, elems);
    if (q.base == nullptr || q.num_slots == 0) continue;
    if ((reinterpret_cast<uintptr_t>(q.base) & 15u) != 0 || (q.slot_bytes & 15u) != 0 ||
        q.slot_bytes < hlkv_layout_slot_bytes(f, layout)) {
      return HLKV_INVALID_ARGUMENT;
    }
    p.pool[f] = DevPool{static_cast<uint8_t*>(q.base), q.slot_bytes, q.num_slots};
  }
  p.jobs = reinterpret_cast<const uint4*>(d_jobs);
  p.err = d_err;
  const uint64_t rows_total = uint64_t{n} * p.rows_per_block;
  if (rows_total >= (uint64_t{1} << 31)) return HLKV_INVALID_ARGUMENT;
  p.rows_total = static_cast<uint32_t>(rows_total);
  p.div_rows = FastDiv(p.rows_per_block);
  p.div_h = FastDiv(layout->kv_heads);
  p.div_t = FastDiv(layout->block_tokens);
  p.T = layout->block_tokens;
  p.H = layout->kv_heads;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint64_t rows_per_cta = kThreads / (layout->head_dim / (8 * kChunks));
  const uint64_t want = (p.rows_total + rows_per_cta - 1) / rows_per_cta;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 16;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  switch (layout->head_dim) {
    case 64: transcode_kernel<64><<<grid, kThreads, 0, s>>>(p); break;
    case 128: transcode_kernel<128><<<grid, kThreads, 0, s>>>(p); break;
    default: transcode_kernel<256><<<grid, kThreads, 0, s>>>(p); break;
  }
  return cuda_status(cudaGetLastError());
}
