// Kernel (2): append-encode of FP16 tokens into heterogeneous KV blocks.
//
// Target k writes token d_targets[k].token of block d_targets[k].block_id,
// found through the device descriptor table.  The token is 2*H rows of D
// binary16 values ([K,V][head][dim]); each row is one group of the reference's
// quantize_reference (project2_quant/src/cpu_quant.cpp:97-170) on the binary32
// values of the inputs, stored at row (kv*T + token)*H + h of the block's
// layout (codes first, then the per-row parameters).
//
// A row is handled by D/16 lanes (8 for D = 128), 16 elements per lane from two
// 16-byte loads (chunks l and l + D/16 of the row, so each warp-wide load is
// contiguous); the per-row encode (group statistics by shuffle reductions, the
// reference's scale rules, RNE codes) is dev::encode_row in row_encode.cuh.  Two
// chunks per lane halve the per-row work (target and descriptor loads and checks,
// index arithmetic, scale division) per element against one chunk per lane.
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "row_encode.cuh"
#include "hlkv.h"

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
  const uint4* table;
  const uint2* targets;
  const uint4* tokens;
  uint32_t* err;
  uint32_t rows_total;  // n * 2H < 2^31
  FastDiv two_h;        // 2H
  uint32_t table_size, T, H, layout_id;
  uint64_t token_bytes;    // the whole token array
  uint32_t prefetch_ctas;  // CTAs that warm L2 with it first (0: none)
};

constexpr int kChunks = 2;  // 8-value chunks per lane

// 6 CTAs of 256 per SM (40 registers): the kernel waits on its row chain (target ->
// descriptor -> store) more than it issues, so more resident warps pay; measured 22 us per
// decode step against 23.8 us at 4 CTAs (64 registers).
constexpr int kMinCtasPerSm = 6;

template <int kD>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) append_encode_kernel(const Params p) {
  constexpr int kLanes = kD / (8 * kChunks);
  constexpr int kRowsPerIter = kThreads / kLanes;
  const uint32_t lane = threadIdx.x % kLanes;
  const uint32_t mask = dev::row_mask<kD, kChunks>();
  bool waited = false;
  if (threadIdx.x == 0 && blockIdx.x < p.prefetch_ctas) {
    // Launched to overlap kernel (3): the first wave asks L2 for the whole token array (the
    // tokens were complete before kernel (3) started), one bulk prefetch per 16 KB, so the
    // row loads after the wait find them in L2.
    const uint64_t per = ((p.token_bytes + p.prefetch_ctas - 1) / p.prefetch_ctas + 15) & ~uint64_t{15};
    uint64_t b = uint64_t{blockIdx.x} * per;
    const uint64_t e = b + per < p.token_bytes ? b + per : p.token_bytes;
    const char* base = reinterpret_cast<const char*>(p.tokens);
    for (; b < e; b += 16384u) {
      const uint32_t size = static_cast<uint32_t>(e - b < 16384u ? e - b : 16384u);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + b), "r"(size) : "memory");
    }
  }
  for (uint32_t g = blockIdx.x * kRowsPerIter + threadIdx.x / kLanes; g < p.rows_total;
       g += gridDim.x * kRowsPerIter) {
    // Everything below is uniform over the lanes of row g.
    const uint32_t k = p.two_h.div(g);
    const uint32_t r = g - k * p.two_h.d;
    const uint32_t kv = r >= p.H ? 1u : 0u, h = r - kv * p.H;

    // The token row does not depend on the descriptor: both loads go out together.  Launched
    // with programmatic serialization after kernel (3), the first token loads are issued
    // before waiting for kernel (3), which writes the targets and the descriptor table.
    uint4 raw[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) raw[c] = __ldcs(p.tokens + uint64_t{g} * (kD / 8) + c * kLanes + lane);
    if (!waited) {
      dev::wait_for_prerequisites();
      waited = true;
    }
    const uint2 t = __ldg(p.targets + k);
    uint32_t bad = 0, f = 0, slot = 0;
    const uint32_t id = t.x, tok = t.y;
    if (id >= p.table_size) {
      bad = dev::kErrBlockIdRange;
    } else {
      const uint4 d = __ldg(p.table + id);
      f = d.y & 0xFu;
      const uint32_t mode = (d.y >> 4) & 3u, layout = (d.y >> 6) & 0xFu;
      slot = d.x;
      if (d.w != id) bad = dev::kErrDescMismatch;
      else if (f == dev::kInvalidFormat) bad = dev::kErrNotExecutable;
      else if (f > 3 || p.pool[f].base == nullptr || p.pool[f].num_slots == 0) bad = dev::kErrBadFormat;
      else if (layout != p.layout_id) bad = dev::kErrLayout;
      else if (f != dev::kFp16 && mode != 0) bad = dev::kErrScaleMode;
      else if (tok >= p.T) bad = dev::kErrTokenRange;
      else if (slot >= p.pool[f].num_slots) bad = dev::kErrSlotRange;
    }
    if (bad) {
      if (r == 0 && lane == 0) atomicOr(p.err, bad);  // once per target
      continue;
    }

    const uint32_t row = (kv * p.T + tok) * p.H + h;
    uint8_t* payload = p.pool[f].base + uint64_t{slot} * p.pool[f].slot_bytes;
    const uint32_t e = dev::encode_row<kD, kChunks>(f, raw, lane, mask, payload, row, p.code_bytes[f]);
    if (e != 0 && lane == 0) atomicOr(p.err, e);
  }
}

}  // namespace
}  // namespace hlkv

namespace hlkv {

// hlkv_append_encode; with overlap_previous the kernel is launched with programmatic stream
// serialization (its prologue may run while the kernel before it finishes; see the kernel)
// and its first wave prefetches the tokens into L2 meanwhile.
int launch_append_encode(const HlkvPools* pools, const HlkvLayout* layout, const HlkvExecDescriptor* d_table,
                         uint32_t table_size, const HlkvAppendTarget* d_targets, uint32_t n,
                         const uint16_t* d_tokens, uint32_t* d_err, bool overlap_previous,
                         cudaStream_t s) {
  if (pools == nullptr || !layout_ok(layout) || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n == 0) return HLKV_OK;
  if (d_targets == nullptr || d_tokens == nullptr || (table_size > 0 && d_table == nullptr) ||
      (reinterpret_cast<uintptr_t>(d_tokens) & 15u) != 0) {
    return HLKV_INVALID_ARGUMENT;
  }
  Params p{};
  const uint64_t rows = uint64_t{2} * layout->block_tokens * layout->kv_heads;
  const uint64_t elems = rows * layout->head_dim;
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
  p.table = reinterpret_cast<const uint4*>(d_table);
  p.targets = reinterpret_cast<const uint2*>(d_targets);
  p.tokens = reinterpret_cast<const uint4*>(d_tokens);
  p.err = d_err;
  const uint64_t rows_total = uint64_t{n} * 2 * layout->kv_heads;
  if (rows_total >= (uint64_t{1} << 31)) return HLKV_INVALID_ARGUMENT;
  p.rows_total = static_cast<uint32_t>(rows_total);
  p.two_h = FastDiv(2 * layout->kv_heads);
  p.table_size = table_size;
  p.T = layout->block_tokens;
  p.H = layout->kv_heads;
  p.layout_id = layout->layout_id;
  const int lanes = static_cast<int>(layout->head_dim / (8 * kChunks));
  const uint64_t rows_per_cta = kThreads / lanes;
  const uint64_t want = (p.rows_total + rows_per_cta - 1) / rows_per_cta;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 16;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  p.token_bytes = rows_total * layout->head_dim * 2;  // a multiple of 16 (head_dim >= 64)
  const unsigned first_wave = static_cast<unsigned>(sm_count()) * kMinCtasPerSm;
  p.prefetch_ctas = overlap_previous ? (grid < first_wave ? grid : first_wave) : 0u;
  void (*kernel)(Params) = layout->head_dim == 64    ? append_encode_kernel<64>
                           : layout->head_dim == 128 ? append_encode_kernel<128>
                                                     : append_encode_kernel<256>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_previous ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, p));
}

}  // namespace hlkv

extern "C" int hlkv_append_encode(const HlkvPools* pools, const HlkvLayout* layout,
                                  const HlkvExecDescriptor* d_table, uint32_t table_size,
                                  const HlkvAppendTarget* d_targets, uint32_t n,
                                  const uint16_t* d_tokens, uint32_t* d_err, hlkv_stream_t stream) {
  return hlkv::launch_append_encode(pools, layout, d_table, table_size, d_targets, n, d_tokens, d_err, false,
                                    reinterpret_cast<cudaStream_t>(stream));
}
