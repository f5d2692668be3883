// Kernel (1): heterogeneous gather-dequant.
//
// For each sequence i and block j, reads descriptor_table[arena[seg_i.offset + j]]
// (the device view of hl::alloc, hetero_block_table.hpp:22-25), decodes the
// block payload from the pool of its format and writes 2*T*H*D binary16
// values to the output.  Per element the result equals the reference's
// dequantize_reference_to_fp16 (cpu_dequant.cpp:127-141) bit for bit.
//
// Structure (HBM-bound; no tensor cores):
//  * persistent grid: one wave of CTAs (SMs x resident CTAs); CTA c owns the
//    global block indices w = c, c + G, c + 2G, ... so every CTA gets a mix of
//    formats.  When a chunk holds fewer than two blocks per CTA, each block is
//    split into 2, 4 or 8 tile ranges ("pieces") owned the same way, so small
//    batches still occupy every SM;
//  * the segments are scanned in chunks of 256 sequences (block-wide prefix
//    sum in shared memory), so the kernel needs no host-side prefix and no
//    scratch memory;
//  * the descriptor chain segment -> arena -> table (three dependent loads) of
//    up to 256 owned blocks is resolved in parallel, one block per thread, into
//    shared memory; blocks are then streamed back to back without a barrier;
//  * per block the format is CTA-uniform and selects one of four instantiations
//    of the streaming loop; each thread handles 8-element
//    chunks: a 16-byte (FP16), 8-byte (FP8) or 4-byte (INT4) coalesced load,
//    register-level byte/nibble unpack into the warp's shared-memory tile;
//    one lane writes each 2 KB tile to HBM with a TMA bulk store
//    (cp.async.bulk, no multicast).  Row parameters are read through the
//    read-only path (16 threads share a row).
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr int kThreads = 256;
constexpr int kMinCtasPerSm = 4;  // 64 registers per thread
constexpr int kUnroll = 4;        // chunks per lane per tile: 2 KB tiles
constexpr uint32_t kTileChunks = 32 * kUnroll;  // 8-element chunks per warp tile

struct DevPool {
  const uint8_t* base;
  uint64_t slot_bytes;
  uint32_t num_slots;
};

struct Params {
  DevPool pool[4];
  uint64_t code_bytes[4];  // size of the code region of a slot, per format
  const uint4* table;
  const uint32_t* arena;
  const uint2* segs;
  uint16_t* out;
  const uint64_t* out_offsets;
  uint32_t* err;
  uint64_t block_elems;
  uint32_t table_size, arena_size, nseq;
  uint32_t T, H, layout_id, rows_per_kv;
};

struct Item {
  const uint8_t* payload;
  uint16_t* out;
  uint32_t fmt;         // 0..3 (| kWide: block-wide parameters in prm), or kSkip
  uint32_t valid_rows;  // rows per K/V half holding valid tokens: valid_tokens * H
  uint32_t tile_begin;  // warp tiles [tile_begin, tile_end) of the block are streamed
  uint32_t tile_end;
  float2 prm;           // block-wide {scale, bias} (scale modes 1 and 2)
};
constexpr uint32_t kSkip = 0xFFu;
constexpr uint32_t kWide = 0x100u;

// Resolves block j of sequence `seq` into an Item; on a failed check the item
// is skipped and its bit collected in *s_err (this CTA's shared error word,
// written to *p.err once the CTA is done).  Check order matches the oracle's
// resolve_block().
__device__ Item resolve(const Params& p, uint32_t seq, uint64_t j, uint64_t blocks_before, uint32_t* s_err) {
  Item it{nullptr, nullptr, kSkip, 0, 0, 0, make_float2(0.0f, 0.0f)};
  uint32_t bad = 0;
  const uint64_t base = p.out_offsets ? p.out_offsets[seq] : blocks_before * p.block_elems;
  if (base & 7u) {
    bad = dev::kErrOutAlign;
  } else {
    const uint64_t pos = uint64_t{p.segs[seq].x} + j;
    if (pos >= p.arena_size) {
      bad = dev::kErrArenaRange;
    } else {
      const uint32_t id = p.arena[pos];
      if (id >= p.table_size) {
        bad = dev::kErrBlockIdRange;
      } else {
        const uint4 d = __ldg(p.table + id);  // {slot, info, scale_ref, block_id}
        const uint32_t f = d.y & 0xFu, mode = (d.y >> 4) & 3u, layout = (d.y >> 6) & 0xFu,
                       vt = (d.y >> 10) & 0x3FFu;
        if (d.w != id) bad = dev::kErrDescMismatch;
        else if (f == dev::kInvalidFormat) bad = dev::kErrNotExecutable;
        else if (f > 3 || p.pool[f].base == nullptr || p.pool[f].num_slots == 0) bad = dev::kErrBadFormat;
        else if (layout != p.layout_id) bad = dev::kErrLayout;
        else if (f != dev::kFp16 && (mode > 2 || (mode != 0 && !dev::block_params(f, mode, d.z, &it.prm))))
          bad = dev::kErrScaleMode;
        else if (vt > p.T) bad = dev::kErrValidTokens;
        else if (d.x >= p.pool[f].num_slots) bad = dev::kErrSlotRange;
        else {
          it.payload = p.pool[f].base + uint64_t{d.x} * p.pool[f].slot_bytes;
          it.out = p.out + base + j * p.block_elems;
          it.fmt = f | (f != dev::kFp16 && mode != 0 ? kWide : 0u);
          it.valid_rows = vt * p.H;
        }
      }
    }
  }
  if (bad) atomicOr(s_err, bad);
  return it;
}

// Streams one block.  kD = head_dim; 8-element chunk v covers row v / (kD/8).
//
// Each warp owns consecutive 2 KB output tiles (128 chunks; lane l handles
// chunks l, l+32, ... of the tile).  Per tile: the lanes issue their kUnroll
// coalesced loads (codes plus, for FP8/INT4, the row parameters through the
// read-only path; 16 lanes share a row), convert in registers, write the
// binary16 results into the warp's shared-memory tile, and lane 0 writes the
// tile to global memory with one TMA bulk store.  Bulk stores reach the DRAM
// write ceiling with few resident warps, where per-thread stores need twice
// the occupancy this kernel's registers allow.  Only __syncwarp is needed.
//
// One instantiation per format (kF): the load widths, the parameter loads and the
// conversion are straight-line code, with no format test per chunk.  The format is
// CTA-uniform per block, so stream_item's switch costs one branch per block.
template <int kD, uint32_t kF>
__device__ __forceinline__ void stream_block(const Params& p, const Item& it, uint4* tile) {
  constexpr uint32_t kChunksPerRowLog2 = kD == 64 ? 3 : (kD == 128 ? 4 : 5);
  constexpr uint32_t kTile = 32 * kUnroll;  // chunks per warp tile
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nchunks = static_cast<uint32_t>(p.block_elems >> 3);
  const uint32_t rpk = p.rows_per_kv;
  constexpr uint32_t f = kF;
  const bool wide = (it.fmt & kWide) != 0;  // the same item for every warp of the CTA
  const uint8_t* payload = it.payload;
  const uint8_t* params = payload + p.code_bytes[f];
  uint4* out = reinterpret_cast<uint4*>(it.out);

  for (uint32_t t = it.tile_begin + warp; t < it.tile_end; t += kThreads / 32) {
    const uint32_t t0 = t * kTile;
    uint4 raw[kUnroll];
    float2 prm[kUnroll];
    uint32_t live = 0;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint32_t v = t0 + u * 32 + lane;
      const uint32_t row = v >> kChunksPerRowLog2;
      const uint32_t r = row >= rpk ? row - rpk : row;
      raw[u] = make_uint4(0u, 0u, 0u, 0u);
      prm[u] = make_float2(0.0f, 0.0f);
      if (v < nchunks && r < it.valid_rows) {
        live |= 1u << u;
        if constexpr (f == dev::kFp16) {
          raw[u] = dev::ld_stream256(reinterpret_cast<const uint4*>(payload) + v);
        } else if constexpr (f == dev::kInt4) {
          raw[u].x = dev::ld_stream256(reinterpret_cast<const uint32_t*>(payload) + v);
          prm[u] = wide ? it.prm : __ldg(reinterpret_cast<const float2*>(params) + row);
        } else {
          const uint2 c = dev::ld_stream256(reinterpret_cast<const uint2*>(payload) + v);
          raw[u].x = c.x;
          raw[u].y = c.y;
          prm[u].x = wide ? it.prm.x : __ldg(reinterpret_cast<const float*>(params) + row);
        }
      }
    }
    // The previous bulk store of this warp must have finished reading the tile.
    if (lane == 0) dev::bulk_wait_read_all();
    __syncwarp();
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint4 o = make_uint4(0u, 0u, 0u, 0u);
      if (live & (1u << u)) {
        if constexpr (f == dev::kFp16) o = dev::canon_f16x8(raw[u]);
        else if constexpr (f == dev::kInt4) o = dev::int4x8_to_f16(raw[u].x, prm[u].x, prm[u].y);
        else o = dev::fp8x8_to_f16_bits<f>(make_uint2(raw[u].x, raw[u].y), prm[u].x);
      }
      tile[u * 32 + lane] = o;
    }
    dev::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const uint32_t n = min(kTile, nchunks - t0);
      dev::bulk_store(out + t0, tile, n * 16u);
      dev::bulk_commit();
    }
  }
}

template <int kD>
__device__ __forceinline__ void stream_item(const Params& p, const Item& it, uint4* tile) {
  switch (it.fmt & 0xFFu) {
    case dev::kFp16: stream_block<kD, dev::kFp16>(p, it, tile); break;
    case dev::kE4M3: stream_block<kD, dev::kE4M3>(p, it, tile); break;
    case dev::kE5M2: stream_block<kD, dev::kE5M2>(p, it, tile); break;
    default: stream_block<kD, dev::kInt4>(p, it, tile); break;
  }
}

// Block-wide exclusive prefix sum of one uint64 per thread; returns the total.
__device__ uint64_t exclusive_scan(uint64_t x, uint64_t* s_out, uint64_t* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = lane < kThreads / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < kThreads / 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kThreads / 32) s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const uint64_t before = (warp > 0 ? s_warp[warp - 1] : 0) + incl - x;
  s_out[threadIdx.x] = before;
  const uint64_t total = s_warp[kThreads / 32 - 1];
  if (threadIdx.x == kThreads - 1) s_out[kThreads] = total;
  __syncthreads();
  return total;
}

using dev::allow_dependents_to_launch;
using dev::wait_for_prerequisites;

// Before wait_for_prerequisites() the kernel reads only the segments, the output offsets,
// the arena and the descriptor table (the segment scan and the block resolution of the
// first batch); pools, the output and *p.err are touched only after it.  So, launched
// with programmatic serialization after a kernel that writes none of those four inputs
// (the gather of the previous layer), this launch's prologue overlaps that kernel's tail.
template <int kD>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) gather_dequant_kernel(const Params p) {
  __shared__ uint64_t s_prefix[kThreads + 1];
  __shared__ uint64_t s_warp[kThreads / 32];
  __shared__ Item s_item[kThreads];
  __shared__ __align__(128) uint4 s_tile[kThreads / 32][32 * kUnroll];  // one output tile per warp
  __shared__ uint32_t s_err;

  allow_dependents_to_launch();
  if (threadIdx.x == 0) s_err = 0;  // ordered before use by the scan's barriers
  bool waited = false;
  const uint64_t G = gridDim.x, c = blockIdx.x;
  const uint32_t ntiles = static_cast<uint32_t>(((p.block_elems >> 3) + kTileChunks - 1) / kTileChunks);
  uint64_t base = 0;   // blocks before the current chunk of sequences
  uint64_t pbase = 0;  // pieces before the current chunk
  for (uint32_t chunk = 0; chunk < p.nseq; chunk += kThreads) {
    const uint32_t cnt = min(p.nseq - chunk, static_cast<uint32_t>(kThreads));
    const uint64_t len = threadIdx.x < cnt ? p.segs[chunk + threadIdx.x].y : 0u;
    const uint64_t total = exclusive_scan(len, s_prefix, s_warp);
    const uint64_t end = base + total;
    // Pieces: a chunk with fewer than 2 blocks per CTA splits every block into `parts`
    // tile ranges (each at least 8 tiles, one per warp), so that every CTA gets work.
    uint32_t parts = 1;
    while (parts < 8 && total * parts < 2 * G && ntiles >= 16 * parts) parts *= 2;
    const uint64_t pend = pbase + total * parts;
    // First owned piece >= pbase: q = c (mod G).
    uint64_t first = pbase + (c + G - pbase % G) % G;
    for (; first < pend; first += uint64_t{kThreads} * G) {
      const uint64_t q = first + threadIdx.x * G;
      if (q < pend) {
        const uint64_t lq = q - pbase;
        const uint64_t local = lq / parts;
        uint32_t lo = 0, hi = cnt;  // last s with s_prefix[s] <= local
        while (hi - lo > 1) {
          const uint32_t mid = (lo + hi) >> 1;
          if (s_prefix[mid] <= local) lo = mid; else hi = mid;
        }
        Item it = resolve(p, chunk + lo, local - s_prefix[lo], base + s_prefix[lo], &s_err);
        const uint32_t per_part = (ntiles + parts - 1) / parts;
        it.tile_begin = static_cast<uint32_t>(lq % parts) * per_part;
        it.tile_end = min(ntiles, it.tile_begin + per_part);
        s_item[threadIdx.x] = it;
      }
      __syncthreads();
      if (!waited) {  // uniform over the CTA
        wait_for_prerequisites();
        waited = true;
      }
      const uint32_t n_items =
          static_cast<uint32_t>(min(uint64_t{kThreads}, (pend - first + G - 1) / G));
      for (uint32_t k = 0; k < n_items; ++k) {
        const Item it = s_item[k];
        if (it.fmt != kSkip) stream_item<kD>(p, it, s_tile[threadIdx.x >> 5]);
      }
      __syncthreads();  // s_item is rewritten by the next batch
    }
    base = end;
    pbase = pend;
    __syncthreads();  // s_prefix is rewritten by the next chunk
  }
  // Shared memory must outlive the bulk stores that read it.
  if ((threadIdx.x & 31) == 0) dev::bulk_wait_all();
  __syncthreads();
  if (threadIdx.x == 0 && s_err != 0) {
    if (!waited) wait_for_prerequisites();
    atomicOr(p.err, s_err);
  }
}

// Grid = one wave of SMs x resident CTAs (more waves measured no faster).
template <int kD>
int grid_for() {
  static thread_local int cached_device = -1;
  static thread_local int cached_grid = 0;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  if (device != cached_device) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gather_dequant_kernel<kD>, kThreads,
                                                      0) != cudaSuccess) {
      return 0;
    }
    cached_grid = sm_count() * (per_sm > 0 ? per_sm : 1);
    cached_device = device;
  }
  return cached_grid;
}

}  // namespace
}  // namespace hlkv

extern "C" int hlkv_gather_dequant_ex(const HlkvPools* pools, const HlkvLayout* layout,
                                      const HlkvExecDescriptor* d_table, uint32_t table_size,
                                      const uint32_t* d_arena, uint32_t arena_size,
                                      const HlkvSegment* d_segs, uint32_t nseq, uint16_t* d_out,
                                      const uint64_t* d_out_offsets, uint32_t* d_err, uint32_t flags,
                                      hlkv_stream_t stream) {
  using namespace hlkv;
  if ((flags & ~uint32_t{HLKV_LAUNCH_OVERLAP_PREVIOUS}) != 0) return HLKV_INVALID_ARGUMENT;
  if (pools == nullptr || !layout_ok(layout) || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (nseq == 0) return HLKV_OK;
  if (d_segs == nullptr || d_out == nullptr || (reinterpret_cast<uintptr_t>(d_out) & 15u) != 0) {
    return HLKV_INVALID_ARGUMENT;
  }
  if ((table_size > 0 && d_table == nullptr) || (arena_size > 0 && d_arena == nullptr)) {
    return HLKV_INVALID_ARGUMENT;
  }
  Params p{};
  const uint64_t rows = uint64_t{2} * layout->block_tokens * layout->kv_heads;
  p.block_elems = rows * layout->head_dim;
  for (int f = 0; f < 4; ++f) {
    const HlkvPool& q = pools->pool[f];
    p.code_bytes[f] = layout_code_bytes(f, p.block_elems);
    if (q.base == nullptr || q.num_slots == 0) continue;
    if ((reinterpret_cast<uintptr_t>(q.base) & 15u) != 0 || (q.slot_bytes & 15u) != 0 ||
        q.slot_bytes < hlkv_layout_slot_bytes(f, layout)) {
      return HLKV_INVALID_ARGUMENT;
    }
    p.pool[f] = DevPool{static_cast<const uint8_t*>(q.base), q.slot_bytes, q.num_slots};
  }
  p.table = reinterpret_cast<const uint4*>(d_table);
  p.arena = d_arena;
  p.segs = reinterpret_cast<const uint2*>(d_segs);
  p.out = d_out;
  p.out_offsets = d_out_offsets;
  p.err = d_err;
  p.table_size = table_size;
  p.arena_size = arena_size;
  p.nseq = nseq;
  p.T = layout->block_tokens;
  p.H = layout->kv_heads;
  p.layout_id = layout->layout_id;
  p.rows_per_kv = layout->block_tokens * layout->kv_heads;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  void (*kernel)(Params) = nullptr;
  int grid = 0;
  switch (layout->head_dim) {
    case 64: kernel = gather_dequant_kernel<64>; grid = grid_for<64>(); break;
    case 128: kernel = gather_dequant_kernel<128>; grid = grid_for<128>(); break;
    default: kernel = gather_dequant_kernel<256>; grid = grid_for<256>(); break;
  }
  if (grid <= 0) {
    const cudaError_t e = cudaGetLastError();
    return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidDevice);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & HLKV_LAUNCH_OVERLAP_PREVIOUS) ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, p));
}

extern "C" int hlkv_gather_dequant(const HlkvPools* pools, const HlkvLayout* layout,
                                   const HlkvExecDescriptor* d_table, uint32_t table_size,
                                   const uint32_t* d_arena, uint32_t arena_size,
                                   const HlkvSegment* d_segs, uint32_t nseq, uint16_t* d_out,
                                   const uint64_t* d_out_offsets, uint32_t* d_err,
                                   hlkv_stream_t stream) {
  return hlkv_gather_dequant_ex(pools, layout, d_table, table_size, d_arena, arena_size, d_segs, nseq,
                                d_out, d_out_offsets, d_err, 0u, stream);
}
