// Kernel (3): device-side application of an hl::alloc::ExecDelta.
//
// The protocol (hetero_block_table.hpp:100-114; the reference only simulates it
// on the host in tests/project1/exec_mirror.hpp:23-49): descriptor patches are
// self-addressed (table[p.block_id] = p) and id patches are {offset, block_id}
// (arena[offset] = block_id); targets are unique within each list, so every
// patch is an independent store and one grid-stride pass applies both lists.
// Each descriptor patch is one 16-byte load and one 16-byte store.  The patch
// lists may be pinned host memory read in place (under unified addressing a
// kernel reads page-locked host memory at its host address), which saves the
// upload copy.  The same pass can also copy n_copy 8-byte words from src to dst
// (a decode step's append targets, from pinned host memory to the device).
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
    apply_delta_kernel(uint4* __restrict__ table, uint32_t table_size, uint32_t* __restrict__ arena,
                       uint32_t arena_size, const uint4* __restrict__ desc, uint32_t n_desc,
                       const uint2* __restrict__ ids, uint32_t n_id, const uint2* __restrict__ copy_src,
                       uint2* __restrict__ copy_dst, uint32_t n_copy, uint32_t* err) {
  // A kernel launched after this one with programmatic serialization (the decode step's
  // encoder) may start now; it waits for this grid before it reads what this grid writes.
  dev::allow_dependents_to_launch();
  const uint64_t n_patch = uint64_t{n_desc} + n_id;
  const uint64_t total = n_patch + n_copy;
  const uint64_t stride = uint64_t{gridDim.x} * kThreads;
  uint32_t bad = 0;
  for (uint64_t k = uint64_t{blockIdx.x} * kThreads + threadIdx.x; k < total; k += stride) {
    if (k < n_desc) {
      const uint4 p = __ldcs(desc + k);
      if (p.w < table_size) table[p.w] = p; else bad = dev::kErrPatchRange;
    } else if (k < n_patch) {
      const uint2 p = __ldcs(ids + (k - n_desc));
      if (p.x < arena_size) arena[p.x] = p.y; else bad = dev::kErrPatchRange;
    } else {
      copy_dst[k - n_patch] = __ldcs(copy_src + (k - n_patch));
    }
  }
  if (bad) atomicOr(err, bad);
}

}  // namespace

int launch_apply_delta(uint4* table, uint32_t table_size, uint32_t* arena, uint32_t arena_size,
                       const uint4* desc, uint32_t n_desc, const uint2* ids, uint32_t n_id,
                       const uint2* copy_src, uint2* copy_dst, uint32_t n_copy, uint32_t* err,
                       cudaStream_t s) {
  const uint64_t total = uint64_t{n_desc} + n_id + n_copy;
  if (total == 0) return HLKV_OK;
  const uint64_t want = (total + kThreads - 1) / kThreads;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  apply_delta_kernel<<<grid, kThreads, 0, s>>>(table, table_size, arena, arena_size, desc, n_desc,
                                               ids, n_id, copy_src, copy_dst, n_copy, err);
  return cuda_status(cudaGetLastError());
}

}  // namespace hlkv

extern "C" int hlkv_apply_delta(HlkvExecDescriptor* d_table, uint32_t table_size, uint32_t* d_arena,
                                uint32_t arena_size, const HlkvExecDescriptor* d_desc_patches,
                                uint32_t n_desc, const HlkvIdPatch* d_id_patches, uint32_t n_id,
                                uint32_t* d_err, hlkv_stream_t stream) {
  if (d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n_desc == 0 && n_id == 0) return HLKV_OK;
  if ((n_desc > 0 && (d_desc_patches == nullptr || (table_size > 0 && d_table == nullptr))) ||
      (n_id > 0 && (d_id_patches == nullptr || (arena_size > 0 && d_arena == nullptr)))) {
    return HLKV_INVALID_ARGUMENT;
  }
  return hlkv::launch_apply_delta(reinterpret_cast<uint4*>(d_table), table_size, d_arena, arena_size,
                                  reinterpret_cast<const uint4*>(d_desc_patches), n_desc,
                                  reinterpret_cast<const uint2*>(d_id_patches), n_id, nullptr, nullptr, 0,
                                  d_err, reinterpret_cast<cudaStream_t>(stream));
}
