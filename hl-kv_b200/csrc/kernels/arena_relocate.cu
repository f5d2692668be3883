// Relocation of the device id arena after a host compaction (HeteroBlockTable::compact_arena).
//
// Each move copies a live segment's entries from `from` to `to`.  A compaction packs the
// segments towards offset 0 in offset order, so a destination can overlap sources that
// other moves (and the move itself) still have to read: the copy runs in two phases
// through a scratch buffer, one launch each -- gather every moved segment to
// scratch[move.scratch ...], then scatter it to its new offset.  Stream order between
// the two launches is the only synchronization; no kernel waits on another.
//
// Offsets and scratch positions are multiples of 8 entries and a segment's capacity is a
// multiple of 8 entries, so each copy moves whole 16-byte vectors up to the length
// rounded up to 4 entries, all inside the segment's own storage.  One warp per move,
// grid-stride over the moves; a move outside the arena or the scratch is skipped with
// HLKV_ERR_PATCH_RANGE.
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr int kThreads = 256;

template <bool kGather>
__global__ void __launch_bounds__(kThreads)
    relocate_kernel(uint32_t* __restrict__ arena, uint32_t arena_size, const uint4* __restrict__ moves,
                    uint32_t n, uint32_t* __restrict__ scratch, uint64_t scratch_entries, uint32_t* err) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = uint64_t{gridDim.x} * (kThreads / 32);
  uint32_t bad = 0;
  for (uint64_t m = (uint64_t{blockIdx.x} * kThreads + threadIdx.x) / 32; m < n; m += warps) {
    const uint4 mv = __ldg(moves + m);  // {from, to, length, scratch}
    const uint64_t len4 = (uint64_t{mv.z} + 3u) & ~uint64_t{3};
    if (((mv.x | mv.y | mv.w) & 7u) != 0 || uint64_t{mv.x} + len4 > arena_size ||
        uint64_t{mv.y} + len4 > arena_size || uint64_t{mv.w} + len4 > scratch_entries) {
      bad = dev::kErrPatchRange;
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(kGather ? arena + mv.x : scratch + mv.w);
    uint4* dst = reinterpret_cast<uint4*>(kGather ? scratch + mv.w : arena + mv.y);
    for (uint64_t v = lane; v < len4 / 4; v += 32) dst[v] = src[v];
  }
  if (bad && lane == 0) atomicOr(err, bad);
}

}  // namespace

int launch_relocate(uint32_t* arena, uint32_t arena_size, const HlkvSegmentMove* moves, uint32_t n,
                    uint32_t* scratch, uint64_t scratch_entries, uint32_t* err, cudaStream_t s) {
  if (n == 0) return HLKV_OK;
  const uint64_t want = (uint64_t{n} * 32 + kThreads - 1) / kThreads;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  const uint4* mv = reinterpret_cast<const uint4*>(moves);
  relocate_kernel<true><<<grid, kThreads, 0, s>>>(arena, arena_size, mv, n, scratch, scratch_entries, err);
  if (const cudaError_t e = cudaGetLastError(); e != cudaSuccess) return cuda_status(e);
  relocate_kernel<false><<<grid, kThreads, 0, s>>>(arena, arena_size, mv, n, scratch, scratch_entries, err);
  return cuda_status(cudaGetLastError());
}

}  // namespace hlkv

extern "C" uint64_t hlkv_segment_moves_scratch_entries(const HlkvSegmentMove* moves, size_t n) {
  if (moves == nullptr || n == 0) return 0;
  return uint64_t{moves[n - 1].scratch} + ((uint64_t{moves[n - 1].length} + 7u) & ~uint64_t{7});
}

extern "C" int hlkv_arena_relocate(uint32_t* d_arena, uint32_t arena_size, const HlkvSegmentMove* moves,
                                   uint32_t n, uint32_t* d_scratch, uint64_t scratch_entries, uint32_t* d_err,
                                   hlkv_stream_t stream) {
  if (d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n == 0) return HLKV_OK;
  if (d_arena == nullptr || moves == nullptr || d_scratch == nullptr ||
      (reinterpret_cast<uintptr_t>(d_arena) & 15u) != 0 || (reinterpret_cast<uintptr_t>(d_scratch) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(moves) & 15u) != 0) {
    return HLKV_INVALID_ARGUMENT;
  }
  return hlkv::launch_relocate(d_arena, arena_size, moves, n, d_scratch, scratch_entries, d_err,
                               reinterpret_cast<cudaStream_t>(stream));
}
