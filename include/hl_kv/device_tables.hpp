#pragma once
// hl::kv::DeviceTables -- the GPU-resident copy of a HeteroBlockTable's
// device-facing state (descriptor table + id arena), kept current with deltas.
//
// The reference defines the protocol (hetero_block_table.hpp:100-114,
// hl_allocator_abi.md section 5) but only simulates the device side on the
// host (tests/project1/exec_mirror.hpp).  Here sync() runs it for real, in
// stream order on the caller's stream:
//   1. table.collect_delta() on the host;
//   2. grow the device arena when delta.arena_size exceeds its capacity.  The
//      arena lives in a reserved virtual address range (CUDA virtual memory
//      management, reached through the runtime's driver entry points): growth
//      maps more device memory behind the same address, with a quarter to
//      spare -- no copy, no stream drain, and the arena pointer never changes.
//      Where the driver offers no virtual memory management, growth falls back
//      to a larger allocation, a device-to-device copy and a stream drain.  The
//      descriptor table is allocated once at max_blocks entries;
//   3. copy the patches into pinned staging;
//   4. run kernel (3) (hlkv_apply_delta), which reads the staged patches in
//      place: under unified addressing a kernel reads page-locked host memory
//      directly, so no upload copy is queued.  Deltas of 1 MiB or more are
//      first copied to the device in one transfer, which is faster for them.
// collect() is the host part (1 and 3) and flush() the queued part, so host table
// work can run while the stream is busy.
// Kernels issued later on the same stream see the updated tables.  One
// DeviceTables per table and device, used from the table's first delta on;
// not thread-safe (like the table).
#include <cuda_runtime_api.h>

#include <cstdint>
#include <memory>
#include <span>

#include "hl_allocator/hetero_block_table.hpp"
#include "hl_quant/cuda_dequant.hpp"

namespace hl::kv {

using hl::quant::cuda::DeviceStatus;

class DeviceTables {
 public:
  /// Binds to the current CUDA device.  Nothing is allocated before sync().
  DeviceTables();
  ~DeviceTables();
  DeviceTables(const DeviceTables&) = delete;
  DeviceTables& operator=(const DeviceTables&) = delete;

  /// collect_delta() + upload + apply on `stream`: collect() then flush().
  [[nodiscard]] DeviceStatus sync(alloc::HeteroBlockTable& table, cudaStream_t stream);
  /// Host half of sync(): moves the table's pending changes into this object (merged
  /// with changes collected earlier and not yet flushed, later patches winning) and
  /// copies them into pinned staging.  Queues nothing; it waits only until the previous
  /// flush's upload and kernel (3) are done with the staging buffers.
  [[nodiscard]] DeviceStatus collect(alloc::HeteroBlockTable& table);
  /// Device half of sync(): queues kernel (3) for what collect() gathered, on
  /// `stream`.  A no-op when nothing is pending.
  [[nodiscard]] DeviceStatus flush(cudaStream_t stream);
  /// flush(stream), and the same kernel (3) launch copies n_copy 8-byte words from
  /// copy_src (device-readable: device memory or page-locked host memory) to copy_dst
  /// (device memory).  The decode step moves its append targets this way.
  [[nodiscard]] DeviceStatus flush(cudaStream_t stream, const void* copy_src, void* copy_dst,
                                   std::uint32_t n_copy);
  /// flush(stream, copy_src, copy_dst, n_copy) that leaves the staging buffers marked busy
  /// past the next operation queued on `stream`: no event is recorded after kernel (3), so a
  /// kernel queued next may overlap it (programmatic dependent launch).  The caller queues
  /// that kernel and then calls release_staging(stream).
  [[nodiscard]] DeviceStatus flush_deferred(cudaStream_t stream, const void* copy_src, void* copy_dst,
                                            std::uint32_t n_copy);
  /// Records the staging buffers' release on `stream` after a flush_deferred (no-op otherwise).
  [[nodiscard]] DeviceStatus release_staging(cudaStream_t stream);
  /// Uploads and applies an already collected delta.
  [[nodiscard]] DeviceStatus apply(const alloc::ExecDelta& delta, cudaStream_t stream);
  /// Applies an arena compaction (HeteroBlockTable::compact_arena) on `stream`: flushes
  /// what collect() gathered, makes the segment moves (two launches through a scratch
  /// buffer), sets the arena size to new_arena_size and, when more than a quarter of
  /// headroom above it is mapped, waits for the device to go idle and unmaps the rest.
  /// No counterpart in the reference.
  [[nodiscard]] DeviceStatus relocate(std::span<const alloc::SegmentMove> moves, std::uint32_t new_arena_size,
                                      cudaStream_t stream);
  /// Device memory behind the arena, in bytes.
  [[nodiscard]] std::uint64_t arena_capacity_bytes() const noexcept {
    return std::uint64_t{arena_capacity_} * sizeof(std::uint32_t);
  }

  [[nodiscard]] const alloc::BlockExecDescriptor* table() const noexcept { return d_table_; }
  [[nodiscard]] std::uint32_t table_size() const noexcept { return table_size_; }
  [[nodiscard]] const std::uint32_t* arena() const noexcept { return d_arena_; }
  [[nodiscard]] std::uint32_t arena_size() const noexcept { return arena_size_; }
  /// Device word that kernel (3) reports HLKV_ERR_PATCH_RANGE into.
  [[nodiscard]] std::uint32_t* error_word() const noexcept { return d_err_; }

 private:
  [[nodiscard]] DeviceStatus stage(const alloc::ExecDelta& delta);
  [[nodiscard]] DeviceStatus upload_and_apply(const alloc::ExecDelta& delta, cudaStream_t stream,
                                              const void* copy_src, void* copy_dst, std::uint32_t n_copy);
  [[nodiscard]] DeviceStatus ensure_error_word(cudaStream_t stream);
  [[nodiscard]] DeviceStatus launch(const void* desc, std::uint32_t n_desc, const void* ids, std::uint32_t n_id,
                                    const void* copy_src, void* copy_dst, std::uint32_t n_copy,
                                    cudaStream_t stream);
  [[nodiscard]] DeviceStatus grow_arena(std::uint32_t entries, cudaStream_t stream);

  struct ArenaSpace;                     // the reserved address range and its mapped chunks
  std::unique_ptr<ArenaSpace> space_;    // null: no virtual memory management (plain allocation)
  bool space_tried_ = false;
  std::uint32_t* d_scratch_ = nullptr;   // relocation scratch
  std::uint64_t scratch_entries_ = 0;
  void* h_moves_ = nullptr;              // pinned staging of relocation moves
  std::size_t h_moves_bytes_ = 0;
  cudaEvent_t moves_free_ = nullptr;     // recorded after the relocation reads the moves

  int device_ = 0;
  alloc::BlockExecDescriptor* d_table_ = nullptr;
  std::uint32_t table_size_ = 0;
  std::uint32_t* d_arena_ = nullptr;
  std::uint32_t arena_size_ = 0;
  std::uint32_t arena_capacity_ = 0;
  std::uint32_t* d_err_ = nullptr;
  static constexpr std::size_t kCopyDeltaBytes = std::size_t{1} << 20;  // copied, not read in place
  void* h_staging_ = nullptr;    // pinned
  void* staging_dev_ = nullptr;  // its device address (not an allocation)
  std::size_t staging_bytes_ = 0;
  unsigned char* d_staging_ = nullptr;  // device copy of large deltas
  std::size_t d_staging_bytes_ = 0;
  cudaEvent_t staging_free_ = nullptr;  // recorded after kernel (3), the staging's reader
  bool defer_release_ = false;    // inside flush_deferred: no staging event after kernel (3)
  bool release_pending_ = false;  // a flush_deferred read the staging; release_staging records it
  alloc::ExecDelta delta_;    // collected, not yet flushed
  alloc::ExecDelta scratch_;  // the next collect_delta() before merging into delta_
  bool pending_ = false;
};

}  // namespace hl::kv
