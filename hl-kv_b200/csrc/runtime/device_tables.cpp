// hl::kv::DeviceTables (include/hl_kv/device_tables.hpp).
#include "hl_kv/device_tables.hpp"

#include <cuda.h>  // types of the virtual memory management calls (reached at run time)
#include <cuda_runtime_api.h>

#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "hlkv.h"

namespace hlkv {
int cuda_status(cudaError_t e) noexcept;
int launch_apply_delta(uint4* table, uint32_t table_size, uint32_t* arena, uint32_t arena_size,
                       const uint4* desc, uint32_t n_desc, const uint2* ids, uint32_t n_id,
                       const uint2* copy_src, uint2* copy_dst, uint32_t n_copy, uint32_t* err,
                       cudaStream_t s);
int launch_relocate(uint32_t* arena, uint32_t arena_size, const HlkvSegmentMove* moves, uint32_t n,
                    uint32_t* scratch, uint64_t scratch_entries, uint32_t* err, cudaStream_t s);
}

namespace hl::kv {
namespace {

using quant::QuantStatus;

DeviceStatus from_cuda(cudaError_t e) {
  (void)hlkv::cuda_status(e);
  return e == cudaSuccess ? DeviceStatus{} : DeviceStatus{QuantStatus::kCudaError, e};
}

template <typename T>
cudaError_t device_alloc(T** p, std::size_t bytes) {
  return cudaMalloc(reinterpret_cast<void**>(p), bytes);
}

// Makes `device` current for the scope of one call.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev_) == cudaSuccess && prev_ != device) {
      ok_ = cudaSetDevice(device) == cudaSuccess;
      restore_ = true;
    }
  }
  ~DeviceGuard() {
    if (restore_) (void)cudaSetDevice(prev_);
  }
  [[nodiscard]] bool ok() const noexcept { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = true;
  bool restore_ = false;
};

// The driver's virtual memory management calls, looked up once through the runtime
// (cudaGetDriverEntryPoint), so the library needs no link-time dependency on the driver.
struct VmmCalls {
  CUresult (*granularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags) = nullptr;
  CUresult (*reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
  CUresult (*release_range)(CUdeviceptr, size_t) = nullptr;
  CUresult (*create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long) = nullptr;
  CUresult (*release)(CUmemGenericAllocationHandle) = nullptr;
  CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
  CUresult (*unmap)(CUdeviceptr, size_t) = nullptr;
  CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
  bool ok = false;
};

const VmmCalls& vmm() {
  static VmmCalls calls;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name, auto& fn) {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult found{};
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &found) != cudaSuccess ||
          found != cudaDriverEntryPointSuccess || p == nullptr) {
        return false;
      }
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(p);
      return true;
    };
    calls.ok = get("cuMemGetAllocationGranularity", calls.granularity) && get("cuMemAddressReserve", calls.reserve) &&
               get("cuMemAddressFree", calls.release_range) && get("cuMemCreate", calls.create) &&
               get("cuMemRelease", calls.release) && get("cuMemMap", calls.map) && get("cuMemUnmap", calls.unmap) &&
               get("cuMemSetAccess", calls.set_access);
  });
  return calls;
}

}  // namespace

// The arena's device storage under virtual memory management: one address range
// reserved for the largest possible arena (2^32 - 1 entries), backed from its start by
// physical chunks mapped as the arena grows and unmapped from its end when it shrinks.
// Every mapped byte belongs to the arena, and kernels never read past the arena's size,
// which is at most the mapped size.
struct DeviceTables::ArenaSpace {
  CUdeviceptr base = 0;
  size_t reserved = 0;
  size_t granularity = 0;
  size_t mapped = 0;
  int device = 0;
  struct Chunk {
    CUmemGenericAllocationHandle handle;
    size_t bytes;
  };
  std::vector<Chunk> chunks;

  CUmemAllocationProp prop() const {
    CUmemAllocationProp p{};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = device;
    return p;
  }

  // Reserves the range; false (nothing held) when the driver cannot.
  bool open(int dev) {
    const VmmCalls& v = vmm();
    if (!v.ok) return false;
    device = dev;
    const CUmemAllocationProp p = prop();
    if (v.granularity(&granularity, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM) != CUDA_SUCCESS || granularity == 0) {
      return false;
    }
    const size_t want = size_t{0xFFFFFFFFull} * sizeof(std::uint32_t);
    reserved = (want + granularity - 1) / granularity * granularity;
    // Aligned to the granularity, so that every chunk maps at an aligned address.
    if (v.reserve(&base, reserved, granularity, 0, 0) != CUDA_SUCCESS) {
      base = 0;
      return false;
    }
    return true;
  }

  // Maps chunks at the end of the mapped part until at least `bytes` are mapped.
  bool grow(size_t bytes) {
    const VmmCalls& v = vmm();
    if (bytes > reserved) return false;
    while (mapped < bytes) {
      // Pieces of about an eighth of what is mapped (at least one granule, at most 256 MiB):
      // few map calls as the arena grows, and fine enough for trim() to give most of it back.
      size_t chunk = mapped / 8;
      if (chunk > (size_t{256} << 20)) chunk = size_t{256} << 20;
      chunk = (chunk + granularity - 1) / granularity * granularity;
      if (chunk < granularity) chunk = granularity;
      if (mapped + chunk > reserved) chunk = reserved - mapped;
      const CUmemAllocationProp p = prop();
      CUmemGenericAllocationHandle h{};
      if (v.create(&h, chunk, &p, 0) != CUDA_SUCCESS) return false;
      if (v.map(base + mapped, chunk, 0, h, 0) != CUDA_SUCCESS) {
        (void)v.release(h);
        return false;
      }
      CUmemAccessDesc access{};
      access.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
      access.location.id = device;
      access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
      if (v.set_access(base + mapped, chunk, &access, 1) != CUDA_SUCCESS) {
        (void)v.unmap(base + mapped, chunk);
        (void)v.release(h);
        return false;
      }
      chunks.push_back(Chunk{h, chunk});
      mapped += chunk;
    }
    return true;
  }

  // Unmaps whole chunks from the end while at least `keep` bytes stay mapped.  The
  // caller has made sure that no queued work reads the unmapped part.
  void trim(size_t keep) {
    const VmmCalls& v = vmm();
    while (!chunks.empty() && mapped - chunks.back().bytes >= keep) {
      const Chunk c = chunks.back();
      chunks.pop_back();
      mapped -= c.bytes;
      (void)v.unmap(base + mapped, c.bytes);
      (void)v.release(c.handle);
    }
  }

  ~ArenaSpace() {
    trim(0);
    if (base != 0) (void)vmm().release_range(base, reserved);
  }
};

DeviceTables::DeviceTables() { (void)cudaGetDevice(&device_); }

DeviceTables::~DeviceTables() {
  DeviceGuard g(device_);
  if (staging_free_ != nullptr) {
    (void)cudaEventSynchronize(staging_free_);
    (void)cudaEventDestroy(staging_free_);
  }
  // The owner must not destroy the tables while kernels that read them are
  // queued; a device-wide sync makes the frees below safe regardless.
  (void)cudaDeviceSynchronize();
  if (moves_free_ != nullptr) (void)cudaEventDestroy(moves_free_);
  if (d_table_ != nullptr) (void)cudaFree(d_table_);
  if (space_ == nullptr && d_arena_ != nullptr) (void)cudaFree(d_arena_);
  space_.reset();
  if (d_scratch_ != nullptr) (void)cudaFree(d_scratch_);
  if (h_moves_ != nullptr) (void)cudaFreeHost(h_moves_);
  if (d_err_ != nullptr) (void)cudaFree(d_err_);
  if (d_staging_ != nullptr) (void)cudaFree(d_staging_);
  if (h_staging_ != nullptr) (void)cudaFreeHost(h_staging_);
}

DeviceStatus DeviceTables::stage(const alloc::ExecDelta& delta) {
  DeviceGuard g(device_);
  if (!g.ok()) return from_cuda(cudaErrorInvalidDevice);
  const std::size_t n_desc = delta.descriptor_patches.size(), n_id = delta.id_patches.size();
  const std::size_t bytes = 16 * n_desc + 8 * n_id;
  // The last flush's upload and kernel (3) must be done with both staging buffers.
  if (staging_free_ != nullptr) {
    if (const cudaError_t e = cudaEventSynchronize(staging_free_); e != cudaSuccess) return from_cuda(e);
  }
  if (bytes > staging_bytes_) {
    std::size_t cap = staging_bytes_ == 0 ? std::size_t{64} << 10 : staging_bytes_;
    while (cap < bytes) cap *= 2;
    if (h_staging_ != nullptr) (void)cudaFreeHost(h_staging_);
    h_staging_ = nullptr;
    staging_dev_ = nullptr;
    staging_bytes_ = 0;
    if (const cudaError_t e = cudaMallocHost(&h_staging_, cap); e != cudaSuccess) return from_cuda(e);
    // Kernel (3) reads the staged patches in place: the device address of the pinned
    // buffer (its host address under unified addressing).
    cudaPointerAttributes attr{};
    if (const cudaError_t e = cudaPointerGetAttributes(&attr, h_staging_); e != cudaSuccess) return from_cuda(e);
    if (attr.devicePointer == nullptr) return from_cuda(cudaErrorNotSupported);
    staging_dev_ = attr.devicePointer;
    staging_bytes_ = cap;
  }
  auto* h = static_cast<unsigned char*>(h_staging_);
  if (n_desc > 0) std::memcpy(h, delta.descriptor_patches.data(), 16 * n_desc);
  if (n_id > 0) std::memcpy(h + 16 * n_desc, delta.id_patches.data(), 8 * n_id);
  return {};
}

DeviceStatus DeviceTables::sync(alloc::HeteroBlockTable& table, cudaStream_t stream) {
  if (DeviceStatus s = collect(table); !s.ok()) return s;
  return flush(stream);
}

DeviceStatus DeviceTables::collect(alloc::HeteroBlockTable& table) {
  if (!pending_) {
    table.collect_delta(delta_);
  } else {
    // A second collect before a flush: merge, later patches winning and one patch per
    // target (kernel (3) applies each list in parallel).
    table.collect_delta(scratch_);
    delta_.descriptor_table_size = scratch_.descriptor_table_size;
    delta_.arena_size = scratch_.arena_size;
    auto merge = [](auto& into, const auto& later, auto key) {
      std::unordered_map<std::uint32_t, std::size_t> at;
      at.reserve(into.size() + later.size());
      for (std::size_t i = 0; i < into.size(); ++i) at[key(into[i])] = i;
      for (const auto& p : later) {
        const auto [it, fresh] = at.try_emplace(key(p), into.size());
        if (fresh) into.push_back(p); else into[it->second] = p;
      }
    };
    merge(delta_.descriptor_patches, scratch_.descriptor_patches,
          [](const alloc::BlockExecDescriptor& d) { return d.block_id; });
    merge(delta_.id_patches, scratch_.id_patches, [](const alloc::IdPatch& d) { return d.offset; });
  }
  pending_ = true;
  return stage(delta_);
}

DeviceStatus DeviceTables::flush(cudaStream_t stream) { return flush(stream, nullptr, nullptr, 0); }

DeviceStatus DeviceTables::flush(cudaStream_t stream, const void* copy_src, void* copy_dst,
                                 std::uint32_t n_copy) {
  if (pending_) {
    pending_ = false;
    return upload_and_apply(delta_, stream, copy_src, copy_dst, n_copy);
  }
  if (n_copy == 0) return {};
  DeviceGuard g(device_);
  if (!g.ok()) return from_cuda(cudaErrorInvalidDevice);
  if (DeviceStatus s = ensure_error_word(stream); !s.ok()) return s;
  return launch(nullptr, 0, nullptr, 0, copy_src, copy_dst, n_copy, stream);
}

DeviceStatus DeviceTables::flush_deferred(cudaStream_t stream, const void* copy_src, void* copy_dst,
                                          std::uint32_t n_copy) {
  defer_release_ = true;
  const DeviceStatus s = flush(stream, copy_src, copy_dst, n_copy);
  defer_release_ = false;
  return s;
}

DeviceStatus DeviceTables::release_staging(cudaStream_t stream) {
  if (!release_pending_) return {};
  release_pending_ = false;
  DeviceGuard g(device_);
  if (!g.ok()) return from_cuda(cudaErrorInvalidDevice);
  if (const cudaError_t e = cudaEventRecord(staging_free_, stream); e != cudaSuccess) return from_cuda(e);
  return {};
}

DeviceStatus DeviceTables::apply(const alloc::ExecDelta& delta, cudaStream_t stream) {
  if (DeviceStatus s = stage(delta); !s.ok()) return s;
  return upload_and_apply(delta, stream, nullptr, nullptr, 0);
}

DeviceStatus DeviceTables::ensure_error_word(cudaStream_t stream) {
  if (d_err_ != nullptr) return {};
  if (const cudaError_t e = device_alloc(&d_err_, sizeof(std::uint32_t)); e != cudaSuccess) {
    d_err_ = nullptr;
    return from_cuda(e);
  }
  if (const cudaError_t e = cudaMemsetAsync(d_err_, 0, sizeof(std::uint32_t), stream); e != cudaSuccess) {
    return from_cuda(e);
  }
  if (const cudaError_t e = cudaEventCreateWithFlags(&staging_free_, cudaEventDisableTiming); e != cudaSuccess) {
    staging_free_ = nullptr;
    return from_cuda(e);
  }
  return {};
}

DeviceStatus DeviceTables::launch(const void* desc, std::uint32_t n_desc, const void* ids, std::uint32_t n_id,
                                  const void* copy_src, void* copy_dst, std::uint32_t n_copy,
                                  cudaStream_t stream) {
  const int st = hlkv::launch_apply_delta(
      reinterpret_cast<uint4*>(d_table_), table_size_, d_arena_, arena_size_, static_cast<const uint4*>(desc),
      n_desc, static_cast<const uint2*>(ids), n_id, static_cast<const uint2*>(copy_src),
      static_cast<uint2*>(copy_dst), n_copy, d_err_, stream);
  if (st != HLKV_OK) {
    return DeviceStatus{static_cast<QuantStatus>(st), static_cast<cudaError_t>(hlkv_last_cuda_error())};
  }
  return {};
}

DeviceStatus DeviceTables::upload_and_apply(const alloc::ExecDelta& delta, cudaStream_t stream,
                                            const void* copy_src, void* copy_dst, std::uint32_t n_copy) {
  DeviceGuard g(device_);
  if (!g.ok()) return from_cuda(cudaErrorInvalidDevice);
  if (DeviceStatus s = ensure_error_word(stream); !s.ok()) return s;
  if (delta.descriptor_table_size != table_size_) {
    // A table has a fixed size; this happens once, on the first delta.
    if (const cudaError_t e = cudaStreamSynchronize(stream); e != cudaSuccess) return from_cuda(e);
    if (d_table_ != nullptr) (void)cudaFree(d_table_);
    d_table_ = nullptr;
    table_size_ = 0;
    if (delta.descriptor_table_size > 0) {
      if (const cudaError_t e = device_alloc(&d_table_, std::size_t{delta.descriptor_table_size} * 16);
          e != cudaSuccess) {
        d_table_ = nullptr;
        return from_cuda(e);
      }
    }
    table_size_ = delta.descriptor_table_size;
  }
  if (delta.arena_size > arena_capacity_) {
    if (DeviceStatus st = grow_arena(delta.arena_size, stream); !st.ok()) return st;
  }
  arena_size_ = delta.arena_size;

  const std::size_t n_desc = delta.descriptor_patches.size(), n_id = delta.id_patches.size();
  if (n_desc + n_id == 0) {
    return n_copy == 0 ? DeviceStatus{} : launch(nullptr, 0, nullptr, 0, copy_src, copy_dst, n_copy, stream);
  }
  // Small deltas (a decode step's) are read by kernel (3) in place from pinned memory;
  // large ones (a big table's first sync) go through one copy, since a DMA copy moves
  // megabytes faster than the kernel's 16-byte reads across PCIe (2.3 M patches: 1.07 ms
  // read in place, about 0.76 ms copied).
  const std::size_t bytes = 16 * n_desc + 8 * n_id;
  const unsigned char* d = static_cast<const unsigned char*>(staging_dev_);
  if (bytes >= kCopyDeltaBytes) {
    if (bytes > d_staging_bytes_) {
      if (d_staging_ != nullptr) {
        if (const cudaError_t e = cudaStreamSynchronize(stream); e != cudaSuccess) return from_cuda(e);
        (void)cudaFree(d_staging_);
      }
      d_staging_ = nullptr;
      d_staging_bytes_ = 0;
      if (const cudaError_t e = device_alloc(&d_staging_, staging_bytes_); e != cudaSuccess) {
        d_staging_ = nullptr;
        return from_cuda(e);
      }
      d_staging_bytes_ = staging_bytes_;
    }
    if (const cudaError_t e = cudaMemcpyAsync(d_staging_, h_staging_, bytes, cudaMemcpyHostToDevice, stream);
        e != cudaSuccess) {
      return from_cuda(e);
    }
    d = static_cast<const unsigned char*>(d_staging_);
  }
  if (DeviceStatus s = launch(d, static_cast<std::uint32_t>(n_desc), d + 16 * n_desc,
                              static_cast<std::uint32_t>(n_id), copy_src, copy_dst, n_copy, stream);
      !s.ok()) {
    return s;
  }
  // The staging buffers are free again once kernel (3) has read them (flush_deferred: once
  // the caller's next launch has been queued, release_staging records it).
  if (defer_release_) {
    release_pending_ = true;
    return {};
  }
  if (const cudaError_t e = cudaEventRecord(staging_free_, stream); e != cudaSuccess) return from_cuda(e);
  return {};
}

DeviceStatus DeviceTables::grow_arena(std::uint32_t entries, cudaStream_t stream) {
  // Room for a quarter more than asked, and at least double the old capacity, so that
  // growth stays rare.
  std::uint64_t cap = arena_capacity_ == 0 ? 1024 : 2ull * arena_capacity_;
  const std::uint64_t want = std::uint64_t{entries} + entries / 4;
  if (cap < want) cap = want;
  if (cap > 0xFFFFFFFFull) cap = 0xFFFFFFFFull;
  if (!space_tried_) {
    space_tried_ = true;
    auto space = std::make_unique<ArenaSpace>();
    if (d_arena_ == nullptr && space->open(device_)) space_ = std::move(space);
  }
  if (space_ != nullptr) {
    // Map more memory behind the same address: no copy, queued kernels keep reading the
    // part that is already mapped.
    if (!space_->grow(static_cast<size_t>(cap) * sizeof(std::uint32_t))) return from_cuda(cudaErrorMemoryAllocation);
    d_arena_ = reinterpret_cast<std::uint32_t*>(space_->base);
    const std::uint64_t mapped_entries = space_->mapped / sizeof(std::uint32_t);
    arena_capacity_ = static_cast<std::uint32_t>(mapped_entries > 0xFFFFFFFFull ? 0xFFFFFFFFull : mapped_entries);
    return {};
  }
  std::uint32_t* fresh = nullptr;
  if (const cudaError_t e = device_alloc(&fresh, cap * 4); e != cudaSuccess) return from_cuda(e);
  if (d_arena_ != nullptr) {
    // Keep the contents (the protocol grows the arena, it never rewrites it).
    if (const cudaError_t e = cudaMemcpyAsync(fresh, d_arena_, std::size_t{arena_size_} * 4,
                                              cudaMemcpyDeviceToDevice, stream);
        e != cudaSuccess) {
      (void)cudaFree(fresh);
      return from_cuda(e);
    }
    // The old buffer may still be read by queued kernels on this stream.
    if (const cudaError_t e = cudaStreamSynchronize(stream); e != cudaSuccess) return from_cuda(e);
    (void)cudaFree(d_arena_);
  }
  d_arena_ = fresh;
  arena_capacity_ = static_cast<std::uint32_t>(cap);
  return {};
}

DeviceStatus DeviceTables::relocate(std::span<const alloc::SegmentMove> moves, std::uint32_t new_arena_size,
                                    cudaStream_t stream) {
  if (DeviceStatus st = flush(stream); !st.ok()) return st;
  DeviceGuard g(device_);
  if (!g.ok()) return from_cuda(cudaErrorInvalidDevice);
  if (DeviceStatus st = ensure_error_word(stream); !st.ok()) return st;
  if (!moves.empty()) {
    if (d_arena_ == nullptr) return from_cuda(cudaErrorInvalidValue);
    const std::uint64_t need = alloc::IdArena::scratch_entries(moves);
    if (need > scratch_entries_) {
      if (d_scratch_ != nullptr) {
        if (const cudaError_t e = cudaStreamSynchronize(stream); e != cudaSuccess) return from_cuda(e);
        (void)cudaFree(d_scratch_);
      }
      d_scratch_ = nullptr;
      scratch_entries_ = 0;
      if (const cudaError_t e = device_alloc(&d_scratch_, need * sizeof(std::uint32_t)); e != cudaSuccess) {
        d_scratch_ = nullptr;
        return from_cuda(e);
      }
      scratch_entries_ = need;
    }
    const std::size_t bytes = moves.size() * sizeof(alloc::SegmentMove);
    if (moves_free_ == nullptr) {
      if (const cudaError_t e = cudaEventCreateWithFlags(&moves_free_, cudaEventDisableTiming); e != cudaSuccess) {
        moves_free_ = nullptr;
        return from_cuda(e);
      }
    } else if (const cudaError_t e = cudaEventSynchronize(moves_free_); e != cudaSuccess) {
      return from_cuda(e);  // the previous relocation has read the staged moves
    }
    if (bytes > h_moves_bytes_) {
      if (h_moves_ != nullptr) (void)cudaFreeHost(h_moves_);
      h_moves_ = nullptr;
      h_moves_bytes_ = 0;
      if (const cudaError_t e = cudaMallocHost(&h_moves_, bytes); e != cudaSuccess) {
        h_moves_ = nullptr;
        return from_cuda(e);
      }
      h_moves_bytes_ = bytes;
    }
    std::memcpy(h_moves_, moves.data(), bytes);
    cudaPointerAttributes attr{};
    if (const cudaError_t e = cudaPointerGetAttributes(&attr, h_moves_); e != cudaSuccess) return from_cuda(e);
    const int rs = hlkv::launch_relocate(d_arena_, arena_size_, static_cast<const HlkvSegmentMove*>(attr.devicePointer),
                                         static_cast<std::uint32_t>(moves.size()), d_scratch_, scratch_entries_,
                                         d_err_, stream);
    if (rs != HLKV_OK) {
      return DeviceStatus{static_cast<quant::QuantStatus>(rs), static_cast<cudaError_t>(hlkv_last_cuda_error())};
    }
    if (const cudaError_t e = cudaEventRecord(moves_free_, stream); e != cudaSuccess) return from_cuda(e);
  }
  arena_size_ = new_arena_size;
  // Give back mapped memory beyond a quarter of headroom, once nothing queued can read it.
  if (space_ != nullptr) {
    const std::uint64_t keep_entries = std::uint64_t{new_arena_size} + new_arena_size / 4;
    const size_t keep = static_cast<size_t>(keep_entries) * sizeof(std::uint32_t);
    if (space_->mapped > keep + space_->granularity) {
      if (const cudaError_t e = cudaDeviceSynchronize(); e != cudaSuccess) return from_cuda(e);
      space_->trim(keep);
      const std::uint64_t mapped_entries = space_->mapped / sizeof(std::uint32_t);
      arena_capacity_ = static_cast<std::uint32_t>(mapped_entries > 0xFFFFFFFFull ? 0xFFFFFFFFull : mapped_entries);
    }
  }
  return {};
}

}  // namespace hl::kv
