// Launch helpers shared by the kernels: device attributes cached per device,
// the per-thread last CUDA error, and cache-hinted loads and stores.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "hlkv.h"

namespace hlkv {

/// Records `e` as this thread's last CUDA error and maps it to an HLKV status.
int cuda_status(cudaError_t e) noexcept;

/// Number of SMs of the current device (cached per device).
int sm_count() noexcept;

/// Bytes of the code region of a layout slot (the parameters follow it).
uint64_t layout_code_bytes(int format, uint64_t elems);
/// A layout the kernels support (block_tokens 1..512, head_dim 64/128/256, ...).
bool layout_ok(const HlkvLayout* l);

// Division by a run-time constant d >= 1 through a multiply and a shift
// (Granlund and Montgomery, "Division by invariant integers using multiplication",
// 1994, theorem 4.2 with N = 31): with l = ceil(log2 d) and m = ceil(2^(31+l) / d),
// floor(n / d) = floor(n * m / 2^(31+l)) for every 0 <= n < 2^31.
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) : d(divisor) {
    uint32_t l = 0;
    while ((uint64_t{1} << l) < d) ++l;
    if (d > 1) {
      m = static_cast<uint32_t>(((uint64_t{1} << (31 + l)) + d - 1) / d);
      s = l - 1;
    }
  }
  // n < 2^31
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return d == 1 ? n : __umulhi(n, m) >> s; }
};

namespace dev {

// Programmatic dependent launch (griddepcontrol, sm_90 and later).  launch_dependents lets a
// kernel launched after this one with programmatic stream serialization start its CTAs
// before this grid has finished; wait blocks until every grid this one depends on has
// completed and its memory is visible (a no-op for an ordinary launch).
__device__ __forceinline__ void allow_dependents_to_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_for_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Streaming (evict-first) global loads and stores: the payload is read once and
// the FP16 output is consumed by another kernel, so neither should displace
// the descriptor table and arena from L2.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ uint2 ld_stream(const uint2* p) { return __ldcs(p); }
__device__ __forceinline__ uint32_t ld_stream(const uint32_t* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) { __stcs(p, v); }

// Streaming loads that also ask L2 to fill 256-byte sectors (the .L2::256B prefetch-size
// hint): a warp's 4-byte INT4 loads cover 128 bytes, and the hint fetches the next 128
// with them.  Used by the gather, where it measured +2 % on INT4 and neutral elsewhere.
__device__ __forceinline__ uint4 ld_stream256(const uint4* p) {
  uint4 v;
  asm("ld.global.cs.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream256(const uint2* p) {
  uint2 v;
  asm("ld.global.cs.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream256(const uint32_t* p) {
  uint32_t v;
  asm("ld.global.cs.L2::256B.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

}  // namespace dev
}  // namespace hlkv

namespace hlkv {
namespace dev {

// ---- TMA bulk copies (cp.async.bulk, no multicast) -------------------------------------------
// Shared -> global bulk store of `bytes` (multiple of 16; both addresses 16-byte aligned),
// tracked in the issuing thread's bulk group.
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(ssrc));
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               :: "l"(gdst), "r"(s), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until this thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until this thread's committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace dev
}  // namespace hlkv
