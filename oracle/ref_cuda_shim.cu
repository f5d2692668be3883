// extern "C" entry to the reference's own GPU kernel, hl::quant::cuda::
// dequantize_fp8_to_fp16 (project2_quant/src/dequant_kernel.cu:171-191), compiled
// from the reference sources for sm_100a by oracle/build.py.  TEST AND BENCH
// INFRASTRUCTURE ONLY: the GPU parity test compares this library's drop-in with it,
// and bench.py times it beside ours on the contiguous FP8 workload.  Nothing in the
// product links or loads it.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "hl_quant/cuda_dequant.hpp"

extern "C" __attribute__((visibility("default"))) int ref_cuda_dequantize_fp8_to_fp16(
    int format, const void* d_in, std::size_t n, const void* d_params, std::size_t group_size,
    std::uint16_t* d_out, void* stream, int* cuda_error) {
  const hl::quant::cuda::DeviceStatus s = hl::quant::cuda::dequantize_fp8_to_fp16(
      static_cast<hl::quant::QuantFormat>(format), static_cast<const std::byte*>(d_in), n,
      static_cast<const hl::quant::AffineParams*>(d_params), group_size, d_out,
      static_cast<cudaStream_t>(stream));
  if (cuda_error != nullptr) *cuda_error = static_cast<int>(s.cuda_error);
  return static_cast<int>(s.status);
}
