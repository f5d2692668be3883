#pragma once
// hl_quant GPU entry points (C++), built for sm_100a.
//
// dequantize_fp8_to_fp16 is the drop-in for the reference's
// project2_quant/include/hl_quant/cuda_dequant.hpp:47-50 (same signature,
// statuses and numerical contract: out[i] = fp16_rn(decode_fp8(in[i]) *
// params[i / group_size].scale), bit-exact against dequantize_reference_to_fp16,
// NaN codes included).  The other two are the device counterparts of the
// reference's CPU quantize_reference / dequantize_reference_to_fp16 for every
// format (see include/hlkv.h for the per-group value checks).
// emulate_fp8_to_fp16_on_host (cuda_dequant.hpp:52-71 of the reference) runs the
// flat decoder's per-element arithmetic on the host, in both of its traversals.
#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <span>

#include "hl_quant/quant_types.hpp"

namespace hl::quant::cuda {

struct DeviceStatus {
  QuantStatus status = QuantStatus::kOk;
  cudaError_t cuda_error = cudaSuccess;
  [[nodiscard]] bool ok() const noexcept { return status == QuantStatus::kOk; }
};

/// Asynchronous on `stream`.  kUnsupportedFormat unless E4M3/E5M2; kInvalidArgument
/// for group_size == 0, n > kMaxElements or null pointers (n > 0); n == 0 is a no-op.
[[nodiscard]] DeviceStatus dequantize_fp8_to_fp16(QuantFormat format, const std::byte* d_in,
                                                  std::size_t n, const AffineParams* d_params,
                                                  std::size_t group_size, std::uint16_t* d_out,
                                                  cudaStream_t stream) noexcept;

/// Device dequantize_reference_to_fp16; groups with non-finite parameters (or a
/// non-zero FP8 bias) are skipped and flagged with HLKV_ERR_NONFINITE in *d_err.
[[nodiscard]] DeviceStatus dequantize_to_fp16(QuantFormat format, const std::byte* d_packed,
                                              std::size_t packed_size, std::size_t n,
                                              const AffineParams* d_params, std::size_t n_params,
                                              std::size_t group_size, std::uint16_t* d_out,
                                              std::size_t out_size, std::uint32_t* d_err,
                                              cudaStream_t stream) noexcept;

/// Device quantize_reference; groups with a non-finite input (or an INT4 range
/// that overflows) are skipped and flagged with HLKV_ERR_NONFINITE in *d_err.
[[nodiscard]] DeviceStatus quantize(QuantFormat format, const float* d_in, std::size_t n,
                                    std::size_t group_size, AffineParams* d_params,
                                    std::size_t n_params, std::byte* d_packed,
                                    std::size_t packed_size, std::uint32_t* d_err,
                                    cudaStream_t stream) noexcept;

/// Which traversal of the flat decoder to run on the host.
enum class HostPath : std::uint8_t {
  kScalar,  ///< one value at a time (the decoder's per-element path)
  kVector,  ///< chunks of 8 values within one group, then the tail one at a time
};

/// The flat FP8 decoder's arithmetic on the CPU: out[i] = fp16_rn(decode_fp8(in[i]) *
/// params[i / group_size].scale), n = in.size(), the bits the device writes (NaN results as
/// dequantize_reference_to_fp16 gives them).  For checking the arithmetic where no GPU is
/// present; it does not exercise device instructions, indexing or launch shapes.  Checked in
/// this order, `out` untouched on failure:
///   format is kFp8E4M3 or kFp8E5M2                          else kUnsupportedFormat
///   group_size >= 1, n <= kMaxElements                      else kInvalidArgument
///   params.size() == num_groups(n, group_size)              else kInvalidArgument
///   out.size() >= n                                         else kBufferTooSmall
/// kVector takes the scalar traversal when a chunk of 8 would straddle two groups
/// (group_size % 8 != 0 and group_size < n).  Both traversals give the same values.
[[nodiscard]] QuantStatus emulate_fp8_to_fp16_on_host(QuantFormat format, std::span<const std::byte> in,
                                                      std::span<const AffineParams> params,
                                                      std::size_t group_size, std::span<std::uint16_t> out,
                                                      HostPath path) noexcept;

}  // namespace hl::quant::cuda
