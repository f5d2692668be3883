#pragma once
// Host dequantization of hl_quant (drop-in for the reference's
// project2_quant/include/hl_quant/cpu_dequant.hpp:15-54: the same declarations,
// statuses and results bit for bit; the implementation is this library's own,
// hl-kv_b200/csrc/quant/host_codec.cpp).  The kernels of include/hlkv.h compute
// exactly these values on the device.
//
// Values, binary32 arithmetic with round to nearest even:
//   FP16  x = decode_fp16(q)
//   FP8   x = decode_fp8(q) * scale                 (bias must be 0)
//   INT4  x = fma(float(q), scale, bias)            (one rounding)
#include <cstddef>
#include <cstdint>
#include <span>

#include "hl_quant/quant_types.hpp"

namespace hl::quant {

/// Exact binary16 -> binary32.  +-Inf stay infinite; every NaN becomes the quiet NaN of the
/// same sign (0x7FC00000 | sign).
[[nodiscard]] float decode_fp16(std::uint16_t bits) noexcept;

/// Exact OCP E4M3 -> binary32; S.1111.111 is NaN.
[[nodiscard]] float decode_fp8_e4m3(std::uint8_t bits) noexcept;

/// Exact OCP E5M2 -> binary32; S.11111.00 is +-Inf, S.11111.{01,10,11} NaN.
[[nodiscard]] float decode_fp8_e5m2(std::uint8_t bits) noexcept;

/// Decodes `num_elements` values of `format` from `packed` into `out`.  Checked in this
/// order, `out` untouched on failure:
///   is_valid(format)                                          else kUnsupportedFormat
///   num_elements <= kMaxElements                              else kInvalidArgument
///   is_valid_group_size(format, group_size)                   else kInvalidArgument
///   params.size() == num_groups(num_elements, group_size)     else kInvalidArgument
///   every scale and bias finite; FP8 bias == 0                else kInvalidArgument
///   packed.size() >= packed_bytes(format, num_elements)       else kBufferTooSmall
///   out.size() >= num_elements                                else kBufferTooSmall
[[nodiscard]] QuantStatus dequantize_reference(QuantFormat format,
                                               std::span<const std::byte> packed,
                                               std::size_t num_elements,
                                               std::span<const AffineParams> params,
                                               std::size_t group_size,
                                               std::span<float> out) noexcept;

/// dequantize_reference() rounded to binary16 by encode_fp16 (two roundings: the binary32
/// value, then binary16), as raw bit patterns.  Same checks and statuses.
[[nodiscard]] QuantStatus dequantize_reference_to_fp16(QuantFormat format,
                                                       std::span<const std::byte> packed,
                                                       std::size_t num_elements,
                                                       std::span<const AffineParams> params,
                                                       std::size_t group_size,
                                                       std::span<std::uint16_t> out) noexcept;

}  // namespace hl::quant
