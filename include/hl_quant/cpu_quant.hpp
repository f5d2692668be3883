#pragma once
// Host quantization of hl_quant (drop-in for the reference's
// project2_quant/include/hl_quant/cpu_quant.hpp:22-47: the same declarations,
// statuses and results bit for bit; the implementation is this library's own,
// hl-kv_b200/csrc/quant/host_codec.cpp).  These are the host API of the format
// codecs, not a fallback of the kernels: the CUDA path is include/hlkv.h.
//
// Parameters per group of `group_size` consecutive values:
//   FP8   scale = max(amax / max_finite, FLT_MIN), or 1 when amax == 0; bias 0;
//         code = round-to-nearest-even, saturating encode of x / scale (IEEE division).
//   INT4  scale = (max - min) / 15, bias = min (std::minmax_element: the first minimum
//         and the last maximum); code = clamp(rint((x - min) / scale), 0, 15), or 0 when
//         scale == 0.  Two codes per byte, low nibble first; a trailing half byte is 0.
#include <cstddef>
#include <cstdint>
#include <span>

#include "hl_quant/quant_types.hpp"

namespace hl::quant {

/// binary32 -> binary16, round to nearest even; beyond the range -> +-Inf; NaN -> the quiet
/// NaN of the same sign (0x7E00 | sign).
[[nodiscard]] std::uint16_t encode_fp16(float x) noexcept;

/// binary32 -> OCP E4M3, round to nearest even, saturating (beyond 448 and +-Inf -> +-448);
/// NaN -> S.1111.111.
[[nodiscard]] std::uint8_t encode_fp8_e4m3(float x) noexcept;

/// binary32 -> OCP E5M2, round to nearest even, saturating (beyond 57344 and +-Inf ->
/// +-57344); NaN -> S.11111.11.
[[nodiscard]] std::uint8_t encode_fp8_e5m2(float x) noexcept;

/// Quantizes `in` into `packed_out` (packed_bytes(format, in.size()) bytes written) and
/// `params_out`.  Checked in this order, outputs untouched on failure:
///   is_valid(format)                                          else kUnsupportedFormat
///   in.size() <= kMaxElements                                 else kInvalidArgument
///   is_valid_group_size(format, group_size)                   else kInvalidArgument
///   params_out.size() == num_groups(in.size(), group_size)    else kInvalidArgument
///   FP8/INT4: every input finite, every INT4 group range finite else kInvalidArgument
///   packed_out.size() >= packed_bytes(format, in.size())      else kBufferTooSmall
/// FP16 takes any input (non-finite values are representable).
[[nodiscard]] QuantStatus quantize_reference(QuantFormat format, std::span<const float> in,
                                             std::size_t group_size,
                                             std::span<AffineParams> params_out,
                                             std::span<std::byte> packed_out) noexcept;

}  // namespace hl::quant
