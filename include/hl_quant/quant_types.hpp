#pragma once
// KV storage formats (drop-in for the reference's
// project2_quant/include/hl_quant/quant_types.hpp: same codes, traits and size
// rules; the code is this library's own).
//
// A format code is the 4-bit `format` field of hl::alloc::BlockExecDescriptor.
// Decoding, binary32 arithmetic with round-to-nearest-even:
//   FP16        x = decode_fp16(q)
//   FP8_E4M3    x = decode_e4m3(q) * scale        (bias must be 0)
//   FP8_E5M2    x = decode_e5m2(q) * scale        (bias must be 0)
//   INT4_PACKED x = fmaf(float(q), scale, bias)   q in [0, 15], one rounding
// (scale, bias) apply to groups of `group_size` consecutive elements.  INT4
// element i lives in byte i/2, low nibble first; groups start on byte
// boundaries and the padding nibble of a trailing partial byte is zero.
// Code 4 (INT2) is retired and rejected.
#include <cstddef>
#include <cstdint>
#include <limits>
#include <string_view>

namespace hl::quant {

enum class QuantFormat : std::uint8_t {
  kFp16 = 0,
  kFp8E4M3 = 1,    ///< OCP E4M3 ("FN"): bias 7, no Inf, NaN = S.1111.111, max 448
  kFp8E5M2 = 2,    ///< OCP E5M2: bias 15, IEEE Inf/NaN, max 57344
  kInt4Packed = 3,
};

inline constexpr std::size_t kNumQuantFormats = 4;
inline constexpr std::uint8_t kRetiredInt2Code = 4;

enum class ElementKind : std::uint8_t { kFloat, kUnsignedInt };

enum class QuantStatus : std::uint8_t {
  kOk = 0,
  kInvalidArgument,
  kBufferTooSmall,
  kUnsupportedFormat,
  kCudaError,
};

[[nodiscard]] const char* to_string(QuantStatus status) noexcept;

struct AffineParams {
  float scale;
  float bias;
};
static_assert(sizeof(AffineParams) == 8);

struct FormatTraits {
  std::string_view name;
  ElementKind kind;
  std::uint8_t bits_per_element;
  std::uint8_t exponent_bits;
  std::uint8_t mantissa_bits;
  std::int8_t exponent_bias;
  bool has_infinity;
  bool uses_params;
  bool uses_bias;
  std::uint32_t max_code;
  float max_finite;
};

[[nodiscard]] constexpr bool is_valid(QuantFormat f) noexcept {
  return static_cast<std::size_t>(f) < kNumQuantFormats;
}

/// Precondition: is_valid(f).
[[nodiscard]] constexpr FormatTraits format_traits(QuantFormat f) noexcept {
  constexpr FormatTraits kTable[kNumQuantFormats] = {
      {"FP16", ElementKind::kFloat, 16, 5, 10, 15, true, false, false, 0x7BFFu, 65504.0f},
      {"FP8_E4M3", ElementKind::kFloat, 8, 4, 3, 7, false, true, false, 0x7Eu, 448.0f},
      {"FP8_E5M2", ElementKind::kFloat, 8, 5, 2, 15, true, true, false, 0x7Bu, 57344.0f},
      {"INT4_PACKED", ElementKind::kUnsignedInt, 4, 0, 0, 0, false, true, true, 15u, 15.0f},
  };
  return is_valid(f) ? kTable[static_cast<std::size_t>(f)]
                     : FormatTraits{"INVALID", ElementKind::kFloat, 0, 0, 0, 0, false, false, false,
                                    0u, 0.0f};
}

inline constexpr std::size_t kMaxElements = std::numeric_limits<std::size_t>::max() / 2;

[[nodiscard]] constexpr std::size_t elements_per_byte(QuantFormat f) noexcept {
  const std::size_t bits = format_traits(f).bits_per_element;
  return (bits == 0 || bits > 8) ? 0 : 8 / bits;
}

[[nodiscard]] constexpr std::size_t packed_bytes(QuantFormat f, std::size_t n) noexcept {
  const std::size_t bits = format_traits(f).bits_per_element;
  if (bits >= 8) return n * (bits / 8);
  const std::size_t per = 8 / bits;
  return n / per + (n % per != 0);
}

[[nodiscard]] constexpr std::size_t num_groups(std::size_t n, std::size_t group_size) noexcept {
  return group_size == 0 ? 0 : n / group_size + (n % group_size != 0);
}

[[nodiscard]] constexpr bool is_valid_group_size(QuantFormat f, std::size_t group_size) noexcept {
  if (!is_valid(f)) return false;
  if (!format_traits(f).uses_params) return group_size == 0;
  return group_size > 0 && group_size % elements_per_byte(f) == 0;
}

}  // namespace hl::quant
