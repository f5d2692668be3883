// Host codecs of hl_quant: the reference's CPU API (project2_quant/include/hl_quant/
// cpu_quant.hpp:22-47 and cpu_dequant.hpp:15-54) and the host emulation of the flat FP8
// decoder (cuda_dequant.hpp:52-71).  Results equal the reference's bit for bit; the
// implementation is this library's own:
//  * encoding rounds in binary64, where |x| divided by the target's spacing at |x| is exact
//    (a 24-bit significand rescaled by a power of two), with std::nearbyint under the default
//    rounding mode doing the round-half-even; the code is then (binade - emin) << mbits plus
//    that integer, which also covers subnormal targets and a carry into the next binade;
//  * FP8 decoding goes through two 256-entry tables built once from the format parameters;
//    FP16 decoding rescales the integer significand with std::ldexp (exact).
// Built with -ffp-contract=off and without fast-math: every product, quotient and fma below
// rounds once, as the reference's arithmetic does.
#include <array>
#include <bit>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <span>

#include "hl_quant/cpu_dequant.hpp"
#include "hl_quant/cpu_quant.hpp"
#include "hl_quant/cuda_dequant.hpp"
#include "hl_quant/quant_types.hpp"

namespace hl::quant {
namespace {

// A binary floating-point format narrower than binary32.
struct Minifloat {
  int mbits;               // stored significand bits
  int emin;                // unbiased exponent of the smallest normal
  int width;               // bits below the sign bit
  std::uint32_t max_mag;   // magnitude code of the largest finite value
  std::uint32_t nan_mag;   // magnitude code an encoder writes for NaN
  std::uint32_t over_mag;  // magnitude code for +-Inf and overflow: Inf, or max_mag when saturating
  bool has_inf;            // the code after max_mag is Inf (IEEE-style specials)
};
constexpr Minifloat kHalf{10, -14, 15, 0x7BFFu, 0x7E00u, 0x7C00u, true};
constexpr Minifloat kE4M3{3, -6, 7, 0x7Eu, 0x7Fu, 0x7Eu, false};
constexpr Minifloat kE5M2{2, -14, 7, 0x7Bu, 0x7Fu, 0x7Bu, true};

std::uint32_t encode(const Minifloat& m, float x) noexcept {
  const std::uint32_t bits = std::bit_cast<std::uint32_t>(x);
  const std::uint32_t sign = (bits >> 31) << m.width;
  const std::uint32_t mag = bits & 0x7FFFFFFFu;
  if (mag > 0x7F800000u) return sign | m.nan_mag;
  if (mag == 0x7F800000u) return sign | m.over_mag;
  // Binade of |x|, clamped at the target's smallest normal: the target's values there are
  // spaced 2^(e - mbits) apart.
  int e = mag >= 0x00800000u ? static_cast<int>(mag >> 23) - 127 : m.emin;
  if (e < m.emin) e = m.emin;
  const double units = std::nearbyint(std::ldexp(static_cast<double>(std::fabs(x)), m.mbits - e));
  const std::uint64_t code = (static_cast<std::uint64_t>(e - m.emin) << m.mbits) +
                             static_cast<std::uint64_t>(units);
  return sign | (code > m.max_mag ? m.over_mag : static_cast<std::uint32_t>(code));
}

float decode(const Minifloat& m, std::uint32_t code) noexcept {
  const bool neg = ((code >> m.width) & 1u) != 0;
  const std::uint32_t mag = code & ((1u << m.width) - 1u);
  if (mag > m.max_mag) {
    if (m.has_inf && mag == m.max_mag + 1u) return neg ? -std::numeric_limits<float>::infinity()
                                                       : std::numeric_limits<float>::infinity();
    return std::bit_cast<float>((neg ? 0x80000000u : 0u) | 0x7FC00000u);  // quiet NaN, sign kept
  }
  const std::uint32_t field = mag >> m.mbits, frac = mag & ((1u << m.mbits) - 1u);
  const float v = field == 0
                      ? std::ldexp(static_cast<float>(frac), m.emin - m.mbits)
                      : std::ldexp(static_cast<float>(frac | (1u << m.mbits)),
                                   m.emin + static_cast<int>(field) - 1 - m.mbits);
  return neg ? -v : v;
}

using Table8 = std::array<float, 256>;
Table8 make_table(const Minifloat& m) noexcept {
  Table8 t{};
  for (std::uint32_t c = 0; c < 256; ++c) t[c] = decode(m, c);
  return t;
}
const Table8& e4m3_table() noexcept {
  static const Table8 t = make_table(kE4M3);
  return t;
}
const Table8& e5m2_table() noexcept {
  static const Table8 t = make_table(kE5M2);
  return t;
}

std::uint32_t code_at(QuantFormat f, const std::byte* packed, std::size_t i) noexcept {
  switch (f) {
    case QuantFormat::kFp16: {
      std::uint16_t h;
      std::memcpy(&h, packed + 2 * i, 2);
      return h;
    }
    case QuantFormat::kInt4Packed:
      return (std::to_integer<std::uint32_t>(packed[i / 2]) >> (4 * (i & 1))) & 0xFu;
    default:
      return std::to_integer<std::uint32_t>(packed[i]);
  }
}

// The binary32 value of element i (its group's parameters already fetched).
float value_of(QuantFormat f, std::uint32_t q, AffineParams p) noexcept {
  switch (f) {
    case QuantFormat::kFp16: return decode(kHalf, q);
    case QuantFormat::kFp8E4M3: return e4m3_table()[q] * p.scale;
    case QuantFormat::kFp8E5M2: return e5m2_table()[q] * p.scale;
    default: return std::fma(static_cast<float>(q), p.scale, p.bias);
  }
}

// The argument checks of dequantize_reference and dequantize_reference_to_fp16, in order.
QuantStatus check_decode(QuantFormat f, std::size_t packed_size, std::size_t n,
                         std::span<const AffineParams> params, std::size_t group_size,
                         std::size_t out_size) noexcept {
  if (!is_valid(f)) return QuantStatus::kUnsupportedFormat;
  if (n > kMaxElements || !is_valid_group_size(f, group_size) ||
      params.size() != num_groups(n, group_size)) {
    return QuantStatus::kInvalidArgument;
  }
  const bool fp8 = f == QuantFormat::kFp8E4M3 || f == QuantFormat::kFp8E5M2;
  for (const AffineParams& p : params) {
    if (!std::isfinite(p.scale) || !std::isfinite(p.bias) || (fp8 && p.bias != 0.0f)) {
      return QuantStatus::kInvalidArgument;
    }
  }
  if (packed_size < packed_bytes(f, n) || out_size < n) return QuantStatus::kBufferTooSmall;
  return QuantStatus::kOk;
}

// Calls fn(i, value) for every element, walking group by group.
template <typename Fn>
void for_each_value(QuantFormat f, const std::byte* packed, std::size_t n,
                    std::span<const AffineParams> params, std::size_t group_size, Fn&& fn) noexcept {
  if (f == QuantFormat::kFp16) {
    for (std::size_t i = 0; i < n; ++i) fn(i, decode(kHalf, code_at(f, packed, i)));
    return;
  }
  for (std::size_t g = 0, b = 0; b < n; ++g, b += group_size) {
    const std::size_t e = n - b < group_size ? n : b + group_size;
    const AffineParams p = params[g];
    for (std::size_t i = b; i < e; ++i) fn(i, value_of(f, code_at(f, packed, i), p));
  }
}

}  // namespace

std::uint16_t encode_fp16(float x) noexcept { return static_cast<std::uint16_t>(encode(kHalf, x)); }
std::uint8_t encode_fp8_e4m3(float x) noexcept { return static_cast<std::uint8_t>(encode(kE4M3, x)); }
std::uint8_t encode_fp8_e5m2(float x) noexcept { return static_cast<std::uint8_t>(encode(kE5M2, x)); }

float decode_fp16(std::uint16_t bits) noexcept { return decode(kHalf, bits); }
float decode_fp8_e4m3(std::uint8_t bits) noexcept { return e4m3_table()[bits]; }
float decode_fp8_e5m2(std::uint8_t bits) noexcept { return e5m2_table()[bits]; }

QuantStatus quantize_reference(QuantFormat format, std::span<const float> in, std::size_t group_size,
                               std::span<AffineParams> params_out,
                               std::span<std::byte> packed_out) noexcept {
  if (!is_valid(format)) return QuantStatus::kUnsupportedFormat;
  const std::size_t n = in.size();
  if (n > kMaxElements || !is_valid_group_size(format, group_size) ||
      params_out.size() != num_groups(n, group_size)) {
    return QuantStatus::kInvalidArgument;
  }
  const bool int4 = format == QuantFormat::kInt4Packed;
  if (format != QuantFormat::kFp16) {
    for (const float x : in) {
      if (!std::isfinite(x)) return QuantStatus::kInvalidArgument;
    }
  }
  // Per-group extremes for INT4: the first minimum and the last maximum, which decide the
  // sign of a zero bias when -0 and +0 both occur.
  struct Range {
    float lo, hi;
  };
  auto extremes = [&](std::size_t b, std::size_t e) {
    Range r{in[b], in[b]};
    for (std::size_t i = b; i < e; ++i) {
      if (in[i] < r.lo) r.lo = in[i];
      if (!(in[i] < r.hi)) r.hi = in[i];
    }
    return r;
  };
  if (int4) {
    for (std::size_t b = 0; b < n; b += group_size) {
      const Range r = extremes(b, n - b < group_size ? n : b + group_size);
      if (!std::isfinite(r.hi - r.lo)) return QuantStatus::kInvalidArgument;
    }
  }
  const std::size_t bytes = packed_bytes(format, n);
  if (packed_out.size() < bytes) return QuantStatus::kBufferTooSmall;

  std::byte* out = packed_out.data();
  if (format == QuantFormat::kFp16) {
    for (std::size_t i = 0; i < n; ++i) {
      const std::uint16_t h = encode_fp16(in[i]);
      std::memcpy(out + 2 * i, &h, 2);
    }
    return QuantStatus::kOk;
  }
  if (int4) std::memset(out, 0, bytes);
  for (std::size_t g = 0, b = 0; b < n; ++g, b += group_size) {
    const std::size_t e = n - b < group_size ? n : b + group_size;
    if (int4) {
      const Range x = extremes(b, e);
      const float lo = x.lo, scale = (x.hi - lo) / 15.0f;
      params_out[g] = AffineParams{scale, lo};
      if (!(scale > 0.0f)) continue;  // a constant group: every code 0
      for (std::size_t i = b; i < e; ++i) {
        const float r = std::nearbyint((in[i] - lo) / scale);
        const std::uint32_t q = r <= 0.0f ? 0u : (r >= 15.0f ? 15u : static_cast<std::uint32_t>(r));
        out[i / 2] |= static_cast<std::byte>(q << (4 * (i & 1)));
      }
      continue;
    }
    const Minifloat& m = format == QuantFormat::kFp8E4M3 ? kE4M3 : kE5M2;
    float amax = 0.0f;
    for (std::size_t i = b; i < e; ++i) {
      const float a = std::fabs(in[i]);
      if (amax < a) amax = a;
    }
    float scale = 1.0f;
    if (amax > 0.0f) {
      scale = amax / format_traits(format).max_finite;
      if (scale < std::numeric_limits<float>::min()) scale = std::numeric_limits<float>::min();
    }
    params_out[g] = AffineParams{scale, 0.0f};
    for (std::size_t i = b; i < e; ++i) out[i] = static_cast<std::byte>(encode(m, in[i] / scale));
  }
  return QuantStatus::kOk;
}

QuantStatus dequantize_reference(QuantFormat format, std::span<const std::byte> packed,
                                 std::size_t num_elements, std::span<const AffineParams> params,
                                 std::size_t group_size, std::span<float> out) noexcept {
  const QuantStatus st = check_decode(format, packed.size(), num_elements, params, group_size, out.size());
  if (st != QuantStatus::kOk) return st;
  for_each_value(format, packed.data(), num_elements, params, group_size,
                 [&](std::size_t i, float v) { out[i] = v; });
  return QuantStatus::kOk;
}

QuantStatus dequantize_reference_to_fp16(QuantFormat format, std::span<const std::byte> packed,
                                         std::size_t num_elements, std::span<const AffineParams> params,
                                         std::size_t group_size, std::span<std::uint16_t> out) noexcept {
  const QuantStatus st = check_decode(format, packed.size(), num_elements, params, group_size, out.size());
  if (st != QuantStatus::kOk) return st;
  for_each_value(format, packed.data(), num_elements, params, group_size,
                 [&](std::size_t i, float v) { out[i] = encode_fp16(v); });
  return QuantStatus::kOk;
}

namespace cuda {

QuantStatus emulate_fp8_to_fp16_on_host(QuantFormat format, std::span<const std::byte> in,
                                        std::span<const AffineParams> params, std::size_t group_size,
                                        std::span<std::uint16_t> out, HostPath path) noexcept {
  if (format != QuantFormat::kFp8E4M3 && format != QuantFormat::kFp8E5M2) {
    return QuantStatus::kUnsupportedFormat;
  }
  const std::size_t n = in.size();
  if (group_size == 0 || n > kMaxElements || params.size() != num_groups(n, group_size)) {
    return QuantStatus::kInvalidArgument;
  }
  if (out.size() < n) return QuantStatus::kBufferTooSmall;
  const Table8& t = format == QuantFormat::kFp8E4M3 ? e4m3_table() : e5m2_table();
  auto one = [&](std::size_t i) {
    out[i] = encode_fp16(t[std::to_integer<std::uint32_t>(in[i])] * params[i / group_size].scale);
  };
  std::size_t i = 0;
  if (path == HostPath::kVector && (group_size % 8 == 0 || group_size >= n)) {
    // Whole chunks of 8 lie in one group: one parameter fetch per chunk.
    for (; i + 8 <= n; i += 8) {
      const float s = params[i / group_size].scale;
      for (std::size_t k = 0; k < 8; ++k) {
        out[i + k] = encode_fp16(t[std::to_integer<std::uint32_t>(in[i + k])] * s);
      }
    }
  }
  for (; i < n; ++i) one(i);
  return QuantStatus::kOk;
}

}  // namespace cuda
}  // namespace hl::quant
