// Device-side element codecs shared by the sm_100a kernels.
//
// Decode contract (the reference's dequantize_reference_to_fp16,
// project2_quant/src/cpu_dequant.cpp:93-141, on its x86-64 build):
//   FP16  out = code, except NaN codes which become sign|0x7E00
//   FP8   out = fp16_rn(fp32(decode(code)) * scale)             (two roundings)
//         NaN codes -> sign|0x7E00; E5M2 +-Inf * 0 -> 0xFE00 (the SSE default NaN)
//   INT4  out = fp16_rn(fmaf(float(q), scale, bias))            (one fused rounding)
// Parameters must be finite, as the reference requires.  No fast-math anywhere:
// products that are binary32 subnormals must not be flushed.
//
// Encode contract (quantize_reference, project2_quant/src/cpu_quant.cpp:27-170):
// round-to-nearest-even with integer arithmetic, FP8 saturating, FP16 overflow to Inf.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace hlkv {
namespace dev {

enum : uint32_t { kFp16 = 0, kE4M3 = 1, kE5M2 = 2, kInt4 = 3, kInvalidFormat = 15 };

// Error bits (the HLKV_ERR_* values of include/hlkv.h).
enum : uint32_t {
  kErrNotExecutable = 1u << 0,
  kErrBadFormat = 1u << 1,
  kErrSlotRange = 1u << 2,
  kErrArenaRange = 1u << 3,
  kErrBlockIdRange = 1u << 4,
  kErrValidTokens = 1u << 5,
  kErrLayout = 1u << 6,
  kErrScaleMode = 1u << 7,
  kErrDescMismatch = 1u << 8,
  kErrNonFinite = 1u << 9,
  kErrTokenRange = 1u << 10,
  kErrPatchRange = 1u << 11,
  kErrOutAlign = 1u << 12,
};

__device__ __forceinline__ uint32_t f16_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }

// Two binary32 values -> two binary16 (RNE) packed lo | hi << 16.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ---- FP16 ------------------------------------------------------------------------------------

// NaN halves (magnitude > 0x7C00) of a packed pair become sign|0x7E00.
__device__ __forceinline__ uint32_t canon_f16x2(uint32_t w) {
  const uint32_t nan = __vcmpgtu2(w & 0x7FFF7FFFu, 0x7C007C00u);  // 0xFFFF per NaN half
  return (w & ~nan) | (nan & ((w & 0x80008000u) | 0x7E007E00u));
}

// Any NaN half among 8: magnitude + 0x3FF reaches bit 15 exactly for magnitudes > 0x7C00.
__device__ __forceinline__ bool f16x8_has_nan(uint4 v) {
  const uint32_t any = ((v.x & 0x7FFF7FFFu) + 0x03FF03FFu) | ((v.y & 0x7FFF7FFFu) + 0x03FF03FFu) |
                       ((v.z & 0x7FFF7FFFu) + 0x03FF03FFu) | ((v.w & 0x7FFF7FFFu) + 0x03FF03FFu);
  return (any & 0x80008000u) != 0;
}

__device__ __forceinline__ uint4 canon_f16x8(uint4 v) {
  if (!f16x8_has_nan(v)) return v;
  return make_uint4(canon_f16x2(v.x), canon_f16x2(v.y), canon_f16x2(v.z), canon_f16x2(v.w));
}

// ---- FP8 decode ------------------------------------------------------------------------------

// Exact value of a finite FP8 code: the code's exponent and mantissa bits are
// placed in the binary32 exponent/mantissa fields (a binary32 normal or
// subnormal) and rebiased by an exact power-of-two multiply.
template <uint32_t kKind>
__device__ __forceinline__ float fp8_finite_value(uint32_t b) {
  if constexpr (kKind == kE4M3) {
    return __fmul_rn(__uint_as_float(((b & 0x80u) << 24) | ((b & 0x7Fu) << 20)), 0x1p120f);
  } else {
    return __fmul_rn(__uint_as_float(((b & 0x80u) << 24) | ((b & 0x7Fu) << 21)), 0x1p112f);
  }
}

// One element, including NaN and Inf codes.
template <uint32_t kKind>
__device__ __forceinline__ uint32_t fp8_to_f16(uint32_t b, float scale) {
  if constexpr (kKind == kE4M3) {
    if ((b & 0x7Fu) == 0x7Fu) return ((b & 0x80u) << 8) | 0x7E00u;
  } else {
    if ((b & 0x7Cu) == 0x7Cu) {
      if (b & 3u) return ((b & 0x80u) << 8) | 0x7E00u;  // NaN
      if (scale == 0.0f) return 0xFE00u;                // Inf * 0: SSE default NaN
      const float inf = __int_as_float((b & 0x80u) ? 0xFF800000 : 0x7F800000);
      return f16_bits(__fmul_rn(inf, scale));
    }
  }
  return f16_bits(__fmul_rn(fp8_finite_value<kKind>(b), scale));
}

// True when any of the 4 codes of `w` is a NaN (E4M3: magnitude 0x7F) or an
// Inf/NaN (E5M2: exponent bits 0x7C all set).  With the magnitude masked to
// 7 bits, adding 1 (E4M3) or 4 (E5M2) per byte carries into bit 7 exactly for
// those codes, and no byte carries into its neighbour.
template <uint32_t kKind>
__device__ __forceinline__ bool fp8_has_special(uint32_t w) {
  if constexpr (kKind == kE4M3) return (((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u) != 0;
  else return (((w & 0x7C7C7C7Cu) + 0x04040404u) & 0x80808080u) != 0;
}

// Per-element path for 8 codes that include a NaN or Inf code (rare): kept out
// of line so the common path stays small in registers.
template <uint32_t kKind>
__device__ __noinline__ uint4 fp8x8_to_f16_special(uint2 c, float scale) {
  uint32_t r[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w = k < 2 ? c.x : c.y;
    const uint32_t sh = (k & 1) * 16;
    r[k] = fp8_to_f16<kKind>((w >> sh) & 0xFFu, scale) |
           (fp8_to_f16<kKind>((w >> (sh + 8)) & 0xFFu, scale) << 16);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Eight codes (little-endian in a uint2) -> eight binary16 in a uint4, with each code's
// bits placed in a binary32 pattern instead of converted (fp8x8_to_f16 below gives the
// same results).  Kernel (1) uses this form: on the mixed cache it measured 2 % faster
// there, while the conversion form is faster where instruction issue bounds the kernel.
//
// fp8_finite_value(b) = bits(b) * 2^k exactly (k = 120 for E4M3, 112 for
// E5M2), so decode(b) * scale = bits(b) * (scale * 2^k) as real numbers, and
// one rounding of the same real gives the same binary32 -- provided
// scale * 2^k is itself exact, i.e. |scale| < 2^(128-k).  That folds the
// rebias into one multiply per row; larger scales take the two-multiply form.
template <uint32_t kKind>
__device__ __forceinline__ float fp8_fold_bits(uint32_t b) {
  if constexpr (kKind == kE4M3) return __uint_as_float(((b & 0x80u) << 24) | ((b & 0x7Fu) << 20));
  else return __uint_as_float(((b & 0x80u) << 24) | ((b & 0x7Fu) << 21));
}

template <uint32_t kKind>
__device__ __forceinline__ uint4 fp8x8_to_f16_bits(uint2 c, float scale) {
  if (fp8_has_special<kKind>(c.x) | fp8_has_special<kKind>(c.y)) {
    return fp8x8_to_f16_special<kKind>(c, scale);
  }
  constexpr float kRebias = kKind == kE4M3 ? 0x1p120f : 0x1p112f;
  constexpr float kFoldLimit = kKind == kE4M3 ? 0x1p8f : 0x1p16f;
  uint32_t r[4];
  if (fabsf(scale) < kFoldLimit) {
    const float folded = __fmul_rn(scale, kRebias);  // exact
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t w = k < 2 ? c.x : c.y;
      const uint32_t sh = (k & 1) * 16;
      const float lo = __fmul_rn(fp8_fold_bits<kKind>((w >> sh) & 0xFFu), folded);
      const float hi = __fmul_rn(fp8_fold_bits<kKind>((w >> (sh + 8)) & 0xFFu), folded);
      r[k] = pack_f16x2(lo, hi);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t w = k < 2 ? c.x : c.y;
      const uint32_t sh = (k & 1) * 16;
      const float lo = __fmul_rn(fp8_finite_value<kKind>((w >> sh) & 0xFFu), scale);
      const float hi = __fmul_rn(fp8_finite_value<kKind>((w >> (sh + 8)) & 0xFFu), scale);
      r[k] = pack_f16x2(lo, hi);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Two finite codes (little-endian in the low 16 bits of w) -> their values as binary16.
// Every finite E4M3 and E5M2 value is a binary16 value, so the conversion is exact.
template <uint32_t kKind>
__device__ __forceinline__ float2 fp8x2_exact(uint32_t w) {
  const unsigned short c = static_cast<unsigned short>(w & 0xFFFFu);
  uint32_t h;
  if constexpr (kKind == kE4M3) {
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(c));
  } else {
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h) : "h"(c));
  }
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Eight codes (little-endian in a uint2) -> eight binary16 in a uint4: per element the
// binary32 product of the code's exact value and the scale, rounded to binary16 -- the
// reference's fp16_rn(fp32(decode(q)) * scale).  Codes are converted two at a time to
// their exact binary16 values, widened to binary32 (exact), multiplied, and packed.
template <uint32_t kKind>
__device__ __forceinline__ uint4 fp8x8_to_f16(uint2 c, float scale) {
  if (fp8_has_special<kKind>(c.x) | fp8_has_special<kKind>(c.y)) {
    return fp8x8_to_f16_special<kKind>(c, scale);
  }
  uint32_t r[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w = k < 2 ? c.x : c.y;
    const float2 v = fp8x2_exact<kKind>(w >> ((k & 1) * 16));
    r[k] = pack_f16x2(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// ---- block-wide parameters --------------------------------------------------------------

// The dequantization parameters {scale, bias} that a quantized block's descriptor carries
// for all its rows, by scale mode (ScaleMode, block_descriptor.hpp:61-72):
//   1 kInlineF32: the binary32 bits of scale_ref (inline_scale_f32), bias 0;
//   2 kInlineF16Pair: binary16 scale in bits 0..15 and bias in bits 16..31, widened exactly.
__device__ __forceinline__ float2 block_params_value(uint32_t mode, uint32_t scale_ref) {
  if (mode == 1) return make_float2(__uint_as_float(scale_ref), 0.0f);
  return make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(scale_ref & 0xFFFFu))),
                     __half2float(__ushort_as_half(static_cast<unsigned short>(scale_ref >> 16))));
}

// The block is then one group of the reference's dequantize_reference_to_fp16, which
// rejects non-finite parameters and a nonzero FP8 bias.  Tested on the bits: a value is
// finite when its exponent field is not all ones; a binary16 bias is 0 when its low 15
// bits are.
__device__ __forceinline__ bool block_params_ok(uint32_t f, uint32_t mode, uint32_t scale_ref) {
  if (mode == 1) return ((scale_ref >> 23) & 0xFFu) != 0xFFu;
  return ((scale_ref >> 10) & 0x1Fu) != 0x1Fu && ((scale_ref >> 26) & 0x1Fu) != 0x1Fu &&
         (f == kInt4 || (scale_ref & 0x7FFF0000u) == 0u);
}

// Both of the above: false when rejected, else the parameters in *out.
__device__ __forceinline__ bool block_params(uint32_t f, uint32_t mode, uint32_t scale_ref, float2* out) {
  if (!block_params_ok(f, mode, scale_ref)) return false;
  *out = block_params_value(mode, scale_ref);
  return true;
}

// ---- INT4 decode -----------------------------------------------------------------------------

// q (0..15) as binary32, exactly: (2^23 + q) - 2^23.
__device__ __forceinline__ float nibble_value(uint32_t q) {
  return __fsub_rn(__uint_as_float(0x4B000000u | q), 8388608.0f);
}

// Eight nibbles (element 2k in the low nibble of byte k) -> eight binary16.
// The low and high nibbles are split into two byte vectors; a byte permute
// then places one code in the low byte of the binary32 pattern of 2^23, so
// (2^23 + q) - 2^23 recovers q exactly.
__device__ __forceinline__ uint4 int4x8_to_f16(uint32_t w, float scale, float bias) {
  const uint32_t lo4 = w & 0x0F0F0F0Fu;         // elements 0, 2, 4, 6
  const uint32_t hi4 = (w >> 4) & 0x0F0F0F0Fu;  // elements 1, 3, 5, 7
  uint32_t r[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // selector: byte k of the first operand, then bytes 1..3 of 0x4B000000 (= 0x4B, 0, 0 high).
    const uint32_t sel = static_cast<uint32_t>(k) | 0x7650u;
    const float qlo = __fsub_rn(__uint_as_float(__byte_perm(lo4, 0x4B000000u, sel)), 8388608.0f);
    const float qhi = __fsub_rn(__uint_as_float(__byte_perm(hi4, 0x4B000000u, sel)), 8388608.0f);
    r[k] = pack_f16x2(__fmaf_rn(qlo, scale, bias), __fmaf_rn(qhi, scale, bias));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

__device__ __forceinline__ uint32_t int4_to_f16(uint32_t q, float scale, float bias) {
  return f16_bits(__fmaf_rn(nibble_value(q), scale, bias));
}

// ---- encoders --------------------------------------------------------------------------------

// binary32 -> minifloat with round-to-nearest-even on the integer significand
// (the method of project2_quant/src/cpu_quant.cpp:27-64).
template <uint32_t kEBits, uint32_t kMBits, int kBias, bool kSaturate, uint32_t kMaxCode,
          uint32_t kNanCode, uint32_t kInfCode>
__device__ __forceinline__ uint32_t encode_minifloat(float x) {
  const uint32_t bits = __float_as_uint(x);
  const uint32_t sign = (bits >> 31) << (kEBits + kMBits);
  const uint32_t mag = bits & 0x7FFFFFFFu;
  constexpr uint32_t kOverflow = kSaturate ? kMaxCode : kInfCode;
  if (mag > 0x7F800000u) return sign | kNanCode;
  if (mag == 0x7F800000u) return sign | kOverflow;
  constexpr int kEmin = 1 - kBias;
  int binade, lsb_exp;
  uint32_t sig;
  if (mag >= 0x00800000u) {
    const int e = static_cast<int>(mag >> 23) - 127;
    sig = (mag & 0x007FFFFFu) | 0x00800000u;
    lsb_exp = e - 23;
    binade = e < kEmin ? kEmin : e;
  } else {
    sig = mag;
    lsb_exp = -149;
    binade = kEmin;
  }
  const int drop = (binade - static_cast<int>(kMBits)) - lsb_exp;  // >= 1
  uint32_t kept = 0;  // drop >= 32: sig < 2^24 is below half a spacing, rounds to 0
  if (drop < 32) {
    kept = sig >> drop;
    const uint32_t rest = sig & ((1u << drop) - 1u);
    const uint32_t half = 1u << (drop - 1);
    if (rest > half || (rest == half && (kept & 1u))) kept += 1u;
  }
  const uint32_t code = (static_cast<uint32_t>(binade - kEmin) << kMBits) + kept;
  return sign | (code > kMaxCode ? kOverflow : code);
}

__device__ __forceinline__ uint32_t encode_e4m3(float x) {
  return encode_minifloat<4, 3, 7, true, 0x7Eu, 0x7Fu, 0u>(x);
}
__device__ __forceinline__ uint32_t encode_e5m2(float x) {
  return encode_minifloat<5, 2, 15, true, 0x7Bu, 0x7Fu, 0x7Cu>(x);
}
__device__ __forceinline__ uint32_t encode_f16(float x) {
  return encode_minifloat<5, 10, 15, false, 0x7BFFu, 0x7E00u, 0x7C00u>(x);
}

// Two binary32 -> two FP8 codes (lo in bits 0..7, hi in bits 8..15), round to nearest
// even, saturating to the largest finite code: the hardware conversion.  For every
// finite binary32 input it equals encode_e4m3 / encode_e5m2 bit for bit (checked
// exhaustively over all 2^32 patterns on sm_100a); NaN and Inf never reach it (the
// encoders reject non-finite groups and x / scale stays finite).
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e5m2x2(float lo, float hi) {
  unsigned short r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ bool finite_f32(float x) {
  return (__float_as_uint(x) & 0x7F800000u) != 0x7F800000u;
}

}  // namespace dev
}  // namespace hlkv
