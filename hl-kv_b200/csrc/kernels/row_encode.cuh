// Row encoder shared by kernel (2) (append-encode) and the transcode kernel: one
// parameter group = one row of kD binary16 values, handled by kD/(8 kChunks) lanes.
// Each lane holds kChunks chunks of 8 values; chunk c of lane l is the row's chunk
// c * lanes + l, so that each chunk-wide load or store of a warp is contiguous.  Per row it is the reference's quantize_reference
// (project2_quant/src/cpu_quant.cpp:97-170) on the binary32 values of the inputs:
//   FP16  encode_fp16 of an FP16 value: the value itself, NaN canonicalized;
//   FP8   amax -> scale = max(amax / max_finite, FLT_MIN) (1 when amax == 0),
//         code = RNE-saturating encode of x / scale (IEEE division; the encode is the
//         hardware cvt.rn.satfinite, equal to the reference's integer RNE);
//   INT4  (min, first index) and (max, last index), which is what std::minmax_element
//         returns and what makes the bias bits of +-0 ties exact;
//         scale = (max - min) / 15, q = clamp(rint((x - min) / scale), 0, 15).
// A row with a non-finite input (or an INT4 range that overflows) is rejected as
// quantize_reference rejects it: nothing is written and kErrNonFinite is returned.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "codec.cuh"

namespace hlkv {
namespace dev {

// Reductions over the kLanes lanes of one row.  `mask` names exactly those lanes, so
// rows of one warp may take different branches.
template <int kLanes>
__device__ __forceinline__ float lanes_max(uint32_t mask, float v) {
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(mask, v, o, kLanes));
  return v;
}

// Min with the lowest index among equal values, max with the highest.
template <int kLanes>
__device__ __forceinline__ void lanes_minmax(uint32_t mask, float& mn, uint32_t& imn, float& mx,
                                             uint32_t& imx) {
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) {
    const float omn = __shfl_xor_sync(mask, mn, o, kLanes);
    const uint32_t oimn = __shfl_xor_sync(mask, imn, o, kLanes);
    const float omx = __shfl_xor_sync(mask, mx, o, kLanes);
    const uint32_t oimx = __shfl_xor_sync(mask, imx, o, kLanes);
    if (omn < mn || (omn == mn && oimn < imn)) { mn = omn; imn = oimn; }
    if (omx > mx || (omx == mx && oimx > imx)) { mx = omx; imx = oimx; }
  }
}

// Per-halfword unsigned max and min of two packed pairs (native on sm_90 and later).
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// The lane mask of the kD/(8 kChunks) lanes that share this thread's row.
template <int kD, int kChunks = 1>
__device__ __forceinline__ uint32_t row_mask() {
  constexpr int kLanes = kD / (8 * kChunks);
  return kLanes == 32 ? 0xFFFFFFFFu : ((1u << kLanes) - 1u) << ((threadIdx.x % 32) / kLanes * kLanes);
}

// ---- the exact quotient shortcut -----------------------------------------------------
//
// Both encoders round a quotient q = RN(v / s) once more: to an FP8 code (RNE,
// saturating) or to an integer (rint).  With y = RN(1/s), the products v*y*(1 -+ e),
// e = 2^-21, each rounded to binary32, lie at least 5 * 2^-24 * |v/s| below and above
// v/s, while RN(v/s) lies within 2^-24 * |v/s| of it (v a binary16 value or a
// difference of two, s > 0, no underflow or overflow for such inputs).  Both final
// roundings are monotone, so when the two ends round to the same result, RN(v/s)
// rounds to it too; otherwise (within a few units of a rounding boundary, about one
// value in 2^17) the quotient is computed with an IEEE division.  The results equal
// the division-based ones bit for bit.
constexpr float kBracketLo = 1.0f - 0x1p-21f;
constexpr float kBracketHi = 1.0f + 0x1p-21f;

// Order-preserving 16-bit key of a binary16 pattern (two per word): -x < -y < -0 < +0 < y.
// Negative halves are complemented, positive ones get the sign bit set; the prmt
// selector 0xBB99 replicates each half's sign bit over that half.
__device__ __forceinline__ uint32_t f16x2_keys(uint32_t w) {
  uint32_t neg;
  asm("prmt.b32 %0, %1, 0, 0xBB99;" : "=r"(neg) : "r"(w));
  return w ^ (neg | 0x80008000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  const uint32_t h = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// rint(v) for 0 <= v < 2^22 as an integer: the addition rounds to nearest even.
__device__ __forceinline__ uint32_t rint_u(float v) {
  return __float_as_uint(__fadd_rn(v, 12582912.0f)) - 0x4B400000u;
}

// Encodes one row (this lane's kChunks x 8 binary16 values in `raw`) in format f into row
// `row` of a slot laid out as codes then per-row parameters (`payload`, code region of
// `code_bytes`).  Uniform over the row's lanes; returns 0 or kErrNonFinite.
template <int kD, int kChunks = 1>
__device__ __forceinline__ uint32_t encode_row(uint32_t f, const uint4 (&raw)[kChunks], uint32_t lane,
                                               uint32_t mask, uint8_t* payload, uint32_t row,
                                               uint64_t code_bytes) {
  constexpr int kLanes = kD / (8 * kChunks);
  constexpr int kW = 4 * kChunks;  // 32-bit words (two values each) per lane
  constexpr int kV = 8 * kChunks;  // values per lane
  if (f == kFp16) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      reinterpret_cast<uint4*>(payload + uint64_t{row} * kD * 2)[c * kLanes + lane] = canon_f16x8(raw[c]);
    }
    return 0;
  }
  uint32_t w[kW];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    w[4 * c] = raw[c].x;
    w[4 * c + 1] = raw[c].y;
    w[4 * c + 2] = raw[c].z;
    w[4 * c + 3] = raw[c].w;
  }
  // A row with an Inf or NaN (exponent field all ones) is found from the row statistics
  // each format reduces anyway: the largest magnitude bits for FP8, the extreme keys for
  // INT4.
  float x[kV];
#pragma unroll
  for (int i = 0; i < kW; ++i) {
    x[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xFFFFu)));
    x[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
  }

  if (f == kE4M3 || f == kE5M2) {
    // amax on the magnitude bits (unsigned order = magnitude order; Inf and NaN patterns
    // are the ones from 0x7C00 up).
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kW; ++i) m = max_u16x2(m, w[i] & 0x7FFF7FFFu);
    m = max(m & 0xFFFFu, m >> 16);
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(mask, m, o, kLanes));
    if (m >= 0x7C00u) return kErrNonFinite;
    const float amax = __half2float(__ushort_as_half(static_cast<unsigned short>(m)));
    // RN(amax / max_finite) without a division.  With y = RN(1/max_finite), q0 = RN(amax y)
    // and r = amax - q0 max_finite (exact in one FMA), RN(q0 + r y) equals the IEEE
    // quotient for every positive finite binary16 amax and both constants (448 = 7 x 2^6,
    // 57344 = 7 x 2^13): checked exhaustively over the 31743 inputs of each.
    const float max_finite = f == kE4M3 ? 448.0f : 57344.0f;
    const float inv_max = f == kE4M3 ? 0x1.24924ap-9f : 0x1.24924ap-16f;
    float scale = 1.0f;
    if (amax > 0.0f) {
      const float q0 = __fmul_rn(amax, inv_max);
      const float q = __fmaf_rn(__fmaf_rn(-q0, max_finite, amax), inv_max, q0);
      scale = q < 1.17549435e-38f ? 1.17549435e-38f : q;  // std::max(q, FLT_MIN)
    }
    const float y = __frcp_rn(scale);
    const float ylo = __fmul_rn(y, kBracketLo), yhi = __fmul_rn(y, kBracketHi);
    uint32_t c[kW];
    uint32_t diff = 0;  // nonzero when the two ends of some bracket round apart
#pragma unroll
    for (int i = 0; i < kW; ++i) {
      const float a0 = __fmul_rn(x[2 * i], ylo), a1 = __fmul_rn(x[2 * i + 1], ylo);
      const float b0 = __fmul_rn(x[2 * i], yhi), b1 = __fmul_rn(x[2 * i + 1], yhi);
      const uint32_t lo = f == kE4M3 ? cvt_e4m3x2(a0, a1) : cvt_e5m2x2(a0, a1);
      const uint32_t hi = f == kE4M3 ? cvt_e4m3x2(b0, b1) : cvt_e5m2x2(b0, b1);
      diff |= lo ^ hi;
      c[i] = lo;
    }
    if (diff != 0) {  // near an FP8 rounding boundary: the divisions themselves
#pragma unroll
      for (int i = 0; i < kW; ++i) {
        const float q0 = __fdiv_rn(x[2 * i], scale), q1 = __fdiv_rn(x[2 * i + 1], scale);
        c[i] = f == kE4M3 ? cvt_e4m3x2(q0, q1) : cvt_e5m2x2(q0, q1);
      }
    }
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      reinterpret_cast<uint2*>(payload + uint64_t{row} * kD)[k * kLanes + lane] =
          make_uint2(c[4 * k] | c[4 * k + 1] << 16, c[4 * k + 2] | c[4 * k + 3] << 16);
    }
    if (lane == 0) reinterpret_cast<float*>(payload + code_bytes)[row] = scale;
    return 0;
  }

  // INT4: min and max through order-preserving keys; one shuffle per round carries both
  // (the min key low, the complement of the max key high).
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;  // two halves each, folded below
#pragma unroll
  for (int i = 0; i < kW; ++i) {
    const uint32_t k = f16x2_keys(w[i]);
    kmin = min_u16x2(kmin, k);
    kmax = max_u16x2(kmax, k);
  }
  kmin = min(kmin & 0xFFFFu, kmin >> 16);
  kmax = max(kmax & 0xFFFFu, kmax >> 16);
  uint32_t both = kmin | (0xFFFFu - kmax) << 16;
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) both = min_u16x2(both, __shfl_xor_sync(mask, both, o, kLanes));
  kmin = both & 0xFFFFu;
  kmax = 0xFFFFu - (both >> 16);
  // Keys of +Inf and NaN are 0xFC00 and above; of -Inf and negative NaN, 0x03FF and below.
  if (kmax >= 0xFC00u || kmin <= 0x03FFu) return kErrNonFinite;
  float mn, mx;
  // -0 and +0 compare equal: std::minmax_element then returns the first minimum and the
  // last maximum by index, which decides the sign of a zero bias.  Only a row whose
  // minimum is -0 with values >= +0 present, or whose maximum is +0 with values <= -0
  // present, can hold both; it takes the index-tracking reduction.  The lane's values
  // are visited in increasing row index (chunk by chunk).
  if ((kmin == 0x7FFFu && kmax >= 0x8000u) || (kmax == 0x8000u && kmin <= 0x7FFFu)) {
    mn = x[0];
    mx = x[0];
    uint32_t imn = lane * 8, imx = lane * 8;
#pragma unroll
    for (int i = 1; i < kV; ++i) {
      const uint32_t idx = ((i / 8) * kLanes + lane) * 8 + i % 8;
      if (x[i] < mn) { mn = x[i]; imn = idx; }
      if (!(x[i] < mx)) { mx = x[i]; imx = idx; }
    }
    lanes_minmax<kLanes>(mask, mn, imn, mx, imx);
  } else {
    mn = key_to_float(kmin);
    mx = key_to_float(kmax);
  }
  const float range = __fsub_rn(mx, mn);
  if (!finite_f32(range)) return kErrNonFinite;
  const float scale = __fdiv_rn(range, 15.0f);
  uint32_t word[kChunks];
#pragma unroll
  for (int k = 0; k < kChunks; ++k) word[k] = 0;
  if (scale > 0.0f) {
    const float y = __frcp_rn(scale);
    const float ylo = __fmul_rn(y, kBracketLo), yhi = __fmul_rn(y, kBracketHi);
    // 0 <= d <= range, so d/scale <= 15 / (1 - 2^-24) and both ends round to integers in
    // [0, 15]: the clamp is a no-op and the low 4 bits of RN(v + 1.5 x 2^23) are the code.
    uint32_t diff = 0;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const float d = __fsub_rn(x[i], mn);
      const uint32_t qa = __float_as_uint(__fadd_rn(__fmul_rn(d, ylo), 12582912.0f));
      const uint32_t qb = __float_as_uint(__fadd_rn(__fmul_rn(d, yhi), 12582912.0f));
      diff |= qa ^ qb;
      word[i / 8] |= (qa & 0xFu) << (4 * (i % 8));
    }
    if (diff != 0) {  // near a .5 boundary: the divisions themselves
#pragma unroll
      for (int k = 0; k < kChunks; ++k) word[k] = 0;
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const uint32_t q = rint_u(__fdiv_rn(__fsub_rn(x[i], mn), scale));
        word[i / 8] |= min(q, 15u) << (4 * (i % 8));
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    reinterpret_cast<uint32_t*>(payload + uint64_t{row} * (kD / 2))[k * kLanes + lane] = word[k];
  }
  if (lane == 0) reinterpret_cast<float2*>(payload + code_bytes)[row] = make_float2(scale, mn);
  return 0;
}

}  // namespace dev
}  // namespace hlkv
