// Row encoder shared by kernel (2) (append-encode) and the transcode kernel: one
// parameter group = one row of kD binary16 values, handled by kD/8 lanes, 8 values
// per lane.  Per row it is the reference's quantize_reference
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

template <int kLanes>
__device__ __forceinline__ bool lanes_any(uint32_t mask, bool b) {
  uint32_t v = b;
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) v |= __shfl_xor_sync(mask, v, o, kLanes);
  return v != 0;
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

// The lane mask of the kD/8 lanes that share this thread's row.
template <int kD>
__device__ __forceinline__ uint32_t row_mask() {
  constexpr int kLanes = kD / 8;
  return kLanes == 32 ? 0xFFFFFFFFu : ((1u << kLanes) - 1u) << ((threadIdx.x % 32) / kLanes * kLanes);
}

// Encodes one row (this lane's 8 binary16 values in `raw`) in format f into row `row` of
// a slot laid out as codes then per-row parameters (`payload`, code region of
// `code_bytes`).  Uniform over the row's lanes; returns 0 or kErrNonFinite.
template <int kD>
__device__ __forceinline__ uint32_t encode_row(uint32_t f, uint4 raw, uint32_t lane, uint32_t mask,
                                               uint8_t* payload, uint32_t row, uint64_t code_bytes) {
  constexpr int kLanes = kD / 8;
  if (f == kFp16) {
    reinterpret_cast<uint4*>(payload + uint64_t{row} * kD * 2)[lane] = canon_f16x8(raw);
    return 0;
  }
  float x[8];
  {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xFFFFu)));
      x[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
    }
  }
  bool nonfinite = false;
#pragma unroll
  for (int i = 0; i < 8; ++i) nonfinite |= !finite_f32(x[i]);
  if (lanes_any<kLanes>(mask, nonfinite)) return kErrNonFinite;

  if (f == kE4M3 || f == kE5M2) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(x[i]));
    const float amax = lanes_max<kLanes>(mask, a);
    const float max_finite = f == kE4M3 ? 448.0f : 57344.0f;
    float scale = 1.0f;
    if (amax > 0.0f) {
      const float q = __fdiv_rn(amax, max_finite);
      scale = q < 1.17549435e-38f ? 1.17549435e-38f : q;  // std::max(q, FLT_MIN)
    }
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fdiv_rn(x[i], scale);
    uint32_t lo, hi;
    if (f == kE4M3) {
      lo = cvt_e4m3x2(y[0], y[1]) | cvt_e4m3x2(y[2], y[3]) << 16;
      hi = cvt_e4m3x2(y[4], y[5]) | cvt_e4m3x2(y[6], y[7]) << 16;
    } else {
      lo = cvt_e5m2x2(y[0], y[1]) | cvt_e5m2x2(y[2], y[3]) << 16;
      hi = cvt_e5m2x2(y[4], y[5]) | cvt_e5m2x2(y[6], y[7]) << 16;
    }
    reinterpret_cast<uint2*>(payload + uint64_t{row} * kD)[lane] = make_uint2(lo, hi);
    if (lane == 0) reinterpret_cast<float*>(payload + code_bytes)[row] = scale;
    return 0;
  }
  float mn = x[0], mx = x[0];
  uint32_t imn = lane * 8, imx = lane * 8;
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    if (x[i] < mn) { mn = x[i]; imn = lane * 8 + i; }
    if (!(x[i] < mx)) { mx = x[i]; imx = lane * 8 + i; }
  }
  lanes_minmax<kLanes>(mask, mn, imn, mx, imx);
  const float range = __fsub_rn(mx, mn);
  if (!finite_f32(range)) return kErrNonFinite;
  const float scale = __fdiv_rn(range, 15.0f);
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t q = 0;
    if (scale > 0.0f) {
      const float rq = rintf(__fdiv_rn(__fsub_rn(x[i], mn), scale));
      q = static_cast<uint32_t>(rq < 0.0f ? 0.0f : (15.0f < rq ? 15.0f : rq));
    }
    word |= q << (4 * i);
  }
  reinterpret_cast<uint32_t*>(payload + uint64_t{row} * (kD / 2))[lane] = word;
  if (lane == 0) reinterpret_cast<float2*>(payload + code_bytes)[row] = make_float2(scale, mn);
  return 0;
}

}  // namespace dev
}  // namespace hlkv
