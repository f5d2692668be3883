// Flat (contiguous) device codecs.
//
//  * hlkv_dequantize_fp8_to_fp16: drop-in for the reference's
//    hl::quant::cuda::dequantize_fp8_to_fp16 (dequant_kernel.cu:171-191):
//    any alignment, any group size; an 8-element path (8-byte load, 16-byte
//    store) when the pointers are aligned and every 8-element chunk lies in one
//    group, a per-element path for the rest.
//  * hlkv_dequantize_to_fp16 / hlkv_quantize: device counterparts of
//    dequantize_reference_to_fp16 / quantize_reference for every format.
//    Host-side argument rules are the reference's; value checks (finite
//    parameters / inputs, INT4 range) happen per group on the device.
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr int kThreads = 256;
constexpr uint64_t kMaxElements = ~uint64_t{0} / 2;  // quant_types.hpp:105

uint64_t packed_bytes(uint32_t f, uint64_t n) {
  return f == dev::kFp16 ? 2 * n : (f == dev::kInt4 ? n / 2 + (n & 1) : n);
}

unsigned grid_for(uint64_t work, uint64_t per_cta) {
  const uint64_t want = (work + per_cta - 1) / per_cta;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 16;
  return static_cast<unsigned>(want == 0 ? 1 : (want < cap ? want : cap));
}

// Parameters usable for decoding: finite, and bias 0 unless INT4 (cpu_dequant.cpp:77-90).
__device__ __forceinline__ bool params_ok(uint32_t f, float2 sb) {
  return dev::finite_f32(sb.x) && dev::finite_f32(sb.y) && (f == dev::kInt4 || sb.y == 0.0f);
}

// ---- decode ---------------------------------------------------------------------------------

// 8 elements per thread; requires aligned pointers and chunks inside one group
// (cpg = 8-element chunks per group, or all-ones for a single group).
// kVecUnroll chunks per thread per pass: every load of a pass is issued before the
// first conversion, so each thread keeps kVecUnroll code loads (and their scale loads)
// in flight; a short array then occupies the whole GPU in a single pass.
constexpr uint32_t kVecUnroll = 8;  // at 2^28 values: 0.889 of the copy peak, 4 chunks: 0.849

template <uint32_t kF, typename Index, bool kCheck>
__global__ void __launch_bounds__(kThreads)
    dequant_vec8(const uint8_t* __restrict__ in, const float2* __restrict__ params, Index cpg,
                 uint64_t nchunks, uint4* __restrict__ out, uint32_t* err) {
  constexpr uint64_t kPass = uint64_t{kThreads} * kVecUnroll;
  uint32_t bad = 0;
  for (uint64_t base = uint64_t{blockIdx.x} * kPass; base < nchunks; base += uint64_t{gridDim.x} * kPass) {
    uint4 raw[kVecUnroll];
    float2 sb[kVecUnroll];
#pragma unroll
    for (uint32_t j = 0; j < kVecUnroll; ++j) {
      const uint64_t c = base + j * kThreads + threadIdx.x;
      raw[j] = make_uint4(0u, 0u, 0u, 0u);
      sb[j] = make_float2(0.0f, 0.0f);
      if (c < nchunks) {
        if constexpr (kF == dev::kFp16) {
          raw[j] = dev::ld_stream(reinterpret_cast<const uint4*>(in) + c);
        } else if constexpr (kF == dev::kInt4) {
          raw[j].x = dev::ld_stream(reinterpret_cast<const uint32_t*>(in) + c);
          sb[j] = __ldg(params + static_cast<Index>(c) / cpg);
        } else {
          const uint2 v = dev::ld_stream(reinterpret_cast<const uint2*>(in) + c);
          raw[j].x = v.x;
          raw[j].y = v.y;
          sb[j] = __ldg(params + static_cast<Index>(c) / cpg);
        }
      }
    }
#pragma unroll
    for (uint32_t j = 0; j < kVecUnroll; ++j) {
      const uint64_t c = base + j * kThreads + threadIdx.x;
      if (c >= nchunks) continue;
      if constexpr (kF == dev::kFp16) {
        out[c] = dev::canon_f16x8(raw[j]);
      } else {
        if (kCheck && !params_ok(kF, sb[j])) {
          bad = dev::kErrNonFinite;
          continue;
        }
        if constexpr (kF == dev::kInt4) {
          out[c] = dev::int4x8_to_f16(raw[j].x, sb[j].x, sb[j].y);
        } else {
          out[c] = dev::fp8x8_to_f16<kF>(make_uint2(raw[j].x, raw[j].y), sb[j].x);
        }
      }
    }
  }
  if (bad) atomicOr(err, bad);
}

template <uint32_t kF, typename Index, bool kCheck>
__global__ void __launch_bounds__(kThreads)
    dequant_scalar(const uint8_t* __restrict__ in, const float2* __restrict__ params, Index group,
                   uint64_t begin, uint64_t end, uint16_t* __restrict__ out, uint32_t* err) {
  const uint64_t stride = uint64_t{gridDim.x} * kThreads;
  uint32_t bad = 0;
  for (uint64_t i = begin + uint64_t{blockIdx.x} * kThreads + threadIdx.x; i < end; i += stride) {
    if constexpr (kF == dev::kFp16) {
      const uint32_t h = uint32_t{in[2 * i]} | (uint32_t{in[2 * i + 1]} << 8);
      out[i] = static_cast<uint16_t>(dev::canon_f16x2(h) & 0xFFFFu);
    } else {
      const float2 sb = __ldg(params + static_cast<Index>(i) / group);
      if (kCheck && !params_ok(kF, sb)) { bad = dev::kErrNonFinite; continue; }
      if constexpr (kF == dev::kInt4) {
        out[i] = static_cast<uint16_t>(dev::int4_to_f16((in[i / 2] >> (4 * (i & 1))) & 0xFu, sb.x, sb.y));
      } else {
        out[i] = static_cast<uint16_t>(dev::fp8_to_f16<kF>(in[i], sb.x));
      }
    }
  }
  if (bad) atomicOr(err, bad);
}

template <uint32_t kF, typename Index, bool kCheck>
void launch_dequant(const uint8_t* in, uint64_t n, const float2* params, uint64_t group,
                    uint16_t* out, uint32_t* err, cudaStream_t s) {
  const bool single = kF == dev::kFp16 || group >= n;
  const uint64_t in_align = kF == dev::kFp16 ? 16 : (kF == dev::kInt4 ? 4 : 8);
  const bool aligned = (reinterpret_cast<uintptr_t>(in) % in_align) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) % 16) == 0;
  uint64_t done = 0;
  if (aligned && n >= 8 && (single || group % 8 == 0)) {
    const uint64_t nchunks = n / 8;
    const Index cpg = single ? static_cast<Index>(~Index{0}) : static_cast<Index>(group / 8);
    dequant_vec8<kF, Index, kCheck><<<grid_for(nchunks, uint64_t{kThreads} * kVecUnroll), kThreads, 0, s>>>(
        in, params, cpg, nchunks, reinterpret_cast<uint4*>(out), err);
    done = nchunks * 8;
  }
  if (done < n) {
    const Index g = single ? static_cast<Index>(~Index{0}) : static_cast<Index>(group);
    dequant_scalar<kF, Index, kCheck><<<grid_for(n - done, kThreads), kThreads, 0, s>>>(
        in, params, g, done, n, out, err);
  }
}

template <bool kCheck>
int dispatch_dequant(uint32_t f, const uint8_t* in, uint64_t n, const float2* params, uint64_t group,
                     uint16_t* out, uint32_t* err, cudaStream_t s) {
  const bool small = n <= 0xFFFFFFFFull;
#define HLKV_DQ(F)                                                                  \
  (small ? launch_dequant<F, uint32_t, kCheck>(in, n, params, group, out, err, s)   \
         : launch_dequant<F, uint64_t, kCheck>(in, n, params, group, out, err, s))
  switch (f) {
    case dev::kFp16: HLKV_DQ(dev::kFp16); break;
    case dev::kE4M3: HLKV_DQ(dev::kE4M3); break;
    case dev::kE5M2: HLKV_DQ(dev::kE5M2); break;
    default: HLKV_DQ(dev::kInt4); break;
  }
#undef HLKV_DQ
  return cuda_status(cudaGetLastError());
}

// ---- encode ---------------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads)
    quantize_f16(const float* __restrict__ in, uint64_t n, uint16_t* __restrict__ out) {
  const uint64_t stride = uint64_t{gridDim.x} * kThreads;
  for (uint64_t i = uint64_t{blockIdx.x} * kThreads + threadIdx.x; i < n; i += stride) {
    out[i] = static_cast<uint16_t>(dev::encode_f16(in[i]));
  }
}

// One warp per group.  Element i of a group goes to lane (i - begin) % 32, so
// per-lane scans run in index order; ties break on the element index.
template <uint32_t kF>
__global__ void __launch_bounds__(kThreads)
    quantize_groups(const float* __restrict__ in, uint64_t n, uint64_t group, uint64_t groups,
                    float2* __restrict__ params, uint8_t* __restrict__ packed, uint32_t* err) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = uint64_t{gridDim.x} * (kThreads / 32);
  for (uint64_t gi = (uint64_t{blockIdx.x} * kThreads + threadIdx.x) / 32; gi < groups; gi += warps) {
    const uint64_t b = gi * group, e = b + group < n ? b + group : n;
    bool nonfinite = false;
    float amax = 0.0f, mn = __int_as_float(0x7F800000), mx = __int_as_float(0xFF800000);
    uint64_t imn = ~uint64_t{0}, imx = 0;
    for (uint64_t i = b + lane; i < e; i += 32) {
      const float x = in[i];
      nonfinite |= !dev::finite_f32(x);
      amax = fmaxf(amax, fabsf(x));
      if (x < mn || imn == ~uint64_t{0}) { mn = x; imn = i; }
      if (!(x < mx)) { mx = x; imx = i; }
    }
    if (__any_sync(0xFFFFFFFFu, nonfinite)) {
      if (lane == 0) atomicOr(err, dev::kErrNonFinite);
      continue;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      const float omn = __shfl_xor_sync(0xFFFFFFFFu, mn, o);
      const uint64_t oimn = __shfl_xor_sync(0xFFFFFFFFu, imn, o);
      const float omx = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
      const uint64_t oimx = __shfl_xor_sync(0xFFFFFFFFu, imx, o);
      if (omn < mn || (omn == mn && oimn < imn)) { mn = omn; imn = oimn; }
      if (omx > mx || (omx == mx && oimx > imx)) { mx = omx; imx = oimx; }
    }
    float scale, bias = 0.0f;
    if constexpr (kF == dev::kInt4) {
      const float range = __fsub_rn(mx, mn);
      if (!dev::finite_f32(range)) {
        if (lane == 0) atomicOr(err, dev::kErrNonFinite);
        continue;
      }
      scale = __fdiv_rn(range, 15.0f);
      bias = mn;
      for (uint64_t u = b / 2 + lane; 2 * u < e; u += 32) {
        uint32_t byte = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint64_t i = 2 * u + k;
          uint32_t q = 0;
          if (i < e && scale > 0.0f) {
            const float rq = rintf(__fdiv_rn(__fsub_rn(in[i], mn), scale));
            q = static_cast<uint32_t>(rq < 0.0f ? 0.0f : (15.0f < rq ? 15.0f : rq));
          }
          byte |= q << (4 * k);
        }
        packed[u] = static_cast<uint8_t>(byte);
      }
    } else {
      scale = 1.0f;
      if (amax > 0.0f) {
        const float q = __fdiv_rn(amax, kF == dev::kE4M3 ? 448.0f : 57344.0f);
        scale = q < 1.17549435e-38f ? 1.17549435e-38f : q;
      }
      for (uint64_t i = b + lane; i < e; i += 32) {
        const float y = __fdiv_rn(in[i], scale);
        packed[i] = static_cast<uint8_t>(kF == dev::kE4M3 ? dev::encode_e4m3(y) : dev::encode_e5m2(y));
      }
    }
    if (lane == 0) params[gi] = make_float2(scale, bias);
  }
}

bool group_ok(uint32_t f, uint64_t g) {
  if (f == dev::kFp16) return g == 0;
  return g > 0 && (f != dev::kInt4 || g % 2 == 0);
}

uint64_t num_groups(uint64_t n, uint64_t g) { return g == 0 ? 0 : n / g + (n % g != 0); }

}  // namespace
}  // namespace hlkv

extern "C" int hlkv_dequantize_fp8_to_fp16(int format, const void* d_in, size_t n,
                                           const float* d_params, size_t group_size,
                                           uint16_t* d_out, hlkv_stream_t stream) {
  using namespace hlkv;
  if (format != HLKV_FP8_E4M3 && format != HLKV_FP8_E5M2) return HLKV_UNSUPPORTED_FORMAT;
  if (group_size == 0 || n > kMaxElements) return HLKV_INVALID_ARGUMENT;
  if (n == 0) return HLKV_OK;
  if (d_in == nullptr || d_params == nullptr || d_out == nullptr) return HLKV_INVALID_ARGUMENT;
  return dispatch_dequant<false>(static_cast<uint32_t>(format), static_cast<const uint8_t*>(d_in), n,
                                 reinterpret_cast<const float2*>(d_params), group_size, d_out,
                                 nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int hlkv_dequantize_to_fp16(int format, const void* d_packed, size_t packed_size,
                                       size_t n, const float* d_params, size_t n_params,
                                       size_t group_size, uint16_t* d_out, size_t out_size,
                                       uint32_t* d_err, hlkv_stream_t stream) {
  using namespace hlkv;
  if (format < 0 || format > 3) return HLKV_UNSUPPORTED_FORMAT;
  const uint32_t f = static_cast<uint32_t>(format);
  if (n > kMaxElements || !group_ok(f, group_size) || n_params != num_groups(n, group_size)) {
    return HLKV_INVALID_ARGUMENT;
  }
  if (packed_size < packed_bytes(f, n) || out_size < n) return HLKV_BUFFER_TOO_SMALL;
  if (n == 0) return HLKV_OK;
  if (d_packed == nullptr || d_out == nullptr || d_err == nullptr ||
      (f != dev::kFp16 && d_params == nullptr)) {
    return HLKV_INVALID_ARGUMENT;
  }
  return dispatch_dequant<true>(f, static_cast<const uint8_t*>(d_packed), n,
                                reinterpret_cast<const float2*>(d_params), group_size, d_out, d_err,
                                reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int hlkv_quantize(int format, const float* d_in, size_t n, size_t group_size,
                             float* d_params, size_t n_params, void* d_packed, size_t packed_size,
                             uint32_t* d_err, hlkv_stream_t stream) {
  using namespace hlkv;
  if (format < 0 || format > 3) return HLKV_UNSUPPORTED_FORMAT;
  const uint32_t f = static_cast<uint32_t>(format);
  if (n > kMaxElements || !group_ok(f, group_size) || n_params != num_groups(n, group_size)) {
    return HLKV_INVALID_ARGUMENT;
  }
  if (packed_size < packed_bytes(f, n)) return HLKV_BUFFER_TOO_SMALL;
  if (n == 0) return HLKV_OK;
  if (d_in == nullptr || d_packed == nullptr || d_err == nullptr ||
      (f != dev::kFp16 && d_params == nullptr)) {
    return HLKV_INVALID_ARGUMENT;
  }
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* packed = static_cast<uint8_t*>(d_packed);
  auto* params = reinterpret_cast<float2*>(d_params);
  const uint64_t groups = num_groups(n, group_size);
  const unsigned grid = grid_for(groups, kThreads / 32);
  switch (f) {
    case dev::kFp16:
      if ((reinterpret_cast<uintptr_t>(d_packed) & 1u) != 0) return HLKV_INVALID_ARGUMENT;
      quantize_f16<<<grid_for(n, kThreads), kThreads, 0, s>>>(d_in, n, static_cast<uint16_t*>(d_packed));
      break;
    case dev::kE4M3:
      quantize_groups<dev::kE4M3><<<grid, kThreads, 0, s>>>(d_in, n, group_size, groups, params, packed, d_err);
      break;
    case dev::kE5M2:
      quantize_groups<dev::kE5M2><<<grid, kThreads, 0, s>>>(d_in, n, group_size, groups, params, packed, d_err);
      break;
    default:
      quantize_groups<dev::kInt4><<<grid, kThreads, 0, s>>>(d_in, n, group_size, groups, params, packed, d_err);
      break;
  }
  return cuda_status(cudaGetLastError());
}
