// Kernel (2): append-encode of FP16 tokens into heterogeneous KV blocks.
//
// Target k writes token d_targets[k].token of block d_targets[k].block_id,
// found through the device descriptor table.  The token is 2*H rows of D
// binary16 values ([K,V][head][dim]); each row is one group of the reference's
// quantize_reference (project2_quant/src/cpu_quant.cpp:97-170) on the binary32
// values of the inputs, stored at row (kv*T + token)*H + h of the block's
// layout (codes first, then the per-row parameters).
//
// A row is handled by D/8 lanes (16 for D = 128), 8 elements per lane from one
// 16-byte load; group statistics use shuffle reductions across those lanes:
//   FP8   amax -> scale = max(amax / max_finite, FLT_MIN) (1 when amax == 0),
//         code = RNE-saturating encode of x / scale (IEEE division; the encode is
//         the hardware cvt.rn.satfinite, equal to the reference's integer RNE);
//   INT4  (min, first index) and (max, last index), which is what
//         std::minmax_element returns and what makes the bias bits of +-0
//         ties exact; scale = (max - min) / 15, q = clamp(rint((x - min)/scale)).
#include <cuda_runtime.h>

#include <cstdint>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr int kThreads = 256;

struct DevPool {
  uint8_t* base;
  uint64_t slot_bytes;
  uint32_t num_slots;
};

struct Params {
  DevPool pool[4];
  uint64_t code_bytes[4];
  const uint4* table;
  const uint2* targets;
  const uint4* tokens;
  uint32_t* err;
  uint64_t rows_total;  // n * 2H
  uint32_t table_size, T, H, layout_id;
};

// Reductions over the kLanes lanes of one row.  `mask` names exactly those
// lanes, so rows of one warp may take different branches.
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

template <int kD>
__global__ void __launch_bounds__(kThreads) append_encode_kernel(const Params p) {
  constexpr int kLanes = kD / 8;
  constexpr int kRowsPerIter = kThreads / kLanes;
  const uint32_t lane = threadIdx.x % kLanes;
  const uint32_t mask =
      kLanes == 32 ? 0xFFFFFFFFu : ((1u << kLanes) - 1u) << ((threadIdx.x % 32) / kLanes * kLanes);
  const uint32_t two_h = 2 * p.H;
  for (uint64_t g = uint64_t{blockIdx.x} * kRowsPerIter + threadIdx.x / kLanes; g < p.rows_total;
       g += uint64_t{gridDim.x} * kRowsPerIter) {
    // Everything below is uniform over the lanes of row g.
    const uint64_t k = g / two_h;
    const uint32_t r = static_cast<uint32_t>(g % two_h);
    const uint32_t kv = r / p.H, h = r % p.H;

    // The token row does not depend on the descriptor: both loads go out together.
    const uint2 t = __ldg(p.targets + k);
    const uint4 raw = __ldcs(p.tokens + g * kLanes + lane);
    uint32_t bad = 0, f = 0, slot = 0;
    const uint32_t id = t.x, tok = t.y;
    if (id >= p.table_size) {
      bad = dev::kErrBlockIdRange;
    } else {
      const uint4 d = __ldg(p.table + id);
      f = d.y & 0xFu;
      const uint32_t mode = (d.y >> 4) & 3u, layout = (d.y >> 6) & 0xFu;
      slot = d.x;
      if (d.w != id) bad = dev::kErrDescMismatch;
      else if (f == dev::kInvalidFormat) bad = dev::kErrNotExecutable;
      else if (f > 3 || p.pool[f].base == nullptr || p.pool[f].num_slots == 0) bad = dev::kErrBadFormat;
      else if (layout != p.layout_id) bad = dev::kErrLayout;
      else if (f != dev::kFp16 && mode != 0) bad = dev::kErrScaleMode;
      else if (tok >= p.T) bad = dev::kErrTokenRange;
      else if (slot >= p.pool[f].num_slots) bad = dev::kErrSlotRange;
    }
    if (bad) {
      if (r == 0 && lane == 0) atomicOr(p.err, bad);  // once per target
      continue;
    }

    const uint32_t row = (kv * p.T + tok) * p.H + h;
    uint8_t* payload = p.pool[f].base + uint64_t{slot} * p.pool[f].slot_bytes;
    if (f == dev::kFp16) {  // encode_fp16 of an FP16 value: itself, NaN canonicalized
      reinterpret_cast<uint4*>(payload + uint64_t{row} * kD * 2)[lane] = dev::canon_f16x8(raw);
      continue;
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
    for (int i = 0; i < 8; ++i) nonfinite |= !dev::finite_f32(x[i]);
    if (lanes_any<kLanes>(mask, nonfinite)) {  // quantize_reference rejects the group
      if (lane == 0) atomicOr(p.err, dev::kErrNonFinite);
      continue;
    }

    if (f == dev::kE4M3 || f == dev::kE5M2) {
      float a = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(x[i]));
      const float amax = lanes_max<kLanes>(mask, a);
      const float max_finite = f == dev::kE4M3 ? 448.0f : 57344.0f;
      float scale = 1.0f;
      if (amax > 0.0f) {
        const float q = __fdiv_rn(amax, max_finite);
        scale = q < 1.17549435e-38f ? 1.17549435e-38f : q;  // std::max(q, FLT_MIN)
      }
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = __fdiv_rn(x[i], scale);
      uint32_t lo, hi;
      if (f == dev::kE4M3) {
        lo = dev::cvt_e4m3x2(y[0], y[1]) | dev::cvt_e4m3x2(y[2], y[3]) << 16;
        hi = dev::cvt_e4m3x2(y[4], y[5]) | dev::cvt_e4m3x2(y[6], y[7]) << 16;
      } else {
        lo = dev::cvt_e5m2x2(y[0], y[1]) | dev::cvt_e5m2x2(y[2], y[3]) << 16;
        hi = dev::cvt_e5m2x2(y[4], y[5]) | dev::cvt_e5m2x2(y[6], y[7]) << 16;
      }
      reinterpret_cast<uint2*>(payload + uint64_t{row} * kD)[lane] = make_uint2(lo, hi);
      if (lane == 0) reinterpret_cast<float*>(payload + p.code_bytes[f])[row] = scale;
    } else {
      float mn = x[0], mx = x[0];
      uint32_t imn = lane * 8, imx = lane * 8;
#pragma unroll
      for (int i = 1; i < 8; ++i) {
        if (x[i] < mn) { mn = x[i]; imn = lane * 8 + i; }
        if (!(x[i] < mx)) { mx = x[i]; imx = lane * 8 + i; }
      }
      lanes_minmax<kLanes>(mask, mn, imn, mx, imx);
      const float range = __fsub_rn(mx, mn);
      if (!dev::finite_f32(range)) {
        if (lane == 0) atomicOr(p.err, dev::kErrNonFinite);
        continue;
      }
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
      if (lane == 0) {
        reinterpret_cast<float2*>(payload + p.code_bytes[dev::kInt4])[row] = make_float2(scale, mn);
      }
    }
  }
}

}  // namespace
}  // namespace hlkv

extern "C" int hlkv_append_encode(const HlkvPools* pools, const HlkvLayout* layout,
                                  const HlkvExecDescriptor* d_table, uint32_t table_size,
                                  const HlkvAppendTarget* d_targets, uint32_t n,
                                  const uint16_t* d_tokens, uint32_t* d_err, hlkv_stream_t stream) {
  using namespace hlkv;
  if (pools == nullptr || !layout_ok(layout) || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n == 0) return HLKV_OK;
  if (d_targets == nullptr || d_tokens == nullptr || (table_size > 0 && d_table == nullptr) ||
      (reinterpret_cast<uintptr_t>(d_tokens) & 15u) != 0) {
    return HLKV_INVALID_ARGUMENT;
  }
  Params p{};
  const uint64_t rows = uint64_t{2} * layout->block_tokens * layout->kv_heads;
  const uint64_t elems = rows * layout->head_dim;
  for (int f = 0; f < 4; ++f) {
    const HlkvPool& q = pools->pool[f];
    p.code_bytes[f] = layout_code_bytes(f, elems);
    if (q.base == nullptr || q.num_slots == 0) continue;
    if ((reinterpret_cast<uintptr_t>(q.base) & 15u) != 0 || (q.slot_bytes & 15u) != 0 ||
        q.slot_bytes < hlkv_layout_slot_bytes(f, layout)) {
      return HLKV_INVALID_ARGUMENT;
    }
    p.pool[f] = DevPool{static_cast<uint8_t*>(q.base), q.slot_bytes, q.num_slots};
  }
  p.table = reinterpret_cast<const uint4*>(d_table);
  p.targets = reinterpret_cast<const uint2*>(d_targets);
  p.tokens = reinterpret_cast<const uint4*>(d_tokens);
  p.err = d_err;
  p.rows_total = uint64_t{n} * 2 * layout->kv_heads;
  p.table_size = table_size;
  p.T = layout->block_tokens;
  p.H = layout->kv_heads;
  p.layout_id = layout->layout_id;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int lanes = static_cast<int>(layout->head_dim / 8);
  const uint64_t rows_per_cta = kThreads / lanes;
  const uint64_t want = (p.rows_total + rows_per_cta - 1) / rows_per_cta;
  const uint64_t cap = uint64_t{static_cast<uint32_t>(sm_count())} * 16;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  switch (layout->head_dim) {
    case 64: append_encode_kernel<64><<<grid, kThreads, 0, s>>>(p); break;
    case 128: append_encode_kernel<128><<<grid, kThreads, 0, s>>>(p); break;
    default: append_encode_kernel<256><<<grid, kThreads, 0, s>>>(p); break;
  }
  return cuda_status(cudaGetLastError());
}
