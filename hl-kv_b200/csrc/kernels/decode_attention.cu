// Decode attention fused with the heterogeneous dequantization: one query token per
// sequence attends to the sequence's cached keys and values, read straight from the
// quantized blocks (FP16 / E4M3 / E5M2 / INT4 block by block) through the descriptor
// table, without materialising FP16 K/V in HBM.  This is the "fused dequant into
// attention" step that follows the gather in the reference's plan (ADR-0004); the
// reference has no kernel for it.
//
// Semantics: K and V are exactly the binary16 values kernel (1) would gather (the same
// decoder, dequantize_reference_to_fp16 per row), taken for the valid tokens of each
// block in sequence order.  For query head qh and its KV head h = qh / G:
//   s_t = softmax_scale * <q, k_t>,  p = softmax(s),  out = sum_t p_t v_t,
// in binary32 arithmetic (exp2 with the scale folded in), the result rounded to binary16.
// A sequence without valid tokens gives zeros.
//
// Structure: a CTA of 4 warps works on one (sequence, KV head) unit, or on one share of
// it (split mode: `splits` CTAs per unit), or on an equal range of all units' blocks laid
// end to end (balanced mode), piece by piece.  Per piece, the CTA resolves up to 128 blocks
// at a time (one thread per block: arena -> descriptor -> checks), and the warps take the
// blocks round-robin, prefetching their next block into L2.  Per 16-token tile a warp
// decodes the K and V rows of its head into shared memory (one out-of-line staging routine
// per format), computes S^T = K . Q^T with mma.sync m16n8k16 (FP16 in, FP32 accumulate),
// runs an online softmax in exp2, and adds V^T . P into its O^T accumulators.  The warps'
// (max, sum, outputs) merge in shared memory; the result goes to the output, or to a
// partial slot that a merge launch combines.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "codec.cuh"
#include "common.cuh"
#include "hlkv.h"

namespace hlkv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

struct DevPool {
  const uint8_t* base;
  uint64_t slot_bytes;
  uint32_t num_slots;
};

struct AttnParams {
  DevPool pool[4];
  uint64_t code_bytes[4];
  const uint4* table;
  const uint32_t* arena;
  const uint2* segs;
  const uint16_t* q;
  uint16_t* out;
  uint32_t* err;
  uint32_t table_size, arena_size, nseq;
  uint32_t T, H, layout_id, q_heads;
  float qscale;     // softmax_scale * log2(e)
  uint32_t splits;  // CTAs per (sequence, KV head), each over a contiguous share of the blocks
  float* ws;        // splits > 1 or balanced: kPart floats of partial results per slot
  // Balanced mode: CTA c takes blocks [c W / G, (c + 1) W / G) of all units laid end to end
  // (unit u = seq * H + h holds segs[seq].y blocks; W = prefix[nseq]), one piece per unit
  // that range meets, and writes piece (c, u) to slot c + u.
  uint32_t balanced;
  const uint64_t* prefix;  // [nseq + 1]: H * (blocks of the sequences before)
};

// The CTA of a balanced launch over W blocks and G CTAs that holds block x: CTA c takes
// [floor(c W / G), floor((c + 1) W / G)), so it is the largest c with floor(c W / G) <= x.
__device__ __forceinline__ uint32_t balanced_cta(uint64_t x, uint64_t W, uint64_t G) {
  return static_cast<uint32_t>(((x + 1) * G - 1) / W);
}

// Partial result of one CTA for its (sequence, KV head) and share of the blocks: the max
// (exp2 domain) and the sum per query column, then the unnormalised outputs.
template <int kD>
constexpr uint32_t kPart = 8 + 8 + 8 * kD;

// The checks of kernel (1) for block j of a sequence; returns the format (4 = skip).
__device__ __forceinline__ uint32_t resolve_block(const AttnParams& p, uint2 seg, uint32_t j,
                                                  const uint8_t** payload, uint32_t* vt, uint32_t* wide,
                                                  uint32_t* sref) {
  uint32_t bad = 0, f = 4;
  const uint64_t pos = uint64_t{seg.x} + j;
  if (pos >= p.arena_size) {
    bad = dev::kErrArenaRange;
  } else {
    const uint32_t id = __ldg(p.arena + pos);
    if (id >= p.table_size) {
      bad = dev::kErrBlockIdRange;
    } else {
      const uint4 d = __ldg(p.table + id);
      const uint32_t ff = d.y & 0xFu, mode = (d.y >> 4) & 3u, layout = (d.y >> 6) & 0xFu,
                     v = (d.y >> 10) & 0x3FFu;
      if (d.w != id) bad = dev::kErrDescMismatch;
      else if (ff == dev::kInvalidFormat) bad = dev::kErrNotExecutable;
      else if (ff > 3 || p.pool[ff].base == nullptr || p.pool[ff].num_slots == 0) bad = dev::kErrBadFormat;
      else if (layout != p.layout_id) bad = dev::kErrLayout;
      else if (ff != dev::kFp16 && (mode > 2 || (mode != 0 && !dev::block_params_ok(ff, mode, d.z))))
        bad = dev::kErrScaleMode;
      else if (v > p.T) bad = dev::kErrValidTokens;
      else if (d.x >= p.pool[ff].num_slots) bad = dev::kErrSlotRange;
      else {
        f = ff;
        *payload = p.pool[ff].base + uint64_t{d.x} * p.pool[ff].slot_bytes;
        *vt = v;
        *wide = ff != dev::kFp16 ? mode : 0u;  // 0: per-row parameters
        *sref = d.z;
      }
    }
  }
  if (bad) atomicOr(p.err, bad);
  return f;
}

// ---- tensor-core fragments (mma.sync m16n8k16, FP16 in, FP32 accumulate) ---------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem_row) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s));
}

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = 32 * kAttnWarps;

// Per warp: a 16-token tile of K and of V (binary16, rows padded by 8 halves so that
// ldmatrix rows fall in different banks) and P^T for the tile.
template <int kD>
struct WarpTiles {
  __half k[16][kD + 8];
  __half v[16][kD + 8];
  __half p[8][16 + 8];
};

// Decodes tokens [t0, t0 + 16) of head h's K rows (kv 0) or V rows (kv 1), in format kF,
// into the warp's tile; tokens >= vt become zeros.  Lane l handles 8-element chunks
// l, l+32, ...: 16-lane groups read whole rows, coalesced.  Every load of the tile is
// issued before the first conversion.
// kWide: the block's parameters are the block-wide pair wp for every row, instead of the
// per-row ones at params (a separate instance, so the per-row code has no test of it).
template <int kD, uint32_t kF, bool kWide>
__device__ __forceinline__ void stage_rows(const uint8_t* payload, const uint8_t* params, float2 wp,
                                           uint32_t kv, uint32_t t0, uint32_t vt, uint32_t T, uint32_t H,
                                           uint32_t h, __half (*tile)[kD + 8], uint32_t lane) {
  constexpr int kChunks = kD / 8;              // chunks per row
  constexpr int kPerLane = 16 * kChunks / 32;  // chunks per lane per tile
  uint4 raw[kPerLane];
  float2 prm[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const uint32_t c = i * 32 + lane, r = c / kChunks, e = (c % kChunks) * 8;
    const uint32_t t = t0 + r, row = (kv * T + t) * H + h;
    const uint64_t v = (uint64_t{row} * kD + e) >> 3;  // 8-element chunk index in the slot
    raw[i] = make_uint4(0u, 0u, 0u, 0u);
    prm[i] = make_float2(0.0f, 0.0f);
    if (t < vt) {
      if constexpr (kF == dev::kFp16) {
        raw[i] = dev::ld_stream(reinterpret_cast<const uint4*>(payload) + v);
      } else if constexpr (kF == dev::kInt4) {
        raw[i].x = dev::ld_stream(reinterpret_cast<const uint32_t*>(payload) + v);
        prm[i] = kWide ? wp : __ldg(reinterpret_cast<const float2*>(params) + row);
      } else {
        const uint2 w = dev::ld_stream(reinterpret_cast<const uint2*>(payload) + v);
        raw[i].x = w.x;
        raw[i].y = w.y;
        prm[i].x = kWide ? wp.x : __ldg(reinterpret_cast<const float*>(params) + row);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const uint32_t c = i * 32 + lane, r = c / kChunks, e = (c % kChunks) * 8;
    uint4 o;
    if constexpr (kF == dev::kFp16) {
      o = dev::canon_f16x8(raw[i]);
    } else if constexpr (kF == dev::kInt4) {
      o = dev::int4x8_to_f16(raw[i].x, prm[i].x, prm[i].y);
    } else {
      o = dev::fp8x8_to_f16<kF>(make_uint2(raw[i].x, raw[i].y), prm[i].x);
    }
    // tokens >= vt: zero codes with zero parameters decode to +0 in every format
    *reinterpret_cast<uint4*>(&tile[r][e]) = o;
  }
}

// Pulls the first tile of a block's K and V rows of head h (tokens 0..15), and their row
// parameters, into L2 while the warp still works on its current block: lane l covers the
// row of kv l / 16, token l % 16.  Only called for blocks that passed resolve_block, so
// every address lies inside the block's slot.
template <int kD>
__device__ __forceinline__ void prefetch_block(const uint8_t* payload, uint64_t code_bytes, uint32_t f,
                                               uint32_t vt, uint32_t T, uint32_t H, uint32_t h,
                                               uint32_t lane) {
  const uint32_t kv = lane >> 4, t = lane & 15;
  if (t >= vt) return;
  const uint32_t row = (kv * T + t) * H + h;
  const uint32_t row_bytes = f == dev::kFp16 ? kD * 2 : f == dev::kInt4 ? kD / 2 : kD;
  const uint8_t* a = payload + uint64_t{row} * row_bytes;
  for (uint32_t o = 0; o < row_bytes; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(a + o));
  if (f != dev::kFp16) {
    const uint8_t* q = payload + code_bytes + uint64_t{row} * (f == dev::kInt4 ? 8u : 4u);
    asm volatile("prefetch.global.L2 [%0];" ::"l"(q));
  }
}

template <int kD>
__device__ __noinline__ void stage_tiles(uint32_t f, const uint8_t* payload, const uint8_t* params,
                                         uint32_t t0, uint32_t vt, uint32_t T, uint32_t H, uint32_t h,
                                         WarpTiles<kD>& w, uint32_t lane) {
  // One copy of each format's staging code (out of line, K and V in a loop): the
  // instruction footprint stays small.
#pragma unroll 1
  for (uint32_t kv = 0; kv < 2; ++kv) {
    __half(*tile)[kD + 8] = kv == 0 ? w.k : w.v;
    switch (f) {
      case dev::kFp16: stage_rows<kD, dev::kFp16, false>(payload, params, make_float2(0.0f, 0.0f), kv, t0, vt, T, H, h, tile, lane); break;
      case dev::kE4M3: stage_rows<kD, dev::kE4M3, false>(payload, params, make_float2(0.0f, 0.0f), kv, t0, vt, T, H, h, tile, lane); break;
      case dev::kE5M2: stage_rows<kD, dev::kE5M2, false>(payload, params, make_float2(0.0f, 0.0f), kv, t0, vt, T, H, h, tile, lane); break;
      default: stage_rows<kD, dev::kInt4, false>(payload, params, make_float2(0.0f, 0.0f), kv, t0, vt, T, H, h, tile, lane); break;
    }
  }
}

// The same for a quantized block with block-wide parameters {scale, bias}.
template <int kD>
__device__ __noinline__ void stage_tiles_wide(uint32_t f, const uint8_t* payload, float2 prm, uint32_t t0,
                                              uint32_t vt, uint32_t T, uint32_t H, uint32_t h,
                                              WarpTiles<kD>& w, uint32_t lane) {
#pragma unroll 1
  for (uint32_t kv = 0; kv < 2; ++kv) {
    __half(*tile)[kD + 8] = kv == 0 ? w.k : w.v;
    switch (f) {
      case dev::kE4M3: stage_rows<kD, dev::kE4M3, true>(payload, nullptr, prm, kv, t0, vt, T, H, h, tile, lane); break;
      case dev::kE5M2: stage_rows<kD, dev::kE5M2, true>(payload, nullptr, prm, kv, t0, vt, T, H, h, tile, lane); break;
      default: stage_rows<kD, dev::kInt4, true>(payload, nullptr, prm, kv, t0, vt, T, H, h, tile, lane); break;
    }
  }
}

template <int kD, int kG>
__global__ void __launch_bounds__(kAttnThreads, 4) decode_attention_kernel(const AttnParams p) {
  constexpr int kSteps = kD / 16;  // k-steps of Q.K and m-tiles of V^T.P
  __shared__ __align__(16) unsigned char s_raw[kAttnWarps * sizeof(WarpTiles<kD>) >
                                                       kAttnWarps * (kD * 8 + 16) * 4
                                                   ? kAttnWarps * sizeof(WarpTiles<kD>)
                                                   : kAttnWarps * (kD * 8 + 16) * 4];
  __shared__ const uint8_t* s_payload[kAttnThreads];
  __shared__ uint32_t s_fv[kAttnThreads];  // format | valid_tokens << 8 | scale mode << 30 (format 4: skip)
  __shared__ uint32_t s_sref[kAttnThreads];  // scale_ref of blocks with block-wide parameters
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t grp = lane >> 2, quad = lane & 3;
  WarpTiles<kD>& w = reinterpret_cast<WarpTiles<kD>*>(s_raw)[warp];
  const uint32_t T = p.T, H = p.H;

  // The CTA's pieces: (seq, h, blocks [b0, b1)), each written to the output directly or
  // to a partial slot.  Split mode: one piece.  Balanced mode: the units its range meets.
  uint64_t x = 0, x_end = 0, W = 0;
  if (p.balanced) {
    W = p.prefix[p.nseq];
    x = uint64_t{blockIdx.x} * W / gridDim.x;
    x_end = (uint64_t{blockIdx.x} + 1) * W / gridDim.x;
  }
  for (bool first = true;; first = false) {
  uint32_t seq, h, b0, b1, slot;
  bool direct = false;
  if (!p.balanced) {
    if (!first) break;
    const uint32_t unit = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
    seq = unit / H;
    h = unit % H;
    const uint32_t n = p.segs[seq].y;
    b0 = static_cast<uint32_t>(uint64_t{n} * split / p.splits);
    b1 = static_cast<uint32_t>(uint64_t{n} * (split + 1) / p.splits);
    slot = blockIdx.x;
    direct = p.splits == 1;
  } else {
    if (x >= x_end) break;
    uint32_t lo = 0, hi = p.nseq;  // the sequence s with prefix[s] <= x < prefix[s + 1]
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (p.prefix[mid] <= x) lo = mid; else hi = mid;
    }
    seq = lo;
    const uint32_t n = p.segs[seq].y;  // > 0: x lies inside the sequence's range
    const uint64_t local = x - p.prefix[seq];
    h = static_cast<uint32_t>(local / n);
    b0 = static_cast<uint32_t>(local - uint64_t{h} * n);
    b1 = static_cast<uint32_t>(min(uint64_t{n}, b0 + (x_end - x)));
    x += b1 - b0;
    slot = blockIdx.x + seq * H + h;
  }

  // B fragments of Q^T (k = head_dim, n = query head of the group; columns >= kG are 0).
  uint32_t qb[kSteps][2];
  {
    const uint16_t* qrow = p.q + (uint64_t{seq} * p.q_heads + h * kG + grp) * kD;
#pragma unroll
    for (int k = 0; k < kSteps; ++k) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        qb[k][j] = grp < kG ? __ldg(reinterpret_cast<const uint32_t*>(qrow + k * 16 + j * 8 + quad * 2)) : 0u;
      }
    }
  }
  // O^T accumulators: m-tile mt covers head_dim rows [16 mt, 16 mt + 16); this lane holds
  // dims 16 mt + grp (+8) for query columns 2 quad, 2 quad + 1.
  float acc[kSteps][4];
#pragma unroll
  for (int mt = 0; mt < kSteps; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};

  const uint2 seg = p.segs[seq];
  // Blocks are resolved (arena -> descriptor -> checks) a batch at a time, one block per
  // thread, so the dependent lookups of a batch overlap instead of preceding each block's
  // payload reads.  Warp w then takes blocks w, w + 4, ... of the batch.
  for (uint32_t base = b0; base < b1; base += kAttnThreads) {
    const uint32_t nb = min(b1 - base, static_cast<uint32_t>(kAttnThreads));
    __syncthreads();  // the previous batch is no longer read
    if (threadIdx.x < nb) {
      const uint8_t* payload = nullptr;
      uint32_t vt = 0;
      uint32_t wide = 0, sref = 0;
      const uint32_t f = resolve_block(p, seg, base + threadIdx.x, &payload, &vt, &wide, &sref);
      s_payload[threadIdx.x] = payload;
      s_fv[threadIdx.x] = f | vt << 8 | wide << 30;
      s_sref[threadIdx.x] = sref;
    }
    __syncthreads();
  for (uint32_t i = warp; i < nb; i += kAttnWarps) {
    if (i + kAttnWarps < nb) {  // this warp's next block, into L2
      const uint32_t fn = s_fv[i + kAttnWarps] & 0xFFu, vn = (s_fv[i + kAttnWarps] >> 8) & 0x3FFu;
      if (fn <= 3 && vn > 0) prefetch_block<kD>(s_payload[i + kAttnWarps], p.code_bytes[fn], fn, vn, T, H, h, lane);
    }
    const uint32_t f = s_fv[i] & 0xFFu, vt = (s_fv[i] >> 8) & 0x3FFu;
    if (f > 3 || vt == 0) continue;
    const uint32_t wmode = s_fv[i] >> 30;  // 0: per-row parameters
    const uint8_t* payload = s_payload[i];
    const uint8_t* params = payload + p.code_bytes[f];
    for (uint32_t t0 = 0; t0 < vt; t0 += 16) {
      if (wmode != 0) stage_tiles_wide<kD>(f, payload, dev::block_params_value(wmode, s_sref[i]), t0, vt, T, H, h, w, lane);
      else stage_tiles<kD>(f, payload, params, t0, vt, T, H, h, w, lane);
      __syncwarp();
      // S^T (16 tokens x 8 query columns) = K . Q^T
      float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int k = 0; k < kSteps; ++k) {
        uint32_t a[4];
        ldsm_x4(a, &w.k[(lane & 7) + ((lane >> 3) & 1) * 8][k * 16 + (lane >> 4) * 8]);
        mma16816(s, a, qb[k][0], qb[k][1]);
      }
      // online softmax per query column; this lane: tokens grp, grp + 8; columns 2quad, 2quad+1
      const bool v0 = t0 + grp < vt, v1 = t0 + grp + 8 < vt;
      float pr[4];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float x0 = v0 ? s[c] * p.qscale : -INFINITY;
        const float x1 = v1 ? s[2 + c] * p.qscale : -INFINITY;
        float mx = fmaxf(x0, x1);
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
        const float mn = fmaxf(m[c], mx);  // finite: token t0 is valid
        const float alpha = exp2f(m[c] - mn);
        pr[c] = exp2f(x0 - mn);
        pr[2 + c] = exp2f(x1 - mn);
        float sum = pr[c] + pr[2 + c];
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
        l[c] = l[c] * alpha + sum;
        m[c] = mn;
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          acc[mt][c] *= alpha;
          acc[mt][2 + c] *= alpha;
        }
      }
      // P^T -> shared (query column major), read back as the B fragment of V^T . P
      w.p[quad * 2][grp] = __float2half_rn(pr[0]);
      w.p[quad * 2 + 1][grp] = __float2half_rn(pr[1]);
      w.p[quad * 2][grp + 8] = __float2half_rn(pr[2]);
      w.p[quad * 2 + 1][grp + 8] = __float2half_rn(pr[3]);
      __syncwarp();
      const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(&w.p[grp][quad * 2]);
      const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(&w.p[grp][quad * 2 + 8]);
      // O^T (head_dim x 8) += V^T . P
#pragma unroll
      for (int mt = 0; mt < kSteps; ++mt) {
        uint32_t a[4];
        ldsm_x4_trans(a, &w.v[(lane & 7) + (lane >> 4) * 8][mt * 16 + ((lane >> 3) & 1) * 8]);
        mma16816(acc[mt], a, pb0, pb1);
      }
      __syncwarp();  // the tiles are rewritten next
    }
  }
  }

  // ---- merge the warps: per query column the max, the sum and the head_dim outputs ----
  __syncthreads();  // the tiles are dead; their space holds the merge buffers
  float* s_o = reinterpret_cast<float*>(s_raw);                 // [warp][8][kD]
  float* s_ml = s_o + kAttnWarps * 8 * kD;                      // [warp][8][2]
#pragma unroll
  for (int mt = 0; mt < kSteps; ++mt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      s_o[(warp * 8 + quad * 2 + c) * kD + mt * 16 + grp] = acc[mt][c];
      s_o[(warp * 8 + quad * 2 + c) * kD + mt * 16 + grp + 8] = acc[mt][2 + c];
    }
  }
  if (grp == 0) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      s_ml[(warp * 8 + quad * 2 + c) * 2] = m[c];
      s_ml[(warp * 8 + quad * 2 + c) * 2 + 1] = l[c];
    }
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < kG * kD; i += kAttnThreads) {
    const uint32_t g = i / kD, e = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int wi = 0; wi < kAttnWarps; ++wi) M = fmaxf(M, s_ml[(wi * 8 + g) * 2]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int wi = 0; wi < kAttnWarps; ++wi) {
        const float mw = s_ml[(wi * 8 + g) * 2];
        const float a = mw == -INFINITY ? 0.0f : exp2f(mw - M);
        L = fmaf(s_ml[(wi * 8 + g) * 2 + 1], a, L);
        O = fmaf(s_o[(wi * 8 + g) * kD + e], a, O);
      }
    }
    if (direct) {
      const float r = L > 0.0f ? O / L : 0.0f;
      p.out[(uint64_t{seq} * p.q_heads + h * kG + g) * kD + e] = __half_as_ushort(__float2half_rn(r));
    } else {
      float* wp = p.ws + uint64_t{slot} * kPart<kD>;
      wp[16 + g * kD + e] = O;
      if (e == 0) {
        wp[g] = M;
        wp[8 + g] = L;
      }
    }
  }
  __syncthreads();  // the merge buffers are read before the next piece stages tiles
  }
}

// Merges the splits' partial results of one (sequence, query head) per CTA, kD threads.
template <int kD>
__global__ void __launch_bounds__(kD) decode_attention_merge(const float* __restrict__ ws, uint32_t splits,
                                                            uint32_t H, uint32_t group, uint32_t q_heads,
                                                            uint16_t* __restrict__ out) {
  const uint32_t seq = blockIdx.x / q_heads, qh = blockIdx.x % q_heads;
  const uint32_t h = qh / group, g = qh % group, e = threadIdx.x;
  const float* w = ws + uint64_t{seq * H + h} * splits * kPart<kD>;
  float M = -INFINITY;
  // Unrolled, so that each thread keeps several partials' loads in flight.
#pragma unroll 8
  for (uint32_t s = 0; s < splits; ++s) M = fmaxf(M, w[uint64_t{s} * kPart<kD> + g]);
  float L = 0.0f, O = 0.0f;
  if (M != -INFINITY) {
#pragma unroll 8
    for (uint32_t s = 0; s < splits; ++s) {
      const float* ps = w + uint64_t{s} * kPart<kD>;
      const float a = ps[g] == -INFINITY ? 0.0f : exp2f(ps[g] - M);
      L = fmaf(ps[8 + g], a, L);
      O = fmaf(ps[16 + g * kD + e], a, O);
    }
  }
  const float r = L > 0.0f ? O / L : 0.0f;
  out[(uint64_t{seq} * q_heads + qh) * kD + e] = __half_as_ushort(__float2half_rn(r));
}

// prefix[0] = 0, prefix[i + 1] = prefix[i] + H * segs[i].y: one CTA, a chunked block scan.
__global__ void __launch_bounds__(kAttnThreads) attention_prefix(const uint2* __restrict__ segs, uint32_t nseq,
                                                                 uint32_t H, uint64_t* __restrict__ prefix) {
  __shared__ uint64_t s_tot[kAttnWarps];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) prefix[0] = 0;
  uint64_t carry = 0;
  for (uint32_t base = 0; base < nseq; base += kAttnThreads) {
    const uint32_t i = base + threadIdx.x;
    uint64_t v = i < nseq ? uint64_t{segs[i].y} * H : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t n = __shfl_up_sync(0xFFFFFFFFu, v, o);
      if (lane >= static_cast<uint32_t>(o)) v += n;
    }
    if (lane == 31) s_tot[warp] = v;
    __syncthreads();
    uint64_t before = 0, total = 0;
#pragma unroll
    for (int wi = 0; wi < kAttnWarps; ++wi) {
      before += wi < static_cast<int>(warp) ? s_tot[wi] : 0;
      total += s_tot[wi];
    }
    if (i < nseq) prefix[i + 1] = carry + before + v;
    carry += total;
    __syncthreads();  // s_tot is rewritten by the next chunk
  }
}

// Merges a balanced launch's partials of one (sequence, query head) per CTA, kD threads:
// the slots c + u of the CTAs c whose ranges meet unit u.
template <int kD>
__global__ void __launch_bounds__(kD)
    decode_attention_merge_balanced(const float* __restrict__ ws, const uint64_t* __restrict__ prefix,
                                    const uint2* __restrict__ segs, uint32_t nseq, uint32_t H, uint32_t group,
                                    uint32_t q_heads, uint32_t ctas, uint16_t* __restrict__ out) {
  const uint32_t seq = blockIdx.x / q_heads, qh = blockIdx.x % q_heads;
  const uint32_t h = qh / group, g = qh % group, e = threadIdx.x;
  const uint32_t n = segs[seq].y;
  float M = -INFINITY, L = 0.0f, O = 0.0f;
  if (n > 0) {
    const uint64_t W = prefix[nseq], u = uint64_t{seq} * H + h;
    const uint64_t start = prefix[seq] + uint64_t{h} * n;
    const uint32_t c0 = balanced_cta(start, W, ctas), c1 = balanced_cta(start + n - 1, W, ctas);
    // With more CTAs than blocks some ranges are empty: those CTAs wrote no slot.  With
    // ctas <= W every range holds at least one block, and the test is skipped.
    const bool sparse = ctas > W;
    auto empty = [&](uint32_t c) { return sparse && uint64_t{c} * W / ctas == (uint64_t{c} + 1) * W / ctas; };
    // Unrolled, so that each thread keeps several partials' loads in flight.
#pragma unroll 8
    for (uint32_t c = c0; c <= c1; ++c) {
      if (!empty(c)) M = fmaxf(M, ws[(c + u) * kPart<kD> + g]);
    }
    if (M != -INFINITY) {
#pragma unroll 8
      for (uint32_t c = c0; c <= c1; ++c) {
        if (empty(c)) continue;
        const float* ps = ws + (c + u) * kPart<kD>;
        const float a = ps[g] == -INFINITY ? 0.0f : exp2f(ps[g] - M);
        L = fmaf(ps[8 + g], a, L);
        O = fmaf(ps[16 + g * kD + e], a, O);
      }
    }
  }
  const float r = L > 0.0f ? O / L : 0.0f;
  out[(uint64_t{seq} * q_heads + qh) * kD + e] = __half_as_ushort(__float2half_rn(r));
}

template <int kD>
cudaError_t launch_for_group(uint32_t group, const AttnParams& p, unsigned grid, cudaStream_t s) {
  switch (group) {
    case 1: decode_attention_kernel<kD, 1><<<grid, kAttnThreads, 0, s>>>(p); break;
    case 2: decode_attention_kernel<kD, 2><<<grid, kAttnThreads, 0, s>>>(p); break;
    case 4: decode_attention_kernel<kD, 4><<<grid, kAttnThreads, 0, s>>>(p); break;
    default: decode_attention_kernel<kD, 8><<<grid, kAttnThreads, 0, s>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace

int launch_attention(const HlkvPools* pools, const HlkvLayout* layout, const HlkvExecDescriptor* d_table,
                     uint32_t table_size, const uint32_t* d_arena, uint32_t arena_size,
                     const HlkvSegment* d_segs, uint32_t nseq, const uint16_t* d_q, uint32_t q_heads,
                     float softmax_scale, uint32_t splits, void* d_ws, size_t ws_bytes, uint16_t* d_out,
                     uint32_t* d_err, hlkv_stream_t stream, bool balanced) {
  if (pools == nullptr || !layout_ok(layout) || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (layout->head_dim != 64 && layout->head_dim != 128) return HLKV_INVALID_ARGUMENT;
  const uint32_t H = layout->kv_heads;
  if (q_heads == 0 || q_heads % H != 0) return HLKV_INVALID_ARGUMENT;
  const uint32_t group = q_heads / H;
  if (group != 1 && group != 2 && group != 4 && group != 8) return HLKV_INVALID_ARGUMENT;
  if (!(softmax_scale > 0.0f) || !std::isfinite(softmax_scale)) return HLKV_INVALID_ARGUMENT;
  if (splits == 0) return HLKV_INVALID_ARGUMENT;
  if (nseq == 0) return HLKV_OK;
  if (d_segs == nullptr || d_q == nullptr || d_out == nullptr ||
      (table_size > 0 && d_table == nullptr) || (arena_size > 0 && d_arena == nullptr)) {
    return HLKV_INVALID_ARGUMENT;
  }
  // Balanced mode: `splits` is the CTA count (at most 2^20, so slot and range arithmetic
  // stays in 64 bits).
  if (balanced ? splits > (1u << 20) || uint64_t{nseq} * H > 0x7FFFFFFFull
               : uint64_t{nseq} * H * splits > 0x7FFFFFFFull) {
    return HLKV_INVALID_ARGUMENT;
  }
  if (uint64_t{nseq} * q_heads > 0x7FFFFFFFull) return HLKV_INVALID_ARGUMENT;
  if (balanced || splits > 1) {
    if (d_ws == nullptr || (reinterpret_cast<uintptr_t>(d_ws) & 15u) != 0) return HLKV_INVALID_ARGUMENT;
    const size_t need = balanced ? hlkv_decode_attention_balanced_workspace_bytes(nseq, H, layout->head_dim, splits)
                                 : hlkv_decode_attention_workspace_bytes(nseq, H, layout->head_dim, splits);
    if (ws_bytes < need) return HLKV_BUFFER_TOO_SMALL;
  }
  AttnParams p{};
  const uint64_t elems = uint64_t{2} * layout->block_tokens * H * layout->head_dim;
  for (int f = 0; f < 4; ++f) {
    const HlkvPool& q = pools->pool[f];
    p.code_bytes[f] = layout_code_bytes(f, elems);
    if (q.base == nullptr || q.num_slots == 0) continue;
    if ((reinterpret_cast<uintptr_t>(q.base) & 15u) != 0 || (q.slot_bytes & 15u) != 0 ||
        q.slot_bytes < hlkv_layout_slot_bytes(f, layout)) {
      return HLKV_INVALID_ARGUMENT;
    }
    p.pool[f] = DevPool{static_cast<const uint8_t*>(q.base), q.slot_bytes, q.num_slots};
  }
  p.table = reinterpret_cast<const uint4*>(d_table);
  p.arena = d_arena;
  p.segs = reinterpret_cast<const uint2*>(d_segs);
  p.q = d_q;
  p.out = d_out;
  p.err = d_err;
  p.table_size = table_size;
  p.arena_size = arena_size;
  p.nseq = nseq;
  p.T = layout->block_tokens;
  p.H = H;
  p.layout_id = layout->layout_id;
  p.q_heads = q_heads;
  p.qscale = softmax_scale * kLog2e;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (balanced) {
    // workspace: prefix[nseq + 1] (16-byte aligned), then the partial slots
    const size_t prefix_bytes = (size_t{nseq} + 1) * sizeof(uint64_t);
    uint64_t* prefix = static_cast<uint64_t*>(d_ws);
    p.splits = 1;
    p.balanced = 1;
    p.prefix = prefix;
    p.ws = reinterpret_cast<float*>(static_cast<unsigned char*>(d_ws) + (prefix_bytes + 15) / 16 * 16);
    attention_prefix<<<1, kAttnThreads, 0, s>>>(p.segs, nseq, H, prefix);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
      e = layout->head_dim == 64 ? launch_for_group<64>(group, p, splits, s) : launch_for_group<128>(group, p, splits, s);
    }
    if (e == cudaSuccess) {
      if (layout->head_dim == 64) {
        decode_attention_merge_balanced<64><<<nseq * q_heads, 64, 0, s>>>(p.ws, prefix, p.segs, nseq, H, group,
                                                                           q_heads, splits, d_out);
      } else {
        decode_attention_merge_balanced<128><<<nseq * q_heads, 128, 0, s>>>(p.ws, prefix, p.segs, nseq, H, group,
                                                                             q_heads, splits, d_out);
      }
      e = cudaGetLastError();
    }
    return cuda_status(e);
  }
  p.splits = splits;
  p.ws = splits > 1 ? static_cast<float*>(d_ws) : nullptr;
  const unsigned grid = nseq * H * splits;
  cudaError_t e = layout->head_dim == 64 ? launch_for_group<64>(group, p, grid, s)
                                         : launch_for_group<128>(group, p, grid, s);
  if (e == cudaSuccess && splits > 1) {
    if (layout->head_dim == 64) {
      decode_attention_merge<64><<<nseq * q_heads, 64, 0, s>>>(p.ws, splits, H, group, q_heads, d_out);
    } else {
      decode_attention_merge<128><<<nseq * q_heads, 128, 0, s>>>(p.ws, splits, H, group, q_heads, d_out);
    }
    e = cudaGetLastError();
  }
  return cuda_status(e);
}

}  // namespace hlkv

extern "C" size_t hlkv_decode_attention_workspace_bytes(uint32_t nseq, uint32_t kv_heads, uint32_t head_dim,
                                                        uint32_t splits) {
  if (head_dim != 64 && head_dim != 128) return 0;
  const uint64_t part = head_dim == 64 ? hlkv::kPart<64> : hlkv::kPart<128>;
  return splits <= 1 ? 0 : static_cast<size_t>(uint64_t{nseq} * kv_heads * splits * part * sizeof(float));
}

extern "C" int hlkv_decode_attention(const HlkvPools* pools, const HlkvLayout* layout,
                                     const HlkvExecDescriptor* d_table, uint32_t table_size,
                                     const uint32_t* d_arena, uint32_t arena_size,
                                     const HlkvSegment* d_segs, uint32_t nseq, const uint16_t* d_q,
                                     uint32_t q_heads, float softmax_scale, uint16_t* d_out,
                                     uint32_t* d_err, hlkv_stream_t stream) {
  return hlkv::launch_attention(pools, layout, d_table, table_size, d_arena, arena_size, d_segs, nseq, d_q,
                                q_heads, softmax_scale, 1, nullptr, 0, d_out, d_err, stream, false);
}

extern "C" size_t hlkv_decode_attention_balanced_workspace_bytes(uint32_t nseq, uint32_t kv_heads,
                                                                 uint32_t head_dim, uint32_t ctas) {
  if (head_dim != 64 && head_dim != 128) return 0;
  const uint64_t part = head_dim == 64 ? hlkv::kPart<64> : hlkv::kPart<128>;
  const uint64_t prefix = ((uint64_t{nseq} + 1) * sizeof(uint64_t) + 15) / 16 * 16;
  return static_cast<size_t>(prefix + (uint64_t{ctas} + uint64_t{nseq} * kv_heads) * part * sizeof(float));
}

extern "C" int hlkv_decode_attention_balanced(const HlkvPools* pools, const HlkvLayout* layout,
                                              const HlkvExecDescriptor* d_table, uint32_t table_size,
                                              const uint32_t* d_arena, uint32_t arena_size,
                                              const HlkvSegment* d_segs, uint32_t nseq, const uint16_t* d_q,
                                              uint32_t q_heads, float softmax_scale, uint32_t ctas,
                                              void* d_workspace, size_t workspace_bytes, uint16_t* d_out,
                                              uint32_t* d_err, hlkv_stream_t stream) {
  return hlkv::launch_attention(pools, layout, d_table, table_size, d_arena, arena_size, d_segs, nseq, d_q,
                                q_heads, softmax_scale, ctas, d_workspace, workspace_bytes, d_out, d_err,
                                stream, true);
}

extern "C" int hlkv_decode_attention_split(const HlkvPools* pools, const HlkvLayout* layout,
                                           const HlkvExecDescriptor* d_table, uint32_t table_size,
                                           const uint32_t* d_arena, uint32_t arena_size,
                                           const HlkvSegment* d_segs, uint32_t nseq, const uint16_t* d_q,
                                           uint32_t q_heads, float softmax_scale, uint32_t splits,
                                           void* d_workspace, size_t workspace_bytes, uint16_t* d_out,
                                           uint32_t* d_err, hlkv_stream_t stream) {
  return hlkv::launch_attention(pools, layout, d_table, table_size, d_arena, arena_size, d_segs, nseq, d_q,
                                q_heads, softmax_scale, splits, d_workspace, workspace_bytes, d_out, d_err,
                                stream, false);
}

// ---- split attention without a caller workspace -------------------------------------------
//
// For callers that cannot allocate device memory when they call: hosts that bind this C ABI
// with no device allocator of their own (a cgo or plain C serving loop has no caching
// allocator to draw a workspace from), and engines that reserve all free HBM for their KV
// pools at start-up, so that a later cudaMalloc fails.  cudaMalloc and cudaFree are also not
// stream-ordered: a pair of them around every decode step would serialize the step against
// all other work in flight on the device.  These callers get the split partials in a fixed
// scratch array that is part of this library's device image instead.

namespace {

// HLKV_NOALLOC_SCRATCH_BYTES (16 MiB) of split partials per device: at head_dim 128 that is
// 4033 CTAs of partials, e.g. 16 sequences x 8 KV heads x 31 splits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[HLKV_NOALLOC_SCRATCH_BYTES];

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoallocDevices] = {};

// The scratch's address on the current device.  The first call on each device looks it up
// with cudaGetSymbolAddress, with that device current, and caches it; later calls only read
// the cache.
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hlkv::cuda_status(e);
  if (dev < 0 || dev >= kNoallocDevices) return HLKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return hlkv::cuda_status(e);
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 255u) != 0) {
      return hlkv::cuda_status(cudaErrorInvalidSymbol);
    }
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return HLKV_OK;
}

}  // namespace

// Nothing in the scratch has to start at zero, so nothing is cleared: every CTA of the split
// launch writes its whole partial (max, sum and outputs; -inf, 0 and 0 for an empty share)
// before the merge launch reads it.  All calls on one device share the one scratch, so calls
// that overlap on the GPU (on different streams, unordered) race on it.
extern "C" int hlkv_decode_attention_split_noalloc(const HlkvPools* pools, const HlkvLayout* layout,
                                                   const HlkvExecDescriptor* d_table, uint32_t table_size,
                                                   const uint32_t* d_arena, uint32_t arena_size,
                                                   const HlkvSegment* d_segs, uint32_t nseq,
                                                   const uint16_t* d_q, uint32_t q_heads,
                                                   float softmax_scale, uint32_t splits, uint16_t* d_out,
                                                   uint32_t* d_err, hlkv_stream_t stream) {
  if (layout != nullptr && splits > 1 && nseq > 0) {
    const uint64_t units = uint64_t{nseq} * layout->kv_heads;
    // Grids of 2^31 CTAs or more are rejected by launch_attention; below that the size fits.
    if (units <= 0x7FFFFFFFull && units * splits <= 0x7FFFFFFFull &&
        hlkv_decode_attention_workspace_bytes(nseq, layout->kv_heads, layout->head_dim, splits) >
            HLKV_NOALLOC_SCRATCH_BYTES) {
      return HLKV_BUFFER_TOO_SMALL;
    }
  }
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != HLKV_OK) return st;
  return hlkv::launch_attention(pools, layout, d_table, table_size, d_arena, arena_size, d_segs, nseq, d_q,
                                q_heads, softmax_scale, splits, scratch, HLKV_NOALLOC_SCRATCH_BYTES, d_out,
                                d_err, stream, false);
}
