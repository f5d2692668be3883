// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers around the reference's own CPU library (hl_quant's
// cpu_quant / cpu_dequant, hl_allocator), compiled from the reference's
// sources by oracle/build.py into oracle/_ref/libhlkv_ref.so.  Tests use it to
// pin the C restatement in oracle/hlkv_oracle.c and to generate the fixtures in
// tests/golden/; bench.py's reference arm times ref_gather_dequant as the
// reference's CPU path.  The product never loads it.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <thread>
#include <vector>

#include "hl_allocator/block_descriptor.hpp"
#include "hl_quant/cpu_dequant.hpp"
#include "hl_quant/cpu_quant.hpp"
#include "hl_quant/quant_types.hpp"

namespace q = hl::quant;
namespace a = hl::alloc;

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API void ref_encode_array(int format, const float* in, std::size_t n, std::uint16_t* out) {
  for (std::size_t i = 0; i < n; ++i) {
    out[i] = format == 0 ? q::encode_fp16(in[i])
             : format == 1 ? q::encode_fp8_e4m3(in[i])
                           : q::encode_fp8_e5m2(in[i]);
  }
}

REF_API void ref_decode_array(int format, const std::uint16_t* in, std::size_t n, float* out) {
  for (std::size_t i = 0; i < n; ++i) {
    out[i] = format == 0 ? q::decode_fp16(in[i])
             : format == 1 ? q::decode_fp8_e4m3(static_cast<std::uint8_t>(in[i]))
                           : q::decode_fp8_e5m2(static_cast<std::uint8_t>(in[i]));
  }
}

REF_API int ref_quantize(int format, const float* in, std::size_t n, std::size_t group,
                         float* params, std::size_t n_params, std::uint8_t* packed,
                         std::size_t packed_size) {
  return static_cast<int>(q::quantize_reference(
      static_cast<q::QuantFormat>(format), std::span<const float>(in, n), group,
      std::span<q::AffineParams>(reinterpret_cast<q::AffineParams*>(params), n_params),
      std::span<std::byte>(reinterpret_cast<std::byte*>(packed), packed_size)));
}

REF_API int ref_dequantize(int format, const std::uint8_t* packed, std::size_t packed_size,
                           std::size_t n, const float* params, std::size_t n_params,
                           std::size_t group, float* out, std::size_t out_size) {
  return static_cast<int>(q::dequantize_reference(
      static_cast<q::QuantFormat>(format),
      std::span<const std::byte>(reinterpret_cast<const std::byte*>(packed), packed_size), n,
      std::span<const q::AffineParams>(reinterpret_cast<const q::AffineParams*>(params), n_params),
      group, std::span<float>(out, out_size)));
}

REF_API int ref_dequantize_to_fp16(int format, const std::uint8_t* packed,
                                   std::size_t packed_size, std::size_t n, const float* params,
                                   std::size_t n_params, std::size_t group, std::uint16_t* out,
                                   std::size_t out_size) {
  return static_cast<int>(q::dequantize_reference_to_fp16(
      static_cast<q::QuantFormat>(format),
      std::span<const std::byte>(reinterpret_cast<const std::byte*>(packed), packed_size), n,
      std::span<const q::AffineParams>(reinterpret_cast<const q::AffineParams*>(params), n_params),
      group, std::span<std::uint16_t>(out, out_size)));
}

// The reference's CPU path for a heterogeneous gather: walk each sequence's
// segment through the arena to the descriptor (the device view defined in
// hetero_block_table.hpp:22-25), locate the payload at
// pool_base[format] + slot * slot_bytes (block_descriptor.hpp:144-145), and
// call dequantize_reference_to_fp16 once per row-sized parameter group of the
// payload layout shared with the oracle and the kernels.  Blocks are split
// over std::thread workers.  Returns the OR of the per-block check bits (same
// bits as the oracle and the kernels).
struct RefPool {
  const std::uint8_t* base;
  std::uint64_t slot_bytes;
  std::uint32_t num_slots;
  std::uint32_t pad;
};

namespace {

std::size_t packed(q::QuantFormat f, std::size_t n) { return q::packed_bytes(f, n); }

std::uint32_t resolve(const RefPool* pools, std::uint32_t T, std::uint32_t layout_id,
                      const a::BlockExecDescriptor* table, std::uint32_t table_size,
                      const std::uint32_t* arena, std::uint32_t arena_size, std::uint64_t pos,
                      const a::BlockExecDescriptor** out) {
  if (pos >= arena_size) return 1u << 3;
  const std::uint32_t id = arena[pos];
  if (id >= table_size) return 1u << 4;
  const a::BlockExecDescriptor& d = table[id];
  if (d.block_id != id) return 1u << 8;
  const auto f = static_cast<std::uint32_t>(d.format());
  if (d.format() == a::kInvalidFormat) return 1u << 0;
  if (f > 3 || pools[f].base == nullptr || pools[f].num_slots == 0) return 1u << 1;
  if (d.layout() != layout_id) return 1u << 6;
  if (f != 0 && d.scale_mode() != a::ScaleMode::kNone) return 1u << 7;
  if (d.valid_tokens() > T) return 1u << 5;
  if (d.slot >= pools[f].num_slots) return 1u << 2;
  *out = &d;
  return 0;
}

}  // namespace

REF_API std::uint32_t ref_gather_dequant(const RefPool* pools, std::uint32_t T, std::uint32_t H,
                                         std::uint32_t D, std::uint32_t layout_id,
                                         const std::uint32_t* table_words,
                                         std::uint32_t table_size, const std::uint32_t* arena,
                                         std::uint32_t arena_size, const std::uint32_t* segs,
                                         std::uint32_t nseq, const std::uint64_t* out_offsets,
                                         std::uint16_t* out, const std::uint64_t* prefix,
                                         int threads) {
  if (nseq == 0) return 0;
  const auto* table = reinterpret_cast<const a::BlockExecDescriptor*>(table_words);
  const std::uint64_t total = prefix[nseq];
  const std::size_t rows = std::size_t{2} * T * H, rows_per_kv = std::size_t{T} * H;
  const std::size_t belems = rows * D;
  if (threads < 1) threads = 1;
  std::vector<std::uint32_t> errs(static_cast<std::size_t>(threads), 0);
  auto work = [&](int t) {
    const std::uint64_t b = total * static_cast<std::uint64_t>(t) / threads;
    const std::uint64_t e = total * static_cast<std::uint64_t>(t + 1) / threads;
    std::uint32_t seq = 0;
    std::uint32_t err = 0;
    for (std::uint64_t w = b; w < e; ++w) {
      while (seq + 1 < nseq && prefix[seq + 1] <= w) ++seq;
      const std::uint64_t j = w - prefix[seq];
      const std::uint64_t base = out_offsets ? out_offsets[seq] : prefix[seq] * belems;
      if (base % 8 != 0) { err |= 1u << 12; continue; }
      const a::BlockExecDescriptor* d = nullptr;
      if (const std::uint32_t bad = resolve(pools, T, layout_id, table, table_size, arena,
                                            arena_size, std::uint64_t{segs[2 * seq]} + j, &d)) {
        err |= bad;
        continue;
      }
      const auto fi = static_cast<std::uint32_t>(d->format());
      const auto f = static_cast<q::QuantFormat>(fi);
      const std::uint8_t* payload = pools[fi].base + std::size_t{d->slot} * pools[fi].slot_bytes;
      const std::size_t code_bytes = packed(f, belems);
      std::uint16_t* o = out + base + j * belems;
      for (std::size_t r = 0; r < rows; ++r) {
        const std::size_t r_in_kv = r < rows_per_kv ? r : r - rows_per_kv;
        if (r_in_kv >= std::size_t{d->valid_tokens()} * H) {
          std::memset(o + r * D, 0, 2 * D);
          continue;
        }
        const auto* codes = reinterpret_cast<const std::byte*>(payload + packed(f, r * D));
        q::AffineParams p{0.0f, 0.0f};
        std::size_t np = 0, group = 0;
        if (fi == 1 || fi == 2) {
          std::memcpy(&p.scale, payload + code_bytes + 4 * r, 4);
          np = 1;
          group = D;
        } else if (fi == 3) {
          std::memcpy(&p, payload + code_bytes + 8 * r, 8);
          np = 1;
          group = D;
        }
        (void)q::dequantize_reference_to_fp16(f, std::span<const std::byte>(codes, packed(f, D)),
                                              D, std::span<const q::AffineParams>(&p, np), group,
                                              std::span<std::uint16_t>(o + r * D, D));
      }
    }
    errs[static_cast<std::size_t>(t)] = err;
  };
  if (threads == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
    for (std::thread& th : pool) th.join();
  }
  std::uint32_t err = 0;
  for (const std::uint32_t e : errs) err |= e;
  return err;
}
