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
  if (f != 0 && d.scale_mode() == a::ScaleMode::kExternal) return 1u << 7;
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
      const bool block_wide = fi != 0 && (d->scale_mode() == a::ScaleMode::kInlineF32 ||
                                          d->scale_mode() == a::ScaleMode::kInlineF16Pair);
      if (block_wide) {
        // One group for the whole block: parameters the reference's dequantizer rejects
        // (non-finite, or an FP8 bias) reject the block, output untouched.
        q::AffineParams bp{0.0f, 0.0f};
        if (d->scale_mode() == a::ScaleMode::kInlineF32) {
          bp.scale = d->inline_scale_f32();
        } else {
          bp.scale = q::decode_fp16(static_cast<std::uint16_t>(d->scale_ref & 0xFFFFu));
          bp.bias = q::decode_fp16(static_cast<std::uint16_t>(d->scale_ref >> 16));
        }
        std::vector<std::uint16_t> probe(D);
        if (q::dequantize_reference_to_fp16(f, std::span<const std::byte>(reinterpret_cast<const std::byte*>(payload), packed(f, D)),
                                            D, std::span<const q::AffineParams>(&bp, 1), D,
                                            std::span<std::uint16_t>(probe)) != q::QuantStatus::kOk) {
          err |= 1u << 7;
          continue;
        }
      }
      for (std::size_t r = 0; r < rows; ++r) {
        const std::size_t r_in_kv = r < rows_per_kv ? r : r - rows_per_kv;
        if (r_in_kv >= std::size_t{d->valid_tokens()} * H) {
          std::memset(o + r * D, 0, 2 * D);
          continue;
        }
        const auto* codes = reinterpret_cast<const std::byte*>(payload + packed(f, r * D));
        q::AffineParams p{0.0f, 0.0f};
        std::size_t np = 0, group = 0;
        if (block_wide && d->scale_mode() == a::ScaleMode::kInlineF32) {
          // one binary32 scale for the whole block: the reference's own accessor
          p.scale = d->inline_scale_f32();
          np = 1;
          group = D;
        } else if (block_wide) {
          // binary16 scale in bits 0..15, bias in 16..31 (hl_allocator_abi.md, scale modes)
          p.scale = q::decode_fp16(static_cast<std::uint16_t>(d->scale_ref & 0xFFFFu));
          p.bias = q::decode_fp16(static_cast<std::uint16_t>(d->scale_ref >> 16));
          np = 1;
          group = D;
        } else if (fi == 1 || fi == 2) {
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

// ---- a CPU-built workload for the reference arm of bench.py --------------------------------
// Built entirely with the reference's own code: its HeteroBlockTable (scrambled
// free lists, sequences, collect_delta/batch_segments for the device view) and
// its quantize_reference (one group per row) on seeded N(0,1) FP16 values.
#include <algorithm>
#include <cmath>
#include <memory>

#include "hl_allocator/hetero_block_table.hpp"

namespace {

struct SplitMix {
  std::uint64_t s;
  std::uint64_t next() {
    std::uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float normal() {
    const double u1 = 1.0 - static_cast<double>(next() >> 11) * 0x1.0p-53;
    const double u2 = static_cast<double>(next() >> 11) * 0x1.0p-53;
    return static_cast<float>(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
  }
};

struct RefWorkload {
  std::uint32_t T, H, D, layout_id;
  std::vector<std::uint32_t> table_words, arena, segs;
  RefPool pools[15]{};
  std::vector<std::vector<std::uint8_t>> pool_bytes = std::vector<std::vector<std::uint8_t>>(4);
  std::uint64_t info[16]{};  // table_size, arena_size, nseq, total_blocks, slots[4], slot_bytes[4]
};

}  // namespace

REF_API void* ref_workload_build(const std::uint8_t* fmts, const std::uint32_t* lens,
                                 std::uint32_t nseq, std::uint32_t T, std::uint32_t H,
                                 std::uint32_t D, std::uint32_t layout_id, std::uint64_t seed,
                                 std::uint32_t outlier_channels, float outlier_scale, int threads) {
  auto w = std::make_unique<RefWorkload>();
  w->T = T; w->H = H; w->D = D; w->layout_id = layout_id;
  const std::size_t rows = std::size_t{2} * T * H, elems = rows * D;
  std::uint32_t counts[4] = {0, 0, 0, 0};
  std::size_t total = 0;
  for (std::uint32_t i = 0; i < nseq; ++i) {
    for (std::uint32_t j = 0; j < lens[i]; ++j) counts[fmts[total + j] & 3]++;
    total += lens[i];
  }
  std::size_t slot_bytes[4];
  for (int f = 0; f < 4; ++f) {
    const auto qf = static_cast<q::QuantFormat>(f);
    const std::size_t params = f == 0 ? 0 : (f == 3 ? 8 * rows : 4 * rows);
    slot_bytes[f] = (q::packed_bytes(qf, elems) + params + 15) / 16 * 16;
  }
  a::TableConfig cfg;
  cfg.max_blocks = static_cast<std::uint32_t>(std::max<std::size_t>(total, 1));
  cfg.block_tokens = T;
  for (int f = 0; f < 4; ++f) {
    if (counts[f] > 0) {
      cfg.pools.push_back({a::FormatId{static_cast<std::uint8_t>(f)},
                           static_cast<std::uint32_t>(slot_bytes[f]), counts[f]});
    }
  }
  if (cfg.pools.empty()) cfg.pools.push_back({a::FormatId{0}, static_cast<std::uint32_t>(slot_bytes[0]), 1});
  a::HeteroBlockTable table(cfg);
  SplitMix rng{seed};
  {  // scramble: allocate every slot, release in a seeded order
    std::vector<a::BlockHandle> hs;
    for (const a::PoolConfig& p : cfg.pools) {
      for (std::uint32_t k = 0; k < p.num_slots; ++k) {
        a::AllocRequest r;
        r.format = p.format;
        r.layout = layout_id;
        hs.push_back(table.allocate(r).value());
      }
    }
    for (std::size_t i = hs.size(); i > 1; --i) std::swap(hs[i - 1], hs[rng.next() % i]);
    for (const a::BlockHandle h : hs) (void)table.release(h);
  }
  std::vector<a::SequenceHandle> seqs;
  total = 0;
  for (std::uint32_t i = 0; i < nseq; ++i) {
    seqs.push_back(table.create_sequence().value());
    for (std::uint32_t j = 0; j < lens[i]; ++j) {
      a::AllocRequest r;
      r.format = a::FormatId{static_cast<std::uint8_t>(fmts[total + j] & 3)};
      r.valid_tokens = T;
      r.layout = layout_id;
      (void)table.append_block(seqs.back(), r).value();
    }
    total += lens[i];
  }
  a::ExecDelta delta;
  table.collect_delta(delta);
  w->table_words.resize(std::size_t{delta.descriptor_table_size} * 4);
  for (const a::BlockExecDescriptor& p : delta.descriptor_patches) {
    std::memcpy(&w->table_words[std::size_t{p.block_id} * 4], &p, 16);
  }
  w->arena.assign(std::max<std::size_t>(delta.arena_size, 1), 0xFFFFFFFFu);
  for (const a::IdPatch& p : delta.id_patches) w->arena[p.offset] = p.block_id;
  w->arena.resize(delta.arena_size);
  std::vector<a::SequenceSegment> segs;
  (void)table.batch_segments(seqs, segs);
  for (const a::SequenceSegment& s : segs) {
    w->segs.push_back(s.offset);
    w->segs.push_back(s.length);
  }
  // Payloads: per slot, seeded N(0,1) values (outlier channels scaled), rounded to
  // FP16, then quantize_reference per row.
  std::vector<std::uint32_t> outlier(std::size_t{H} * D, 0);
  for (std::uint32_t h = 0; h < H; ++h) {
    for (std::uint32_t k = 0; k < outlier_channels && k < D; ++k) outlier[h * D + rng.next() % D] = 1;
  }
  for (int f = 0; f < 4; ++f) {
    if (counts[f] == 0) continue;
    const auto qf = static_cast<q::QuantFormat>(f);
    std::vector<std::uint8_t>& bytes = w->pool_bytes[f];
    bytes.assign(std::size_t{counts[f]} * slot_bytes[f], 0);
    auto fill = [&](std::uint32_t s0, std::uint32_t s1) {
      std::vector<float> x(elems);
      std::vector<q::AffineParams> prm(rows);
      for (std::uint32_t s = s0; s < s1; ++s) {
        SplitMix g{seed * 0x100000001B3ull + static_cast<std::uint64_t>(f) * 0x1000003ull + s};
        for (std::size_t e = 0; e < elems; ++e) {
          float v = g.normal();
          if (outlier[e % (std::size_t{H} * D)]) v *= outlier_scale;
          x[e] = q::decode_fp16(q::encode_fp16(v));
        }
        std::uint8_t* dst = bytes.data() + std::size_t{s} * slot_bytes[f];
        const std::size_t cb = q::packed_bytes(qf, elems);
        (void)q::quantize_reference(qf, x, f == 0 ? 0 : D,
                                    std::span<q::AffineParams>(prm.data(), f == 0 ? 0 : rows),
                                    std::span<std::byte>(reinterpret_cast<std::byte*>(dst), cb));
        for (std::size_t r = 0; r < rows && f != 0; ++r) {
          if (f == 3) std::memcpy(dst + cb + 8 * r, &prm[r], 8);
          else std::memcpy(dst + cb + 4 * r, &prm[r].scale, 4);
        }
      }
    };
    const int nt = std::max(1, threads);
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t) {
      pool.emplace_back(fill, static_cast<std::uint32_t>(std::uint64_t{counts[f]} * t / nt),
                        static_cast<std::uint32_t>(std::uint64_t{counts[f]} * (t + 1) / nt));
    }
    for (std::thread& th : pool) th.join();
    w->pools[f] = RefPool{bytes.data(), slot_bytes[f], counts[f], 0};
    w->info[4 + f] = counts[f];
    w->info[8 + f] = slot_bytes[f];
  }
  w->info[0] = delta.descriptor_table_size;
  w->info[1] = delta.arena_size;
  w->info[2] = nseq;
  w->info[3] = total;
  return w.release();
}

REF_API const std::uint64_t* ref_workload_info(void* w) { return static_cast<RefWorkload*>(w)->info; }
REF_API const std::uint32_t* ref_workload_table(void* w) { return static_cast<RefWorkload*>(w)->table_words.data(); }
REF_API const std::uint32_t* ref_workload_arena(void* w) { return static_cast<RefWorkload*>(w)->arena.data(); }
REF_API const std::uint32_t* ref_workload_segs(void* w) { return static_cast<RefWorkload*>(w)->segs.data(); }
REF_API const std::uint8_t* ref_workload_pool(void* w, int f) {
  return static_cast<RefWorkload*>(w)->pool_bytes[f & 3].data();
}

REF_API std::uint32_t ref_workload_gather(void* wp, std::uint16_t* out, int threads) {
  auto* w = static_cast<RefWorkload*>(wp);
  const std::uint32_t nseq = static_cast<std::uint32_t>(w->info[2]);
  std::vector<std::uint64_t> prefix(nseq + 1, 0);
  for (std::uint32_t i = 0; i < nseq; ++i) prefix[i + 1] = prefix[i] + w->segs[2 * i + 1];
  return ref_gather_dequant(w->pools, w->T, w->H, w->D, w->layout_id, w->table_words.data(),
                            static_cast<std::uint32_t>(w->info[0]), w->arena.data(),
                            static_cast<std::uint32_t>(w->info[1]), w->segs.data(), nseq, nullptr,
                            out, prefix.data(), threads);
}

REF_API void ref_workload_free(void* w) { delete static_cast<RefWorkload*>(w); }

// The CPU baseline of the decode-append step: quantize_reference on each row of D
// binary32 values (one parameter group per row, format fmt[r]: E4M3, E5M2 or INT4), rows split over
// `threads` std::thread workers.  codes: row r at codes + r * D (packed_bytes of the
// format used); params: {scale, bias} per row.  Returns the number of rows rejected.
REF_API std::size_t ref_quantize_rows(const std::uint8_t* fmt, const float* in, std::size_t rows,
                                      std::size_t D, float* params, std::uint8_t* codes,
                                      int threads) {
  if (threads < 1) threads = 1;
  std::vector<std::size_t> bad(static_cast<std::size_t>(threads), 0);
  auto work = [&](int t) {
    const std::size_t lo = rows * static_cast<std::size_t>(t) / static_cast<std::size_t>(threads);
    const std::size_t hi = rows * static_cast<std::size_t>(t + 1) / static_cast<std::size_t>(threads);
    for (std::size_t r = lo; r < hi; ++r) {
      const auto f = static_cast<q::QuantFormat>(fmt[r]);
      const q::QuantStatus s = q::quantize_reference(
          f, std::span<const float>(in + r * D, D), D,
          std::span<q::AffineParams>(reinterpret_cast<q::AffineParams*>(params + 2 * r), 1),
          std::span<std::byte>(reinterpret_cast<std::byte*>(codes + r * D), D));
      if (s != q::QuantStatus::kOk) ++bad[static_cast<std::size_t>(t)];
    }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
  for (std::thread& th : pool) th.join();
  std::size_t n = 0;
  for (const std::size_t b : bad) n += b;
  return n;
}
