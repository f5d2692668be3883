// table_trace.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A seeded random walk over the whole public API of hl::alloc::HeteroBlockTable
// that records every observable result (statuses, handles, 32-byte records,
// deltas, batch segments, CSR tables, stats, validate() status) into a stream
// of uint32 words.  The same source is compiled twice:
//   - against the reference headers and sources (oracle/build.py ->
//     oracle/_ref/libhlkv_ref.so), which yields the expected stream;
//   - against this repository's include/ and libhlkv.so (tests build it into
//     tests/_build/), which yields the stream under test.
// Equal streams mean the drop-in table behaves like the reference's, call for
// call.  The op mix follows the reference's randomized stress test
// (tests/project1/test_hetero_block_table.cpp:675-784) and adds the direct
// block API, stale handles, invalid arguments and every query.  Every random
// draw is its own statement: argument evaluation order is unspecified in C++.
#include <array>
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "hl_allocator/hetero_block_table.hpp"

namespace {

using namespace hl::alloc;

struct Rng {
  std::uint64_t s;
  std::uint64_t next() {
    std::uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  std::uint32_t below(std::uint32_t n) { return n == 0 ? 0 : static_cast<std::uint32_t>(next() % n); }
};

struct Tracer {
  std::vector<std::uint32_t> w;
  void put(std::uint32_t v) { w.push_back(v); }
  void put(Status s) { w.push_back(0x5000u | static_cast<std::uint32_t>(s)); }
  void put_exec(const BlockExecDescriptor& d) {
    std::uint32_t b[4];
    std::memcpy(b, &d, 16);
    for (std::uint32_t x : b) put(x);
  }
  void put_record(const BlockDescriptor& d) {
    std::uint32_t b[8];
    std::memcpy(b, &d, 32);
    for (std::uint32_t x : b) put(x);
  }
};

}  // namespace

extern "C" __attribute__((visibility("default"))) std::size_t table_trace_run(
    std::uint64_t seed, std::uint32_t steps, std::uint32_t max_blocks, std::uint32_t slots_fp16,
    std::uint32_t slots_fp8, std::uint32_t slots_int4, std::uint32_t* out, std::size_t cap) {
  Rng rng{seed};
  Tracer tr;
  TableConfig cfg;
  cfg.max_blocks = max_blocks;
  cfg.block_tokens = 16;
  cfg.pools = {{FormatId{0}, 65536, slots_fp16}, {FormatId{1}, 33792, slots_fp8},
               {FormatId{3}, 18432, slots_int4}};
  tr.put(HeteroBlockTable::validate_config(cfg));
  HeteroBlockTable t(cfg);
  const std::array<FormatId, 5> formats{FormatId{0}, FormatId{1}, FormatId{3}, FormatId{9},
                                        kInvalidFormat};
  std::vector<SequenceHandle> seqs;      // live sequences
  std::vector<SequenceHandle> all_seqs;  // every handle ever issued (for stale handles)
  std::vector<BlockHandle> blocks;       // every block handle ever issued
  std::vector<BlockHandle> transcoding;
  std::vector<BlockHandle> standalone;   // allocate()d outside any sequence
  ExecDelta delta;

  auto pick_format = [&](bool mostly_valid) {
    const std::uint32_t r = rng.below(mostly_valid ? 40 : 5);
    return r < 3 ? formats[r] : (r < 5 ? formats[r] : formats[r % 3]);
  };
  auto request = [&](bool odd) {
    AllocRequest r;
    r.format = pick_format(!odd);
    r.valid_tokens = odd ? rng.below(18) : rng.below(17);
    r.layout = odd ? rng.below(17) : 1;
    r.scale_mode = static_cast<ScaleMode>(odd ? rng.below(5) : 0);
    r.scale_ref = static_cast<std::uint32_t>(rng.next());
    return r;
  };
  auto any_block = [&]() -> BlockHandle {
    if (blocks.empty() || rng.below(16) == 0) {
      const std::uint32_t id = rng.below(max_blocks + 2);
      const std::uint32_t gen = rng.below(3);
      return BlockHandle{id, gen};
    }
    return blocks[rng.below(static_cast<std::uint32_t>(blocks.size()))];
  };
  auto live_block = [&]() -> BlockHandle {
    if (seqs.empty()) return any_block();
    const Result<std::span<const std::uint32_t>> ids =
        t.sequence_block_ids(seqs[rng.below(static_cast<std::uint32_t>(seqs.size()))]);
    if (!ids.ok() || ids.value().empty()) return any_block();
    const std::span<const std::uint32_t> v = ids.value();
    return t.handle_of(v[rng.below(static_cast<std::uint32_t>(v.size()))]);
  };
  auto any_seq = [&]() -> SequenceHandle {
    if (all_seqs.empty() || rng.below(10) == 0) {
      const std::uint32_t id = rng.below(8);
      const std::uint32_t gen = rng.below(2);
      return SequenceHandle{id, gen};
    }
    if (!seqs.empty() && rng.below(4) != 0) {
      return seqs[rng.below(static_cast<std::uint32_t>(seqs.size()))];
    }
    return all_seqs[rng.below(static_cast<std::uint32_t>(all_seqs.size()))];
  };
  auto drop_seq = [&](SequenceHandle s) {
    for (std::size_t i = 0; i < seqs.size(); ++i) {
      if (seqs[i] == s) {
        seqs.erase(seqs.begin() + static_cast<std::ptrdiff_t>(i));
        return;
      }
    }
  };
  auto dump_delta = [&]() {
    t.collect_delta(delta);
    tr.put(0xDE17A000u);
    tr.put(delta.descriptor_table_size);
    tr.put(delta.arena_size);
    tr.put(static_cast<std::uint32_t>(delta.descriptor_patches.size()));
    for (const BlockExecDescriptor& p : delta.descriptor_patches) tr.put_exec(p);
    tr.put(static_cast<std::uint32_t>(delta.id_patches.size()));
    for (const IdPatch& p : delta.id_patches) {
      tr.put(p.offset);
      tr.put(p.block_id);
    }
  };

  for (std::uint32_t step = 0; step < steps; ++step) {
    const std::uint32_t op = rng.below(24);
    tr.put(0xA0000000u | op);
    switch (op) {
      case 0: {
        const Result<SequenceHandle> s = t.create_sequence();
        tr.put(s.status());
        if (s.ok()) {
          seqs.push_back(s.value());
          all_seqs.push_back(s.value());
          tr.put(s.value().id);
          tr.put(s.value().generation);
        }
        break;
      }
      case 1: case 2: case 3: {
        const SequenceHandle s = any_seq();
        const Result<BlockHandle> b = t.append_block(s, request(op == 3));
        tr.put(b.status());
        if (b.ok()) {
          blocks.push_back(b.value());
          tr.put(b.value().id);
          tr.put(b.value().generation);
        }
        break;
      }
      case 4: {
        const BlockHandle h = live_block();
        tr.put(t.seal(h));
        const SequenceHandle s = any_seq();
        tr.put(t.append_shared_block(s, h));
        break;
      }
      case 5: {
        const BlockHandle h = live_block();
        (void)t.seal(h);
        const Result<FormatChange> fc = t.begin_format_change(h, pick_format(true));
        tr.put(fc.status());
        if (fc.ok()) {
          tr.put(static_cast<std::uint32_t>(fc.value().from_format));
          tr.put(fc.value().from_slot);
          tr.put(static_cast<std::uint32_t>(fc.value().to_format));
          tr.put(fc.value().to_slot);
          transcoding.push_back(h);
        }
        break;
      }
      case 6: {
        if (transcoding.empty()) {
          tr.put(t.commit_format_change(any_block(), ScaleMode::kNone, 0));
          break;
        }
        const std::uint32_t i = rng.below(static_cast<std::uint32_t>(transcoding.size()));
        const std::uint32_t how = rng.below(3);
        const auto mode = static_cast<ScaleMode>(rng.below(5));
        const auto ref = static_cast<std::uint32_t>(rng.next());
        const Status s = how == 0 ? t.abort_format_change(transcoding[i])
                                  : t.commit_format_change(transcoding[i], mode, ref);
        tr.put(s);
        if (s == Status::kOk) transcoding.erase(transcoding.begin() + i);
        break;
      }
      case 7: {
        const BlockHandle h = live_block();
        const auto r = static_cast<Residency>(rng.below(4));
        tr.put(t.set_residency(h, r));
        break;
      }
      case 8: case 9: {
        const BlockHandle h = live_block();
        const std::uint32_t n = rng.below(18);
        tr.put(t.set_valid_tokens(h, n));
        break;
      }
      case 10: {
        if (seqs.empty()) break;
        const SequenceHandle s =
            rng.below(8) == 0 ? any_seq() : seqs[rng.below(static_cast<std::uint32_t>(seqs.size()))];
        const Status st = t.release_sequence(s);
        tr.put(st);
        if (st == Status::kOk) drop_seq(s);
        break;
      }
      case 11: {
        const Result<BlockHandle> b = t.allocate(request(rng.below(4) == 0));
        tr.put(b.status());
        if (b.ok()) {
          blocks.push_back(b.value());
          tr.put(b.value().id);
          tr.put(b.value().generation);
          if (rng.below(2) == 0) {
            tr.put(t.release(b.value()));
          } else {
            standalone.push_back(b.value());
          }
        }
        break;
      }
      case 12:
        tr.put(t.retain(any_block()));
        break;
      case 13: {
        // Mostly blocks no sequence owns; rarely any block, which drops a
        // sequence's reference (misuse that validate() reports as kCorrupt).
        if (!standalone.empty() && rng.below(64) != 0) {
          const std::uint32_t i = rng.below(static_cast<std::uint32_t>(standalone.size()));
          tr.put(t.release(standalone[i]));
          standalone.erase(standalone.begin() + i);
        } else if (rng.below(8) == 0) {
          tr.put(t.release(any_block()));
        }
        break;
      }
      case 14: {
        const BlockHandle h = any_block();
        const auto mode = static_cast<ScaleMode>(rng.below(5));
        const auto ref = static_cast<std::uint32_t>(rng.next());
        tr.put(t.set_scale(h, mode, ref));
        break;
      }
      case 15: {
        const Result<BlockDescriptor> d = t.lookup(any_block());
        tr.put(d.status());
        if (d.ok()) tr.put_record(d.value());
        break;
      }
      case 16: {
        std::vector<BlockHandle> hs;
        const std::uint32_t n = rng.below(6);
        for (std::uint32_t i = 0; i < n; ++i) hs.push_back(rng.below(3) ? live_block() : any_block());
        std::vector<BlockExecDescriptor> out(n + rng.below(2));
        if (out.size() > 0 && rng.below(6) == 0) out.pop_back();
        const Status st = t.lookup_batch(hs, out);
        tr.put(st);
        if (st == Status::kOk) for (std::uint32_t i = 0; i < n; ++i) tr.put_exec(out[i]);
        break;
      }
      case 17: {
        const BlockHandle h = t.handle_of(rng.below(max_blocks + 2));
        tr.put(h.id);
        tr.put(h.generation);
        const std::uint32_t id = rng.below(max_blocks + 2);
        tr.put_exec(t.device_descriptor(id));
        break;
      }
      case 18: {
        const Result<std::span<const std::uint32_t>> ids = t.sequence_block_ids(any_seq());
        tr.put(ids.status());
        if (ids.ok()) {
          tr.put(static_cast<std::uint32_t>(ids.value().size()));
          for (std::uint32_t id : ids.value()) tr.put(id);
        }
        break;
      }
      case 19:
        dump_delta();
        break;
      case 20: {
        std::vector<SequenceHandle> batch = seqs;
        if (rng.below(6) == 0) batch.push_back(any_seq());
        std::vector<SequenceSegment> segs;
        const Status st = t.batch_segments(batch, segs);
        tr.put(st);
        tr.put(static_cast<std::uint32_t>(segs.size()));
        for (const SequenceSegment& s : segs) {
          tr.put(s.offset);
          tr.put(s.length);
        }
        break;
      }
      case 21: {
        ExecTable et;
        const Status st = t.build_exec_table(seqs, et);
        tr.put(st);
        tr.put(static_cast<std::uint32_t>(et.indptr.size()));
        for (std::uint32_t x : et.indptr) tr.put(x);
        tr.put(static_cast<std::uint32_t>(et.blocks.size()));
        for (const BlockExecDescriptor& d : et.blocks) tr.put_exec(d);
        break;
      }
      case 22: {
        const TableStats st = t.stats();
        tr.put(st.blocks_in_use);
        tr.put(st.blocks_capacity);
        tr.put(st.active_sequences);
        for (std::uint32_t x : st.blocks_per_format) tr.put(x);
        for (std::uint32_t x : st.blocks_per_residency) tr.put(x);
        for (std::uint32_t x : st.blocks_per_state) tr.put(x);
        for (std::uint64_t x : {st.valid_tokens, st.token_capacity_in_use, st.payload_bytes_in_use,
                                st.format_changes_committed, st.arena_entries,
                                st.arena_live_entries, st.arena_reserved_entries,
                                st.arena_free_entries, st.pending_descriptor_patches,
                                st.pending_id_patches}) {
          tr.put(static_cast<std::uint32_t>(x));
          tr.put(static_cast<std::uint32_t>(x >> 32));
        }
        for (FormatId f : formats) {
          tr.put(t.has_pool(f) ? 1u : 0u);
          tr.put(t.free_slots(f));
          tr.put(t.pool_slots(f));
          tr.put(t.slot_bytes(f));
        }
        tr.put(t.blocks_in_use());
        tr.put(t.max_blocks());
        tr.put(t.block_tokens());
        tr.put(static_cast<std::uint32_t>(t.pending_descriptor_patches()));
        tr.put(static_cast<std::uint32_t>(t.pending_id_patches()));
        break;
      }
      default:
        tr.put(t.validate().status);
        break;
    }
  }
  // Drain: finish transcodes, release everything, final delta.
  for (const BlockHandle h : transcoding) tr.put(t.abort_format_change(h));
  for (const SequenceHandle s : seqs) tr.put(t.release_sequence(s));
  dump_delta();
  tr.put(t.validate().status);
  tr.put(t.blocks_in_use());
  const std::size_t n = tr.w.size();
  if (out != nullptr) {
    for (std::size_t i = 0; i < n && i < cap; ++i) out[i] = tr.w[i];
  }
  return n;
}
