// Host-side tests of the drop-in C++ API (hl::alloc), linked against libhlkv.so.
//
// Restates the reference's own unit and behaviour tests
// (tests/project1/test_block_descriptor.cpp, test_id_arena.cpp,
// test_hetero_block_table.cpp) in a self-contained harness: every case prints
// "ok <name>" or "FAIL <name>: <what>", and the process exits non-zero on any
// failure.  tests/test_table.py builds and runs it.
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "hl_allocator/hetero_block_table.hpp"

using namespace hl::alloc;

namespace {

int g_failures = 0;
std::string g_current;

#define CHECK(cond)                                                                    \
  do {                                                                                 \
    if (!(cond)) {                                                                     \
      std::printf("FAIL %s: %s (line %d)\n", g_current.c_str(), #cond, __LINE__);      \
      ++g_failures;                                                                    \
      return;                                                                          \
    }                                                                                  \
  } while (0)

struct Case {
  const char* name;
  void (*fn)();
};
std::vector<Case>& cases() {
  static std::vector<Case> v;
  return v;
}
struct Register {
  Register(const char* n, void (*f)()) { cases().push_back({n, f}); }
};
#define TEST(name)                         \
  void name();                             \
  const Register reg_##name(#name, name);  \
  void name()

constexpr FormatId kFp16{0}, kFp8{1}, kInt4{3}, kUnconfigured{9};

TableConfig small_config(std::uint32_t blocks = 8, std::uint32_t a = 4, std::uint32_t b = 4,
                         std::uint32_t c = 4) {
  TableConfig cfg;
  cfg.max_blocks = blocks;
  cfg.block_tokens = 16;
  cfg.pools = {{kFp16, 4096, a}, {kFp8, 2048, b}, {kInt4, 1088, c}};
  return cfg;
}

AllocRequest req(FormatId f, std::uint32_t tokens = 0) {
  AllocRequest r;
  r.format = f;
  r.valid_tokens = tokens;
  return r;
}

bool non_executable(const BlockExecDescriptor& d) {
  return d.format() == kInvalidFormat && d.slot == kNoSlot;
}

// Host simulation of the device tables, as the reference's ExecMirror.
struct Mirror {
  std::vector<BlockExecDescriptor> table;
  std::vector<std::uint32_t> arena;
  bool apply(const ExecDelta& d) {
    if (table.size() < d.descriptor_table_size) {
      BlockExecDescriptor g{0xABABABABu, 0xABABABABu, 0xABABABABu, 0xABABABABu};
      table.resize(d.descriptor_table_size, g);
    }
    if (arena.size() < d.arena_size) arena.resize(d.arena_size, 0xDEADBEEFu);
    std::vector<std::uint8_t> seen(table.size(), 0), seen_a(arena.size(), 0);
    for (const BlockExecDescriptor& p : d.descriptor_patches) {
      if (p.block_id >= table.size() || seen[p.block_id]) return false;
      seen[p.block_id] = 1;
      table[p.block_id] = p;
    }
    for (const IdPatch& p : d.id_patches) {
      if (p.offset >= arena.size() || seen_a[p.offset]) return false;
      seen_a[p.offset] = 1;
      arena[p.offset] = p.block_id;
    }
    return true;
  }
  std::vector<BlockExecDescriptor> read(SequenceSegment s) const {
    std::vector<BlockExecDescriptor> out;
    for (std::uint32_t j = 0; j < s.length; ++j) out.push_back(table.at(arena.at(std::size_t{s.offset} + j)));
    return out;
  }
  bool matches(const HeteroBlockTable& t) const {
    if (table.size() != t.max_blocks()) return false;
    for (std::uint32_t id = 0; id < t.max_blocks(); ++id) {
      if (!(table[id] == t.device_descriptor(id))) return false;
    }
    return true;
  }
};

std::vector<BlockExecDescriptor> device_view(const HeteroBlockTable& t, SequenceHandle s) {
  std::vector<BlockExecDescriptor> out;
  const Result<std::span<const std::uint32_t>> ids = t.sequence_block_ids(s);
  for (const std::uint32_t id : ids.value()) out.push_back(t.device_descriptor(id));
  return out;
}

// ---- ABI (test_block_descriptor.cpp) -----------------------------------------------------

TEST(AbiSizesAndAlignment) {
  CHECK(sizeof(BlockExecDescriptor) == 16 && alignof(BlockExecDescriptor) == 16);
  CHECK(sizeof(BlockDescriptor) == 32 && alignof(BlockDescriptor) == 32);
  CHECK(kAbiVersion == 1);
}

TEST(AbiGoldenInfoWord) {
  constexpr std::uint32_t info = BlockExecDescriptor::pack_info(FormatId{5}, ScaleMode::kInlineF32, 3, 16);
  static_assert(info == 0x000040D5u);
  CHECK(info == 0x000040D5u);
}

TEST(AbiGoldenByteLayout) {
  BlockDescriptor d{};
  d.exec.slot = 0x04030201u;
  d.exec.info = BlockExecDescriptor::pack_info(FormatId{2}, ScaleMode::kExternal, 0, 512);
  d.exec.scale_ref = 0x0C0B0A09u;
  d.exec.block_id = 0x100F0E0Du;
  d.generation = 0x14131211u;
  d.set_state(BlockState::kSealed);
  d.set_residency(Residency::kHost);
  d.set_pending_format(FormatId{7});
  d.set_refcount(0xABCD);
  d.pending_slot = 0x1C1B1A19u;
  d.reserved = 0;
  std::array<std::uint8_t, 32> bytes{};
  std::memcpy(bytes.data(), &d, 32);
  const std::array<std::uint8_t, 32> expected = {
      0x01, 0x02, 0x03, 0x04, 0x32, 0x00, 0x08, 0x00, 0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x0E, 0x0F, 0x10,
      0x11, 0x12, 0x13, 0x14, 0x76, 0xCD, 0xAB, 0x00, 0x19, 0x1A, 0x1B, 0x1C, 0x00, 0x00, 0x00, 0x00};
  CHECK(bytes == expected);
}

TEST(AbiFieldsRoundTripAtLimits) {
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    for (std::uint32_t m = 0; m < 4; ++m) {
      for (const std::uint32_t layout : {0u, 1u, kMaxLayoutId}) {
        for (const std::uint32_t tokens : {0u, 1u, 16u, kMaxBlockTokens}) {
          BlockExecDescriptor e{};
          e.info = BlockExecDescriptor::pack_info(FormatId{static_cast<std::uint8_t>(f)},
                                                  static_cast<ScaleMode>(m), layout, tokens);
          CHECK(static_cast<std::uint32_t>(e.format()) == f);
          CHECK(static_cast<std::uint32_t>(e.scale_mode()) == m);
          CHECK(e.layout() == layout && e.valid_tokens() == tokens && e.info_reserved() == 0);
        }
      }
    }
  }
}

TEST(AbiSettersKeepNeighbours) {
  BlockExecDescriptor e{};
  e.info = BlockExecDescriptor::pack_info(FormatId{14}, ScaleMode::kInlineF16Pair, kMaxLayoutId, kMaxBlockTokens);
  e.set_valid_tokens(7);
  CHECK(static_cast<std::uint32_t>(e.format()) == 14 && e.scale_mode() == ScaleMode::kInlineF16Pair);
  CHECK(e.layout() == kMaxLayoutId && e.valid_tokens() == 7);
  e.set_format(FormatId{1});
  e.set_scale_mode(ScaleMode::kNone);
  CHECK(e.valid_tokens() == 7 && e.layout() == kMaxLayoutId);
  BlockDescriptor d{};
  d.set_refcount(kMaxRefcount);
  d.set_state(BlockState::kTranscoding);
  d.set_residency(Residency::kDropped);
  d.set_pending_format(FormatId{14});
  CHECK(d.refcount() == kMaxRefcount && d.state() == BlockState::kTranscoding);
  CHECK(d.residency() == Residency::kDropped && static_cast<std::uint32_t>(d.pending_format()) == 14);
  CHECK(d.control_reserved() == 0);
  e.set_valid_tokens(0xFFFFFFFFu);  // masked, never spilled into the reserved bits
  CHECK(e.info_reserved() == 0 && static_cast<std::uint32_t>(e.format()) == 1);
  BlockExecDescriptor s{};
  float v = 0.0123f;
  std::memcpy(&s.scale_ref, &v, 4);
  CHECK(s.inline_scale_f32() == 0.0123f);
  std::vector<BlockDescriptor> many(257);
  for (const BlockDescriptor& x : many) {
    const auto a = reinterpret_cast<std::uintptr_t>(&x);
    CHECK(a % 32 == 0 && a / 64 == (a + 31) / 64);
  }
}

// ---- IdArena (test_id_arena.cpp) ---------------------------------------------------------

TEST(ArenaFirstReserveUsesSmallestClass) {
  IdArena arena;
  IdArena::Segment seg;
  CHECK(arena.view(seg).empty() && IdArena::kernel_view(seg) == (SequenceSegment{0, 0}));
  CHECK(arena.reserve(seg, 1) == Status::kOk);
  CHECK(seg.capacity == IdArena::kMinSegment && seg.offset == 0 && seg.length == 0);
  CHECK(arena.size() == IdArena::kMinSegment);
  CHECK(arena.reserve(seg, IdArena::kMinSegment) == Status::kOk && arena.size() == IdArena::kMinSegment);
  const IdArena::Segment live[] = {seg};
  CHECK(arena.validate(live).empty());
}

TEST(ArenaGrowthRelocatesAndPreserves) {
  IdArena arena;
  IdArena::Segment a, b;
  std::vector<std::uint32_t> expect_a;
  for (std::uint32_t i = 0; i < 100; ++i) {
    CHECK(arena.reserve(a, a.length + 1) == Status::kOk);
    arena.push_back(a, 1000 + i);
    expect_a.push_back(1000 + i);
    if (i % 3 == 0) {
      CHECK(arena.reserve(b, b.length + 1) == Status::kOk);
      arena.push_back(b, i);
    }
  }
  const auto v = arena.view(a);
  CHECK(std::vector<std::uint32_t>(v.begin(), v.end()) == expect_a);
  CHECK(a.capacity == 128 && b.length == 34 && b.capacity == 64);
  const IdArena::Segment live[] = {a, b};
  CHECK(arena.validate(live).empty());
  CHECK(arena.free_entries() + a.capacity + b.capacity == arena.size());
}

TEST(ArenaPatchesUniqueFinal) {
  IdArena arena;
  IdArena::Segment seg;
  for (std::uint32_t i = 0; i < 20; ++i) {
    CHECK(arena.reserve(seg, seg.length + 1) == Status::kOk);
    arena.push_back(seg, 7 * i);
  }
  std::vector<IdPatch> patches;
  arena.collect(patches);
  std::set<std::uint32_t> offsets;
  for (const IdPatch& p : patches) CHECK(offsets.insert(p.offset).second && p.offset < arena.size());
  for (std::uint32_t j = 0; j < seg.length; ++j) {
    const auto it = std::find_if(patches.begin(), patches.end(),
                                 [&](IdPatch p) { return p.offset == seg.offset + j; });
    CHECK(it != patches.end() && it->block_id == 7 * j);
  }
  CHECK(arena.pending_patches() == 0);
  arena.collect(patches);
  CHECK(patches.empty());
}

TEST(ArenaReleasedSegmentsReused) {
  IdArena arena;
  IdArena::Segment a, b, c;
  CHECK(arena.reserve(a, 5) == Status::kOk && arena.reserve(b, 5) == Status::kOk);
  const std::uint32_t a_off = a.offset;
  arena.release(a);
  CHECK(a.capacity == 0);
  CHECK(arena.reserve(c, 3) == Status::kOk && c.offset == a_off);
  CHECK(arena.size() == 2 * IdArena::kMinSegment);
  const IdArena::Segment live[] = {b, c};
  CHECK(arena.validate(live).empty());
}

TEST(ArenaLimitsAndValidate) {
  IdArena arena;
  IdArena::Segment seg;
  CHECK(arena.reserve(seg, IdArena::kMaxSegment + 1) == Status::kCapacityExceeded);
  CHECK(seg.capacity == 0 && arena.size() == 0);
  IdArena::Segment a, b;
  CHECK(arena.reserve(a, 1) == Status::kOk && arena.reserve(b, 1) == Status::kOk);
  const IdArena::Segment leak[] = {a};
  CHECK(!arena.validate(leak).empty());
  const IdArena::Segment overlap[] = {a, a, b};
  CHECK(!arena.validate(overlap).empty());
  IdArena::Segment bogus = a;
  bogus.capacity = 12;
  const IdArena::Segment badcap[] = {bogus, b};
  CHECK(!arena.validate(badcap).empty());
  bogus = a;
  bogus.length = bogus.capacity + 1;
  const IdArena::Segment badlen[] = {bogus, b};
  CHECK(!arena.validate(badlen).empty());
}

// ---- HeteroBlockTable (test_hetero_block_table.cpp) -----------------------------------------

TEST(TableRejectsInvalidConfigs) {
  CHECK(HeteroBlockTable::validate_config(small_config()) == Status::kOk);
  TableConfig c = small_config();
  c.max_blocks = 0;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c = small_config();
  c.block_tokens = 0;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c.block_tokens = kMaxBlockTokens + 1;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c.block_tokens = kMaxBlockTokens;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kOk);
  c = small_config();
  c.pools.clear();
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c = small_config();
  c.pools.push_back({kFp16, 4096, 1});
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c = small_config();
  c.pools.push_back({kInvalidFormat, 16, 1});
  CHECK(HeteroBlockTable::validate_config(c) == Status::kUnknownFormat);
  c = small_config();
  c.pools[0].slot_bytes = 0;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c = small_config();
  c.pools[0].num_slots = 0;
  CHECK(HeteroBlockTable::validate_config(c) == Status::kInvalidArgument);
  c = small_config();
  c.max_blocks = 0;
  bool threw = false;
  try {
    HeteroBlockTable t{c};
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
}

TEST(TableFreshIsConsistent) {
  const HeteroBlockTable t(small_config());
  CHECK(t.max_blocks() == 8 && t.blocks_in_use() == 0 && t.free_slots(kFp16) == 4);
  CHECK(t.slot_bytes(kFp8) == 2048 && !t.has_pool(kUnconfigured));
  CHECK(t.free_slots(kUnconfigured) == 0 && t.free_slots(kInvalidFormat) == 0);
  CHECK(t.validate().ok());
}

TEST(TableAllocationOrderIsDeterministic) {
  HeteroBlockTable t(small_config());
  for (std::uint32_t i = 0; i < 3; ++i) {
    const Result<BlockHandle> h = t.allocate(req(kFp16));
    CHECK(h.ok() && h.value().id == i && t.lookup(h.value()).value().exec.slot == i);
  }
  const Result<BlockHandle> h = t.allocate(req(kInt4));
  CHECK(h.ok() && h.value().id == 3 && t.lookup(h.value()).value().exec.slot == 0);
}

TEST(TableDescriptorReflectsRequest) {
  HeteroBlockTable t(small_config());
  AllocRequest r = req(kFp8, 5);
  r.layout = 2;
  r.scale_mode = ScaleMode::kInlineF32;
  r.scale_ref = 0x3F800000u;
  const BlockHandle h = t.allocate(r).value();
  const BlockDescriptor d = t.lookup(h).value();
  CHECK(d.exec.format() == kFp8 && d.exec.valid_tokens() == 5 && d.exec.layout() == 2);
  CHECK(d.exec.scale_mode() == ScaleMode::kInlineF32 && d.exec.inline_scale_f32() == 1.0f);
  CHECK(d.exec.block_id == h.id && d.state() == BlockState::kOpen);
  CHECK(d.residency() == Residency::kDevice && d.refcount() == 1 && d.pending_slot == kNoSlot);
}

TEST(TableRejectsInvalidRequestsAndExhaustion) {
  HeteroBlockTable t(small_config(8, 2, 4, 4));
  CHECK(t.allocate(req(kUnconfigured)).status() == Status::kUnknownFormat);
  CHECK(t.allocate(req(kInvalidFormat)).status() == Status::kUnknownFormat);
  CHECK(t.allocate(req(kFp16, 17)).status() == Status::kInvalidArgument);
  AllocRequest r = req(kFp16);
  r.layout = kMaxLayoutId + 1;
  CHECK(t.allocate(r).status() == Status::kInvalidArgument);
  r = req(kFp16);
  r.scale_mode = static_cast<ScaleMode>(4);
  CHECK(t.allocate(r).status() == Status::kInvalidArgument);
  CHECK(t.allocate(req(kFp16)).ok() && t.allocate(req(kFp16)).ok());
  CHECK(t.allocate(req(kFp16)).status() == Status::kOutOfSlots);
  for (int i = 0; i < 6; ++i) CHECK(t.allocate(req(i < 4 ? kFp8 : kInt4)).ok());
  CHECK(t.allocate(req(kInt4)).status() == Status::kOutOfBlocks);
  CHECK(t.validate().ok());
}

TEST(TableStaleHandlesAndRefcounts) {
  HeteroBlockTable t(small_config());
  const BlockHandle h = t.allocate(req(kFp16)).value();
  CHECK(t.retain(h) == Status::kOk && t.release(h) == Status::kOk);
  CHECK(t.lookup(h).ok());
  CHECK(t.release(h) == Status::kOk);
  CHECK(t.lookup(h).status() == Status::kStaleHandle);
  CHECK(t.release(h) == Status::kStaleHandle && t.retain(h) == Status::kStaleHandle);
  CHECK(t.lookup(BlockHandle{100, 0}).status() == Status::kInvalidHandle);
  const BlockHandle h2 = t.allocate(req(kFp16)).value();
  CHECK(h2.id == h.id && h2.generation == h.generation + 1);  // LIFO reuse, new generation
  CHECK(t.handle_of(h2.id) == h2 && t.handle_of(7) == kInvalidBlock && t.handle_of(99) == kInvalidBlock);
  bool threw = false;
  try {
    (void)t.lookup(h).value();
  } catch (const BadResultAccess& e) {
    threw = e.status() == Status::kStaleHandle;
  }
  CHECK(threw);
}

TEST(TableStateMachine) {
  HeteroBlockTable t(small_config());
  const BlockHandle h = t.allocate(req(kFp16, 3)).value();
  CHECK(t.set_valid_tokens(h, 16) == Status::kOk);
  CHECK(t.set_valid_tokens(h, 17) == Status::kInvalidArgument);
  CHECK(t.begin_format_change(h, kInt4).status() == Status::kInvalidState);  // open
  CHECK(t.seal(h) == Status::kOk && t.seal(h) == Status::kInvalidState);
  CHECK(t.set_valid_tokens(h, 1) == Status::kInvalidState);
  CHECK(t.set_residency(h, static_cast<Residency>(3)) == Status::kInvalidArgument);
  CHECK(t.set_residency(h, Residency::kHost) == Status::kOk);
  CHECK(t.begin_format_change(h, kInt4).status() == Status::kNotDeviceResident);
  CHECK(t.set_residency(h, Residency::kDevice) == Status::kOk);
  CHECK(t.begin_format_change(h, kUnconfigured).status() == Status::kUnknownFormat);
  CHECK(t.begin_format_change(h, kFp16).status() == Status::kInvalidArgument);
  const Result<FormatChange> fc = t.begin_format_change(h, kInt4);
  CHECK(fc.ok() && fc.value().from_format == kFp16 && fc.value().to_format == kInt4);
  CHECK(t.set_residency(h, Residency::kHost) == Status::kInvalidState);
  CHECK(t.set_scale(h, ScaleMode::kNone, 0) == Status::kInvalidState);
  CHECK(t.release(h) == Status::kInvalidState);  // last reference while transcoding
  CHECK(t.free_slots(kInt4) == 3 && t.free_slots(kFp16) == 3);
  CHECK(t.abort_format_change(h) == Status::kOk && t.free_slots(kInt4) == 4);
  CHECK(t.abort_format_change(h) == Status::kInvalidState);
  CHECK(t.begin_format_change(h, kInt4).ok());
  CHECK(t.commit_format_change(h, static_cast<ScaleMode>(4), 0) == Status::kInvalidArgument);
  CHECK(t.commit_format_change(h, ScaleMode::kInlineF32, 0x3F800000u) == Status::kOk);
  const BlockDescriptor d = t.lookup(h).value();
  CHECK(d.exec.format() == kInt4 && d.state() == BlockState::kSealed && d.pending_slot == kNoSlot);
  CHECK(t.free_slots(kFp16) == 4 && t.free_slots(kInt4) == 3 && t.stats().format_changes_committed == 1);
  CHECK(t.validate().ok());
}

TEST(TableSequencesSharingAndCsr) {
  HeteroBlockTable t(small_config(16, 8, 8, 8));
  const SequenceHandle a = t.create_sequence().value();
  const SequenceHandle b = t.create_sequence().value();
  const BlockHandle p = t.append_block(a, req(kFp16, 16)).value();
  CHECK(t.append_shared_block(b, p) == Status::kInvalidState);  // open blocks are not shared
  CHECK(t.seal(p) == Status::kOk && t.append_shared_block(b, p) == Status::kOk);
  CHECK(t.lookup(p).value().refcount() == 2);
  CHECK(t.append_block(b, req(kFp8, 1)).ok());
  ExecTable et;
  const std::vector<SequenceHandle> batch{a, b};
  CHECK(t.build_exec_table(batch, et) == Status::kOk);
  CHECK(et.indptr == (std::vector<std::uint32_t>{0, 1, 3}) && et.blocks[0] == et.blocks[1]);
  CHECK(t.release_sequence(a) == Status::kOk && t.lookup(p).value().refcount() == 1);
  CHECK(t.release_sequence(a) == Status::kStaleHandle);
  CHECK(t.sequence_block_ids(a).status() == Status::kStaleHandle);
  const SequenceHandle c = t.create_sequence().value();
  CHECK(c.id == a.id && c.generation == a.generation + 1);
  CHECK(t.set_residency(p, Residency::kDropped) == Status::kOk);
  const std::vector<SequenceHandle> bb{b};
  CHECK(t.build_exec_table(bb, et) == Status::kNotDeviceResident && et.blocks.empty());
  CHECK(t.release_sequence(b) == Status::kOk && t.blocks_in_use() == 0);
  CHECK(t.validate().ok());
}

TEST(DeltaFirstInitializesWholeTable) {
  HeteroBlockTable t(small_config());
  ExecDelta d;
  t.collect_delta(d);
  CHECK(d.descriptor_table_size == 8 && d.arena_size == 0 && d.id_patches.empty());
  CHECK(d.descriptor_patches.size() == 8);
  for (std::uint32_t i = 0; i < 8; ++i) {
    CHECK(d.descriptor_patches[i].block_id == i && non_executable(d.descriptor_patches[i]));
  }
  Mirror m;
  CHECK(m.apply(d) && m.matches(t));
  t.collect_delta(d);
  CHECK(d.descriptor_patches.empty() && d.id_patches.empty());
}

TEST(DeltaOnlyChangedRecords) {
  HeteroBlockTable t(small_config());
  ExecDelta d;
  t.collect_delta(d);
  const SequenceHandle s = t.create_sequence().value();
  const BlockHandle b = t.append_block(s, req(kFp16, 1)).value();
  CHECK(t.set_valid_tokens(b, 2) == Status::kOk && t.set_valid_tokens(b, 3) == Status::kOk);
  CHECK(t.pending_descriptor_patches() == 1 && t.pending_id_patches() == 1);
  t.collect_delta(d);
  CHECK(d.descriptor_patches.size() == 1 && d.descriptor_patches[0] == t.lookup(b).value().exec);
  CHECK(d.descriptor_patches[0].valid_tokens() == 3);
  CHECK(d.id_patches.size() == 1 && d.id_patches[0].block_id == b.id);
  CHECK(t.seal(b) == Status::kOk);
  t.collect_delta(d);
  CHECK(d.descriptor_patches.empty() && d.id_patches.empty());
}

TEST(DeltaNonResidentAndFreedBecomeNonExecutable) {
  HeteroBlockTable t(small_config());
  Mirror m;
  ExecDelta d;
  const SequenceHandle s = t.create_sequence().value();
  const BlockHandle a = t.append_block(s, req(kFp16, 16)).value();
  const BlockHandle b = t.append_block(s, req(kInt4, 16)).value();
  CHECK(t.set_residency(b, Residency::kHost) == Status::kOk);
  t.collect_delta(d);
  CHECK(m.apply(d) && m.matches(t));
  CHECK(non_executable(m.table[b.id]) && !non_executable(m.table[a.id]));
  ExecTable et;
  const std::vector<SequenceHandle> batch{s};
  CHECK(t.build_exec_table(batch, et) == Status::kNotDeviceResident);
  std::vector<SequenceSegment> segs;
  CHECK(t.batch_segments(batch, segs) == Status::kOk && m.read(segs[0]) == device_view(t, s));
  CHECK(t.set_residency(b, Residency::kDevice) == Status::kOk && t.release_sequence(s) == Status::kOk);
  t.collect_delta(d);
  CHECK(m.apply(d) && m.matches(t) && non_executable(m.table[a.id]) && non_executable(m.table[b.id]));
}

TEST(DeltaSharedChangeIsOnePatch) {
  HeteroBlockTable t(small_config(16, 8, 8, 8));
  Mirror m;
  ExecDelta d;
  std::vector<SequenceHandle> seqs;
  for (int i = 0; i < 3; ++i) seqs.push_back(t.create_sequence().value());
  const BlockHandle prefix = t.append_block(seqs[0], req(kFp16, 16)).value();
  CHECK(t.seal(prefix) == Status::kOk);
  CHECK(t.append_shared_block(seqs[1], prefix) == Status::kOk);
  CHECK(t.append_shared_block(seqs[2], prefix) == Status::kOk);
  for (const SequenceHandle s : seqs) CHECK(t.append_block(s, req(kFp8, 1)).ok());
  t.collect_delta(d);
  CHECK(m.apply(d));
  CHECK(t.begin_format_change(prefix, kInt4).ok());
  CHECK(t.commit_format_change(prefix, ScaleMode::kInlineF32, 0x3F800000u) == Status::kOk);
  t.collect_delta(d);
  CHECK(d.descriptor_patches.size() == 1 && d.id_patches.empty() && m.apply(d));
  std::vector<SequenceSegment> segs;
  CHECK(t.batch_segments(seqs, segs) == Status::kOk);
  ExecTable ref;
  CHECK(t.build_exec_table(seqs, ref) == Status::kOk);
  std::vector<BlockExecDescriptor> seen;
  for (const SequenceSegment& s : segs) for (const auto& x : m.read(s)) seen.push_back(x);
  CHECK(seen == ref.blocks);
  for (std::size_t i = 0; i < 3; ++i) CHECK(seen[2 * i].format() == kInt4);
}

TEST(DeltaRelocationCarriedByIdPatches) {
  HeteroBlockTable t(small_config(64, 64, 64, 64));
  Mirror m;
  ExecDelta d;
  const SequenceHandle a = t.create_sequence().value();
  const SequenceHandle b = t.create_sequence().value();
  for (int i = 0; i < 20; ++i) {
    CHECK(t.append_block(a, req(kFp16, 16)).ok());
    if (i % 4 == 0) CHECK(t.append_block(b, req(kFp8, 16)).ok());
    if (i % 7 == 0) {
      t.collect_delta(d);
      CHECK(m.apply(d));
    }
  }
  t.collect_delta(d);
  CHECK(m.apply(d) && d.arena_size == t.stats().arena_entries);
  std::vector<SequenceSegment> segs;
  const std::vector<SequenceHandle> batch{a, b};
  CHECK(t.batch_segments(batch, segs) == Status::kOk && segs[0].length == 20);
  CHECK(m.read(segs[0]) == device_view(t, a) && m.read(segs[1]) == device_view(t, b));
  CHECK(t.validate().ok());
}

TEST(DeltaBatchSegmentsValidatesHandles) {
  HeteroBlockTable t(small_config());
  const SequenceHandle s = t.create_sequence().value();
  std::vector<SequenceSegment> segs{{1, 2}};
  const std::vector<SequenceHandle> ok{s};
  CHECK(t.batch_segments(ok, segs) == Status::kOk && segs == (std::vector<SequenceSegment>{{0, 0}}));
  const std::vector<SequenceHandle> bad{s, kInvalidSequence};
  CHECK(t.batch_segments(bad, segs) == Status::kInvalidHandle && segs.empty());
}

TEST(StatsReportArenaAndPending) {
  HeteroBlockTable t(small_config());
  ExecDelta d;
  CHECK(t.stats().pending_descriptor_patches == 8);
  t.collect_delta(d);
  const SequenceHandle s = t.create_sequence().value();
  CHECK(t.append_block(s, req(kFp16, 4)).ok());
  const TableStats st = t.stats();
  CHECK(st.arena_entries == IdArena::kMinSegment && st.arena_live_entries == 1);
  CHECK(st.arena_reserved_entries == IdArena::kMinSegment && st.arena_free_entries == 0);
  CHECK(st.pending_descriptor_patches == 1 && st.pending_id_patches == 1 && st.valid_tokens == 4);
  CHECK(st.payload_bytes_in_use == 4096 && st.blocks_per_format[0] == 1);
  CHECK(t.release_sequence(s) == Status::kOk && t.stats().arena_free_entries == IdArena::kMinSegment);
}

TEST(StressRandomOperationsAgainstMirror) {
  TableConfig cfg;
  cfg.max_blocks = 96;
  cfg.block_tokens = 16;
  cfg.pools = {{kFp16, 4096, 48}, {kFp8, 2048, 48}, {kInt4, 1088, 64}};
  HeteroBlockTable t(cfg);
  Mirror m;
  ExecDelta d;
  std::mt19937 rng(20261011);
  auto pick = [&](std::size_t n) { return static_cast<std::size_t>(rng() % n); };
  const std::array<FormatId, 3> formats{kFp16, kFp8, kInt4};
  const std::array<Residency, 3> res{Residency::kDevice, Residency::kHost, Residency::kDropped};
  std::vector<SequenceHandle> seqs;
  std::vector<BlockHandle> transcoding;
  auto random_block = [&]() -> BlockHandle {
    if (seqs.empty()) return kInvalidBlock;
    const Result<std::span<const std::uint32_t>> r = t.sequence_block_ids(seqs[pick(seqs.size())]);
    const auto ids = r.value();
    return ids.empty() ? kInvalidBlock : t.handle_of(ids[pick(ids.size())]);
  };
  std::size_t comparisons = 0;
  for (int step = 0; step < 20000; ++step) {
    switch (pick(11)) {
      case 0:
        if (auto s = t.create_sequence(); s.ok()) seqs.push_back(s.value());
        break;
      case 1: case 2:
        if (!seqs.empty()) (void)t.append_block(seqs[pick(seqs.size())], req(formats[pick(3)], 16));
        break;
      case 3:
        if (const BlockHandle h = random_block(); h != kInvalidBlock) {
          (void)t.seal(h);
          (void)t.append_shared_block(seqs[pick(seqs.size())], h);
        }
        break;
      case 4:
        if (const BlockHandle h = random_block(); h != kInvalidBlock) {
          (void)t.seal(h);
          if (t.begin_format_change(h, formats[pick(3)]).ok()) transcoding.push_back(h);
        }
        break;
      case 5:
        if (!transcoding.empty()) {
          const std::size_t i = pick(transcoding.size());
          const Status s = pick(2) == 0 ? t.commit_format_change(transcoding[i], ScaleMode::kNone, 0)
                                        : t.abort_format_change(transcoding[i]);
          CHECK(s == Status::kOk);
          transcoding.erase(transcoding.begin() + static_cast<std::ptrdiff_t>(i));
        }
        break;
      case 6:
        if (const BlockHandle h = random_block(); h != kInvalidBlock) (void)t.set_residency(h, res[pick(3)]);
        break;
      case 7:
        if (const BlockHandle h = random_block(); h != kInvalidBlock) {
          (void)t.set_valid_tokens(h, static_cast<std::uint32_t>(pick(17)));
        }
        break;
      default:
        if (!seqs.empty()) {
          const std::size_t i = pick(seqs.size());
          const Status s = t.release_sequence(seqs[i]);
          CHECK(s == Status::kOk || s == Status::kInvalidState);
          if (s == Status::kOk) seqs.erase(seqs.begin() + static_cast<std::ptrdiff_t>(i));
        }
        break;
    }
    if (step % 97 == 0) CHECK(t.validate().ok());
    if (pick(23) == 0) {
      t.collect_delta(d);
      CHECK(m.apply(d) && m.matches(t));
      std::vector<SequenceSegment> segs;
      CHECK(t.batch_segments(seqs, segs) == Status::kOk);
      for (std::size_t i = 0; i < seqs.size(); ++i) CHECK(m.read(segs[i]) == device_view(t, seqs[i]));
      ExecTable ref;
      if (t.build_exec_table(seqs, ref) == Status::kOk) {
        std::vector<BlockExecDescriptor> seen;
        for (const SequenceSegment& s : segs) for (const auto& x : m.read(s)) seen.push_back(x);
        CHECK(seen == ref.blocks);
        ++comparisons;
      }
    }
  }
  CHECK(comparisons > 10);
  for (const BlockHandle h : transcoding) CHECK(t.abort_format_change(h) == Status::kOk);
  for (const SequenceHandle s : seqs) CHECK(t.release_sequence(s) == Status::kOk);
  CHECK(t.blocks_in_use() == 0 && t.free_slots(kFp16) == 48 && t.free_slots(kFp8) == 48);
  CHECK(t.free_slots(kInt4) == 64);
  t.collect_delta(d);
  CHECK(m.apply(d) && m.matches(t) && t.validate().ok());
}

}  // namespace

int main() {
  for (const Case& c : cases()) {
    g_current = c.name;
    const int before = g_failures;
    c.fn();
    if (g_failures == before) std::printf("ok %s\n", c.name);
  }
  std::printf("%zu cases, %d failures\n", cases().size(), g_failures);
  return g_failures == 0 ? 0 : 1;
}
