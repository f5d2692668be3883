// HeteroBlockTable (see include/hl_allocator/hetero_block_table.hpp).
//
// The observable contract follows the reference's
// project1_allocator/src/hetero_block_table.cpp: LIFO free lists primed so the
// first pops return 0, 1, 2, ...; the check order of every call (hence which
// Status wins when several apply); the first delta carrying every record; the
// descriptor dirty list reported in marking order; and device_descriptor()'s
// non-executable form (format 15, slot 0xFFFFFFFF, block_id kept, the other
// info bits and scale_ref of the host record kept).  oracle/table_trace.cpp
// replays the same seeded call stream on both implementations and compares
// every word.
#include "hl_allocator/hetero_block_table.hpp"
#include "hl_allocator/snapshot_io.hpp"

#include <algorithm>
#include <cstring>
#include <limits>
#include <stdexcept>

namespace hl::alloc {
namespace {

constexpr std::uint32_t kIdLimit = 0xFFFF'FFFEu;  // 0xFFFFFFFF is the invalid id

constexpr std::uint32_t raw(FormatId f) noexcept { return static_cast<std::uint32_t>(f); }
constexpr bool scale_mode_ok(ScaleMode m) noexcept { return static_cast<std::uint32_t>(m) <= 3u; }
constexpr bool residency_ok(Residency r) noexcept { return static_cast<std::uint32_t>(r) <= 2u; }

// A LIFO stack whose pops yield 0, 1, ..., count-1 first.
void prime_lifo(std::vector<std::uint32_t>& stack, std::uint32_t count) {
  stack.clear();
  stack.reserve(count);
  for (std::uint32_t v = count; v-- > 0;) stack.push_back(v);
}

ValidationReport corrupt(std::string what) { return {Status::kCorrupt, std::move(what)}; }

}  // namespace

Status HeteroBlockTable::validate_config(const TableConfig& config) noexcept {
  if (config.max_blocks == 0 || config.max_blocks > kIdLimit) return Status::kInvalidArgument;
  if (config.block_tokens == 0 || config.block_tokens > kMaxBlockTokens) {
    return Status::kInvalidArgument;
  }
  if (config.pools.empty()) return Status::kInvalidArgument;
  std::array<bool, kMaxFormats> used{};
  for (const PoolConfig& p : config.pools) {
    if (raw(p.format) >= kMaxFormats) return Status::kUnknownFormat;
    if (used[raw(p.format)]) return Status::kInvalidArgument;
    used[raw(p.format)] = true;
    if (p.slot_bytes == 0 || p.num_slots == 0 || p.num_slots > kIdLimit) {
      return Status::kInvalidArgument;
    }
  }
  return Status::kOk;
}

HeteroBlockTable::HeteroBlockTable(const TableConfig& config) : block_tokens_(config.block_tokens) {
  if (const Status s = validate_config(config); s != Status::kOk) {
    throw std::invalid_argument(std::string("HeteroBlockTable: invalid TableConfig: ") +
                                to_string(s));
  }
  records_.resize(config.max_blocks);
  for (std::uint32_t id = 0; id < config.max_blocks; ++id) reset_record(id, 0);
  prime_lifo(free_ids_, config.max_blocks);
  // The device table starts as garbage: the first delta must carry every record.
  is_dirty_.assign(config.max_blocks, 1);
  dirty_ids_.reserve(config.max_blocks);
  for (std::uint32_t id = 0; id < config.max_blocks; ++id) dirty_ids_.push_back(id);
  for (const PoolConfig& pc : config.pools) {
    SlotPool& p = pools_[raw(pc.format)];
    p.present = true;
    p.slot_bytes = pc.slot_bytes;
    p.capacity = pc.num_slots;
    prime_lifo(p.lifo, pc.num_slots);
  }
}

// ---- helpers ---------------------------------------------------------------------------

HeteroBlockTable::SlotPool* HeteroBlockTable::pool(FormatId f) noexcept {
  return raw(f) < kMaxFormats && pools_[raw(f)].present ? &pools_[raw(f)] : nullptr;
}
const HeteroBlockTable::SlotPool* HeteroBlockTable::pool(FormatId f) const noexcept {
  return raw(f) < kMaxFormats && pools_[raw(f)].present ? &pools_[raw(f)] : nullptr;
}

Status HeteroBlockTable::verify(BlockHandle h) const noexcept {
  if (h.id >= records_.size()) return Status::kInvalidHandle;
  const BlockDescriptor& d = records_[h.id];
  return d.generation == h.generation && d.state() != BlockState::kFree ? Status::kOk
                                                                         : Status::kStaleHandle;
}

Status HeteroBlockTable::verify(SequenceHandle s) const noexcept {
  if (s.id >= seqs_.size()) return Status::kInvalidHandle;
  const Seq& q = seqs_[s.id];
  return q.live && q.generation == s.generation ? Status::kOk : Status::kStaleHandle;
}

Status HeteroBlockTable::verify(const AllocRequest& r) const noexcept {
  if (pool(r.format) == nullptr) return Status::kUnknownFormat;
  if (r.valid_tokens > block_tokens_ || r.layout > kMaxLayoutId || !scale_mode_ok(r.scale_mode)) {
    return Status::kInvalidArgument;
  }
  return Status::kOk;
}

void HeteroBlockTable::reset_record(std::uint32_t id, std::uint32_t generation) noexcept {
  BlockDescriptor d{};
  d.exec.slot = kNoSlot;
  d.exec.block_id = id;
  d.exec.set_format(kInvalidFormat);
  d.generation = generation;
  d.set_state(BlockState::kFree);
  d.set_pending_format(kInvalidFormat);
  d.pending_slot = kNoSlot;
  records_[id] = d;
}

void HeteroBlockTable::touch(std::uint32_t id) noexcept {
  if (is_dirty_[id]) return;
  is_dirty_[id] = 1;
  dirty_ids_.push_back(id);  // capacity == max_blocks, never reallocates
}

void HeteroBlockTable::retire(std::uint32_t id) noexcept {
  const BlockDescriptor d = records_[id];
  // The stacks were reserved to their pool size, so these pushes never allocate.
  if (SlotPool* p = pool(d.exec.format()); p != nullptr && d.exec.slot != kNoSlot) {
    p->lifo.push_back(d.exec.slot);
  }
  if (SlotPool* p = pool(d.pending_format()); p != nullptr && d.pending_slot != kNoSlot) {
    p->lifo.push_back(d.pending_slot);
  }
  reset_record(id, d.generation + 1u);  // the generation wraps at 2^32 by design
  free_ids_.push_back(id);
  in_use_ -= 1;
  touch(id);
}

void HeteroBlockTable::drop_reference(std::uint32_t id) noexcept {
  BlockDescriptor& d = records_[id];
  if (d.refcount() == 1) {
    retire(id);
  } else {
    d.set_refcount(d.refcount() - 1);
  }
}

// ---- blocks ------------------------------------------------------------------------------

Result<BlockHandle> HeteroBlockTable::allocate(const AllocRequest& request) {
  if (const Status s = verify(request); s != Status::kOk) return s;
  if (free_ids_.empty()) return Status::kOutOfBlocks;
  SlotPool& p = *pool(request.format);
  if (p.lifo.empty()) return Status::kOutOfSlots;

  const std::uint32_t id = free_ids_.back();
  free_ids_.pop_back();
  const std::uint32_t slot = p.lifo.back();
  p.lifo.pop_back();

  BlockDescriptor& d = records_[id];
  d.exec.slot = slot;
  d.exec.info = BlockExecDescriptor::pack_info(request.format, request.scale_mode, request.layout,
                                               request.valid_tokens);
  d.exec.scale_ref = request.scale_ref;
  d.control = 0;
  d.set_state(BlockState::kOpen);
  d.set_residency(Residency::kDevice);
  d.set_pending_format(kInvalidFormat);
  d.set_refcount(1);
  d.pending_slot = kNoSlot;
  d.reserved = 0;
  in_use_ += 1;
  touch(id);
  return BlockHandle{id, d.generation};
}

Status HeteroBlockTable::retain(BlockHandle handle) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  BlockDescriptor& d = records_[handle.id];
  if (d.refcount() >= kMaxRefcount) return Status::kRefcountOverflow;
  d.set_refcount(d.refcount() + 1);
  return Status::kOk;
}

Status HeteroBlockTable::release(BlockHandle handle) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  const BlockDescriptor& d = records_[handle.id];
  // The last reference of a block being transcoded must wait for commit/abort:
  // a conversion kernel may still read the old slot.
  if (d.refcount() == 1 && d.state() == BlockState::kTranscoding) return Status::kInvalidState;
  drop_reference(handle.id);
  return Status::kOk;
}

Status HeteroBlockTable::set_valid_tokens(BlockHandle handle, std::uint32_t valid_tokens) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() != BlockState::kOpen) return Status::kInvalidState;
  if (valid_tokens > block_tokens_) return Status::kInvalidArgument;
  d.exec.set_valid_tokens(valid_tokens);
  touch(handle.id);
  return Status::kOk;
}

Status HeteroBlockTable::seal(BlockHandle handle) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() != BlockState::kOpen) return Status::kInvalidState;
  d.set_state(BlockState::kSealed);  // host-only: no device change
  return Status::kOk;
}

Status HeteroBlockTable::set_residency(BlockHandle handle, Residency residency) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  if (!residency_ok(residency)) return Status::kInvalidArgument;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() == BlockState::kTranscoding) return Status::kInvalidState;
  d.set_residency(residency);
  touch(handle.id);  // the device record becomes executable or not
  return Status::kOk;
}

Status HeteroBlockTable::set_scale(BlockHandle handle, ScaleMode mode, std::uint32_t scale_ref) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  if (!scale_mode_ok(mode)) return Status::kInvalidArgument;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() == BlockState::kTranscoding) return Status::kInvalidState;
  d.exec.set_scale_mode(mode);
  d.exec.scale_ref = scale_ref;
  touch(handle.id);
  return Status::kOk;
}

Result<FormatChange> HeteroBlockTable::begin_format_change(BlockHandle handle, FormatId target) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() != BlockState::kSealed) return Status::kInvalidState;
  if (d.residency() != Residency::kDevice) return Status::kNotDeviceResident;
  SlotPool* to = pool(target);
  if (to == nullptr) return Status::kUnknownFormat;
  if (target == d.exec.format()) return Status::kInvalidArgument;
  if (to->lifo.empty()) return Status::kOutOfSlots;
  const std::uint32_t to_slot = to->lifo.back();
  to->lifo.pop_back();
  d.pending_slot = to_slot;
  d.set_pending_format(target);
  d.set_state(BlockState::kTranscoding);
  return FormatChange{d.exec.format(), d.exec.slot, target, to_slot};
}

Status HeteroBlockTable::commit_format_change(BlockHandle handle, ScaleMode mode,
                                              std::uint32_t scale_ref) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  if (!scale_mode_ok(mode)) return Status::kInvalidArgument;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() != BlockState::kTranscoding) return Status::kInvalidState;
  pool(d.exec.format())->lifo.push_back(d.exec.slot);
  d.exec.slot = d.pending_slot;
  d.exec.set_format(d.pending_format());
  d.exec.set_scale_mode(mode);
  d.exec.scale_ref = scale_ref;
  d.pending_slot = kNoSlot;
  d.set_pending_format(kInvalidFormat);
  d.set_state(BlockState::kSealed);
  committed_changes_ += 1;
  touch(handle.id);
  return Status::kOk;
}

Status HeteroBlockTable::abort_format_change(BlockHandle handle) {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  BlockDescriptor& d = records_[handle.id];
  if (d.state() != BlockState::kTranscoding) return Status::kInvalidState;
  pool(d.pending_format())->lifo.push_back(d.pending_slot);
  d.pending_slot = kNoSlot;
  d.set_pending_format(kInvalidFormat);
  d.set_state(BlockState::kSealed);
  return Status::kOk;
}

Result<BlockDescriptor> HeteroBlockTable::lookup(BlockHandle handle) const {
  if (const Status s = verify(handle); s != Status::kOk) return s;
  return records_[handle.id];
}

Status HeteroBlockTable::lookup_batch(std::span<const BlockHandle> handles,
                                      std::span<BlockExecDescriptor> out) const {
  if (out.size() < handles.size()) return Status::kInvalidArgument;
  for (std::size_t k = 0; k < handles.size(); ++k) {
    if (const Status s = verify(handles[k]); s != Status::kOk) return s;
    const BlockDescriptor& d = records_[handles[k].id];
    if (d.residency() != Residency::kDevice) return Status::kNotDeviceResident;
    out[k] = d.exec;
  }
  return Status::kOk;
}

BlockHandle HeteroBlockTable::handle_of(std::uint32_t block_id) const noexcept {
  if (block_id >= records_.size() || records_[block_id].state() == BlockState::kFree) {
    return kInvalidBlock;
  }
  return BlockHandle{block_id, records_[block_id].generation};
}

// ---- sequences ---------------------------------------------------------------------------

Result<SequenceHandle> HeteroBlockTable::create_sequence() {
  std::uint32_t id;
  if (!free_seqs_.empty()) {
    id = free_seqs_.back();
    free_seqs_.pop_back();
  } else {
    if (seqs_.size() >= kIdLimit) return Status::kCapacityExceeded;
    // release_sequence() must never allocate: keep room to park every sequence.
    if (free_seqs_.capacity() < seqs_.size() + 1) {
      free_seqs_.reserve(std::max<std::size_t>(8, 2 * (seqs_.size() + 1)));
    }
    id = static_cast<std::uint32_t>(seqs_.size());
    seqs_.emplace_back();
  }
  Seq& q = seqs_[id];
  q.live = true;
  q.seg = IdArena::Segment{};  // storage comes with the first append
  return SequenceHandle{id, q.generation};
}

Result<BlockHandle> HeteroBlockTable::append_block(SequenceHandle seq, const AllocRequest& request) {
  if (const Status s = verify(seq); s != Status::kOk) return s;
  IdArena::Segment& seg = seqs_[seq.id].seg;
  // Room first (may move the segment or throw); nothing can fail after allocate().
  if (const Status s = arena_.reserve(seg, seg.length + 1); s != Status::kOk) return s;
  Result<BlockHandle> block = allocate(request);
  if (!block.ok()) return block.status();
  arena_.push_back(seg, block.value().id);
  return block;
}

Status HeteroBlockTable::append_shared_block(SequenceHandle seq, BlockHandle block) {
  if (const Status s = verify(seq); s != Status::kOk) return s;
  if (const Status s = verify(block); s != Status::kOk) return s;
  // Open blocks still receive appends; only immutable ones may be shared.
  if (records_[block.id].state() == BlockState::kOpen) return Status::kInvalidState;
  IdArena::Segment& seg = seqs_[seq.id].seg;
  if (const Status s = arena_.reserve(seg, seg.length + 1); s != Status::kOk) return s;
  if (const Status s = retain(block); s != Status::kOk) return s;
  arena_.push_back(seg, block.id);
  return Status::kOk;
}

Status HeteroBlockTable::release_sequence(SequenceHandle seq) {
  if (const Status s = verify(seq); s != Status::kOk) return s;
  Seq& q = seqs_[seq.id];
  const std::span<const std::uint32_t> ids = arena_.view(q.seg);
  // All-or-nothing: check before changing anything.
  const bool busy = std::any_of(ids.begin(), ids.end(), [&](std::uint32_t id) {
    return records_[id].state() == BlockState::kTranscoding;
  });
  if (busy) return Status::kInvalidState;
  for (const std::uint32_t id : ids) drop_reference(id);
  arena_.release(q.seg);
  q.live = false;
  q.generation += 1;
  free_seqs_.push_back(seq.id);
  return Status::kOk;
}

Status HeteroBlockTable::append_tokens(std::span<const SequenceHandle> seqs,
                                       std::span<const FormatId> new_formats, std::uint32_t layout,
                                       std::span<TokenTarget> out, std::size_t& n_done) {
  n_done = 0;
  const std::size_t n = seqs.size();
  if (new_formats.size() < n || out.size() < n) return Status::kInvalidArgument;
  // Each sequence is a chain of dependent random reads (its Seq record, the arena entry of
  // its tail, the tail's record and dirty flag).  Prefetches for sequences further ahead, one
  // link of the chain per distance, keep several chains' misses in flight at once.
  constexpr std::size_t kAheadSeq = 24, kAheadTail = 16, kAheadRecord = 8;
  auto seq_at = [&](std::size_t k) -> const Seq* {
    const std::uint32_t id = seqs[k].id;
    return id < seqs_.size() ? &seqs_[id] : nullptr;
  };
  auto tail_of = [&](const Seq* q) -> const std::uint32_t* {
    return q != nullptr && q->seg.capacity > 0 && q->seg.length > 0
               ? arena_.view(q->seg).data() + (q->seg.length - 1)
               : nullptr;
  };
  for (std::size_t i = 0; i < n; ++i) {
    if (i + kAheadSeq < n) {
      if (const Seq* q = seq_at(i + kAheadSeq)) __builtin_prefetch(q);
    }
    if (i + kAheadTail < n) {
      if (const std::uint32_t* t = tail_of(seq_at(i + kAheadTail))) __builtin_prefetch(t);
    }
    if (i + kAheadRecord < n) {
      if (const std::uint32_t* t = tail_of(seq_at(i + kAheadRecord)); t != nullptr && *t < records_.size()) {
        __builtin_prefetch(&records_[*t], 1);
        __builtin_prefetch(&is_dirty_[*t], 1);
      }
    }

    const SequenceHandle sh = seqs[i];
    if (const Status s = verify(sh); s != Status::kOk) return s;
    if (const std::uint32_t* t = tail_of(&seqs_[sh.id]); t != nullptr) {
      const std::uint32_t tail = *t;
      // lookup(handle_of(tail)): a free (or out-of-range) tail is an invalid handle.
      if (tail >= records_.size() || records_[tail].state() == BlockState::kFree) return Status::kInvalidHandle;
      BlockDescriptor& d = records_[tail];
      const std::uint32_t vt = d.exec.valid_tokens();
      if (vt < block_tokens_) {
        if (d.state() != BlockState::kOpen) return Status::kInvalidState;  // set_valid_tokens
        d.exec.set_valid_tokens(vt + 1);
        touch(tail);
        out[i] = TokenTarget{tail, vt};
        n_done = i + 1;
        continue;
      }
    }
    AllocRequest req;
    req.format = new_formats[i];
    req.valid_tokens = 1;
    req.layout = layout;
    const Result<BlockHandle> r = append_block(sh, req);
    if (!r.ok()) return r.status();
    out[i] = TokenTarget{r.value().id, 0};
    n_done = i + 1;
  }
  return Status::kOk;
}

Result<std::span<const std::uint32_t>> HeteroBlockTable::sequence_block_ids(
    SequenceHandle seq) const {
  if (const Status s = verify(seq); s != Status::kOk) return s;
  return arena_.view(seqs_[seq.id].seg);
}

Status HeteroBlockTable::build_exec_table(std::span<const SequenceHandle> seqs,
                                          ExecTable& out) const {
  out.indptr.clear();
  out.blocks.clear();
  std::uint64_t total = 0;
  for (const SequenceHandle s : seqs) {
    if (const Status st = verify(s); st != Status::kOk) return st;
    total += seqs_[s.id].seg.length;
  }
  if (total > std::numeric_limits<std::uint32_t>::max()) return Status::kInvalidArgument;
  out.indptr.reserve(seqs.size() + 1);
  out.blocks.reserve(total);
  out.indptr.push_back(0);
  for (const SequenceHandle s : seqs) {
    for (const std::uint32_t id : arena_.view(seqs_[s.id].seg)) {
      const BlockDescriptor& d = records_[id];
      if (d.residency() != Residency::kDevice) {
        out.indptr.clear();
        out.blocks.clear();
        return Status::kNotDeviceResident;
      }
      out.blocks.push_back(d.exec);
    }
    out.indptr.push_back(static_cast<std::uint32_t>(out.blocks.size()));
  }
  return Status::kOk;
}

// ---- device-facing state -----------------------------------------------------------------

Status HeteroBlockTable::batch_segments(std::span<const SequenceHandle> seqs,
                                        std::vector<SequenceSegment>& out) const {
  out.clear();
  out.reserve(seqs.size());
  for (const SequenceHandle s : seqs) {
    if (const Status st = verify(s); st != Status::kOk) {
      out.clear();
      return st;
    }
    out.push_back(IdArena::kernel_view(seqs_[s.id].seg));
  }
  return Status::kOk;
}

void HeteroBlockTable::collect_delta(ExecDelta& out) {
  out.descriptor_patches.clear();
  out.descriptor_patches.reserve(dirty_ids_.size());  // may throw; nothing changed yet
  arena_.collect(out.id_patches);                      // strong guarantee
  for (const std::uint32_t id : dirty_ids_) {
    out.descriptor_patches.push_back(device_descriptor(id));
    is_dirty_[id] = 0;
  }
  dirty_ids_.clear();
  out.descriptor_table_size = max_blocks();
  out.arena_size = arena_.size();
}

BlockExecDescriptor HeteroBlockTable::device_descriptor(std::uint32_t block_id) const noexcept {
  BlockExecDescriptor e{};
  if (block_id < records_.size()) {
    const BlockDescriptor& d = records_[block_id];
    e = d.exec;
    if (d.state() != BlockState::kFree && d.residency() == Residency::kDevice) return e;
  }
  e.slot = kNoSlot;  // kernels must never dereference this record
  e.set_format(kInvalidFormat);
  e.block_id = block_id;
  return e;
}

// ---- introspection -----------------------------------------------------------------------

bool HeteroBlockTable::has_pool(FormatId format) const noexcept { return pool(format) != nullptr; }

std::uint32_t HeteroBlockTable::free_slots(FormatId format) const noexcept {
  const SlotPool* p = pool(format);
  return p ? static_cast<std::uint32_t>(p->lifo.size()) : 0u;
}

std::uint32_t HeteroBlockTable::pool_slots(FormatId format) const noexcept {
  const SlotPool* p = pool(format);
  return p ? p->capacity : 0u;
}

std::uint32_t HeteroBlockTable::slot_bytes(FormatId format) const noexcept {
  const SlotPool* p = pool(format);
  return p ? p->slot_bytes : 0u;
}

TableStats HeteroBlockTable::stats() const {
  TableStats st;
  st.blocks_capacity = max_blocks();
  st.format_changes_committed = committed_changes_;
  for (const BlockDescriptor& d : records_) {
    st.blocks_per_state[static_cast<std::size_t>(d.state())] += 1;
    if (d.state() == BlockState::kFree) continue;
    st.blocks_in_use += 1;
    st.blocks_per_format[raw(d.exec.format())] += 1;
    st.blocks_per_residency[static_cast<std::size_t>(d.residency())] += 1;
    st.valid_tokens += d.exec.valid_tokens();
    st.payload_bytes_in_use += slot_bytes(d.exec.format());
    if (d.state() == BlockState::kTranscoding) st.payload_bytes_in_use += slot_bytes(d.pending_format());
  }
  st.token_capacity_in_use = std::uint64_t{st.blocks_in_use} * block_tokens_;
  for (const Seq& q : seqs_) {
    st.active_sequences += q.live ? 1u : 0u;
    st.arena_live_entries += q.seg.length;
    st.arena_reserved_entries += q.seg.capacity;
  }
  st.arena_entries = arena_.size();
  st.arena_free_entries = arena_.free_entries();
  st.pending_descriptor_patches = dirty_ids_.size();
  st.pending_id_patches = arena_.pending_patches();
  return st;
}

// ---- snapshot ------------------------------------------------------------------------
//
// Image layout (host byte order; u32 lists are a count then the values):
//   u64 magic "HLKVSNAP", u32 image version, u32 ABI version,
//   u32 max_blocks, u32 block_tokens, u32 blocks in use, u64 committed format changes,
//   u32 pool count, per pool {u32 format, u32 slot_bytes, u32 capacity, u32 list free slots},
//   the block records (32 B each), u32 list free block ids,
//   u32 sequence count, per sequence {u32 offset, capacity, length, generation, live},
//   u32 list free sequence ids, the id arena (IdArena::snapshot),
//   u64 FNV-1a checksum of everything before it.

namespace {
constexpr std::uint64_t kSnapshotMagic = 0x50414E53564B4C48ull;  // bytes "HLKVSNAP" little-endian
constexpr std::uint32_t kSnapshotVersion = 1;
constexpr std::size_t kSeqBytes = 5 * sizeof(std::uint32_t);
}  // namespace

std::vector<std::byte> HeteroBlockTable::snapshot() const {
  std::vector<std::byte> out;
  detail::SnapshotWriter w(out);
  w.u64(kSnapshotMagic);
  w.u32(kSnapshotVersion);
  w.u32(kAbiVersion);
  w.u32(static_cast<std::uint32_t>(records_.size()));
  w.u32(block_tokens_);
  w.u32(in_use_);
  w.u64(committed_changes_);
  std::uint32_t n_pools = 0;
  for (const SlotPool& p : pools_) n_pools += p.present ? 1u : 0u;
  w.u32(n_pools);
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    const SlotPool& p = pools_[f];
    if (!p.present) continue;
    w.u32(f);
    w.u32(p.slot_bytes);
    w.u32(p.capacity);
    w.u32s(p.lifo);
  }
  w.bytes(records_.data(), records_.size() * sizeof(BlockDescriptor));
  w.u32s(free_ids_);
  w.u32(static_cast<std::uint32_t>(seqs_.size()));
  for (const Seq& q : seqs_) {
    w.u32(q.seg.offset);
    w.u32(q.seg.capacity);
    w.u32(q.seg.length);
    w.u32(q.generation);
    w.u32(q.live ? 1u : 0u);
  }
  w.u32s(free_seqs_);
  arena_.snapshot(w);
  w.u64(detail::snapshot_checksum(out));
  return out;
}

Status HeteroBlockTable::restore(std::span<const std::byte> image, std::unique_ptr<HeteroBlockTable>& out) {
  constexpr std::size_t kSum = sizeof(std::uint64_t);
  if (image.size() < kSum) return Status::kCorrupt;
  const std::span<const std::byte> body = image.first(image.size() - kSum);
  std::uint64_t sum = 0;
  std::memcpy(&sum, image.data() + body.size(), kSum);
  if (sum != detail::snapshot_checksum(body)) return Status::kCorrupt;

  detail::SnapshotReader r(body);
  std::uint64_t magic = 0, committed = 0;
  std::uint32_t version = 0, abi = 0, max_blocks = 0, block_tokens = 0, in_use = 0, n_pools = 0;
  if (!r.u64(magic) || magic != kSnapshotMagic || !r.u32(version) || version != kSnapshotVersion ||
      !r.u32(abi) || abi != kAbiVersion || !r.u32(max_blocks) || !r.u32(block_tokens) || !r.u32(in_use) ||
      !r.u64(committed) || !r.u32(n_pools) || n_pools > kMaxFormats) {
    return Status::kCorrupt;
  }
  TableConfig config;
  config.max_blocks = max_blocks;
  config.block_tokens = block_tokens;
  std::array<std::vector<std::uint32_t>, kMaxFormats> lifos;
  for (std::uint32_t i = 0; i < n_pools; ++i) {
    std::uint32_t f = 0, slot_bytes = 0, capacity = 0;
    if (!r.u32(f) || f >= kMaxFormats || !r.u32(slot_bytes) || !r.u32(capacity) || !r.u32s(lifos[f], capacity)) {
      return Status::kCorrupt;
    }
    config.pools.push_back(PoolConfig{FormatId{static_cast<std::uint8_t>(f)}, slot_bytes, capacity});
  }
  if (validate_config(config) != Status::kOk) return Status::kCorrupt;
  // The records are in the image: bound the allocation by it.
  if (std::size_t{max_blocks} * sizeof(BlockDescriptor) > r.remaining()) return Status::kCorrupt;
  auto t = std::make_unique<HeteroBlockTable>(config);
  if (!r.bytes(t->records_.data(), std::size_t{max_blocks} * sizeof(BlockDescriptor)) ||
      !r.u32s(t->free_ids_, max_blocks)) {
    return Status::kCorrupt;
  }
  t->free_ids_.reserve(max_blocks);
  for (const PoolConfig& pc : config.pools) {
    SlotPool& p = t->pools_[raw(pc.format)];
    p.lifo = std::move(lifos[raw(pc.format)]);
    p.lifo.reserve(p.capacity);  // the stacks never allocate when slots come back
  }
  std::uint32_t n_seqs = 0;
  if (!r.u32(n_seqs) || std::size_t{n_seqs} * kSeqBytes > r.remaining()) return Status::kCorrupt;
  t->seqs_.resize(n_seqs);
  for (Seq& q : t->seqs_) {
    std::uint32_t live = 0;
    if (!r.u32(q.seg.offset) || !r.u32(q.seg.capacity) || !r.u32(q.seg.length) || !r.u32(q.generation) ||
        !r.u32(live) || live > 1) {
      return Status::kCorrupt;
    }
    q.live = live != 0;
  }
  if (!r.u32s(t->free_seqs_, n_seqs) || !t->arena_.restore(r) || r.remaining() != 0) return Status::kCorrupt;
  t->in_use_ = in_use;
  t->committed_changes_ = committed;
  // A fresh table already lists every descriptor as pending; the arena's restore did the
  // same for every entry.
  if (!t->validate().ok()) return Status::kCorrupt;
  out = std::move(t);
  return Status::kOk;
}

ValidationReport HeteroBlockTable::validate() const {
  const std::size_t n = records_.size();
  std::vector<std::uint8_t> listed_free(n, 0);
  for (const std::uint32_t id : free_ids_) {
    if (id >= n || listed_free[id] || records_[id].state() != BlockState::kFree) {
      return corrupt("free id list entry " + std::to_string(id) + " is invalid");
    }
    listed_free[id] = 1;
  }

  std::array<std::vector<std::uint8_t>, kMaxFormats> owned;
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    const SlotPool& p = pools_[f];
    if (!p.present) continue;
    owned[f].assign(p.capacity, 0);
    for (const std::uint32_t s : p.lifo) {
      if (s >= p.capacity || owned[f][s]) {
        return corrupt("pool " + std::to_string(f) + " lists slot " + std::to_string(s) + " badly");
      }
      owned[f][s] = 1;
    }
  }
  auto own = [&](FormatId f, std::uint32_t slot, std::uint32_t id) -> std::string {
    const SlotPool* p = pool(f);
    if (p == nullptr) return "block " + std::to_string(id) + " has no pool";
    if (slot >= p->capacity) return "block " + std::to_string(id) + " slot out of range";
    std::uint8_t& o = owned[raw(f)][slot];
    if (o) return "slot " + std::to_string(slot) + " owned twice";
    o = 1;
    return {};
  };

  std::uint32_t counted = 0;
  for (std::uint32_t id = 0; id < n; ++id) {
    const BlockDescriptor& d = records_[id];
    if (d.exec.block_id != id) return corrupt("block " + std::to_string(id) + ": block_id field");
    if (d.state() == BlockState::kFree) {
      if (!listed_free[id]) return corrupt("block " + std::to_string(id) + ": free but unlisted");
      continue;
    }
    counted += 1;
    if (d.refcount() == 0) return corrupt("block " + std::to_string(id) + ": refcount 0");
    if (d.exec.info_reserved() || d.control_reserved() || d.reserved) {
      return corrupt("block " + std::to_string(id) + ": reserved bits set");
    }
    if (d.exec.valid_tokens() > block_tokens_) return corrupt("valid_tokens above block_tokens");
    if (!residency_ok(d.residency())) return corrupt("invalid residency");
    if (std::string e = own(d.exec.format(), d.exec.slot, id); !e.empty()) return corrupt(e);
    if (d.state() == BlockState::kTranscoding) {
      if (d.pending_format() == d.exec.format()) return corrupt("pending format == format");
      if (std::string e = own(d.pending_format(), d.pending_slot, id); !e.empty()) return corrupt(e);
    } else if (d.pending_slot != kNoSlot || d.pending_format() != kInvalidFormat) {
      return corrupt("pending slot outside a format change");
    }
  }
  if (counted != in_use_) return corrupt("blocks_in_use counter");
  if (free_ids_.size() + counted != n) return corrupt("free id list size");
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    if (pools_[f].present && std::find(owned[f].begin(), owned[f].end(), 0) != owned[f].end()) {
      return corrupt("pool " + std::to_string(f) + " leaked a slot");
    }
  }

  std::vector<std::uint32_t> seq_refs(n, 0);
  std::vector<IdArena::Segment> live;
  std::size_t parked = 0;
  for (std::size_t s = 0; s < seqs_.size(); ++s) {
    const Seq& q = seqs_[s];
    if (!q.live) {
      parked += 1;
      if (q.seg.capacity || q.seg.length) return corrupt("released sequence holds storage");
      continue;
    }
    live.push_back(q.seg);
    for (const std::uint32_t id : arena_.view(q.seg)) {
      if (id >= n || records_[id].state() == BlockState::kFree) {
        return corrupt("sequence " + std::to_string(s) + " references a free block");
      }
      seq_refs[id] += 1;
    }
  }
  for (std::uint32_t id = 0; id < n; ++id) {
    if (seq_refs[id] > records_[id].refcount()) return corrupt("sequence refs above refcount");
  }
  if (parked != free_seqs_.size()) return corrupt("sequence free list size");
  std::vector<std::uint8_t> seen(seqs_.size(), 0);
  for (const std::uint32_t s : free_seqs_) {
    if (s >= seqs_.size() || seqs_[s].live || seen[s]) return corrupt("sequence free list entry");
    seen[s] = 1;
  }
  if (std::string e = arena_.validate(live); !e.empty()) return corrupt(e);

  if (is_dirty_.size() != n || dirty_ids_.capacity() < n) return corrupt("dirty tracking size");
  std::vector<std::uint8_t> in_list(n, 0);
  for (const std::uint32_t id : dirty_ids_) {
    if (id >= n || !is_dirty_[id] || in_list[id]) return corrupt("dirty list entry");
    in_list[id] = 1;
  }
  if (static_cast<std::size_t>(std::count(is_dirty_.begin(), is_dirty_.end(), 1)) != dirty_ids_.size()) {
    return corrupt("dirty flag without a list entry");
  }
  return {};
}

}  // namespace hl::alloc
