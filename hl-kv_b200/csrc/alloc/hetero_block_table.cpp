// HeteroBlockTable (see include/hl_allocator/hetero_block_table.hpp).
//
// What is observable follows the reference (project1_allocator/src/hetero_block_table.cpp)
// and is pinned word for word by oracle/table_trace.cpp against the reference library:
// block ids, slots and sequence ids are reused last-freed-first and are first handed out
// as 0, 1, 2, ...; each call rejects with the same status when several problems apply;
// the first delta carries every descriptor in id order, later ones the changed
// descriptors in first-change order; device_descriptor() of a free or non-resident block
// is the record with format 15 and slot 0xFFFFFFFF.
//
// Storage is this library's own.  Every free list is a stack threaded through the free
// objects themselves (a free block record's `reserved` word, a slot's entry of its pool's
// `below` array, a released sequence's segment offset), sized once at construction, so no
// release path allocates.  Descriptor changes go through an epoch-stamped ChangeQueue,
// like the arena's.  Each block operation is one check-then-edit on its record
// (edit_block below), with the checks in the order the reference applies them.
#include "hl_allocator/hetero_block_table.hpp"
#include "hl_allocator/snapshot_io.hpp"

#include <algorithm>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <utility>

namespace hl::alloc {
namespace {

constexpr std::uint32_t kIdLimit = 0xFFFF'FFFEu;  // 0xFFFFFFFF is the invalid id

constexpr std::uint32_t fmt_index(FormatId f) noexcept { return static_cast<std::uint32_t>(f); }
constexpr bool valid_scale_mode(ScaleMode m) noexcept { return static_cast<std::uint32_t>(m) <= 3u; }
constexpr bool valid_residency(Residency r) noexcept { return static_cast<std::uint32_t>(r) <= 2u; }

ValidationReport corrupt(std::string what) { return {Status::kCorrupt, std::move(what)}; }

// Runs `edit` on the record of a live block, or returns the status that rejected its handle.
template <typename Edit>
Status edit_block(Status found, BlockDescriptor* d, Edit&& edit) {
  return found == Status::kOk ? edit(*d) : found;
}

}  // namespace

Status HeteroBlockTable::validate_config(const TableConfig& config) noexcept {
  if (config.max_blocks == 0 || config.max_blocks > kIdLimit) return Status::kInvalidArgument;
  if (config.block_tokens == 0 || config.block_tokens > kMaxBlockTokens) return Status::kInvalidArgument;
  if (config.pools.empty()) return Status::kInvalidArgument;
  std::uint32_t seen = 0;  // one bit per format (kMaxFormats <= 32)
  static_assert(kMaxFormats <= 32);
  for (const PoolConfig& pc : config.pools) {
    const std::uint32_t f = fmt_index(pc.format);
    if (f >= kMaxFormats) return Status::kUnknownFormat;
    if ((seen >> f) & 1u) return Status::kInvalidArgument;
    seen |= 1u << f;
    if (pc.slot_bytes == 0 || pc.num_slots == 0 || pc.num_slots > kIdLimit) return Status::kInvalidArgument;
  }
  return Status::kOk;
}

HeteroBlockTable::HeteroBlockTable(const TableConfig& config) : block_tokens_(config.block_tokens) {
  if (const Status s = validate_config(config); s != Status::kOk) {
    throw std::invalid_argument(std::string("HeteroBlockTable: invalid TableConfig: ") + to_string(s));
  }
  const std::uint32_t n = config.max_blocks;
  blocks_.resize(n);
  // Every id free, chained 0 -> 1 -> ... so that allocation hands them out in id order.
  for (std::uint32_t id = n; id-- > 0;) {
    init_free_record(id, 0);
    blocks_[id].reserved = free_block_top_;
    free_block_top_ = id;
  }
  for (const PoolConfig& pc : config.pools) {
    SlotStack& st = slots_[fmt_index(pc.format)];
    st.present = true;
    st.slot_bytes = pc.slot_bytes;
    st.capacity = pc.num_slots;
    st.below.resize(pc.num_slots);
    for (std::uint32_t s = pc.num_slots; s-- > 0;) push(st, s);
  }
  // The device copy starts undefined: the first delta carries every descriptor.
  changed_blocks_.grow(n);
  for (std::uint32_t id = 0; id < n; ++id) changed_blocks_.mark(id);
}

// ---- helpers ---------------------------------------------------------------------------

HeteroBlockTable::SlotStack* HeteroBlockTable::stack(FormatId f) noexcept {
  const std::uint32_t i = fmt_index(f);
  return i < kMaxFormats && slots_[i].present ? &slots_[i] : nullptr;
}
const HeteroBlockTable::SlotStack* HeteroBlockTable::stack(FormatId f) const noexcept {
  const std::uint32_t i = fmt_index(f);
  return i < kMaxFormats && slots_[i].present ? &slots_[i] : nullptr;
}

bool HeteroBlockTable::pop(SlotStack& st, std::uint32_t& slot) noexcept {
  if (st.top == kEnd) return false;
  slot = st.top;
  st.top = st.below[slot];
  st.depth -= 1;
  return true;
}

void HeteroBlockTable::push(SlotStack& st, std::uint32_t slot) noexcept {
  st.below[slot] = st.top;
  st.top = slot;
  st.depth += 1;
}

Status HeteroBlockTable::find(BlockHandle h, BlockDescriptor*& out) noexcept {
  const BlockDescriptor* c = nullptr;
  const Status s = std::as_const(*this).find(h, c);
  out = const_cast<BlockDescriptor*>(c);
  return s;
}

Status HeteroBlockTable::find(BlockHandle h, const BlockDescriptor*& out) const noexcept {
  if (h.id >= blocks_.size()) return Status::kInvalidHandle;
  const BlockDescriptor& d = blocks_[h.id];
  if (d.state() == BlockState::kFree || d.generation != h.generation) return Status::kStaleHandle;
  out = &d;
  return Status::kOk;
}

Status HeteroBlockTable::find(SequenceHandle h, SeqRecord*& out) noexcept {
  const SeqRecord* c = nullptr;
  const Status s = std::as_const(*this).find(h, c);
  out = const_cast<SeqRecord*>(c);
  return s;
}

Status HeteroBlockTable::find(SequenceHandle h, const SeqRecord*& out) const noexcept {
  if (h.id >= seq_records_.size()) return Status::kInvalidHandle;
  const SeqRecord& q = seq_records_[h.id];
  if (!q.live || q.generation != h.generation) return Status::kStaleHandle;
  out = &q;
  return Status::kOk;
}

Status HeteroBlockTable::admissible(const AllocRequest& r) const noexcept {
  if (stack(r.format) == nullptr) return Status::kUnknownFormat;
  const bool ok = r.valid_tokens <= block_tokens_ && r.layout <= kMaxLayoutId && valid_scale_mode(r.scale_mode);
  return ok ? Status::kOk : Status::kInvalidArgument;
}

// A free record: not executable (format 15, no slot), its id kept, everything else zero.
// The `reserved` word is set by whoever chains the record into the free ids.
void HeteroBlockTable::init_free_record(std::uint32_t id, std::uint32_t generation) noexcept {
  BlockDescriptor& d = blocks_[id];
  d = BlockDescriptor{};
  d.exec.slot = kNoSlot;
  d.exec.block_id = id;
  d.exec.set_format(kInvalidFormat);
  d.generation = generation;
  d.set_state(BlockState::kFree);
  d.set_pending_format(kInvalidFormat);
  d.pending_slot = kNoSlot;
}

// The last reference is gone: both slots (the current one and, if a change were in flight,
// the pending one) go back to their pools, the record becomes free under the next
// generation and its id goes on top of the free ids.
void HeteroBlockTable::free_block(std::uint32_t id) noexcept {
  const BlockDescriptor old = blocks_[id];
  if (SlotStack* st = stack(old.exec.format()); st != nullptr && old.exec.slot != kNoSlot) {
    push(*st, old.exec.slot);
  }
  if (SlotStack* st = stack(old.pending_format()); st != nullptr && old.pending_slot != kNoSlot) {
    push(*st, old.pending_slot);
  }
  init_free_record(id, old.generation + 1u);  // generations wrap at 2^32 by design
  blocks_[id].reserved = free_block_top_;
  free_block_top_ = id;
  in_use_ -= 1;
  changed_blocks_.mark(id);
}

// Drops one reference; the block is freed exactly when its count goes from 1 to 0.  (A
// record that misuse has already freed -- release() of a block a sequence still lists --
// only has its count field decremented when that sequence later lets go of it, as the
// reference does; it is never freed twice.)
void HeteroBlockTable::unreference(std::uint32_t id) noexcept {
  BlockDescriptor& d = blocks_[id];
  if (d.refcount() == 1) {
    free_block(id);
  } else {
    d.set_refcount(d.refcount() - 1);
  }
}

// ---- blocks ------------------------------------------------------------------------------

Result<BlockHandle> HeteroBlockTable::allocate(const AllocRequest& request) {
  if (const Status s = admissible(request); s != Status::kOk) return s;
  if (free_block_top_ == kEnd) return Status::kOutOfBlocks;
  SlotStack& st = *stack(request.format);
  std::uint32_t slot = 0;
  if (!pop(st, slot)) return Status::kOutOfSlots;
  const std::uint32_t id = free_block_top_;
  BlockDescriptor& d = blocks_[id];
  free_block_top_ = d.reserved;

  const std::uint32_t generation = d.generation;
  d = BlockDescriptor{};
  d.generation = generation;
  d.exec = BlockExecDescriptor{slot,
                               BlockExecDescriptor::pack_info(request.format, request.scale_mode,
                                                              request.layout, request.valid_tokens),
                               request.scale_ref, id};
  d.set_state(BlockState::kOpen);
  d.set_residency(Residency::kDevice);
  d.set_pending_format(kInvalidFormat);
  d.set_refcount(1);
  d.pending_slot = kNoSlot;
  in_use_ += 1;
  changed_blocks_.mark(id);
  return BlockHandle{id, generation};
}

Status HeteroBlockTable::retain(BlockHandle handle) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (b.refcount() >= kMaxRefcount) return Status::kRefcountOverflow;
    b.set_refcount(b.refcount() + 1);
    return Status::kOk;
  });
}

Status HeteroBlockTable::release(BlockHandle handle) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    // A block in a format change keeps its last reference until the change commits or
    // aborts: the transcoding kernel may still read the old slot.
    if (b.refcount() == 1 && b.state() == BlockState::kTranscoding) return Status::kInvalidState;
    unreference(handle.id);
    return Status::kOk;
  });
}

Status HeteroBlockTable::set_valid_tokens(BlockHandle handle, std::uint32_t valid_tokens) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (b.state() != BlockState::kOpen) return Status::kInvalidState;
    if (valid_tokens > block_tokens_) return Status::kInvalidArgument;
    b.exec.set_valid_tokens(valid_tokens);
    changed_blocks_.mark(handle.id);
    return Status::kOk;
  });
}

Status HeteroBlockTable::seal(BlockHandle handle) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (b.state() != BlockState::kOpen) return Status::kInvalidState;
    b.set_state(BlockState::kSealed);  // host bookkeeping only: the device record is unchanged
    return Status::kOk;
  });
}

Status HeteroBlockTable::set_residency(BlockHandle handle, Residency residency) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (!valid_residency(residency)) return Status::kInvalidArgument;
    if (b.state() == BlockState::kTranscoding) return Status::kInvalidState;
    b.set_residency(residency);
    changed_blocks_.mark(handle.id);  // executable on the device or not
    return Status::kOk;
  });
}

Status HeteroBlockTable::set_scale(BlockHandle handle, ScaleMode mode, std::uint32_t scale_ref) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (!valid_scale_mode(mode)) return Status::kInvalidArgument;
    if (b.state() == BlockState::kTranscoding) return Status::kInvalidState;
    b.exec.set_scale_mode(mode);
    b.exec.scale_ref = scale_ref;
    changed_blocks_.mark(handle.id);
    return Status::kOk;
  });
}

Result<FormatChange> HeteroBlockTable::begin_format_change(BlockHandle handle, FormatId target) {
  BlockDescriptor* d = nullptr;
  if (const Status s = find(handle, d); s != Status::kOk) return s;
  if (d->state() != BlockState::kSealed) return Status::kInvalidState;
  if (d->residency() != Residency::kDevice) return Status::kNotDeviceResident;
  SlotStack* to = stack(target);
  if (to == nullptr) return Status::kUnknownFormat;
  if (target == d->exec.format()) return Status::kInvalidArgument;
  std::uint32_t to_slot = 0;
  if (!pop(*to, to_slot)) return Status::kOutOfSlots;
  // Readers still see the old format and slot (no descriptor change) until the commit.
  d->pending_slot = to_slot;
  d->set_pending_format(target);
  d->set_state(BlockState::kTranscoding);
  return FormatChange{d->exec.format(), d->exec.slot, target, to_slot};
}

Status HeteroBlockTable::commit_format_change(BlockHandle handle, ScaleMode mode, std::uint32_t scale_ref) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (!valid_scale_mode(mode)) return Status::kInvalidArgument;
    if (b.state() != BlockState::kTranscoding) return Status::kInvalidState;
    push(*stack(b.exec.format()), b.exec.slot);  // the old payload's slot
    b.exec.slot = b.pending_slot;
    b.exec.set_format(b.pending_format());
    b.exec.set_scale_mode(mode);
    b.exec.scale_ref = scale_ref;
    b.pending_slot = kNoSlot;
    b.set_pending_format(kInvalidFormat);
    b.set_state(BlockState::kSealed);
    committed_changes_ += 1;
    changed_blocks_.mark(handle.id);
    return Status::kOk;
  });
}

Status HeteroBlockTable::abort_format_change(BlockHandle handle) {
  BlockDescriptor* d = nullptr;
  const Status found = find(handle, d);
  return edit_block(found, d, [&](BlockDescriptor& b) {
    if (b.state() != BlockState::kTranscoding) return Status::kInvalidState;
    push(*stack(b.pending_format()), b.pending_slot);
    b.pending_slot = kNoSlot;
    b.set_pending_format(kInvalidFormat);
    b.set_state(BlockState::kSealed);
    return Status::kOk;
  });
}

Result<BlockDescriptor> HeteroBlockTable::lookup(BlockHandle handle) const {
  const BlockDescriptor* d = nullptr;
  if (const Status s = find(handle, d); s != Status::kOk) return s;
  return *d;
}

Status HeteroBlockTable::lookup_batch(std::span<const BlockHandle> handles,
                                      std::span<BlockExecDescriptor> out) const {
  if (out.size() < handles.size()) return Status::kInvalidArgument;
  for (std::size_t k = 0; k < handles.size(); ++k) {
    const BlockDescriptor* d = nullptr;
    if (const Status s = find(handles[k], d); s != Status::kOk) return s;
    if (d->residency() != Residency::kDevice) return Status::kNotDeviceResident;
    out[k] = d->exec;
  }
  return Status::kOk;
}

BlockHandle HeteroBlockTable::handle_of(std::uint32_t block_id) const noexcept {
  const bool live = block_id < blocks_.size() && blocks_[block_id].state() != BlockState::kFree;
  return live ? BlockHandle{block_id, blocks_[block_id].generation} : kInvalidBlock;
}

// ---- sequences ---------------------------------------------------------------------------

Result<SequenceHandle> HeteroBlockTable::create_sequence() {
  std::uint32_t id = free_seq_top_;
  if (id != kEnd) {
    free_seq_top_ = seq_records_[id].seg.offset;
  } else {
    if (seq_records_.size() >= kIdLimit) return Status::kCapacityExceeded;
    id = static_cast<std::uint32_t>(seq_records_.size());
    seq_records_.emplace_back();  // may throw; nothing has changed yet
  }
  SeqRecord& q = seq_records_[id];
  q.seg = IdArena::Segment{};  // storage comes with the first block
  q.live = true;
  return SequenceHandle{id, q.generation};
}

Result<BlockHandle> HeteroBlockTable::append_block(SequenceHandle seq, const AllocRequest& request) {
  SeqRecord* q = nullptr;
  if (const Status s = find(seq, q); s != Status::kOk) return s;
  // The arena room comes first: it may move the segment (or throw) while nothing else has
  // changed, and once the block is allocated nothing can fail.
  if (const Status s = arena_.reserve(q->seg, q->seg.length + 1); s != Status::kOk) return s;
  const Result<BlockHandle> b = allocate(request);
  if (b.ok()) arena_.push_back(q->seg, b.value().id);
  return b;
}

Status HeteroBlockTable::append_shared_block(SequenceHandle seq, BlockHandle block) {
  SeqRecord* q = nullptr;
  if (const Status s = find(seq, q); s != Status::kOk) return s;
  BlockDescriptor* d = nullptr;
  if (const Status s = find(block, d); s != Status::kOk) return s;
  if (d->state() == BlockState::kOpen) return Status::kInvalidState;  // still being appended to
  if (const Status s = arena_.reserve(q->seg, q->seg.length + 1); s != Status::kOk) return s;
  if (const Status s = retain(block); s != Status::kOk) return s;
  arena_.push_back(q->seg, block.id);
  return Status::kOk;
}

Status HeteroBlockTable::release_sequence(SequenceHandle seq) {
  SeqRecord* q = nullptr;
  if (const Status s = find(seq, q); s != Status::kOk) return s;
  const std::span<const std::uint32_t> members = arena_.view(q->seg);
  // All or nothing: a member in a format change blocks the whole release.
  for (const std::uint32_t id : members) {
    if (blocks_[id].state() == BlockState::kTranscoding) return Status::kInvalidState;
  }
  for (const std::uint32_t id : members) unreference(id);
  arena_.release(q->seg);
  q->live = false;
  q->generation += 1;
  q->seg.offset = free_seq_top_;  // chain the id into the free sequence ids
  free_seq_top_ = seq.id;
  return Status::kOk;
}

Status HeteroBlockTable::append_tokens(std::span<const SequenceHandle> seqs, std::span<const FormatId> new_formats,
                                       std::uint32_t layout, std::span<TokenTarget> out, std::size_t& n_done) {
  n_done = 0;
  const std::size_t n = seqs.size();
  if (new_formats.size() < n || out.size() < n) return Status::kInvalidArgument;
  // Sequence i's work is a chain of dependent random reads: its record, the arena entry of
  // its last block, that block's record and change stamp.  Touching the links of the
  // sequences a few places ahead (each link at its own distance) keeps several chains'
  // cache misses in flight.
  auto tail_entry = [&](std::size_t k) -> const std::uint32_t* {
    const std::uint32_t sid = seqs[k].id;
    if (sid >= seq_records_.size()) return nullptr;
    const IdArena::Segment& g = seq_records_[sid].seg;
    return g.capacity != 0 && g.length != 0 ? arena_.view(g).data() + (g.length - 1) : nullptr;
  };
  for (std::size_t i = 0; i < n; ++i) {
    if (i + 24 < n && seqs[i + 24].id < seq_records_.size()) __builtin_prefetch(&seq_records_[seqs[i + 24].id]);
    if (i + 16 < n) {
      if (const std::uint32_t* t = tail_entry(i + 16)) __builtin_prefetch(t);
    }
    if (i + 8 < n) {
      if (const std::uint32_t* t = tail_entry(i + 8); t != nullptr && *t < blocks_.size()) {
        __builtin_prefetch(&blocks_[*t], 1);
      }
    }

    SeqRecord* q = nullptr;
    if (const Status s = find(seqs[i], q); s != Status::kOk) return s;
    const IdArena::Segment& g = q->seg;
    if (g.capacity != 0 && g.length != 0) {
      const std::uint32_t tail = arena_.view(g)[g.length - 1];
      // As lookup(handle_of(tail)): a free tail reads as an invalid handle.
      if (tail >= blocks_.size() || blocks_[tail].state() == BlockState::kFree) return Status::kInvalidHandle;
      BlockDescriptor& b = blocks_[tail];
      const std::uint32_t used = b.exec.valid_tokens();
      if (used < block_tokens_) {  // room in the tail: set_valid_tokens(tail, used + 1)
        if (b.state() != BlockState::kOpen) return Status::kInvalidState;
        b.exec.set_valid_tokens(used + 1);
        changed_blocks_.mark(tail);
        out[i] = TokenTarget{tail, used};
        n_done = i + 1;
        continue;
      }
    }
    AllocRequest next;
    next.format = new_formats[i];
    next.valid_tokens = 1;
    next.layout = layout;
    const Result<BlockHandle> b = append_block(seqs[i], next);
    if (!b.ok()) return b.status();
    out[i] = TokenTarget{b.value().id, 0};
    n_done = i + 1;
  }
  return Status::kOk;
}

Result<std::span<const std::uint32_t>> HeteroBlockTable::sequence_block_ids(SequenceHandle seq) const {
  const SeqRecord* q = nullptr;
  if (const Status s = find(seq, q); s != Status::kOk) return s;
  return arena_.view(q->seg);
}

Status HeteroBlockTable::build_exec_table(std::span<const SequenceHandle> seqs, ExecTable& out) const {
  out.indptr.clear();
  out.blocks.clear();
  // Every handle is checked before anything is built.
  std::uint64_t total = 0;
  for (const SequenceHandle h : seqs) {
    const SeqRecord* q = nullptr;
    if (const Status s = find(h, q); s != Status::kOk) return s;
    total += q->seg.length;
  }
  if (total > std::numeric_limits<std::uint32_t>::max()) return Status::kInvalidArgument;
  out.indptr.reserve(seqs.size() + 1);
  out.blocks.reserve(total);
  out.indptr.push_back(0);
  for (const SequenceHandle h : seqs) {
    for (const std::uint32_t id : arena_.view(seq_records_[h.id].seg)) {
      if (blocks_[id].residency() != Residency::kDevice) {
        out.indptr.clear();
        out.blocks.clear();
        return Status::kNotDeviceResident;
      }
      out.blocks.push_back(blocks_[id].exec);
    }
    out.indptr.push_back(static_cast<std::uint32_t>(out.blocks.size()));
  }
  return Status::kOk;
}

Status HeteroBlockTable::compact_arena(std::vector<SegmentMove>& moves) {
  std::vector<IdArena::Segment*> live;
  live.reserve(seq_records_.size());
  for (SeqRecord& q : seq_records_) {
    if (q.live) live.push_back(&q.seg);
  }
  return arena_.compact(live, moves);
}

// ---- device-facing state -----------------------------------------------------------------

Status HeteroBlockTable::batch_segments(std::span<const SequenceHandle> seqs,
                                        std::vector<SequenceSegment>& out) const {
  out.resize(seqs.size());
  std::size_t k = 0;
  for (const SequenceHandle h : seqs) {
    const SeqRecord* q = nullptr;
    const Status s = find(h, q);
    if (s != Status::kOk) {
      out.clear();  // all or nothing
      return s;
    }
    out[k++] = IdArena::kernel_view(q->seg);
  }
  return Status::kOk;
}

void HeteroBlockTable::collect_delta(ExecDelta& out) {
  // Both outputs are sized before either queue is drained, so a throw changes nothing.
  out.descriptor_patches.resize(changed_blocks_.size());
  arena_.collect(out.id_patches);
  std::size_t k = 0;
  changed_blocks_.drain([&](std::uint32_t id) noexcept { out.descriptor_patches[k++] = device_descriptor(id); });
  out.descriptor_table_size = max_blocks();
  out.arena_size = arena_.size();
}

BlockExecDescriptor HeteroBlockTable::device_descriptor(std::uint32_t block_id) const noexcept {
  BlockExecDescriptor e{};
  bool executable = false;
  if (block_id < blocks_.size()) {
    const BlockDescriptor& d = blocks_[block_id];
    e = d.exec;
    executable = d.state() != BlockState::kFree && d.residency() == Residency::kDevice;
  }
  if (!executable) {  // a record no kernel may follow: no slot, format 15
    e.slot = kNoSlot;
    e.set_format(kInvalidFormat);
    e.block_id = block_id;
  }
  return e;
}

// ---- introspection -----------------------------------------------------------------------

bool HeteroBlockTable::has_pool(FormatId format) const noexcept { return stack(format) != nullptr; }

std::uint32_t HeteroBlockTable::free_slots(FormatId format) const noexcept {
  const SlotStack* st = stack(format);
  return st != nullptr ? st->depth : 0u;
}

std::uint32_t HeteroBlockTable::pool_slots(FormatId format) const noexcept {
  const SlotStack* st = stack(format);
  return st != nullptr ? st->capacity : 0u;
}

std::uint32_t HeteroBlockTable::slot_bytes(FormatId format) const noexcept {
  const SlotStack* st = stack(format);
  return st != nullptr ? st->slot_bytes : 0u;
}

TableStats HeteroBlockTable::stats() const {
  TableStats st;
  st.blocks_capacity = max_blocks();
  st.format_changes_committed = committed_changes_;
  for (const BlockDescriptor& d : blocks_) {
    st.blocks_per_state[static_cast<std::size_t>(d.state())] += 1;
    if (d.state() == BlockState::kFree) continue;
    st.blocks_in_use += 1;
    st.blocks_per_format[fmt_index(d.exec.format())] += 1;
    st.blocks_per_residency[static_cast<std::size_t>(d.residency())] += 1;
    st.valid_tokens += d.exec.valid_tokens();
    st.payload_bytes_in_use += slot_bytes(d.exec.format());
    if (d.state() == BlockState::kTranscoding) st.payload_bytes_in_use += slot_bytes(d.pending_format());
  }
  st.token_capacity_in_use = std::uint64_t{st.blocks_in_use} * block_tokens_;
  for (const SeqRecord& q : seq_records_) {
    if (!q.live) continue;
    st.active_sequences += 1;
    st.arena_live_entries += q.seg.length;
    st.arena_reserved_entries += q.seg.capacity;
  }
  st.arena_entries = arena_.size();
  st.arena_free_entries = arena_.free_entries();
  st.pending_descriptor_patches = changed_blocks_.size();
  st.pending_id_patches = arena_.pending_patches();
  return st;
}

// ---- snapshot ------------------------------------------------------------------------
//
// Image layout (host byte order; u32 lists are a count then the values):
//   u64 magic "HLKVSNAP", u32 image version, u32 ABI version,
//   u32 max_blocks, u32 block_tokens, u32 blocks in use, u64 committed format changes,
//   u32 pool count, per pool {u32 format, slot_bytes, capacity, stack top, stack depth,
//   u32 list `below` links}, the block records (32 B each; free records carry their
//   free-chain link in `reserved`), u32 top of the free block ids,
//   u32 sequence count, per sequence {u32 offset, capacity, length, generation, live},
//   u32 top of the free sequence ids, the id arena (IdArena::snapshot),
//   u64 FNV-1a checksum of everything before it.

namespace {
constexpr std::uint64_t kSnapshotMagic = 0x50414E53564B4C48ull;  // bytes "HLKVSNAP" little-endian
constexpr std::uint32_t kSnapshotVersion = 2;
constexpr std::size_t kSeqBytes = 5 * sizeof(std::uint32_t);
}  // namespace

std::vector<std::byte> HeteroBlockTable::snapshot() const {
  std::vector<std::byte> out;
  detail::SnapshotWriter w(out);
  w.u64(kSnapshotMagic);
  w.u32(kSnapshotVersion);
  w.u32(kAbiVersion);
  w.u32(max_blocks());
  w.u32(block_tokens_);
  w.u32(in_use_);
  w.u64(committed_changes_);
  std::uint32_t n_pools = 0;
  for (const SlotStack& st : slots_) n_pools += st.present ? 1u : 0u;
  w.u32(n_pools);
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    const SlotStack& st = slots_[f];
    if (!st.present) continue;
    w.u32(f);
    w.u32(st.slot_bytes);
    w.u32(st.capacity);
    w.u32(st.top);
    w.u32(st.depth);
    w.u32s(st.below);
  }
  w.bytes(blocks_.data(), blocks_.size() * sizeof(BlockDescriptor));
  w.u32(free_block_top_);
  w.u32(static_cast<std::uint32_t>(seq_records_.size()));
  for (const SeqRecord& q : seq_records_) {
    w.u32(q.seg.offset);
    w.u32(q.seg.capacity);
    w.u32(q.seg.length);
    w.u32(q.generation);
    w.u32(q.live ? 1u : 0u);
  }
  w.u32(free_seq_top_);
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
  struct Stack {
    std::uint32_t top = kEnd, depth = 0;
    std::vector<std::uint32_t> below;
  };
  TableConfig config;
  config.max_blocks = max_blocks;
  config.block_tokens = block_tokens;
  std::array<Stack, kMaxFormats> stacks;
  for (std::uint32_t i = 0; i < n_pools; ++i) {
    std::uint32_t f = 0, slot_bytes = 0, capacity = 0;
    if (!r.u32(f) || f >= kMaxFormats || !r.u32(slot_bytes) || !r.u32(capacity) || !r.u32(stacks[f].top) ||
        !r.u32(stacks[f].depth) || !r.u32s(stacks[f].below, capacity) || stacks[f].below.size() != capacity) {
      return Status::kCorrupt;
    }
    config.pools.push_back(PoolConfig{FormatId{static_cast<std::uint8_t>(f)}, slot_bytes, capacity});
  }
  if (validate_config(config) != Status::kOk) return Status::kCorrupt;
  // The records are in the image: bound the allocation by it.
  if (std::size_t{max_blocks} * sizeof(BlockDescriptor) > r.remaining()) return Status::kCorrupt;
  auto t = std::make_unique<HeteroBlockTable>(config);
  if (!r.bytes(t->blocks_.data(), std::size_t{max_blocks} * sizeof(BlockDescriptor)) ||
      !r.u32(t->free_block_top_)) {
    return Status::kCorrupt;
  }
  for (const PoolConfig& pc : config.pools) {
    SlotStack& st = t->slots_[fmt_index(pc.format)];
    Stack& s = stacks[fmt_index(pc.format)];
    st.top = s.top;
    st.depth = s.depth;
    st.below = std::move(s.below);
  }
  std::uint32_t n_seqs = 0;
  if (!r.u32(n_seqs) || std::size_t{n_seqs} * kSeqBytes > r.remaining()) return Status::kCorrupt;
  t->seq_records_.resize(n_seqs);
  for (SeqRecord& q : t->seq_records_) {
    std::uint32_t live = 0;
    if (!r.u32(q.seg.offset) || !r.u32(q.seg.capacity) || !r.u32(q.seg.length) || !r.u32(q.generation) ||
        !r.u32(live) || live > 1) {
      return Status::kCorrupt;
    }
    q.live = live != 0;
  }
  if (!r.u32(t->free_seq_top_) || !t->arena_.restore(r) || r.remaining() != 0) return Status::kCorrupt;
  t->in_use_ = in_use;
  t->committed_changes_ = committed;
  // The constructor left every descriptor pending and the arena's restore every entry, so
  // the restored table's first delta is the whole device image.  validate() walks every
  // chain with bounds, so a malformed image cannot loop or index out of range.
  if (!t->validate().ok()) return Status::kCorrupt;
  out = std::move(t);
  return Status::kOk;
}

ValidationReport HeteroBlockTable::validate() const {
  const std::size_t n = blocks_.size();
  // The free block ids: a chain through free records, no repeats, ending at kEnd.
  std::vector<bool> chained(n, false);
  std::size_t free_count = 0;
  for (std::uint32_t id = free_block_top_; id != kEnd; id = blocks_[id].reserved) {
    if (id >= n || chained[id] || blocks_[id].state() != BlockState::kFree) {
      return corrupt("free block chain is broken at id " + std::to_string(id));
    }
    chained[id] = true;
    free_count += 1;
  }

  // Each pool's free slots: a chain of in-range, distinct slots of the stated depth.
  std::array<std::vector<bool>, kMaxFormats> taken;
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    const SlotStack& st = slots_[f];
    if (!st.present) continue;
    if (st.below.size() != st.capacity) return corrupt("pool " + std::to_string(f) + " link array size");
    taken[f].assign(st.capacity, false);
    std::uint32_t depth = 0;
    for (std::uint32_t s = st.top; s != kEnd; s = st.below[s]) {
      if (s >= st.capacity || taken[f][s]) return corrupt("pool " + std::to_string(f) + " free chain is broken");
      taken[f][s] = true;
      depth += 1;
    }
    if (depth != st.depth) return corrupt("pool " + std::to_string(f) + " depth");
  }
  auto take = [&](FormatId f, std::uint32_t slot, std::uint32_t id) -> std::string {
    const SlotStack* st = stack(f);
    if (st == nullptr) return "block " + std::to_string(id) + " has no pool";
    if (slot >= st->capacity) return "block " + std::to_string(id) + " slot out of range";
    if (taken[fmt_index(f)][slot]) return "slot " + std::to_string(slot) + " held twice";
    taken[fmt_index(f)][slot] = true;
    return {};
  };

  std::uint32_t live_blocks = 0;
  for (std::uint32_t id = 0; id < n; ++id) {
    const BlockDescriptor& d = blocks_[id];
    if (d.exec.block_id != id) return corrupt("block " + std::to_string(id) + ": block_id field");
    if (d.state() == BlockState::kFree) {
      if (!chained[id]) return corrupt("block " + std::to_string(id) + ": free but not on the free chain");
      continue;
    }
    live_blocks += 1;
    if (d.refcount() == 0) return corrupt("block " + std::to_string(id) + ": refcount 0");
    if (d.exec.info_reserved() || d.control_reserved() || d.reserved) {
      return corrupt("block " + std::to_string(id) + ": reserved bits set");
    }
    if (d.exec.valid_tokens() > block_tokens_) return corrupt("valid_tokens above block_tokens");
    if (!valid_residency(d.residency())) return corrupt("invalid residency");
    if (std::string e = take(d.exec.format(), d.exec.slot, id); !e.empty()) return corrupt(e);
    if (d.state() == BlockState::kTranscoding) {
      if (d.pending_format() == d.exec.format()) return corrupt("pending format == format");
      if (std::string e = take(d.pending_format(), d.pending_slot, id); !e.empty()) return corrupt(e);
    } else if (d.pending_slot != kNoSlot || d.pending_format() != kInvalidFormat) {
      return corrupt("pending slot outside a format change");
    }
  }
  if (live_blocks != in_use_) return corrupt("blocks_in_use counter");
  if (free_count + live_blocks != n) return corrupt("free block chain length");
  for (std::uint32_t f = 0; f < kMaxFormats; ++f) {
    if (slots_[f].present && std::find(taken[f].begin(), taken[f].end(), false) != taken[f].end()) {
      return corrupt("pool " + std::to_string(f) + " lost a slot");
    }
  }

  // Sequences: live ones reference live blocks (no more often than their refcounts); the
  // released ones are exactly the free sequence chain.
  std::vector<std::uint32_t> refs(n, 0);
  std::vector<IdArena::Segment> live;
  std::size_t released = 0;
  for (std::size_t s = 0; s < seq_records_.size(); ++s) {
    const SeqRecord& q = seq_records_[s];
    if (!q.live) {
      released += 1;
      if (q.seg.capacity != 0 || q.seg.length != 0) return corrupt("released sequence holds storage");
      continue;
    }
    live.push_back(q.seg);
    for (const std::uint32_t id : arena_.view(q.seg)) {
      if (id >= n || blocks_[id].state() == BlockState::kFree) {
        return corrupt("sequence " + std::to_string(s) + " references a free block");
      }
      refs[id] += 1;
    }
  }
  for (std::uint32_t id = 0; id < n; ++id) {
    if (refs[id] > blocks_[id].refcount()) return corrupt("sequence references above refcount");
  }
  std::vector<bool> on_chain(seq_records_.size(), false);
  std::size_t chain_len = 0;
  for (std::uint32_t s = free_seq_top_; s != kEnd; s = seq_records_[s].seg.offset) {
    if (s >= seq_records_.size() || seq_records_[s].live || on_chain[s]) return corrupt("free sequence chain is broken");
    on_chain[s] = true;
    chain_len += 1;
  }
  if (chain_len != released) return corrupt("free sequence chain length");
  if (std::string e = arena_.validate(live); !e.empty()) return corrupt(e);
  if (changed_blocks_.span() != n || !changed_blocks_.consistent()) return corrupt("descriptor change queue");
  return {};
}

}  // namespace hl::alloc
