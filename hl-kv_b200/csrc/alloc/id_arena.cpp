// IdArena (see include/hl_allocator/id_arena.hpp).
//
// The placement policy is the reference's (project1_allocator/src/id_arena.cpp), because
// arena offsets and the patch stream are observable: capacities are 8 << k entries and a
// sequence needing n entries gets the smallest class holding n; a class reuses its most
// recently freed segment before new space is appended; a moved segment's entries are
// written (and queued) in order, and its old segment is freed only after the new one is
// taken.  The storage is this library's own: free segments are stacks linked through a
// side array indexed by 8-entry unit, and the change queue is epoch-stamped.
#include "hl_allocator/id_arena.hpp"
#include "hl_allocator/snapshot_io.hpp"

#include <algorithm>
#include <bit>
#include <cassert>

namespace hl::alloc {
namespace {

constexpr std::uint32_t capacity_of(std::uint32_t cls) noexcept { return IdArena::kMinSegment << cls; }

// The smallest class with capacity >= n (n >= 1): ceil(log2(n)) - 3, at least 0.
constexpr std::uint32_t class_for(std::uint32_t n) noexcept {
  const std::uint32_t bits = static_cast<std::uint32_t>(std::bit_width(n - 1u));
  return bits > 3u ? bits - 3u : 0u;
}

// The class of a segment capacity, or kNumClasses when it is not a class size.
constexpr std::uint32_t class_of_capacity(std::uint32_t cap) noexcept {
  if (!std::has_single_bit(cap) || cap < IdArena::kMinSegment) return IdArena::kNumClasses;
  const std::uint32_t c = static_cast<std::uint32_t>(std::countr_zero(cap)) - 3u;
  return c < IdArena::kNumClasses ? c : IdArena::kNumClasses;
}

static_assert(IdArena::kMinSegment == 8u, "class arithmetic assumes 8-entry minimum segments");
static_assert(class_for(1) == 0 && class_for(8) == 0 && class_for(9) == 1 && class_for(17) == 2);
static_assert(class_for(IdArena::kMaxSegment) == IdArena::kNumClasses - 1);
static_assert(class_of_capacity(64) == 3 && class_of_capacity(48) == IdArena::kNumClasses);

}  // namespace

Status IdArena::obtain(std::uint32_t cls, std::uint32_t& offset) {
  if (free_top_[cls] != kNone) {
    offset = free_top_[cls];
    free_top_[cls] = next_free_[offset / kMinSegment];
    free_len_[cls] -= 1;
    return Status::kOk;
  }
  const std::size_t at = entry_.size();
  const std::size_t grown = at + capacity_of(cls);
  if (grown > kMaxEntries) return Status::kCapacityExceeded;
  // Every allocation before any change: a throw leaves the arena as it was.
  const std::size_t units = grown / kMinSegment;
  if (entry_.capacity() < grown) entry_.reserve(grown > 2 * entry_.capacity() ? grown : 2 * entry_.capacity());
  if (next_free_.capacity() < units) next_free_.reserve(units > 2 * next_free_.capacity() ? units : 2 * next_free_.capacity());
  changed_.grow(grown);
  entry_.resize(grown, 0u);
  next_free_.resize(units, kNone);
  offset = static_cast<std::uint32_t>(at);
  return Status::kOk;
}

void IdArena::park(std::uint32_t cls, std::uint32_t offset) noexcept {
  next_free_[offset / kMinSegment] = free_top_[cls];
  free_top_[cls] = offset;
  free_len_[cls] += 1;
}

Status IdArena::reserve(Segment& seg, std::uint32_t needed) {
  if (needed <= seg.capacity) return Status::kOk;
  if (needed > kMaxSegment) return Status::kCapacityExceeded;
  const std::uint32_t cls = class_for(needed);
  std::uint32_t to = 0;
  if (const Status s = obtain(cls, to); s != Status::kOk) return s;
  // Copy the live entries across (each one a patch for the device), then free the old
  // segment: taking the new one first keeps a segment from being reused by its own move.
  for (std::uint32_t k = 0; k < seg.length; ++k) {
    entry_[to + k] = entry_[seg.offset + k];
    changed_.mark(to + k);
  }
  if (seg.capacity != 0) park(class_of_capacity(seg.capacity), seg.offset);
  seg.offset = to;
  seg.capacity = capacity_of(cls);
  return Status::kOk;
}

void IdArena::push_back(Segment& seg, std::uint32_t block_id) noexcept {
  assert(seg.length < seg.capacity && "IdArena::push_back needs reserve() first");
  const std::uint32_t at = seg.offset + seg.length;
  entry_[at] = block_id;
  changed_.mark(at);
  seg.length += 1;
}

void IdArena::release(Segment& seg) noexcept {
  if (seg.capacity != 0) park(class_of_capacity(seg.capacity), seg.offset);
  seg = Segment{};
}

std::span<const std::uint32_t> IdArena::view(const Segment& seg) const noexcept {
  if (seg.capacity == 0) return {};
  return std::span<const std::uint32_t>(entry_).subspan(seg.offset, seg.length);
}

void IdArena::collect(std::vector<IdPatch>& out) {
  out.resize(changed_.size());  // the only allocation, before the queue is touched
  std::size_t k = 0;
  changed_.drain([&](std::uint32_t off) noexcept { out[k++] = IdPatch{off, entry_[off]}; });
}

Status IdArena::compact(std::span<Segment* const> live, std::vector<SegmentMove>& moves) {
  if (changed_.size() != 0) return Status::kInvalidState;
  // Everything is built aside first; the swap at the end cannot fail.
  std::vector<Segment*> order;
  order.reserve(live.size());
  std::uint64_t total = 0;
  for (Segment* seg : live) {
    if (seg->capacity == 0) continue;
    order.push_back(seg);
    total += seg->capacity;
  }
  std::sort(order.begin(), order.end(), [](const Segment* a, const Segment* b) { return a->offset < b->offset; });
  std::vector<std::uint32_t> packed(total, 0u);
  std::vector<std::uint32_t> links(total / kMinSegment, kNone);
  std::vector<std::uint32_t> offsets(order.size());
  std::vector<SegmentMove> out;
  out.reserve(order.size());
  std::uint64_t at = 0, scratch = 0;
  for (std::size_t k = 0; k < order.size(); ++k) {
    const Segment& seg = *order[k];
    std::copy_n(entry_.begin() + seg.offset, seg.length, packed.begin() + static_cast<std::ptrdiff_t>(at));
    if (at != seg.offset && seg.length != 0) {
      out.push_back(SegmentMove{seg.offset, static_cast<std::uint32_t>(at), seg.length,
                                static_cast<std::uint32_t>(scratch)});
      scratch += (seg.length + 7u) & ~7u;  // 8-entry units keep every copy 32-byte aligned
    }
    offsets[k] = static_cast<std::uint32_t>(at);
    at += seg.capacity;
  }
  if (scratch > kMaxEntries) return Status::kCapacityExceeded;
  for (std::size_t k = 0; k < order.size(); ++k) order[k]->offset = offsets[k];
  entry_.swap(packed);
  next_free_.swap(links);
  free_top_ = no_free_segments();
  free_len_ = {};
  moves.swap(out);
  return Status::kOk;
}

std::uint64_t IdArena::free_entries() const noexcept {
  std::uint64_t total = 0;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) total += std::uint64_t{free_len_[c]} * capacity_of(c);
  return total;
}

// Image: the entries, the free-stack links (one per 8-entry unit), then per class the top
// of its free stack and the stack's length.
void IdArena::snapshot(detail::SnapshotWriter& w) const {
  w.u32s(entry_);
  w.u32s(next_free_);
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    w.u32(free_top_[c]);
    w.u32(free_len_[c]);
  }
}

bool IdArena::restore(detail::SnapshotReader& r) {
  std::vector<std::uint32_t> entries, links;
  if (!r.u32s(entries, kMaxEntries) || entries.size() % kMinSegment != 0) return false;
  if (!r.u32s(links, entries.size() / kMinSegment) || links.size() != entries.size() / kMinSegment) return false;
  std::array<std::uint32_t, kNumClasses> top{}, len{};
  std::uint64_t parked = 0;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    if (!r.u32(top[c]) || !r.u32(len[c])) return false;
    // The stacks' segments fit in the arena (this also bounds the walk below); each
    // stack holds exactly len[c] in-range links and then ends.
    parked += std::uint64_t{len[c]} * capacity_of(c);
    if (parked > entries.size()) return false;
    std::uint32_t at = top[c];
    for (std::uint32_t k = 0; k < len[c]; ++k) {
      if (at == kNone || at % kMinSegment != 0 || std::uint64_t{at} + capacity_of(c) > entries.size()) return false;
      at = links[at / kMinSegment];
    }
    if (at != kNone) return false;
  }
  detail::ChangeQueue changed;
  changed.grow(entries.size());
  for (std::size_t k = 0; k < entries.size(); ++k) changed.mark(static_cast<std::uint32_t>(k));
  entry_ = std::move(entries);
  next_free_ = std::move(links);
  changed_ = std::move(changed);
  free_top_ = top;
  free_len_ = len;
  return true;
}

std::string IdArena::validate(std::span<const Segment> live) const {
  const std::size_t n = entry_.size();
  if (changed_.span() < n) return "arena: change stamps do not cover the arena";
  if (n % kMinSegment != 0 || next_free_.size() != n / kMinSegment) return "arena: link array size";
  if (!changed_.consistent()) return "arena: change queue inconsistent";
  std::vector<bool> owned(n, false);
  auto claim = [&](std::uint64_t off, std::uint32_t cap, const char* what) -> std::string {
    if (off + cap > n) return std::string("arena: ") + what + " segment at " + std::to_string(off) + " out of range";
    for (std::uint64_t k = off; k < off + cap; ++k) {
      if (owned[k]) return "arena: entry " + std::to_string(k) + " in two segments";
      owned[k] = true;
    }
    return {};
  };
  for (const Segment& s : live) {
    if (s.capacity == 0) {
      if (s.length != 0) return "arena: a segment without storage has a length";
      continue;
    }
    if (class_of_capacity(s.capacity) == kNumClasses) return "arena: capacity " + std::to_string(s.capacity) + " is not a class";
    if (s.length > s.capacity) return "arena: length exceeds capacity";
    if (std::string e = claim(s.offset, s.capacity, "live"); !e.empty()) return e;
  }
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    std::uint32_t at = free_top_[c];
    for (std::uint32_t k = 0; k < free_len_[c]; ++k) {
      if (at == kNone || at >= n || at % kMinSegment != 0) {
        return "arena: free stack of class " + std::to_string(c) + " is short or broken";
      }
      if (std::string e = claim(at, capacity_of(c), "free"); !e.empty()) return e;
      at = next_free_[at / kMinSegment];
    }
    if (at != kNone) return "arena: free stack of class " + std::to_string(c) + " is longer than its count";
  }
  for (std::size_t k = 0; k < n; ++k) {
    if (!owned[k]) return "arena: entry " + std::to_string(k) + " belongs to no segment";
  }
  return {};
}

}  // namespace hl::alloc
