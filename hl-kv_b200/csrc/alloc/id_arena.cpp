// IdArena (see include/hl_allocator/id_arena.hpp).
//
// Observable behaviour follows the reference's project1_allocator/src/id_arena.cpp:
// size classes 8 << k (class of `needed` = ceil(log2(needed)) - 3, class 0 for
// needed <= 8), LIFO reuse per class before carving new space at the end,
// relocation copies entries in order and marks each one dirty, and collect()
// reports dirty offsets in marking order.
#include "hl_allocator/id_arena.hpp"
#include "hl_allocator/snapshot_io.hpp"

#include <algorithm>
#include <bit>
#include <cassert>

namespace hl::alloc {
namespace {

constexpr std::uint32_t kClassShift = 3;  // kMinSegment == 1 << 3
static_assert(IdArena::kMinSegment == (1u << kClassShift));

constexpr std::uint32_t class_capacity(std::uint32_t c) noexcept { return IdArena::kMinSegment << c; }

// Smallest class holding `needed` (>= 1) entries.
constexpr std::uint32_t class_holding(std::uint32_t needed) noexcept {
  return needed <= IdArena::kMinSegment
             ? 0u
             : static_cast<std::uint32_t>(std::bit_width(needed - 1u)) - kClassShift;
}

// Class whose capacity is exactly `capacity`, or kNumClasses when there is none.
constexpr std::uint32_t class_exact(std::uint32_t capacity) noexcept {
  if (capacity < IdArena::kMinSegment || !std::has_single_bit(capacity)) return IdArena::kNumClasses;
  const std::uint32_t c = static_cast<std::uint32_t>(std::countr_zero(capacity)) - kClassShift;
  return c < IdArena::kNumClasses ? c : IdArena::kNumClasses;
}

static_assert(class_holding(1) == 0 && class_holding(8) == 0 && class_holding(9) == 1);
static_assert(class_holding(IdArena::kMaxSegment) == IdArena::kNumClasses - 1);
static_assert(class_exact(16) == 1 && class_exact(24) == IdArena::kNumClasses);

// Grows capacity at least geometrically so amortized cost stays O(1).
template <typename T>
void ensure_capacity(std::vector<T>& v, std::size_t n) {
  if (v.capacity() < n) v.reserve(std::max(n, v.capacity() * 2));
}

}  // namespace

Status IdArena::carve_or_reuse(std::uint32_t size_class, std::uint32_t& offset) {
  std::vector<std::uint32_t>& parked = parked_[size_class];
  if (!parked.empty()) {
    offset = parked.back();
    parked.pop_back();
    return Status::kOk;
  }
  const std::size_t old_size = ids_.size();
  const std::size_t new_size = old_size + class_capacity(size_class);
  if (new_size > kMaxEntries) return Status::kCapacityExceeded;
  // Everything the noexcept paths rely on is allocated here, before any state
  // changes: room to mark every entry dirty, and room to park every segment of
  // this class that will ever exist.
  ensure_capacity(ids_, new_size);
  ensure_capacity(is_dirty_, new_size);
  ensure_capacity(dirty_order_, new_size);
  ensure_capacity(parked, std::size_t{carved_[size_class]} + 1);
  ids_.resize(new_size);
  is_dirty_.resize(new_size, 0);
  carved_[size_class] += 1;
  offset = static_cast<std::uint32_t>(old_size);
  return Status::kOk;
}

void IdArena::mark(std::uint32_t offset) noexcept {
  if (is_dirty_[offset]) return;
  is_dirty_[offset] = 1;
  dirty_order_.push_back(offset);  // capacity covers every entry
}

Status IdArena::reserve(Segment& seg, std::uint32_t needed) {
  if (needed <= seg.capacity) return Status::kOk;
  if (needed > kMaxSegment) return Status::kCapacityExceeded;
  const std::uint32_t c = class_holding(needed);
  std::uint32_t dst = 0;
  if (const Status s = carve_or_reuse(c, dst); s != Status::kOk) return s;
  for (std::uint32_t k = 0; k < seg.length; ++k) {
    ids_[dst + k] = ids_[seg.offset + k];
    mark(dst + k);
  }
  if (seg.capacity != 0) parked_[class_exact(seg.capacity)].push_back(seg.offset);
  seg.offset = dst;
  seg.capacity = class_capacity(c);
  return Status::kOk;
}

void IdArena::push_back(Segment& seg, std::uint32_t block_id) noexcept {
  assert(seg.length < seg.capacity && "IdArena::push_back needs reserve() first");
  const std::uint32_t at = seg.offset + seg.length;
  ids_[at] = block_id;
  mark(at);
  seg.length += 1;
}

void IdArena::release(Segment& seg) noexcept {
  if (seg.capacity != 0) parked_[class_exact(seg.capacity)].push_back(seg.offset);
  seg = Segment{};
}

std::span<const std::uint32_t> IdArena::view(const Segment& seg) const noexcept {
  if (seg.capacity == 0) return {};
  return {ids_.data() + seg.offset, seg.length};
}

void IdArena::collect(std::vector<IdPatch>& out) {
  out.clear();
  out.reserve(dirty_order_.size());  // the only allocation, before any state change
  for (const std::uint32_t off : dirty_order_) {
    out.push_back(IdPatch{off, ids_[off]});
    is_dirty_[off] = 0;
  }
  dirty_order_.clear();
}

std::uint64_t IdArena::free_entries() const noexcept {
  std::uint64_t sum = 0;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    sum += std::uint64_t{parked_[c].size()} * class_capacity(c);
  }
  return sum;
}

void IdArena::snapshot(detail::SnapshotWriter& w) const {
  w.u32s(ids_);
  for (std::uint32_t c = 0; c < kNumClasses; ++c) w.u32s(parked_[c]);
  for (std::uint32_t c = 0; c < kNumClasses; ++c) w.u32(carved_[c]);
}

bool IdArena::restore(detail::SnapshotReader& r) {
  std::vector<std::uint32_t> ids;
  if (!r.u32s(ids, kMaxEntries)) return false;
  std::array<std::vector<std::uint32_t>, kNumClasses> parked;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    if (!r.u32s(parked[c], ids.size())) return false;
  }
  std::array<std::uint32_t, kNumClasses> carved{};
  std::uint64_t carved_entries = 0;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    if (!r.u32(carved[c])) return false;
    carved_entries += std::uint64_t{carved[c]} * class_capacity(c);
  }
  // The segments must tile the arena before anything is sized from the counts.
  if (carved_entries != ids.size()) return false;
  const std::size_t n = ids.size();
  ids_ = std::move(ids);
  is_dirty_.assign(n, 1);
  dirty_order_.clear();
  dirty_order_.reserve(n);
  for (std::size_t k = 0; k < n; ++k) dirty_order_.push_back(static_cast<std::uint32_t>(k));
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    parked_[c] = std::move(parked[c]);
    ensure_capacity(parked_[c], std::max<std::size_t>(carved[c], parked_[c].size()));
  }
  carved_ = carved;
  return true;
}

std::string IdArena::validate(std::span<const Segment> live) const {
  const std::size_t n = ids_.size();
  if (is_dirty_.size() != n) return "arena: dirty flags do not cover the arena";
  if (dirty_order_.capacity() < n) return "arena: dirty list cannot hold every entry";
  std::uint64_t carved_entries = 0;
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    carved_entries += std::uint64_t{carved_[c]} * class_capacity(c);
    if (parked_[c].size() > carved_[c] || parked_[c].capacity() < carved_[c]) {
      return "arena: free list of class " + std::to_string(c) + " is inconsistent";
    }
  }
  if (carved_entries != n) return "arena: carved segments do not sum to the arena size";

  std::vector<std::uint8_t> owner(n, 0);
  auto claim = [&](std::uint32_t off, std::uint32_t cap) -> std::string {
    if (class_exact(cap) == kNumClasses) return "arena: capacity " + std::to_string(cap) + " is not a class";
    if (std::uint64_t{off} + cap > n) return "arena: segment at " + std::to_string(off) + " out of range";
    for (std::uint64_t k = off; k < std::uint64_t{off} + cap; ++k) {
      if (owner[k]) return "arena: entry " + std::to_string(k) + " owned twice";
      owner[k] = 1;
    }
    return {};
  };
  for (const Segment& s : live) {
    if (s.capacity == 0) {
      if (s.length != 0) return "arena: storage-less segment with a length";
      continue;
    }
    if (s.length > s.capacity) return "arena: length exceeds capacity";
    if (std::string e = claim(s.offset, s.capacity); !e.empty()) return e;
  }
  for (std::uint32_t c = 0; c < kNumClasses; ++c) {
    for (const std::uint32_t off : parked_[c]) {
      if (std::string e = claim(off, class_capacity(c)); !e.empty()) return e;
    }
  }
  for (std::size_t k = 0; k < n; ++k) {
    if (!owner[k]) return "arena: entry " + std::to_string(k) + " leaked";
  }
  std::vector<std::uint8_t> listed(n, 0);
  for (const std::uint32_t off : dirty_order_) {
    if (off >= n || !is_dirty_[off] || listed[off]) {
      return "arena: dirty list entry " + std::to_string(off) + " inconsistent";
    }
    listed[off] = 1;
  }
  const auto flagged = static_cast<std::size_t>(std::count(is_dirty_.begin(), is_dirty_.end(), 1));
  if (flagged != dirty_order_.size()) return "arena: dirty flag without a list entry";
  return {};
}

}  // namespace hl::alloc
