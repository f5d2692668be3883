#pragma once
// IdArena: per-sequence lists of block ids in one growable uint32 array, with
// the dirty tracking that keeps a device copy current through patches.
//
// Drop-in for the reference's project1_allocator/include/hl_allocator/id_arena.hpp
// (same public API, same observable results: offsets, capacities and patch
// order).  A sequence owns one segment whose capacity is a power-of-two size
// class (8 << k entries, 8 .. 2^31).  A full segment moves to one of the next
// class, copying its entries; freed segments are reused per class, last freed
// first; the array only grows.  Every write queues its entry; collect() turns
// the queued entries into {offset, block_id} patches, each offset once, so a
// device can apply them in any order.
//
// Storage: the entries in one array; the free segments of a class form a stack
// linked through a side array with one slot per 8-entry unit (segments start on
// unit boundaries), so freeing never allocates and never touches an entry -- a
// freed entry still waiting to be patched keeps the id it was written with; the
// entries to patch are a detail::ChangeQueue.  reserve() gives the strong guarantee: all
// allocation happens before any state changes, so push_back(), release() and the
// change bookkeeping never allocate and are noexcept.
#include <array>
#include <cstdint>
#include <span>
#include <string>
#include <vector>

#include "hl_allocator/change_queue.hpp"
#include "hl_allocator/status.hpp"

namespace hl::alloc {

/// arena[offset] = block_id on the device.
struct IdPatch {
  std::uint32_t offset;
  std::uint32_t block_id;
  friend constexpr bool operator==(IdPatch, IdPatch) noexcept = default;
};

/// A live segment's move in an arena compaction: entries [from, from + length) go to
/// [to, to + length).  `scratch` places the segment in a relocation scratch buffer
/// (moves are made in two phases through it; see IdArena::compact).
struct SegmentMove {
  std::uint32_t from;
  std::uint32_t to;
  std::uint32_t length;
  std::uint32_t scratch;
  friend constexpr bool operator==(SegmentMove, SegmentMove) noexcept = default;
};

/// What a kernel needs per sequence: block ids arena[offset .. offset + length).
struct SequenceSegment {
  std::uint32_t offset;
  std::uint32_t length;
  friend constexpr bool operator==(SequenceSegment, SequenceSegment) noexcept = default;
};

namespace detail {
class SnapshotWriter;
class SnapshotReader;
}  // namespace detail

class IdArena {
 public:
  static constexpr std::uint32_t kMinSegment = 8;
  static constexpr std::uint32_t kNumClasses = 29;  // 8 .. 2^31 entries
  static constexpr std::uint32_t kMaxSegment = kMinSegment << (kNumClasses - 1);
  /// Offsets are uint32 and 0xFFFFFFFF is reserved.
  static constexpr std::uint64_t kMaxEntries = 0xFFFF'FFFFull;

  /// A sequence's storage; capacity 0 = no storage yet.
  struct Segment {
    std::uint32_t offset = 0;
    std::uint32_t capacity = 0;
    std::uint32_t length = 0;
  };

  /// Makes seg.capacity >= needed, moving the segment if necessary.
  /// kCapacityExceeded past kMaxSegment or kMaxEntries.  Strong guarantee.
  [[nodiscard]] Status reserve(Segment& seg, std::uint32_t needed);
  /// Appends one id.  Precondition: seg.length < seg.capacity.
  void push_back(Segment& seg, std::uint32_t block_id) noexcept;
  /// Returns the segment's storage to its class free list; seg becomes empty.
  void release(Segment& seg) noexcept;

  [[nodiscard]] std::span<const std::uint32_t> view(const Segment& seg) const noexcept;
  [[nodiscard]] static SequenceSegment kernel_view(const Segment& seg) noexcept {
    return seg.capacity == 0 ? SequenceSegment{0u, seg.length}
                             : SequenceSegment{seg.offset, seg.length};
  }

  /// Packs the `live` segments (every segment that holds storage) to the front of the
  /// arena in their current offset order, each keeping its capacity; empties the free
  /// stacks and shrinks the arena to the packed size.  Each segment's offset is updated;
  /// `moves` receives the moves a device copy must make (segments that hold entries and
  /// whose offset changed), in increasing offset order, with scratch offsets packed in
  /// 8-entry units (scratch_entries() of them in all).  Nothing is queued for patching:
  /// the device copy makes the same moves.  kInvalidState, nothing changed, while
  /// patches are pending (collect() first), since they name pre-compaction offsets.
  /// Strong guarantee.  No counterpart in the reference, whose arena never compacts
  /// (hl_allocator_abi.md, section 9, item 5).
  [[nodiscard]] Status compact(std::span<Segment* const> live, std::vector<SegmentMove>& moves);
  /// Entries of relocation scratch that `moves` needs.
  [[nodiscard]] static std::uint64_t scratch_entries(std::span<const SegmentMove> moves) noexcept {
    return moves.empty() ? 0 : std::uint64_t{moves.back().scratch} + ((moves.back().length + 7u) & ~7u);
  }

  /// Replaces `out` with one patch per changed entry (first change first) and empties the queue.
  void collect(std::vector<IdPatch>& out);

  [[nodiscard]] std::uint32_t size() const noexcept {
    return static_cast<std::uint32_t>(entry_.size());
  }
  [[nodiscard]] std::size_t pending_patches() const noexcept { return changed_.size(); }
  /// Total capacity parked on the free lists.
  [[nodiscard]] std::uint64_t free_entries() const noexcept;

  /// Appends the arena (entries, and per class the top and length of its free stack) to a
  /// table snapshot.
  void snapshot(detail::SnapshotWriter& w) const;
  /// Replaces the arena with one that snapshot() wrote; every entry is then pending, so
  /// the next collect() reports all of them.  False, with nothing changed, on a malformed
  /// image.
  [[nodiscard]] bool restore(detail::SnapshotReader& r);

  /// Checks that `live` plus the free stacks tile the array exactly and that the
  /// change queue is consistent; "" when it holds, else the first problem.
  [[nodiscard]] std::string validate(std::span<const Segment> live) const;

 private:
  static constexpr std::uint32_t kNone = 0xFFFF'FFFFu;  // end of a free stack

  /// A segment of class `cls` for a sequence: the last one freed, else new space at the end.
  [[nodiscard]] Status obtain(std::uint32_t cls, std::uint32_t& offset);
  /// Puts a segment of class `cls` on top of its free stack.
  void park(std::uint32_t cls, std::uint32_t offset) noexcept;

  static constexpr std::array<std::uint32_t, kNumClasses> no_free_segments() {
    std::array<std::uint32_t, kNumClasses> a{};
    for (std::uint32_t& x : a) x = kNone;
    return a;
  }

  std::vector<std::uint32_t> entry_;      // the arena
  std::vector<std::uint32_t> next_free_;  // per 8-entry unit: the free segment under this one
  detail::ChangeQueue changed_;           // entries the device copy lacks, first change first
  std::array<std::uint32_t, kNumClasses> free_top_ = no_free_segments();  // per class, kNone: empty
  std::array<std::uint32_t, kNumClasses> free_len_{};                     // segments on each stack
};

}  // namespace hl::alloc
