#pragma once
// detail::ChangeQueue: the distinct indices of a host array whose device copy must be
// patched, in the order they were first changed.  Shared by IdArena (arena entries) and
// HeteroBlockTable (descriptor records).
//
// An index counts as queued when its stamp equals the current epoch.  drain() hands the
// queue over and starts a new epoch, so clearing costs nothing per entry; every 2^32 - 1
// drains the stamps are reset once.  grow() is the only call that allocates: it makes
// room for indices below n, in the stamps and in the order list, so mark() (each index
// at most once per epoch) never allocates.
#include <cstddef>
#include <cstdint>
#include <span>
#include <vector>

namespace hl::alloc::detail {

class ChangeQueue {
 public:
  /// Room for indices < n (never shrinks).  May throw; nothing changes then.
  void grow(std::size_t n) {
    if (n <= stamp_.size()) return;
    if (order_.capacity() < n) order_.reserve(n > 2 * order_.capacity() ? n : 2 * order_.capacity());
    stamp_.resize(n, 0);  // after the reserve: a throw here leaves the old size in place
  }

  /// Queues index i (< the grown size) unless it is queued already.
  void mark(std::uint32_t i) noexcept {
    if (stamp_[i] == epoch_) return;
    stamp_[i] = epoch_;
    order_.push_back(i);  // capacity covers every index once
  }

  [[nodiscard]] bool queued(std::uint32_t i) const noexcept { return stamp_[i] == epoch_; }
  [[nodiscard]] std::size_t size() const noexcept { return order_.size(); }
  [[nodiscard]] std::size_t span() const noexcept { return stamp_.size(); }
  [[nodiscard]] std::span<const std::uint32_t> order() const noexcept { return order_; }

  /// Calls fn(i) for every queued index in marking order, then empties the queue.
  template <typename Fn>
  void drain(Fn&& fn) noexcept(noexcept(fn(std::uint32_t{}))) {
    for (const std::uint32_t i : order_) fn(i);
    order_.clear();
    if (++epoch_ == 0) {  // the stamps would be ambiguous after a wrap: reset them
      for (std::uint32_t& s : stamp_) s = 0;
      epoch_ = 1;
    }
  }

  /// True when the stamps and the order list agree (every listed index stamped, once).
  [[nodiscard]] bool consistent() const {
    if (order_.capacity() < stamp_.size()) return false;
    std::size_t stamped = 0;
    for (const std::uint32_t s : stamp_) stamped += s == epoch_ ? 1u : 0u;
    if (stamped != order_.size()) return false;
    std::vector<bool> seen(stamp_.size(), false);
    for (const std::uint32_t i : order_) {
      if (i >= stamp_.size() || stamp_[i] != epoch_ || seen[i]) return false;
      seen[i] = true;
    }
    return true;
  }

 private:
  std::vector<std::uint32_t> stamp_;  // per index: the epoch in which it was last queued (0: none)
  std::vector<std::uint32_t> order_;  // queued indices, first marking first
  std::uint32_t epoch_ = 1;
};

}  // namespace hl::alloc::detail
