#pragma once
// Byte-level writer and reader of a table snapshot image (HeteroBlockTable::snapshot /
// restore).  Values are stored in the host's byte order; the image's magic number, read
// back in another byte order, does not match, so such an image is rejected.  The reader
// never reads past its span and reports a short image as failure.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

namespace hl::alloc::detail {

class SnapshotWriter {
 public:
  explicit SnapshotWriter(std::vector<std::byte>& out) : out_(out) {}
  void u32(std::uint32_t v) { put(&v, sizeof v); }
  void u64(std::uint64_t v) { put(&v, sizeof v); }
  void bytes(const void* p, std::size_t n) { put(p, n); }
  /// A count, then the values.
  void u32s(const std::vector<std::uint32_t>& v) {
    u32(static_cast<std::uint32_t>(v.size()));
    put(v.data(), v.size() * sizeof(std::uint32_t));
  }

 private:
  void put(const void* p, std::size_t n) {
    const auto* b = static_cast<const std::byte*>(p);
    out_.insert(out_.end(), b, b + n);
  }
  std::vector<std::byte>& out_;
};

class SnapshotReader {
 public:
  explicit SnapshotReader(std::span<const std::byte> in) : in_(in) {}
  [[nodiscard]] bool u32(std::uint32_t& v) { return get(&v, sizeof v); }
  [[nodiscard]] bool u64(std::uint64_t& v) { return get(&v, sizeof v); }
  [[nodiscard]] bool bytes(void* p, std::size_t n) { return get(p, n); }
  /// A count of at most max_count, then the values.
  [[nodiscard]] bool u32s(std::vector<std::uint32_t>& v, std::size_t max_count) {
    std::uint32_t n = 0;
    if (!u32(n) || n > max_count || std::size_t{n} * sizeof(std::uint32_t) > remaining()) return false;
    v.resize(n);
    return get(v.data(), std::size_t{n} * sizeof(std::uint32_t));
  }
  [[nodiscard]] std::size_t remaining() const noexcept { return in_.size() - pos_; }
  [[nodiscard]] std::size_t position() const noexcept { return pos_; }

 private:
  bool get(void* p, std::size_t n) {
    if (n > remaining()) return false;
    if (n != 0) std::memcpy(p, in_.data() + pos_, n);
    pos_ += n;
    return true;
  }
  std::span<const std::byte> in_;
  std::size_t pos_ = 0;
};

/// FNV-1a (64-bit) over an image, the trailer that detects damaged snapshots.
inline std::uint64_t snapshot_checksum(std::span<const std::byte> bytes) noexcept {
  std::uint64_t h = 0xCBF29CE484222325ull;
  for (const std::byte b : bytes) {
    h ^= static_cast<std::uint64_t>(b);
    h *= 0x100000001B3ull;
  }
  return h;
}

}  // namespace hl::alloc::detail
