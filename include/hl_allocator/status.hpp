#pragma once
// Error reporting of the host table (drop-in for the reference's
// project1_allocator/include/hl_allocator/status.hpp: same codes and values,
// same Result<T> contract).
//
// Expected conditions on the scheduler's hot path (exhausted pool, stale handle,
// wrong state) come back as Status and never throw.  Programming errors throw:
// an invalid TableConfig (std::invalid_argument) and Result<T>::value() on an
// error (BadResultAccess).
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <utility>

namespace hl::alloc {

enum class Status : std::uint8_t {
  kOk = 0,
  kOutOfBlocks,        ///< no free block id
  kOutOfSlots,         ///< the pool of the requested format is full
  kInvalidHandle,      ///< id out of range
  kStaleHandle,        ///< generation mismatch (freed or reused)
  kInvalidState,       ///< not allowed in the block's current state
  kInvalidArgument,    ///< argument outside the documented bounds
  kUnknownFormat,      ///< no pool configured for the format
  kNotDeviceResident,  ///< residency is not kDevice
  kRefcountOverflow,   ///< refcount would pass kMaxRefcount
  kCorrupt,            ///< validate() found an inconsistency
  kCapacityExceeded,   ///< a 32-bit index space is exhausted
};

[[nodiscard]] const char* to_string(Status status) noexcept;

class BadResultAccess : public std::logic_error {
 public:
  explicit BadResultAccess(Status status);
  [[nodiscard]] Status status() const noexcept { return status_; }

 private:
  Status status_;
};

/// A value or a non-OK status.
template <typename T>
class [[nodiscard]] Result {
 public:
  Result(const T& v) : value_(v), status_(Status::kOk) {}             // NOLINT
  Result(T&& v) : value_(std::move(v)), status_(Status::kOk) {}       // NOLINT
  /// An OK result must carry a value, so kOk here becomes kInvalidArgument.
  Result(Status s) : status_(s == Status::kOk ? Status::kInvalidArgument : s) {}  // NOLINT

  [[nodiscard]] bool ok() const noexcept { return status_ == Status::kOk; }
  [[nodiscard]] Status status() const noexcept { return status_; }

  [[nodiscard]] const T& value() const& { return checked(), *value_; }
  [[nodiscard]] T& value() & { return checked(), *value_; }
  /// By value, so that `for (auto x : f().value())` does not dangle.
  [[nodiscard]] T value() && { return checked(), std::move(*value_); }

 private:
  void checked() const {
    if (status_ != Status::kOk) throw BadResultAccess(status_);
  }
  std::optional<T> value_;
  Status status_;
};

}  // namespace hl::alloc
