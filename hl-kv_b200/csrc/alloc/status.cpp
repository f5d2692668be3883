#include "hl_allocator/status.hpp"

#include <string>

namespace hl::alloc {

const char* to_string(Status status) noexcept {
  static constexpr const char* kNames[] = {
      "ok",           "out of blocks",    "out of slots",        "invalid handle",
      "stale handle", "invalid state",    "invalid argument",    "unknown format",
      "not device resident", "refcount overflow", "corrupt", "capacity exceeded"};
  const auto i = static_cast<std::size_t>(status);
  return i < sizeof(kNames) / sizeof(kNames[0]) ? kNames[i] : "unknown status";
}

BadResultAccess::BadResultAccess(Status status)
    : std::logic_error(std::string("hl_allocator: value() of a failed Result: ") + to_string(status)),
      status_(status) {}

}  // namespace hl::alloc
