#pragma once
// HL-KV block descriptor ABI (version 1): the per-block records shared by the
// host table and the GPU kernels.
//
// Drop-in for project1_allocator/include/hl_allocator/block_descriptor.hpp of
// the reference: the names, constants, bit positions and byte layouts below are
// the ABI and must be identical (golden bytes are pinned by the tests), so they
// follow the reference field for field; the code around them is this
// library's own.
//
//   BlockExecDescriptor, 16 bytes (device-facing, one 128-bit load per block):
//     0..3 slot | 4..7 info | 8..11 scale_ref | 12..15 block_id
//     info = format:4 | scale_mode:2 | layout:4 | valid_tokens:10 | zero:12
//   BlockDescriptor, 32 bytes (host record; the first 16 bytes are the exec record):
//     16..19 generation | 20..23 control | 24..27 pending_slot | 28..31 reserved
//     control = state:2 | residency:2 | pending_format:4 | refcount:16 | zero:8
//
// Words are packed with explicit shifts and masks, never C++ bit-fields, so the
// layout does not depend on the compiler (host g++ and device nvcc agree).
#include <bit>
#include <cstddef>
#include <cstdint>
#include <type_traits>

namespace hl::alloc {

static_assert(std::endian::native == std::endian::little,
              "the HL-KV ABI is little-endian (x86-64, AArch64 hosts and NVIDIA GPUs)");

inline constexpr std::uint32_t kAbiVersion = 1;

/// 4-bit storage-format code; the allocator treats it as opaque.  The codes in
/// use are those of hl::quant::QuantFormat (0 FP16, 1 E4M3, 2 E5M2, 3 INT4).
enum class FormatId : std::uint8_t {};

inline constexpr std::uint32_t kMaxFormats = 15;      ///< codes 0..14 name pools
inline constexpr FormatId kInvalidFormat{15};         ///< "not executable"
inline constexpr std::uint32_t kMaxBlockTokens = 512; ///< valid_tokens is 10 bits wide
inline constexpr std::uint32_t kNoSlot = 0xFFFF'FFFFu;

/// How a block's scale metadata is found.
enum class ScaleMode : std::uint8_t {
  kNone = 0,            ///< unscaled, per-tensor, or scales inside the slot payload
  kInlineF32 = 1,       ///< scale_ref = binary32 bits of one per-block scale
  kInlineF16Pair = 2,   ///< scale_ref = binary16 scale (bits 0..15) | binary16 bias (16..31)
  kExternal = 3,        ///< scale_ref indexes an external scale pool
};

enum class BlockState : std::uint8_t {
  kFree = 0,
  kOpen = 1,          ///< tokens may still be appended
  kSealed = 2,        ///< payload immutable; may be shared or re-encoded
  kTranscoding = 3,   ///< sealed, with a format change in flight (two slots live)
};

enum class Residency : std::uint8_t {
  kDevice = 0,   ///< in a device pool slot
  kHost = 1,     ///< offloaded (a tag only in ABI v1)
  kDropped = 2,  ///< payload discarded
};

namespace bits {

[[nodiscard]] constexpr std::uint32_t mask(std::uint32_t width) noexcept {
  return width >= 32u ? ~0u : (1u << width) - 1u;
}
[[nodiscard]] constexpr std::uint32_t get(std::uint32_t word, std::uint32_t shift,
                                          std::uint32_t width) noexcept {
  return (word >> shift) & mask(width);
}
[[nodiscard]] constexpr std::uint32_t set(std::uint32_t word, std::uint32_t shift,
                                          std::uint32_t width, std::uint32_t value) noexcept {
  const std::uint32_t field = mask(width) << shift;
  return (word & ~field) | ((value << shift) & field);
}

// BlockExecDescriptor::info
inline constexpr std::uint32_t kFormatShift = 0, kFormatWidth = 4;
inline constexpr std::uint32_t kScaleModeShift = 4, kScaleModeWidth = 2;
inline constexpr std::uint32_t kLayoutShift = 6, kLayoutWidth = 4;
inline constexpr std::uint32_t kValidTokensShift = 10, kValidTokensWidth = 10;
inline constexpr std::uint32_t kInfoReservedShift = 20;

// BlockDescriptor::control
inline constexpr std::uint32_t kStateShift = 0, kStateWidth = 2;
inline constexpr std::uint32_t kResidencyShift = 2, kResidencyWidth = 2;
inline constexpr std::uint32_t kPendingFormatShift = 4, kPendingFormatWidth = 4;
inline constexpr std::uint32_t kRefcountShift = 8, kRefcountWidth = 16;
inline constexpr std::uint32_t kControlReservedShift = 24;

static_assert(kMaxBlockTokens < (1u << kValidTokensWidth));
static_assert(kMaxFormats < (1u << kFormatWidth));

}  // namespace bits

inline constexpr std::uint32_t kMaxLayoutId = bits::mask(bits::kLayoutWidth);
inline constexpr std::uint32_t kMaxRefcount = bits::mask(bits::kRefcountWidth);

/// Device-facing record.  Payload address = pool_base[format] + slot * slot_bytes[format].
struct alignas(16) BlockExecDescriptor {
  std::uint32_t slot;
  std::uint32_t info;
  std::uint32_t scale_ref;
  std::uint32_t block_id;

  [[nodiscard]] static constexpr std::uint32_t pack_info(FormatId format, ScaleMode scale_mode,
                                                         std::uint32_t layout,
                                                         std::uint32_t valid_tokens) noexcept {
    using namespace bits;
    std::uint32_t w = set(0u, kFormatShift, kFormatWidth, static_cast<std::uint32_t>(format));
    w = set(w, kScaleModeShift, kScaleModeWidth, static_cast<std::uint32_t>(scale_mode));
    w = set(w, kLayoutShift, kLayoutWidth, layout);
    return set(w, kValidTokensShift, kValidTokensWidth, valid_tokens);
  }

  [[nodiscard]] constexpr FormatId format() const noexcept {
    return FormatId{static_cast<std::uint8_t>(bits::get(info, bits::kFormatShift, bits::kFormatWidth))};
  }
  [[nodiscard]] constexpr ScaleMode scale_mode() const noexcept {
    return static_cast<ScaleMode>(bits::get(info, bits::kScaleModeShift, bits::kScaleModeWidth));
  }
  [[nodiscard]] constexpr std::uint32_t layout() const noexcept {
    return bits::get(info, bits::kLayoutShift, bits::kLayoutWidth);
  }
  [[nodiscard]] constexpr std::uint32_t valid_tokens() const noexcept {
    return bits::get(info, bits::kValidTokensShift, bits::kValidTokensWidth);
  }
  [[nodiscard]] constexpr std::uint32_t info_reserved() const noexcept {
    return info >> bits::kInfoReservedShift;
  }
  /// The per-block scale; meaningful for ScaleMode::kInlineF32 only.
  [[nodiscard]] constexpr float inline_scale_f32() const noexcept {
    return std::bit_cast<float>(scale_ref);
  }

  constexpr void set_format(FormatId f) noexcept {
    info = bits::set(info, bits::kFormatShift, bits::kFormatWidth, static_cast<std::uint32_t>(f));
  }
  constexpr void set_scale_mode(ScaleMode m) noexcept {
    info = bits::set(info, bits::kScaleModeShift, bits::kScaleModeWidth,
                     static_cast<std::uint32_t>(m));
  }
  constexpr void set_valid_tokens(std::uint32_t n) noexcept {
    info = bits::set(info, bits::kValidTokensShift, bits::kValidTokensWidth, n);
  }

  friend constexpr bool operator==(const BlockExecDescriptor&,
                                   const BlockExecDescriptor&) noexcept = default;
};

/// Host-side record held by HeteroBlockTable.
struct alignas(32) BlockDescriptor {
  BlockExecDescriptor exec;
  std::uint32_t generation;
  std::uint32_t control;
  std::uint32_t pending_slot;
  std::uint32_t reserved;

  [[nodiscard]] constexpr BlockState state() const noexcept {
    return static_cast<BlockState>(bits::get(control, bits::kStateShift, bits::kStateWidth));
  }
  [[nodiscard]] constexpr Residency residency() const noexcept {
    return static_cast<Residency>(bits::get(control, bits::kResidencyShift, bits::kResidencyWidth));
  }
  [[nodiscard]] constexpr FormatId pending_format() const noexcept {
    return FormatId{static_cast<std::uint8_t>(
        bits::get(control, bits::kPendingFormatShift, bits::kPendingFormatWidth))};
  }
  [[nodiscard]] constexpr std::uint32_t refcount() const noexcept {
    return bits::get(control, bits::kRefcountShift, bits::kRefcountWidth);
  }
  [[nodiscard]] constexpr std::uint32_t control_reserved() const noexcept {
    return control >> bits::kControlReservedShift;
  }

  constexpr void set_state(BlockState s) noexcept {
    control = bits::set(control, bits::kStateShift, bits::kStateWidth, static_cast<std::uint32_t>(s));
  }
  constexpr void set_residency(Residency r) noexcept {
    control = bits::set(control, bits::kResidencyShift, bits::kResidencyWidth,
                        static_cast<std::uint32_t>(r));
  }
  constexpr void set_pending_format(FormatId f) noexcept {
    control = bits::set(control, bits::kPendingFormatShift, bits::kPendingFormatWidth,
                        static_cast<std::uint32_t>(f));
  }
  constexpr void set_refcount(std::uint32_t n) noexcept {
    control = bits::set(control, bits::kRefcountShift, bits::kRefcountWidth, n);
  }

  friend constexpr bool operator==(const BlockDescriptor&,
                                   const BlockDescriptor&) noexcept = default;
};

static_assert(sizeof(BlockExecDescriptor) == 16 && alignof(BlockExecDescriptor) == 16);
static_assert(std::is_trivially_copyable_v<BlockExecDescriptor> &&
              std::is_standard_layout_v<BlockExecDescriptor>);
static_assert(offsetof(BlockExecDescriptor, slot) == 0 && offsetof(BlockExecDescriptor, info) == 4 &&
              offsetof(BlockExecDescriptor, scale_ref) == 8 &&
              offsetof(BlockExecDescriptor, block_id) == 12);
static_assert(sizeof(BlockDescriptor) == 32 && alignof(BlockDescriptor) == 32);
static_assert(64 % alignof(BlockDescriptor) == 0, "a record never straddles a 64-byte line");
static_assert(std::is_trivially_copyable_v<BlockDescriptor> &&
              std::is_standard_layout_v<BlockDescriptor>);
static_assert(offsetof(BlockDescriptor, exec) == 0 && offsetof(BlockDescriptor, generation) == 16 &&
              offsetof(BlockDescriptor, control) == 20 &&
              offsetof(BlockDescriptor, pending_slot) == 24 &&
              offsetof(BlockDescriptor, reserved) == 28);

}  // namespace hl::alloc
