#pragma once
// HeteroBlockTable: host-side manager of KV blocks whose storage format varies
// block by block.  Drop-in for the reference's
// project1_allocator/include/hl_allocator/hetero_block_table.hpp: same public
// API, statuses and deterministic results (ids, slots, arena offsets, delta
// contents and order).
//
// A block has a stable id (guarded by a generation counter) and a slot in the
// fixed-size pool of its current format.  A sequence is a list of block ids in
// an IdArena segment and holds one reference per block; sealed blocks can be
// shared between sequences.  The device-facing state is kept incrementally:
//   descriptor table  BlockExecDescriptor[max_blocks] indexed by block id,
//                     holding device_descriptor(id) (non-executable: format 15,
//                     slot 0xFFFFFFFF, when free or not device-resident);
//   id arena          the IdArena contents.
// collect_delta() hands the changes over as self-addressed patches (applied on
// the GPU by hlkv_apply_delta), batch_segments() gives the per-step
// {offset, length} per sequence, and a kernel reads block j of sequence i as
// descriptor_table[arena[segment_i.offset + j]].  build_exec_table() is the
// O(total blocks) materialized path, kept for cross-checking the incremental one.
//
// Not thread-safe: one owner thread mutates; const calls may run concurrently
// only while nothing mutates.  release() and commit_format_change() free slots
// immediately, so a caller must not free a slot that queued GPU work still
// reads (wait for the step's stream event first).
#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "hl_allocator/block_descriptor.hpp"
#include "hl_allocator/id_arena.hpp"
#include "hl_allocator/status.hpp"

namespace hl::alloc {

struct BlockHandle {
  std::uint32_t id;
  std::uint32_t generation;
  friend constexpr bool operator==(BlockHandle, BlockHandle) noexcept = default;
};
inline constexpr BlockHandle kInvalidBlock{0xFFFF'FFFFu, 0};

struct SequenceHandle {
  std::uint32_t id;
  std::uint32_t generation;
  friend constexpr bool operator==(SequenceHandle, SequenceHandle) noexcept = default;
};
inline constexpr SequenceHandle kInvalidSequence{0xFFFF'FFFFu, 0};

struct PoolConfig {
  FormatId format{};
  std::uint32_t slot_bytes = 0;  ///< > 0
  std::uint32_t num_slots = 0;   ///< > 0
};

struct TableConfig {
  std::uint32_t max_blocks = 0;     ///< 1 .. 2^32-2
  std::uint32_t block_tokens = 16;  ///< 1 .. kMaxBlockTokens
  std::vector<PoolConfig> pools;    ///< formats unique and < kMaxFormats
};

struct AllocRequest {
  FormatId format{};
  std::uint32_t valid_tokens = 0;  ///< <= block_tokens
  std::uint32_t layout = 0;        ///< <= kMaxLayoutId
  ScaleMode scale_mode = ScaleMode::kNone;
  std::uint32_t scale_ref = 0;
};

/// Where a decode step's new token goes: token slot `token` of block `block_id`.
struct TokenTarget {
  std::uint32_t block_id;
  std::uint32_t token;
};

/// Both slots of a format change in flight.
struct FormatChange {
  FormatId from_format;
  std::uint32_t from_slot;
  FormatId to_format;
  std::uint32_t to_slot;
};

/// CSR of exec descriptors: sequence i owns blocks[indptr[i] .. indptr[i+1]).
struct ExecTable {
  std::vector<std::uint32_t> indptr;
  std::vector<BlockExecDescriptor> blocks;
};

/// Device-facing changes since the previous collect_delta().  To apply: grow
/// the arena to arena_size (keeping contents), then table[p.block_id] = p for
/// each descriptor patch and arena[p.offset] = p.block_id for each id patch.
/// Targets are unique within each list, so any order (or a parallel scatter)
/// is valid.  The first delta carries every descriptor.
struct ExecDelta {
  std::vector<BlockExecDescriptor> descriptor_patches;
  std::vector<IdPatch> id_patches;
  std::uint32_t descriptor_table_size = 0;
  std::uint32_t arena_size = 0;
};

struct TableStats {
  std::uint32_t blocks_in_use = 0;
  std::uint32_t blocks_capacity = 0;
  std::uint32_t active_sequences = 0;
  std::array<std::uint32_t, kMaxFormats> blocks_per_format{};
  std::array<std::uint32_t, 4> blocks_per_residency{};
  std::array<std::uint32_t, 4> blocks_per_state{};
  std::uint64_t valid_tokens = 0;
  std::uint64_t token_capacity_in_use = 0;
  std::uint64_t payload_bytes_in_use = 0;
  std::uint64_t format_changes_committed = 0;
  std::uint64_t arena_entries = 0;
  std::uint64_t arena_live_entries = 0;
  std::uint64_t arena_reserved_entries = 0;
  std::uint64_t arena_free_entries = 0;
  std::uint64_t pending_descriptor_patches = 0;
  std::uint64_t pending_id_patches = 0;
};

struct ValidationReport {
  Status status = Status::kOk;
  std::string message;
  [[nodiscard]] bool ok() const noexcept { return status == Status::kOk; }
};

class HeteroBlockTable {
 public:
  /// Throws std::invalid_argument when validate_config(config) != kOk.
  explicit HeteroBlockTable(const TableConfig& config);

  [[nodiscard]] static Status validate_config(const TableConfig& config) noexcept;

  // -- blocks ------------------------------------------------------------------------
  [[nodiscard]] Result<BlockHandle> allocate(const AllocRequest& request);
  [[nodiscard]] Status retain(BlockHandle handle);
  [[nodiscard]] Status release(BlockHandle handle);

  [[nodiscard]] Status set_valid_tokens(BlockHandle handle, std::uint32_t valid_tokens);
  [[nodiscard]] Status seal(BlockHandle handle);
  [[nodiscard]] Status set_residency(BlockHandle handle, Residency residency);
  [[nodiscard]] Status set_scale(BlockHandle handle, ScaleMode mode, std::uint32_t scale_ref);

  /// Reserves a slot of `target`; the block stays readable in its old format.
  [[nodiscard]] Result<FormatChange> begin_format_change(BlockHandle handle, FormatId target);
  [[nodiscard]] Status commit_format_change(BlockHandle handle, ScaleMode mode,
                                            std::uint32_t scale_ref);
  [[nodiscard]] Status abort_format_change(BlockHandle handle);

  [[nodiscard]] Result<BlockDescriptor> lookup(BlockHandle handle) const;
  [[nodiscard]] Status lookup_batch(std::span<const BlockHandle> handles,
                                    std::span<BlockExecDescriptor> out) const;
  [[nodiscard]] BlockHandle handle_of(std::uint32_t block_id) const noexcept;

  // -- sequences ---------------------------------------------------------------------
  [[nodiscard]] Result<SequenceHandle> create_sequence();
  [[nodiscard]] Result<BlockHandle> append_block(SequenceHandle seq, const AllocRequest& request);
  [[nodiscard]] Status append_shared_block(SequenceHandle seq, BlockHandle block);
  [[nodiscard]] Status release_sequence(SequenceHandle seq);
  /// Decode-step driver (no counterpart in the reference): one more token per sequence.
  /// While the tail block has room, set_valid_tokens(tail, vt + 1) and out[i] = {tail, vt};
  /// otherwise append_block(seqs[i], {new_formats[i], 1 valid token, layout}) and
  /// out[i] = {new block, 0}.  The same state, delta and statuses as those public calls made
  /// one sequence at a time; stops at the first failure, n_done = sequences completed.
  [[nodiscard]] Status append_tokens(std::span<const SequenceHandle> seqs,
                                     std::span<const FormatId> new_formats, std::uint32_t layout,
                                     std::span<TokenTarget> out, std::size_t& n_done);
  [[nodiscard]] Result<std::span<const std::uint32_t>> sequence_block_ids(
      SequenceHandle seq) const;
  [[nodiscard]] Status build_exec_table(std::span<const SequenceHandle> seqs,
                                        ExecTable& out) const;

  /// Packs the id arena (IdArena::compact over every live sequence's segment): the
  /// storage a burst of long sequences left behind is given back and the live segments
  /// become contiguous.  `moves` receives the segment moves the device copy of the arena
  /// must make before any later delta is applied (hlkv_device_tables_relocate).  Sequence
  /// contents and handles are unchanged; batch_segments() reports the new offsets.
  /// kInvalidState while id patches are pending: collect the delta first.  No counterpart
  /// in the reference.
  [[nodiscard]] Status compact_arena(std::vector<SegmentMove>& moves);

  // -- device-facing state -----------------------------------------------------------
  [[nodiscard]] Status batch_segments(std::span<const SequenceHandle> seqs,
                                      std::vector<SequenceSegment>& out) const;
  void collect_delta(ExecDelta& out);
  [[nodiscard]] BlockExecDescriptor device_descriptor(std::uint32_t block_id) const noexcept;
  [[nodiscard]] std::size_t pending_descriptor_patches() const noexcept {
    return changed_blocks_.size();
  }
  [[nodiscard]] std::size_t pending_id_patches() const noexcept {
    return arena_.pending_patches();
  }

  // -- introspection -----------------------------------------------------------------
  [[nodiscard]] std::uint32_t block_tokens() const noexcept { return block_tokens_; }
  [[nodiscard]] std::uint32_t max_blocks() const noexcept {
    return static_cast<std::uint32_t>(blocks_.size());
  }
  [[nodiscard]] std::uint32_t blocks_in_use() const noexcept { return in_use_; }
  [[nodiscard]] bool has_pool(FormatId format) const noexcept;
  [[nodiscard]] std::uint32_t free_slots(FormatId format) const noexcept;
  [[nodiscard]] std::uint32_t pool_slots(FormatId format) const noexcept;
  [[nodiscard]] std::uint32_t slot_bytes(FormatId format) const noexcept;

  [[nodiscard]] TableStats stats() const;

  // -- snapshot (no counterpart in the reference, whose ABI v1 lists the missing
  //    snapshot API among its limitations, hl_allocator_abi.md section 9) ------------
  /// A versioned binary image of the whole table: configuration, block records, free
  /// lists, pool stacks, sequences and id arena, with a checksum trailer.
  [[nodiscard]] std::vector<std::byte> snapshot() const;
  /// Rebuilds the table that `image` describes into `out`.  kCorrupt, with `out`
  /// untouched, for an image that is short, damaged (checksum), of another version, ABI
  /// or byte order, or inconsistent (validate()).  The restored table behaves as the
  /// original from then on (same handles, free lists and arena layout), except that
  /// every descriptor and arena entry is pending: its first collect_delta() carries the
  /// whole device image, for a fresh device mirror.
  [[nodiscard]] static Status restore(std::span<const std::byte> image,
                                      std::unique_ptr<HeteroBlockTable>& out);
  [[nodiscard]] ValidationReport validate() const;

 private:
  static constexpr std::uint32_t kEnd = 0xFFFF'FFFFu;  // end of a free chain

  // The free slots of one pool, handed out last-freed-first: a stack threaded through
  // `below` (below[s] = the slot under s while s is free).  Sized once; never allocates.
  struct SlotStack {
    bool present = false;
    std::uint32_t slot_bytes = 0;
    std::uint32_t capacity = 0;
    std::uint32_t top = kEnd;
    std::uint32_t depth = 0;
    std::vector<std::uint32_t> below;
  };
  // A sequence: its arena segment, or -- once released -- a link in the chain of free
  // sequence ids (seg.offset, with capacity and length 0).
  struct SeqRecord {
    IdArena::Segment seg;
    std::uint32_t generation = 0;
    bool live = false;
  };

  [[nodiscard]] Status find(BlockHandle h, BlockDescriptor*& out) noexcept;
  [[nodiscard]] Status find(BlockHandle h, const BlockDescriptor*& out) const noexcept;
  [[nodiscard]] Status find(SequenceHandle h, SeqRecord*& out) noexcept;
  [[nodiscard]] Status find(SequenceHandle h, const SeqRecord*& out) const noexcept;
  [[nodiscard]] Status admissible(const AllocRequest& r) const noexcept;
  [[nodiscard]] SlotStack* stack(FormatId f) noexcept;
  [[nodiscard]] const SlotStack* stack(FormatId f) const noexcept;
  static bool pop(SlotStack& st, std::uint32_t& slot) noexcept;
  static void push(SlotStack& st, std::uint32_t slot) noexcept;
  void init_free_record(std::uint32_t id, std::uint32_t generation) noexcept;
  void unreference(std::uint32_t id) noexcept;
  void free_block(std::uint32_t id) noexcept;

  std::uint32_t block_tokens_;
  std::uint32_t in_use_ = 0;
  std::uint64_t committed_changes_ = 0;
  std::vector<BlockDescriptor> blocks_;   // by id; a free record's `reserved` links the free ids
  std::uint32_t free_block_top_ = kEnd;   // next id allocate() hands out
  std::array<SlotStack, kMaxFormats> slots_{};
  std::vector<SeqRecord> seq_records_;
  std::uint32_t free_seq_top_ = kEnd;     // next id create_sequence() reuses
  IdArena arena_;
  detail::ChangeQueue changed_blocks_;    // ids whose device descriptor is out of date
};

}  // namespace hl::alloc
