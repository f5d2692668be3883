// extern "C" layer of include/hlkv.h over the C++ host objects, and the C++
// hl::quant::cuda entry points over the C kernels' launchers.
#include <cstddef>
#include <cstring>
#include <memory>
#include <new>
#include <span>
#include <vector>

#include "hl_allocator/hetero_block_table.hpp"
#include "hl_kv/device_tables.hpp"
#include "hl_quant/cuda_dequant.hpp"
#include "hlkv.h"

namespace hlkv {
int launch_append_encode(const HlkvPools* pools, const HlkvLayout* layout, const HlkvExecDescriptor* d_table,
                         uint32_t table_size, const HlkvAppendTarget* d_targets, uint32_t n,
                         const uint16_t* d_tokens, uint32_t* d_err, bool overlap_previous, cudaStream_t s);
}

using namespace hl::alloc;

struct hlkv_table {
  HeteroBlockTable t;
  ExecDelta scratch_delta;  // reused by hlkv_table_collect_delta
  explicit hlkv_table(const TableConfig& c) : t(c) {}
  explicit hlkv_table(HeteroBlockTable&& restored) : t(std::move(restored)) {}
};

struct hlkv_device_tables {
  hl::kv::DeviceTables dt;
};

static_assert(sizeof(HlkvExecDescriptor) == sizeof(BlockExecDescriptor));
static_assert(sizeof(HlkvIdPatch) == sizeof(IdPatch));
static_assert(sizeof(HlkvSegment) == sizeof(SequenceSegment));
static_assert(sizeof(HlkvSegmentMove) == sizeof(SegmentMove) && offsetof(HlkvSegmentMove, scratch) ==
                                                                    offsetof(SegmentMove, scratch));
static_assert(sizeof(HlkvHandle) == sizeof(SequenceHandle) && offsetof(HlkvHandle, generation) ==
                                                                  offsetof(SequenceHandle, generation));
static_assert(sizeof(HlkvAppendTarget) == sizeof(TokenTarget) &&
              offsetof(HlkvAppendTarget, token) == offsetof(TokenTarget, token));
static_assert(static_cast<int>(Status::kCapacityExceeded) == HLKV_STATUS_CAPACITY_EXCEEDED);

namespace {

int st(Status s) { return static_cast<int>(s); }
BlockHandle bh(HlkvHandle h) { return BlockHandle{h.id, h.generation}; }
SequenceHandle sh(HlkvHandle h) { return SequenceHandle{h.id, h.generation}; }
HlkvHandle out_of(BlockHandle h) { return HlkvHandle{h.id, h.generation}; }
HlkvHandle out_of(SequenceHandle h) { return HlkvHandle{h.id, h.generation}; }
HlkvExecDescriptor out_of(const BlockExecDescriptor& d) {
  HlkvExecDescriptor r;
  std::memcpy(&r, &d, sizeof(r));
  return r;
}

std::uint8_t narrow(uint32_t v) { return static_cast<std::uint8_t>(v > 0xFFu ? 0xFFu : v); }
FormatId fmt(uint32_t f) { return FormatId{narrow(f)}; }

bool to_config(const HlkvTableConfig* c, TableConfig& out) {
  if (c == nullptr || (c->num_pools > 0 && c->pools == nullptr)) return false;
  out.max_blocks = c->max_blocks;
  out.block_tokens = c->block_tokens;
  out.pools.clear();
  for (uint32_t i = 0; i < c->num_pools; ++i) {
    if (c->pools[i].format > 0xFFu) return false;
    out.pools.push_back(PoolConfig{fmt(c->pools[i].format), c->pools[i].slot_bytes,
                                   c->pools[i].num_slots});
  }
  return true;
}

AllocRequest to_request(const HlkvAllocRequest* r) {
  AllocRequest a;
  a.format = fmt(r->format);
  a.valid_tokens = r->valid_tokens;
  a.layout = r->layout;
  a.scale_mode = static_cast<ScaleMode>(narrow(r->scale_mode));
  a.scale_ref = r->scale_ref;
  return a;
}

}  // namespace

extern "C" {

int hlkv_table_validate_config(const HlkvTableConfig* config) {
  TableConfig c;
  if (!to_config(config, c)) return HLKV_STATUS_INVALID_ARGUMENT;
  return st(HeteroBlockTable::validate_config(c));
}

int hlkv_table_create(const HlkvTableConfig* config, hlkv_table** out) {
  if (out == nullptr) return HLKV_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  TableConfig c;
  if (!to_config(config, c)) return HLKV_STATUS_INVALID_ARGUMENT;
  if (const Status s = HeteroBlockTable::validate_config(c); s != Status::kOk) return st(s);
  try {
    *out = new hlkv_table(c);
  } catch (const std::bad_alloc&) {
    return HLKV_STATUS_CAPACITY_EXCEEDED;
  }
  return HLKV_STATUS_OK;
}

void hlkv_table_destroy(hlkv_table* table) { delete table; }

int hlkv_table_snapshot(const hlkv_table* t, void* buf, size_t cap, size_t* size) {
  if (t == nullptr || size == nullptr) return HLKV_STATUS_INVALID_ARGUMENT;
  std::vector<std::byte> image;
  try {
    image = t->t.snapshot();
  } catch (const std::bad_alloc&) {
    return HLKV_STATUS_CAPACITY_EXCEEDED;
  }
  *size = image.size();
  if (buf == nullptr || cap < image.size()) return buf == nullptr ? HLKV_STATUS_OK : HLKV_STATUS_INVALID_ARGUMENT;
  std::memcpy(buf, image.data(), image.size());
  return HLKV_STATUS_OK;
}

int hlkv_table_restore(const void* buf, size_t size, hlkv_table** out) {
  if (out == nullptr || (buf == nullptr && size > 0)) return HLKV_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  try {
    std::unique_ptr<HeteroBlockTable> table;
    const Status s = HeteroBlockTable::restore(
        std::span<const std::byte>(static_cast<const std::byte*>(buf), size), table);
    if (s != Status::kOk) return st(s);
    *out = new hlkv_table(std::move(*table));
  } catch (const std::bad_alloc&) {
    return HLKV_STATUS_CAPACITY_EXCEEDED;
  }
  return HLKV_STATUS_OK;
}

int hlkv_table_allocate(hlkv_table* t, const HlkvAllocRequest* req, HlkvHandle* out) {
  if (t == nullptr || req == nullptr || out == nullptr) return HLKV_STATUS_INVALID_ARGUMENT;
  const Result<BlockHandle> r = t->t.allocate(to_request(req));
  if (r.ok()) *out = out_of(r.value());
  return st(r.status());
}

int hlkv_table_retain(hlkv_table* t, HlkvHandle b) { return st(t->t.retain(bh(b))); }
int hlkv_table_release(hlkv_table* t, HlkvHandle b) { return st(t->t.release(bh(b))); }
int hlkv_table_set_valid_tokens(hlkv_table* t, HlkvHandle b, uint32_t n) {
  return st(t->t.set_valid_tokens(bh(b), n));
}
int hlkv_table_seal(hlkv_table* t, HlkvHandle b) { return st(t->t.seal(bh(b))); }
int hlkv_table_set_residency(hlkv_table* t, HlkvHandle b, uint32_t r) {
  return st(t->t.set_residency(bh(b), static_cast<Residency>(narrow(r))));
}
int hlkv_table_set_scale(hlkv_table* t, HlkvHandle b, uint32_t mode, uint32_t ref) {
  return st(t->t.set_scale(bh(b), static_cast<ScaleMode>(narrow(mode)), ref));
}

int hlkv_table_begin_format_change(hlkv_table* t, HlkvHandle b, uint32_t target, uint32_t out[4]) {
  const Result<FormatChange> r = t->t.begin_format_change(bh(b), fmt(target));
  if (r.ok() && out != nullptr) {
    out[0] = static_cast<uint32_t>(r.value().from_format);
    out[1] = r.value().from_slot;
    out[2] = static_cast<uint32_t>(r.value().to_format);
    out[3] = r.value().to_slot;
  }
  return st(r.status());
}

int hlkv_table_commit_format_change(hlkv_table* t, HlkvHandle b, uint32_t mode, uint32_t ref) {
  return st(t->t.commit_format_change(bh(b), static_cast<ScaleMode>(narrow(mode)), ref));
}
int hlkv_table_abort_format_change(hlkv_table* t, HlkvHandle b) {
  return st(t->t.abort_format_change(bh(b)));
}

int hlkv_table_lookup(const hlkv_table* t, HlkvHandle b, void* out32) {
  const Result<BlockDescriptor> r = t->t.lookup(bh(b));
  if (r.ok() && out32 != nullptr) std::memcpy(out32, &r.value(), sizeof(BlockDescriptor));
  return st(r.status());
}

int hlkv_table_lookup_batch(const hlkv_table* t, const HlkvHandle* blocks, size_t n,
                            HlkvExecDescriptor* out, size_t out_n) {
  if ((n > 0 && blocks == nullptr) || (out_n > 0 && out == nullptr)) return HLKV_STATUS_INVALID_ARGUMENT;
  std::vector<BlockHandle> hs(n);
  for (size_t i = 0; i < n; ++i) hs[i] = bh(blocks[i]);
  std::vector<BlockExecDescriptor> tmp(out_n);
  const Status s = t->t.lookup_batch(hs, tmp);
  if (s == Status::kOk) {
    for (size_t i = 0; i < n; ++i) out[i] = out_of(tmp[i]);
  }
  return st(s);
}

HlkvHandle hlkv_table_handle_of(const hlkv_table* t, uint32_t block_id) {
  return out_of(t->t.handle_of(block_id));
}

int hlkv_table_create_sequence(hlkv_table* t, HlkvHandle* out) {
  const Result<SequenceHandle> r = t->t.create_sequence();
  if (r.ok() && out != nullptr) *out = out_of(r.value());
  return st(r.status());
}

int hlkv_table_append_block(hlkv_table* t, HlkvHandle seq, const HlkvAllocRequest* req,
                            HlkvHandle* out) {
  if (req == nullptr) return HLKV_STATUS_INVALID_ARGUMENT;
  const Result<BlockHandle> r = t->t.append_block(sh(seq), to_request(req));
  if (r.ok() && out != nullptr) *out = out_of(r.value());
  return st(r.status());
}

int hlkv_table_append_shared_block(hlkv_table* t, HlkvHandle seq, HlkvHandle block) {
  return st(t->t.append_shared_block(sh(seq), bh(block)));
}

int hlkv_table_release_sequence(hlkv_table* t, HlkvHandle seq) {
  return st(t->t.release_sequence(sh(seq)));
}

int hlkv_table_sequence_block_ids(const hlkv_table* t, HlkvHandle seq, uint32_t* out, size_t cap,
                                  size_t* len) {
  const Result<std::span<const std::uint32_t>> r = t->t.sequence_block_ids(sh(seq));
  if (!r.ok()) return st(r.status());
  const std::span<const std::uint32_t> ids = r.value();
  if (len != nullptr) *len = ids.size();
  if (cap < ids.size() || (!ids.empty() && out == nullptr)) return HLKV_STATUS_INVALID_ARGUMENT;
  if (!ids.empty()) std::memcpy(out, ids.data(), ids.size_bytes());
  return HLKV_STATUS_OK;
}

int hlkv_table_batch_segments(const hlkv_table* t, const HlkvHandle* seqs, size_t n,
                              HlkvSegment* out) {
  if (n > 0 && (seqs == nullptr || out == nullptr)) return HLKV_STATUS_INVALID_ARGUMENT;
  std::vector<SequenceHandle> hs(n);
  for (size_t i = 0; i < n; ++i) hs[i] = sh(seqs[i]);
  std::vector<SequenceSegment> segs;
  const Status s = t->t.batch_segments(hs, segs);
  if (s == Status::kOk && !segs.empty()) std::memcpy(out, segs.data(), segs.size() * sizeof(HlkvSegment));
  return st(s);
}

int hlkv_table_append_tokens(hlkv_table* t, const HlkvHandle* seqs, size_t n,
                             const uint32_t* new_formats, uint32_t layout,
                             HlkvAppendTarget* out, size_t* n_done) {
  if (n_done != nullptr) *n_done = 0;
  if (n > 0 && (seqs == nullptr || new_formats == nullptr || out == nullptr)) {
    return HLKV_STATUS_INVALID_ARGUMENT;
  }
  // Reused per thread: no allocation once they have grown to the batch size.
  thread_local std::vector<SequenceHandle> hs;
  thread_local std::vector<FormatId> fs;
  thread_local std::vector<TokenTarget> tg;
  hs.resize(n);
  fs.resize(n);
  tg.resize(n);
  if (n > 0) std::memcpy(hs.data(), seqs, n * sizeof(SequenceHandle));
  for (size_t i = 0; i < n; ++i) fs[i] = fmt(new_formats[i]);
  size_t done = 0;
  const Status s = t->t.append_tokens(hs, fs, layout, tg, done);
  if (done > 0) std::memcpy(out, tg.data(), done * sizeof(HlkvAppendTarget));
  if (n_done != nullptr) *n_done = done;
  return st(s);
}

int hlkv_table_build_exec_table(const hlkv_table* t, const HlkvHandle* seqs, size_t n,
                                uint32_t* indptr, HlkvExecDescriptor* blocks, size_t cap,
                                size_t* total) {
  if (n > 0 && seqs == nullptr) return HLKV_STATUS_INVALID_ARGUMENT;
  std::vector<SequenceHandle> hs(n);
  for (size_t i = 0; i < n; ++i) hs[i] = sh(seqs[i]);
  ExecTable et;
  const Status s = t->t.build_exec_table(hs, et);
  if (total != nullptr) *total = et.blocks.size();
  if (s != Status::kOk) return st(s);
  if (cap < et.blocks.size() || indptr == nullptr || (!et.blocks.empty() && blocks == nullptr)) {
    return HLKV_STATUS_INVALID_ARGUMENT;
  }
  std::memcpy(indptr, et.indptr.data(), et.indptr.size() * sizeof(uint32_t));
  if (!et.blocks.empty()) std::memcpy(blocks, et.blocks.data(), et.blocks.size() * 16);
  return HLKV_STATUS_OK;
}

void hlkv_table_pending(const hlkv_table* t, size_t* n_desc, size_t* n_id) {
  if (n_desc != nullptr) *n_desc = t->t.pending_descriptor_patches();
  if (n_id != nullptr) *n_id = t->t.pending_id_patches();
}

int hlkv_table_collect_delta(hlkv_table* t, HlkvExecDescriptor* desc, size_t desc_cap,
                             HlkvIdPatch* ids, size_t id_cap, size_t* n_desc, size_t* n_id,
                             uint32_t* table_size, uint32_t* arena_size) {
  const size_t nd = t->t.pending_descriptor_patches(), ni = t->t.pending_id_patches();
  if (n_desc != nullptr) *n_desc = nd;
  if (n_id != nullptr) *n_id = ni;
  if (desc_cap < nd || id_cap < ni || (nd > 0 && desc == nullptr) || (ni > 0 && ids == nullptr)) {
    return HLKV_STATUS_INVALID_ARGUMENT;
  }
  t->t.collect_delta(t->scratch_delta);
  const ExecDelta& d = t->scratch_delta;
  if (nd > 0) std::memcpy(desc, d.descriptor_patches.data(), nd * 16);
  if (ni > 0) std::memcpy(ids, d.id_patches.data(), ni * 8);
  if (table_size != nullptr) *table_size = d.descriptor_table_size;
  if (arena_size != nullptr) *arena_size = d.arena_size;
  return HLKV_STATUS_OK;
}

int hlkv_table_compact_arena(hlkv_table* t, HlkvSegmentMove* out, size_t cap, size_t* n_moves) {
  // A compaction makes at most one move per live sequence: check the room before changing
  // anything.
  const std::uint32_t live = t->t.stats().active_sequences;
  if (n_moves != nullptr) *n_moves = 0;
  if (cap < live || (live > 0 && out == nullptr)) return HLKV_STATUS_INVALID_ARGUMENT;
  try {
    std::vector<SegmentMove> moves;
    const Status s = t->t.compact_arena(moves);
    if (s != Status::kOk) return st(s);
    if (!moves.empty()) std::memcpy(out, moves.data(), moves.size() * sizeof(SegmentMove));
    if (n_moves != nullptr) *n_moves = moves.size();
    return HLKV_STATUS_OK;
  } catch (const std::bad_alloc&) {
    return HLKV_STATUS_CAPACITY_EXCEEDED;
  }
}

HlkvExecDescriptor hlkv_table_device_descriptor(const hlkv_table* t, uint32_t block_id) {
  return out_of(t->t.device_descriptor(block_id));
}

uint32_t hlkv_table_block_tokens(const hlkv_table* t) { return t->t.block_tokens(); }
uint32_t hlkv_table_max_blocks(const hlkv_table* t) { return t->t.max_blocks(); }
uint32_t hlkv_table_blocks_in_use(const hlkv_table* t) { return t->t.blocks_in_use(); }
int hlkv_table_has_pool(const hlkv_table* t, uint32_t f) { return t->t.has_pool(fmt(f)) ? 1 : 0; }
uint32_t hlkv_table_free_slots(const hlkv_table* t, uint32_t f) { return t->t.free_slots(fmt(f)); }
uint32_t hlkv_table_pool_slots(const hlkv_table* t, uint32_t f) { return t->t.pool_slots(fmt(f)); }
uint32_t hlkv_table_slot_bytes(const hlkv_table* t, uint32_t f) { return t->t.slot_bytes(fmt(f)); }

void hlkv_table_stats(const hlkv_table* t, uint64_t out[36]) {
  const TableStats s = t->t.stats();
  size_t k = 0;
  out[k++] = s.blocks_in_use;
  out[k++] = s.blocks_capacity;
  out[k++] = s.active_sequences;
  for (const uint32_t v : s.blocks_per_format) out[k++] = v;
  for (const uint32_t v : s.blocks_per_residency) out[k++] = v;
  for (const uint32_t v : s.blocks_per_state) out[k++] = v;
  for (const uint64_t v : {s.valid_tokens, s.token_capacity_in_use, s.payload_bytes_in_use,
                           s.format_changes_committed, s.arena_entries, s.arena_live_entries,
                           s.arena_reserved_entries, s.arena_free_entries,
                           s.pending_descriptor_patches, s.pending_id_patches}) {
    out[k++] = v;
  }
}

int hlkv_table_validate(const hlkv_table* t, char* msg, size_t cap) {
  const ValidationReport r = t->t.validate();
  if (msg != nullptr && cap > 0) {
    const size_t n = r.message.size() < cap - 1 ? r.message.size() : cap - 1;
    std::memcpy(msg, r.message.data(), n);
    msg[n] = '\0';
  }
  return st(r.status);
}

// ---- device tables ------------------------------------------------------------------------

int hlkv_device_tables_create(hlkv_device_tables** out) {
  if (out == nullptr) return HLKV_INVALID_ARGUMENT;
  *out = new (std::nothrow) hlkv_device_tables();
  return *out == nullptr ? HLKV_CUDA_ERROR : HLKV_OK;
}

void hlkv_device_tables_destroy(hlkv_device_tables* dt) { delete dt; }

int hlkv_device_tables_sync(hlkv_device_tables* dt, hlkv_table* t, hlkv_stream_t stream) {
  if (dt == nullptr || t == nullptr) return HLKV_INVALID_ARGUMENT;
  const hl::kv::DeviceStatus s = dt->dt.sync(t->t, reinterpret_cast<cudaStream_t>(stream));
  return static_cast<int>(s.status);
}

int hlkv_device_tables_collect(hlkv_device_tables* dt, hlkv_table* t) {
  if (dt == nullptr || t == nullptr) return HLKV_INVALID_ARGUMENT;
  try {
    return static_cast<int>(dt->dt.collect(t->t).status);
  } catch (const std::bad_alloc&) {
    return HLKV_BUFFER_TOO_SMALL;
  }
}

int hlkv_device_tables_relocate(hlkv_device_tables* dt, const HlkvSegmentMove* moves, size_t n,
                                uint32_t new_arena_size, hlkv_stream_t stream) {
  if (dt == nullptr || (n > 0 && moves == nullptr) || n > 0xFFFFFFFFu) return HLKV_INVALID_ARGUMENT;
  try {
    const std::span<const SegmentMove> mv(reinterpret_cast<const SegmentMove*>(moves), n);
    return static_cast<int>(dt->dt.relocate(mv, new_arena_size, reinterpret_cast<cudaStream_t>(stream)).status);
  } catch (const std::bad_alloc&) {
    return HLKV_BUFFER_TOO_SMALL;
  }
}

uint64_t hlkv_device_tables_arena_capacity_bytes(const hlkv_device_tables* dt) {
  return dt->dt.arena_capacity_bytes();
}

int hlkv_device_tables_flush(hlkv_device_tables* dt, hlkv_stream_t stream) {
  if (dt == nullptr) return HLKV_INVALID_ARGUMENT;
  return static_cast<int>(dt->dt.flush(reinterpret_cast<cudaStream_t>(stream)).status);
}

int hlkv_decode_step_queue(hlkv_device_tables* dt, const HlkvPools* pools, const HlkvLayout* layout,
                           const HlkvAppendTarget* h_targets, HlkvAppendTarget* d_targets, uint32_t n,
                           const uint16_t* d_tokens, uint32_t* d_err, void* start_event,
                           void* encode_event, hlkv_stream_t stream) {
  if (dt == nullptr || pools == nullptr || layout == nullptr || d_err == nullptr) return HLKV_INVALID_ARGUMENT;
  if (n > 0 && (h_targets == nullptr || d_targets == nullptr || d_tokens == nullptr)) {
    return HLKV_INVALID_ARGUMENT;
  }
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Kernel (3) copies the targets while it applies the delta, reading h_targets in place
  // (page-locked host memory is device-readable at its device address): no upload copy.
  const void* src = nullptr;
  if (n > 0) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, h_targets) != cudaSuccess || attr.devicePointer == nullptr) {
      (void)cudaGetLastError();
      return HLKV_INVALID_ARGUMENT;  // pageable memory: not readable by a kernel
    }
    src = attr.devicePointer;
  }
  if (start_event != nullptr) {
    if (cudaEventRecord(static_cast<cudaEvent_t>(start_event), s) != cudaSuccess) return HLKV_CUDA_ERROR;
  }
  // Kernel (3) and then kernel (2) with programmatic serialization: kernel (2)'s first token
  // loads overlap kernel (3), and it waits for kernel (3) before reading the targets and the
  // table.  The staging buffers' release is recorded after kernel (2), so that no event
  // separates the two kernels.
  if (const int f = static_cast<int>(dt->dt.flush_deferred(s, src, d_targets, n).status); f != HLKV_OK) {
    (void)dt->dt.release_staging(s);
    return f;
  }
  if (encode_event != nullptr) {
    if (cudaEventRecord(static_cast<cudaEvent_t>(encode_event), s) != cudaSuccess) {
      (void)dt->dt.release_staging(s);
      return HLKV_CUDA_ERROR;
    }
  }
  // An event between the kernels leaves nothing to overlap: kernel (2) is then launched plainly.
  const int st = hlkv::launch_append_encode(pools, layout, hlkv_device_tables_table(dt), dt->dt.table_size(),
                                            d_targets, n, d_tokens, d_err, encode_event == nullptr, s);
  const int r = static_cast<int>(dt->dt.release_staging(s).status);
  return st != HLKV_OK ? st : r;
}

const HlkvExecDescriptor* hlkv_device_tables_table(const hlkv_device_tables* dt) {
  return reinterpret_cast<const HlkvExecDescriptor*>(dt->dt.table());
}
uint32_t hlkv_device_tables_table_size(const hlkv_device_tables* dt) { return dt->dt.table_size(); }
const uint32_t* hlkv_device_tables_arena(const hlkv_device_tables* dt) { return dt->dt.arena(); }
uint32_t hlkv_device_tables_arena_size(const hlkv_device_tables* dt) { return dt->dt.arena_size(); }
uint32_t* hlkv_device_tables_error_word(const hlkv_device_tables* dt) { return dt->dt.error_word(); }

}  // extern "C"

// ---- C++ hl::quant::cuda over the C entry points --------------------------------------------

namespace hl::quant {

const char* to_string(QuantStatus status) noexcept {
  switch (status) {
    case QuantStatus::kOk: return "ok";
    case QuantStatus::kInvalidArgument: return "invalid argument";
    case QuantStatus::kBufferTooSmall: return "buffer too small";
    case QuantStatus::kUnsupportedFormat: return "unsupported format";
    case QuantStatus::kCudaError: return "CUDA error";
  }
  return "unknown status";
}

namespace cuda {
namespace {
DeviceStatus wrap(int s) {
  return s == HLKV_OK ? DeviceStatus{}
                      : DeviceStatus{static_cast<QuantStatus>(s),
                                     s == HLKV_CUDA_ERROR ? static_cast<cudaError_t>(hlkv_last_cuda_error())
                                                          : cudaSuccess};
}
}  // namespace

DeviceStatus dequantize_fp8_to_fp16(QuantFormat format, const std::byte* d_in, std::size_t n,
                                    const AffineParams* d_params, std::size_t group_size,
                                    std::uint16_t* d_out, cudaStream_t stream) noexcept {
  return wrap(hlkv_dequantize_fp8_to_fp16(static_cast<int>(format), d_in, n,
                                          reinterpret_cast<const float*>(d_params), group_size,
                                          d_out, reinterpret_cast<hlkv_stream_t>(stream)));
}

DeviceStatus dequantize_to_fp16(QuantFormat format, const std::byte* d_packed,
                                std::size_t packed_size, std::size_t n,
                                const AffineParams* d_params, std::size_t n_params,
                                std::size_t group_size, std::uint16_t* d_out, std::size_t out_size,
                                std::uint32_t* d_err, cudaStream_t stream) noexcept {
  return wrap(hlkv_dequantize_to_fp16(static_cast<int>(format), d_packed, packed_size, n,
                                      reinterpret_cast<const float*>(d_params), n_params,
                                      group_size, d_out, out_size, d_err,
                                      reinterpret_cast<hlkv_stream_t>(stream)));
}

DeviceStatus quantize(QuantFormat format, const float* d_in, std::size_t n, std::size_t group_size,
                      AffineParams* d_params, std::size_t n_params, std::byte* d_packed,
                      std::size_t packed_size, std::uint32_t* d_err, cudaStream_t stream) noexcept {
  return wrap(hlkv_quantize(static_cast<int>(format), d_in, n, group_size,
                            reinterpret_cast<float*>(d_params), n_params, d_packed, packed_size,
                            d_err, reinterpret_cast<hlkv_stream_t>(stream)));
}

}  // namespace cuda
}  // namespace hl::quant
