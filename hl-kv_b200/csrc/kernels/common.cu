#include "common.cuh"

namespace hlkv {
namespace {
thread_local cudaError_t g_last_error = cudaSuccess;
}  // namespace

int cuda_status(cudaError_t e) noexcept {
  g_last_error = e;
  return e == cudaSuccess ? HLKV_OK : HLKV_CUDA_ERROR;
}

int sm_count() noexcept {
  static thread_local int cached_device = -1;
  static thread_local int cached = 0;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 1;
  if (device != cached_device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 1;
    cached = n;
    cached_device = device;
  }
  return cached;
}

uint64_t layout_code_bytes(int format, uint64_t elems) {
  switch (format) {
    case HLKV_FP16: return 2 * elems;
    case HLKV_FP8_E4M3:
    case HLKV_FP8_E5M2: return elems;
    case HLKV_INT4: return (elems + 1) / 2;
    default: return 0;
  }
}

bool layout_ok(const HlkvLayout* l) {
  return l != nullptr && l->block_tokens >= 1 && l->block_tokens <= 512 && l->kv_heads >= 1 &&
         (l->head_dim == 64 || l->head_dim == 128 || l->head_dim == 256) && l->layout_id <= 15 &&
         uint64_t{l->block_tokens} * l->kv_heads * l->head_dim <= (uint64_t{1} << 30);
}

}  // namespace hlkv

extern "C" int hlkv_last_cuda_error(void) { return static_cast<int>(hlkv::g_last_error); }

extern "C" uint64_t hlkv_layout_slot_bytes(int format, const HlkvLayout* layout) {
  if (!hlkv::layout_ok(layout) || format < 0 || format > 3) return 0;
  const uint64_t rows = uint64_t{2} * layout->block_tokens * layout->kv_heads;
  const uint64_t elems = rows * layout->head_dim;
  const uint64_t params = format == 0 ? 0 : (format == 3 ? 8 * rows : 4 * rows);
  return hlkv::layout_code_bytes(format, elems) + params;
}
