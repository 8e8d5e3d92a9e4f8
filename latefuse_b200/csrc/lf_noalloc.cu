// lf_lora_apply_noalloc: the fused late-fusion delta for callers that cannot
// allocate device memory.
//
// lf_lora_apply needs a device workspace for the shrink output (n_modules x
// n_tokens x rank elements) and expects the caller to allocate it.  Some callers
// cannot: code running inside a framework that owns every device allocation
// (a serving runtime with a fixed memory plan, a plugin host whose allocator
// must not be bypassed), or code that must not call cudaMalloc at all, because
// cudaMalloc can synchronise the device or fail mid-request once the memory has
// been carved up.  This entry point takes the same inputs and outputs, and
// keeps the workspace in a file-scope device array instead.
//
// The array is a static __device__ object of LF_NOALLOC_SCRATCH_BYTES, so every
// GPU on which the library is loaded holds it until the process exits.  Host
// code cannot use the array's name as a device address (on the host it names a
// stand-in symbol), so the first call on each device, with that device current,
// looks the real address up with cudaGetSymbolAddress and remembers it; make
// that first call before any stream capture.  Every call shares the one array:
// calls whose kernels may overlap on the GPU (different streams without
// ordering between them) race on it.  Nothing in the scratch needs to start at
// zero: the shrink kernel writes every row that the expand kernel then reads.
#include <mutex>

#include "lf_common.cuh"
#include "lf_internal.h"

namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[LF_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" int lf_lora_apply_noalloc(void* stream, int dtype,
                                     const void* x, int64_t ldx,
                                     void* y, int64_t ldy,
                                     int64_t n_tokens, int hidden, int rank,
                                     const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                                     const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                                     int n_slots, int n_modules, const int32_t* modules,
                                     const int64_t* y_col_offsets,
                                     const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                                     int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                                     int32_t* status) {
  using namespace lf;
  const size_t need = lf_lora_workspace_bytes(dtype, n_tokens, rank, n_modules);
  if (need > LF_NOALLOC_SCRATCH_BYTES)
    return set_error(LF_ERR_WORKSPACE,
                     "lf_lora_apply_noalloc: %zu bytes of scratch needed (n_modules x n_tokens x rank elements), "
                     "more than the %zu-byte static scratch; split the batch or use lf_lora_apply",
                     need, size_t(LF_NOALLOC_SCRATCH_BYTES));
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "lf_lora_apply_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(LF_ERR_UNSUPPORTED, "lf_lora_apply_noalloc: device ordinal %d", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // resolved with `dev` current
      if (e != cudaSuccess) return cuda_error(e, "lf_lora_apply_noalloc: cudaGetSymbolAddress");
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  // the shrink + expand launches, with u in the static array (lf_lora_apply's one-launch
  // kernel keeps u on chip and would not use it)
  return apply_entry(false, stream, dtype, x, ldx, y, ldy, n_tokens, hidden, rank, cache_a, a_slot_stride,
                     a_module_stride, cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules,
                     y_col_offsets, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles, n_multi, scratch,
                     LF_NOALLOC_SCRATCH_BYTES, status);
}
