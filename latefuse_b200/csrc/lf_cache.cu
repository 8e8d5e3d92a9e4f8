// Adapter-cache utilities: slot gather, slot write, and the growable
// virtual-memory arena that backs the slot cache.
#include <mutex>
#include <vector>

#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

// dst[i] = bytes of slot slots[i] (bit-exact copy).  grid = (chunks, n).
__global__ void __launch_bounds__(256)
cache_gather_kernel(const uint8_t* __restrict__ src, int64_t slot_stride_b, int64_t offset_b,
                    int64_t row_bytes, int n_slots, const int32_t* __restrict__ slots,
                    uint8_t* __restrict__ dst, int vec16, int32_t* status) {
  const int i = blockIdx.y;
  const int32_t slot = slots[i];
  uint8_t* d = dst + int64_t(i) * row_bytes;
  if (slot < 0 || slot >= n_slots) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(status, LF_STATUS_BAD_SLOT);
    return;
  }
  const uint8_t* s = src + int64_t(slot) * slot_stride_b + offset_b;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t start = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec16) {
    const uint4* s4 = reinterpret_cast<const uint4*>(s);
    uint4* d4 = reinterpret_cast<uint4*>(d);
    for (int64_t k = start; k < row_bytes / 16; k += stride) d4[k] = s4[k];
  } else {
    for (int64_t k = start; k < row_bytes; k += stride) d[k] = s[k];
  }
}

// ---------------------------------------------------------------------------
// virtual-memory arena
// ---------------------------------------------------------------------------
struct Arena {
  int device = 0;
  CUdeviceptr base = 0;
  size_t reserved = 0;
  size_t mapped = 0;
  size_t gran = 0;
  std::vector<std::pair<CUmemGenericAllocationHandle, size_t>> chunks;
  std::mutex mu;
};

struct VmmFns {
  decltype(&cuMemGetAllocationGranularity) granularity = nullptr;
  decltype(&cuMemAddressReserve) reserve = nullptr;
  decltype(&cuMemAddressFree) addr_free = nullptr;
  decltype(&cuMemCreate) create = nullptr;
  decltype(&cuMemRelease) release = nullptr;
  decltype(&cuMemMap) map = nullptr;
  decltype(&cuMemUnmap) unmap = nullptr;
  decltype(&cuMemSetAccess) set_access = nullptr;
  bool ok = false;
};

static const VmmFns& vmm() {
  static VmmFns f = [] {
    VmmFns v;
    v.granularity = reinterpret_cast<decltype(v.granularity)>(get_driver_fn("cuMemGetAllocationGranularity"));
    v.reserve = reinterpret_cast<decltype(v.reserve)>(get_driver_fn("cuMemAddressReserve"));
    v.addr_free = reinterpret_cast<decltype(v.addr_free)>(get_driver_fn("cuMemAddressFree"));
    v.create = reinterpret_cast<decltype(v.create)>(get_driver_fn("cuMemCreate"));
    v.release = reinterpret_cast<decltype(v.release)>(get_driver_fn("cuMemRelease"));
    v.map = reinterpret_cast<decltype(v.map)>(get_driver_fn("cuMemMap"));
    v.unmap = reinterpret_cast<decltype(v.unmap)>(get_driver_fn("cuMemUnmap"));
    v.set_access = reinterpret_cast<decltype(v.set_access)>(get_driver_fn("cuMemSetAccess"));
    v.ok = v.granularity && v.reserve && v.addr_free && v.create && v.release && v.map && v.unmap &&
           v.set_access;
    return v;
  }();
  return f;
}

static int drv_error(CUresult r, const char* what) {
  return set_error(LF_ERR_CUDA, "%s failed with CUresult %d", what, int(r));
}

// Makes `device` current for the duration of a scope (driver calls need a context).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
    cudaFree(nullptr);  // ensure the primary context exists
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace lf

using namespace lf;

extern "C" int lf_cache_gather(void* stream, const void* src, int64_t slot_stride, int64_t offset,
                               int64_t n_elems, int elem_bytes, int n_slots, const int32_t* slots,
                               int n, void* dst, int32_t* status) {
  if (src == nullptr || dst == nullptr || slots == nullptr || n < 0 || n_elems < 0 ||
      (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8) || n_slots <= 0)
    return set_error(LF_ERR_INVALID, "lf_cache_gather: bad arguments");
  if (n == 0 || n_elems == 0) return LF_OK;
  const int64_t row_bytes = n_elems * elem_bytes;
  const int64_t ssb = slot_stride * elem_bytes, ob = offset * elem_bytes;
  const bool vec16 = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0) &&
                     (row_bytes % 16 == 0) && (ssb % 16 == 0) && (ob % 16 == 0);
  const int64_t units = vec16 ? row_bytes / 16 : row_bytes;
  int64_t chunks = (units + 255) / 256;
  if (chunks > 1024) chunks = 1024;
  if (n > 65535) return set_error(LF_ERR_UNSUPPORTED, "lf_cache_gather: n > 65535");
  const dim3 grid{unsigned(chunks), unsigned(n), 1u};
  cache_gather_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), ssb, ob, row_bytes, n_slots, slots,
      static_cast<uint8_t*>(dst), vec16 ? 1 : 0, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch cache_gather");
  count_launch();
  return LF_OK;
}

extern "C" int lf_cache_write_slot(void* stream, void* cache_base, int64_t slot_stride_bytes,
                                   int slot, int n_slots, size_t offset, const void* src,
                                   size_t nbytes) {
  if (cache_base == nullptr || src == nullptr || slot < 0 || slot >= n_slots || slot_stride_bytes <= 0 ||
      offset + nbytes > size_t(slot_stride_bytes))
    return set_error(LF_ERR_INVALID, "lf_cache_write_slot: slot %d / range out of bounds", slot);
  uint8_t* dst = static_cast<uint8_t*>(cache_base) + int64_t(slot) * slot_stride_bytes + offset;
  cudaError_t e = cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync(write_slot)");
  return LF_OK;
}

extern "C" int lf_arena_create(int device, size_t reserve_bytes, void** handle) {
  if (handle == nullptr || reserve_bytes == 0) return set_error(LF_ERR_INVALID, "lf_arena_create: bad arguments");
  *handle = nullptr;
  const VmmFns& f = vmm();
  if (!f.ok) return set_error(LF_ERR_DRIVER, "lf_arena_create: CUDA virtual memory entry points unavailable");
  DeviceGuard guard(device);
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  size_t gran = 0;
  CUresult r = f.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuMemGetAllocationGranularity");
  const size_t reserve = (reserve_bytes + gran - 1) / gran * gran;
  CUdeviceptr base = 0;
  r = f.reserve(&base, reserve, gran, 0, 0);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuMemAddressReserve");
  Arena* a = new Arena();
  a->device = device;
  a->base = base;
  a->reserved = reserve;
  a->gran = gran;
  *handle = a;
  return LF_OK;
}

extern "C" int lf_arena_grow(void* handle, size_t mapped_bytes) {
  if (handle == nullptr) return set_error(LF_ERR_INVALID, "lf_arena_grow: null handle");
  Arena* a = static_cast<Arena*>(handle);
  std::lock_guard<std::mutex> lock(a->mu);
  if (mapped_bytes <= a->mapped) return LF_OK;
  const size_t want = (mapped_bytes + a->gran - 1) / a->gran * a->gran;
  if (want > a->reserved)
    return set_error(LF_ERR_INVALID, "lf_arena_grow: %zu bytes exceed the %zu reserved", want, a->reserved);
  const VmmFns& f = vmm();
  DeviceGuard guard(a->device);
  const size_t chunk = want - a->mapped;
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = a->device;
  CUmemGenericAllocationHandle h;
  CUresult r = f.create(&h, chunk, &prop, 0);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuMemCreate (out of device memory?)");
  r = f.map(a->base + a->mapped, chunk, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    f.release(h);
    return drv_error(r, "cuMemMap");
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = a->device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = f.set_access(a->base + a->mapped, chunk, &acc, 1);
  if (r != CUDA_SUCCESS) {
    f.unmap(a->base + a->mapped, chunk);
    f.release(h);
    return drv_error(r, "cuMemSetAccess");
  }
  a->chunks.emplace_back(h, chunk);
  a->mapped = want;
  return LF_OK;
}

extern "C" void* lf_arena_base(void* handle) {
  return handle ? reinterpret_cast<void*>(static_cast<Arena*>(handle)->base) : nullptr;
}

extern "C" size_t lf_arena_mapped_bytes(void* handle) {
  return handle ? static_cast<Arena*>(handle)->mapped : 0;
}

extern "C" int lf_arena_destroy(void* handle) {
  if (handle == nullptr) return LF_OK;
  Arena* a = static_cast<Arena*>(handle);
  const VmmFns& f = vmm();
  {
    DeviceGuard guard(a->device);
    cudaDeviceSynchronize();  // no kernel may still read the cache
    size_t off = 0;
    for (auto& c : a->chunks) {
      f.unmap(a->base + off, c.second);
      f.release(c.first);
      off += c.second;
    }
    f.addr_free(a->base, a->reserved);
  }
  delete a;
  return LF_OK;
}
