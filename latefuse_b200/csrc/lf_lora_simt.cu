// CUDA-core LoRA kernels: any dtype (f32 / bf16 / f16), any hidden size and rank.
//
// They serve f32 batches (where exact f32 arithmetic is required, so the
// tf32/f16 tensor-core kinds do not apply) and shapes the tcgen05 kernels do
// not tile (rank not in {8,16,32,64}, hidden not a multiple of 64, strides the
// TMA engine cannot describe).  Same contract and rounding as the tcgen05 path:
// the shrink output is rounded to the storage dtype, the expand delta is rounded
// to the storage dtype before it is added, exactly as the reference's
// `out_A`/`out_B` buffers are (src/latefuse/ops/lora.py:26-27,57,75).
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

__device__ __forceinline__ int32_t seg_slot_of(const SimtParams& p, int64_t t) {
  const int g = first_seg_ending_after(p.seg_start, p.seg_len, p.n_segs, t);
  if (g >= p.n_segs) return -1;
  const int64_t s = p.seg_start[g];
  if (t < s) return -1;
  const int32_t slot = p.seg_slot[g];
  if (slot < 0 || slot >= p.n_slots) {
    set_status(p.status, LF_STATUS_BAD_SLOT);
    return -1;
  }
  return slot;
}

// One warp per token row; lanes split the hidden dimension; 8 rank columns per pass.
template <typename T>
__global__ void __launch_bounds__(256) lora_shrink_simt_kernel(const SimtParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (t >= p.n_tokens) return;
  const int32_t slot = seg_slot_of(p, t);
  const T* __restrict__ x = reinterpret_cast<const T*>(p.x) + t * p.ldx;
  const int R = p.rank, H = p.hidden;
  for (int m = 0; m < p.n_modules; ++m) {
    T* u = reinterpret_cast<T*>(p.u) + (int64_t(m) * p.n_tokens + t) * R;
    const T* __restrict__ a =
        slot < 0 ? nullptr : reinterpret_cast<const T*>(p.cache_a[m]) + int64_t(slot) * p.a_slot_stride;
    for (int j0 = 0; j0 < R; j0 += 8) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      if (a != nullptr) {
        for (int h = lane; h < H; h += 32) {
          const float xv = DT<T>::to_f(x[h]);
          const T* ar = a + int64_t(h) * R + j0;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (j0 + i < R) acc[i] = fmaf(xv, DT<T>::to_f(ar[i]), acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
      }
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (j0 + i < R) u[j0 + i] = DT<T>::from_f(acc[i]);
      }
    }
  }
}

// grid = (n_tokens, ceil(hidden / 256), n_modules); one thread per output element.
template <typename T>
__global__ void __launch_bounds__(256) lora_expand_simt_kernel(const SimtParams p) {
  const int64_t t = blockIdx.x;
  const int n = blockIdx.y * blockDim.x + threadIdx.x;
  const int m = blockIdx.z;
  if (n >= p.hidden) return;
  const int32_t slot = seg_slot_of(p, t);
  T* y = reinterpret_cast<T*>(p.y) + t * p.ldy + p.y_col_off[m] + n;
  float d = 0.f;
  if (slot >= 0) {
    const T* __restrict__ u = reinterpret_cast<const T*>(p.u) + (int64_t(m) * p.n_tokens + t) * p.rank;
    const T* __restrict__ b = reinterpret_cast<const T*>(p.cache_b[m]) + int64_t(slot) * p.b_slot_stride + n;
    float acc = 0.f;
    for (int j = 0; j < p.rank; ++j) acc = fmaf(DT<T>::to_f(u[j]), DT<T>::to_f(b[int64_t(j) * p.hidden]), acc);
    d = round_through<T>(acc);
  } else if (p.accumulate) {
    return;  // no segment: y is left untouched
  }
  *y = p.accumulate ? DT<T>::from_f(DT<T>::to_f(*y) + d) : DT<T>::from_f(d);
}

template <typename T>
static int shrink_simt(const SimtParams& p, cudaStream_t s) {
  const int rows_per_block = 8;
  dim3 grid(unsigned((p.n_tokens + rows_per_block - 1) / rows_per_block));
  lora_shrink_simt_kernel<T><<<grid, 256, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch lora_shrink_simt");
  count_launch();
  return LF_OK;
}

template <typename T>
static int expand_simt(const SimtParams& p, cudaStream_t s) {
  dim3 grid(unsigned(p.n_tokens), unsigned((p.hidden + 255) / 256), unsigned(p.n_modules));
  lora_expand_simt_kernel<T><<<grid, 256, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch lora_expand_simt");
  count_launch();
  return LF_OK;
}

int run_shrink_simt(int dtype, const SimtParams& p, cudaStream_t s) {
  switch (dtype) {
    case LF_DTYPE_F32: return shrink_simt<float>(p, s);
    case LF_DTYPE_BF16: return shrink_simt<__nv_bfloat16>(p, s);
    case LF_DTYPE_F16: return shrink_simt<__half>(p, s);
  }
  return set_error(LF_ERR_INVALID, "unknown dtype %d", dtype);
}

int run_expand_simt(int dtype, const SimtParams& p, cudaStream_t s) {
  switch (dtype) {
    case LF_DTYPE_F32: return expand_simt<float>(p, s);
    case LF_DTYPE_BF16: return expand_simt<__nv_bfloat16>(p, s);
    case LF_DTYPE_F16: return expand_simt<__half>(p, s);
  }
  return set_error(LF_ERR_INVALID, "unknown dtype %d", dtype);
}

}  // namespace lf
