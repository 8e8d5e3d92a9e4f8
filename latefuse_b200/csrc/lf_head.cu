// Pooling + L2 normalisation + per-tenant head (gather-GEMV) + masked softmax.
//
// One CTA per batch row.  The pooled row is built in shared memory (f32 copies
// of values rounded to the storage dtype, because the reference materialises
// the pooled tensor in the model dtype), then
//   * normalised:  pooled / max(||pooled||_2, 1e-12)        F.normalize
//   * scored:      logits[j] = round(round(pooled . coef[off+j]) + bias[off+j])
//                  for j < n, 0 for n <= j < n_max         bmm + add on padded heads
//   * squashed:    softmax over the row's own n logits (max-shifted), or a
//                  sigmoid when n == 1; padded lanes are 0.
// The head rows are read in place from the packed head cache by offset, so the
// zero-padded (B, n_max, H) tensor of the reference is never built.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

struct HeadParams {
  const void* hidden;
  int64_t ld_batch;
  int64_t ld_seq;
  const int64_t* mask;
  int32_t batch, seq, H;
  int32_t pooling;
  void* pooled_out;
  void* normed_out;
  const void* coef;
  const void* bias;
  int64_t head_rows;
  const int32_t* head_off;
  const int32_t* head_n;
  int32_t n_max;
  void* logits_out;
  float* probs_out;
  int32_t* status;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

template <typename T>
__global__ void __launch_bounds__(256) head_forward_kernel(const HeadParams p) {
  extern __shared__ float sm[];
  float* pooled = sm;                 // H
  float* logits = sm + p.H;           // n_max
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const T* src = reinterpret_cast<const T*>(p.hidden);

  // ---- pooling (values rounded to T as the reference's pooled tensor is) ----
  float count = 1.f;
  if (p.pooling == LF_POOL_MEAN && p.mask != nullptr) {
    float c = 0.f;
    for (int s = tid; s < p.seq; s += blockDim.x) c += p.mask[int64_t(b) * p.seq + s] != 0 ? 1.f : 0.f;
    c = block_sum(c, red);
    // mask.sum(1) is taken in the model dtype, then clamped at 1e-9
    count = fmaxf(round_through<T>(c), 1e-9f);
  }
  for (int h = tid; h < p.H; h += blockDim.x) {
    float v;
    if (p.pooling == LF_POOL_CLS) {
      v = DT<T>::to_f(src[int64_t(b) * p.ld_batch + h]);
    } else if (p.pooling == LF_POOL_NONE) {
      v = DT<T>::to_f(src[int64_t(b) * p.ld_batch + h]);
    } else {
      float acc = 0.f;
      const T* row = src + int64_t(b) * p.ld_batch + h;
      if (p.mask != nullptr) {
        for (int s = 0; s < p.seq; ++s)
          if (p.mask[int64_t(b) * p.seq + s] != 0) acc += DT<T>::to_f(row[int64_t(s) * p.ld_seq]);
        v = round_through<T>(round_through<T>(acc) / count);
      } else {
        for (int s = 0; s < p.seq; ++s) acc += DT<T>::to_f(row[int64_t(s) * p.ld_seq]);
        v = round_through<T>(acc / float(p.seq));
      }
    }
    pooled[h] = v;
    if (p.pooled_out != nullptr) reinterpret_cast<T*>(p.pooled_out)[int64_t(b) * p.H + h] = DT<T>::from_f(v);
  }
  __syncthreads();

  // ---- L2 normalisation ----
  if (p.normed_out != nullptr) {
    float ss = 0.f;
    for (int h = tid; h < p.H; h += blockDim.x) ss = fmaf(pooled[h], pooled[h], ss);
    ss = block_sum(ss, red);
    const float denom = fmaxf(round_through<T>(sqrtf(ss)), round_through<T>(1e-12f));
    T* out = reinterpret_cast<T*>(p.normed_out) + int64_t(b) * p.H;
    for (int h = tid; h < p.H; h += blockDim.x) out[h] = DT<T>::from_f(pooled[h] / denom);
  }

  // ---- per-tenant head ----
  if (p.coef == nullptr) return;
  int off = p.head_off[b];
  int n = p.head_n[b];
  if (off < 0 || n < 0 || n > p.n_max || int64_t(off) + n > p.head_rows) {
    set_status(p.status, LF_STATUS_BAD_HEAD);
    n = 0;
    off = 0;
  }
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const T* coef = reinterpret_cast<const T*>(p.coef);
  const T* bias = reinterpret_cast<const T*>(p.bias);
  for (int j = warp; j < n; j += nwarps) {
    const T* crow = coef + int64_t(off + j) * p.H;
    float acc = 0.f;
    for (int h = lane; h < p.H; h += 32) acc = fmaf(pooled[h], DT<T>::to_f(crow[h]), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const float dot = round_through<T>(acc);
      logits[j] = round_through<T>(dot + DT<T>::to_f(bias[off + j]));
    }
  }
  __syncthreads();
  if (tid == 0) {
    T* lo = p.logits_out != nullptr ? reinterpret_cast<T*>(p.logits_out) + int64_t(b) * p.n_max : nullptr;
    float* pr = p.probs_out != nullptr ? p.probs_out + int64_t(b) * p.n_max : nullptr;
    if (n == 1) {
      if (pr) pr[0] = 1.f / (1.f + expf(-logits[0]));
    } else if (n > 1) {
      float mx = logits[0];
      for (int j = 1; j < n; ++j) mx = fmaxf(mx, logits[j]);
      float sum = 0.f;
      for (int j = 0; j < n; ++j) sum += expf(logits[j] - mx);
      if (pr)
        for (int j = 0; j < n; ++j) pr[j] = expf(logits[j] - mx) / sum;
    }
    for (int j = 0; j < p.n_max; ++j) {
      if (lo) lo[j] = DT<T>::from_f(j < n ? logits[j] : 0.f);
      if (pr && j >= n) pr[j] = 0.f;
    }
  }
}

int run_head_forward(int dtype, const HeadParams& p, cudaStream_t s) {
  const size_t smem = size_t(p.H + (p.n_max > 0 ? p.n_max : 1)) * sizeof(float);
  if (smem > 200 * 1024) return set_error(LF_ERR_UNSUPPORTED, "head_forward: hidden %d too large", p.H);
  cudaError_t e = cudaSuccess;
  switch (dtype) {
    case LF_DTYPE_F32:
      cudaFuncSetAttribute(head_forward_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      head_forward_kernel<float><<<p.batch, 256, smem, s>>>(p);
      break;
    case LF_DTYPE_BF16:
      cudaFuncSetAttribute(head_forward_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      head_forward_kernel<__nv_bfloat16><<<p.batch, 256, smem, s>>>(p);
      break;
    case LF_DTYPE_F16:
      cudaFuncSetAttribute(head_forward_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      head_forward_kernel<__half><<<p.batch, 256, smem, s>>>(p);
      break;
    default:
      return set_error(LF_ERR_INVALID, "unknown dtype %d", dtype);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch head_forward");
  count_launch();
  return LF_OK;
}

}  // namespace lf

extern "C" int lf_head_forward(void* stream, int dtype, const void* hidden, int64_t ld_batch,
                               int64_t ld_seq, const int64_t* mask, int batch, int seq,
                               int hidden_size, int pooling, void* pooled_out, void* normed_out,
                               const void* coef, const void* bias, int64_t head_rows,
                               const int32_t* head_off, const int32_t* head_n, int n_max,
                               void* logits_out, float* probs_out, int32_t* status) {
  using namespace lf;
  if (dtype != LF_DTYPE_F32 && dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_INVALID, "lf_head_forward: unknown dtype %d", dtype);
  if (hidden == nullptr || batch < 0 || hidden_size <= 0)
    return set_error(LF_ERR_INVALID, "lf_head_forward: bad hidden/batch/hidden_size");
  if (pooling != LF_POOL_CLS && pooling != LF_POOL_MEAN && pooling != LF_POOL_NONE)
    return set_error(LF_ERR_INVALID, "lf_head_forward: unknown pooling %d", pooling);
  if (pooling == LF_POOL_MEAN && seq <= 0)
    return set_error(LF_ERR_INVALID, "lf_head_forward: mean pooling needs seq > 0");
  if (coef != nullptr && (bias == nullptr || head_off == nullptr || head_n == nullptr || n_max <= 0))
    return set_error(LF_ERR_INVALID, "lf_head_forward: head needs bias, head_off, head_n and n_max > 0");
  if (batch == 0) return LF_OK;
  HeadParams p{};
  p.hidden = hidden;
  p.ld_batch = ld_batch;
  p.ld_seq = ld_seq;
  p.mask = mask;
  p.batch = batch;
  p.seq = seq;
  p.H = hidden_size;
  p.pooling = pooling;
  p.pooled_out = pooled_out;
  p.normed_out = normed_out;
  p.coef = coef;
  p.bias = bias;
  p.head_rows = head_rows;
  p.head_off = head_off;
  p.head_n = head_n;
  p.n_max = coef != nullptr ? n_max : 0;
  p.logits_out = logits_out;
  p.probs_out = probs_out;
  p.status = status;
  return run_head_forward(dtype, p, static_cast<cudaStream_t>(stream));
}
