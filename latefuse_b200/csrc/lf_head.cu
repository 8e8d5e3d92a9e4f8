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
//
// lf_head_forward_rows serves the padding-free forward, whose hidden states are
// packed (n_tokens, H): row b is token row_index[b] (its CLS token), optionally
// through the encoder's pooler tanh(W x + b) (pooler_rows_kernel, CUDA cores:
// 16 rows x 64 outputs per CTA, the rows gathered once into shared memory), then
// the same normalisation / head / softmax, launched as a programmatic dependent.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

struct HeadParams {
  const void* hidden;
  const int32_t* row_index;  // CLS / NONE: row b reads hidden row row_index[b] (null: row b)
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
  pdl_wait();  // a pooler kernel before this one has written its rows

  // ---- pooling (values rounded to T as the reference's pooled tensor is) ----
  float count = 1.f;
  if (p.pooling == LF_POOL_MEAN && p.mask != nullptr) {
    float c = 0.f;
    for (int s = tid; s < p.seq; s += blockDim.x) c += p.mask[int64_t(b) * p.seq + s] != 0 ? 1.f : 0.f;
    c = block_sum(c, red);
    // mask.sum(1) is taken in the model dtype, then clamped at 1e-9
    count = fmaxf(round_through<T>(c), 1e-9f);
  }
  const int64_t rb = p.row_index != nullptr ? int64_t(p.row_index[b]) : int64_t(b);
  for (int h = tid; h < p.H; h += blockDim.x) {
    float v;
    if (p.pooling == LF_POOL_CLS || p.pooling == LF_POOL_NONE) {
      v = DT<T>::to_f(src[rb * p.ld_batch + h]);
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
  // eight consecutive elements per lane per step (16-byte loads for 2-byte types)
  // when every head row starts on a 16-byte boundary; element-wise otherwise
  const bool vec = (p.H % 8) == 0 && (reinterpret_cast<uintptr_t>(coef) & 15u) == 0 && sizeof(T) == 2;
  for (int j = warp; j < n; j += nwarps) {
    const T* crow = coef + int64_t(off + j) * p.H;
    float acc = 0.f;
    if constexpr (sizeof(T) == 2) {
      if (vec) {
      for (int h = lane * 8; h < p.H; h += 256) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(crow + h));
        const float4 x0 = *reinterpret_cast<const float4*>(pooled + h);
        const float4 x1 = *reinterpret_cast<const float4*>(pooled + h + 4);
        float2 f = Pack2<T>::unpack(w.x);
        acc = fmaf(x0.x, f.x, acc);
        acc = fmaf(x0.y, f.y, acc);
        f = Pack2<T>::unpack(w.y);
        acc = fmaf(x0.z, f.x, acc);
        acc = fmaf(x0.w, f.y, acc);
        f = Pack2<T>::unpack(w.z);
        acc = fmaf(x1.x, f.x, acc);
        acc = fmaf(x1.y, f.y, acc);
        f = Pack2<T>::unpack(w.w);
        acc = fmaf(x1.z, f.x, acc);
        acc = fmaf(x1.w, f.y, acc);
      }
      } else {
        for (int h = lane; h < p.H; h += 32) acc = fmaf(pooled[h], DT<T>::to_f(crow[h]), acc);
      }
    } else {
      (void)vec;
      for (int h = lane; h < p.H; h += 32) acc = fmaf(pooled[h], DT<T>::to_f(crow[h]), acc);
    }
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


// ---------------------------------------------------------------------------
// pooler: out[b] = round(tanh(round(x[b] . W^T + bias))), x[b] = hidden[row_index[b]]
// (HF's pooler: nn.Linear then nn.Tanh, each output materialised in the dtype).
// Grid (H / 64, ceil(B / 16)); 8 warps, each owning 8 output columns for the
// CTA's 16 rows.  The rows sit in shared memory as f32; W rows are read with
// 16-byte loads, eight elements per lane per step, and reduced across the warp.
// ---------------------------------------------------------------------------
constexpr int kPoolRows = 16, kPoolCols = 64;

struct PoolerParams {
  const void* hidden;
  int64_t ld;
  const int32_t* row_index;
  int32_t batch, H;
  const void* w;   // (H, H) row-major: out column c is row c
  const void* b;   // (H,)
  void* out;       // (B, H)
};

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Pack2<T>::unpack(ws[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 c = __ldg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) pooler_rows_kernel(const PoolerParams p) {
  extern __shared__ float xs[];  // kPoolRows x H
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.y * kPoolRows;
  const int nr = min(kPoolRows, p.batch - r0);
  const T* hid = reinterpret_cast<const T*>(p.hidden);
  pdl_wait();
  for (int i = tid; i < kPoolRows * p.H; i += blockDim.x) {
    const int r = i / p.H, h = i - r * p.H;
    float v = 0.f;
    if (r < nr) {
      const int64_t src = p.row_index != nullptr ? int64_t(p.row_index[r0 + r]) : int64_t(r0 + r);
      v = DT<T>::to_f(hid[src * p.ld + h]);
    }
    xs[i] = v;
  }
  __syncthreads();
  pdl_launch_dependents();
  const T* W = reinterpret_cast<const T*>(p.w);
  const T* bias = reinterpret_cast<const T*>(p.b);
  T* out = reinterpret_cast<T*>(p.out);
  for (int cc = 0; cc < kPoolCols / 8; ++cc) {
    const int c = blockIdx.x * kPoolCols + warp * (kPoolCols / 8) + cc;
    if (c >= p.H) break;
    float acc[kPoolRows];
#pragma unroll
    for (int r = 0; r < kPoolRows; ++r) acc[r] = 0.f;
    for (int h = lane * 8; h < p.H; h += 256) {
      float wv[8];
      load8<T>(W + int64_t(c) * p.H + h, wv);
#pragma unroll
      for (int r = 0; r < kPoolRows; ++r) {
        const float4 a = *reinterpret_cast<const float4*>(xs + r * p.H + h);
        const float4 d = *reinterpret_cast<const float4*>(xs + r * p.H + h + 4);
        float s = acc[r];
        s = fmaf(a.x, wv[0], s); s = fmaf(a.y, wv[1], s); s = fmaf(a.z, wv[2], s); s = fmaf(a.w, wv[3], s);
        s = fmaf(d.x, wv[4], s); s = fmaf(d.y, wv[5], s); s = fmaf(d.z, wv[6], s); s = fmaf(d.w, wv[7], s);
        acc[r] = s;
      }
    }
#pragma unroll
    for (int r = 0; r < kPoolRows; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (lane < nr) {  // lane r writes row r of column c
      float v = 0.f;
#pragma unroll
      for (int r = 0; r < kPoolRows; ++r) v = lane == r ? acc[r] : v;
      const float lin = round_through<T>(v + (bias != nullptr ? DT<T>::to_f(bias[c]) : 0.f));
      out[int64_t(r0 + lane) * p.H + c] = DT<T>::from_f(tanhf(lin));
    }
  }
}

int run_head_forward(int dtype, const HeadParams& p, cudaStream_t s) {
  const size_t smem = size_t(p.H + (p.n_max > 0 ? p.n_max : 1)) * sizeof(float);
  if (smem > 200 * 1024) return set_error(LF_ERR_UNSUPPORTED, "head_forward: hidden %d too large", p.H);
  cudaError_t e = cudaSuccess;
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    return launch_pdl(kern, dim3(p.batch), dim3(256), smem, s, p);
  };
  switch (dtype) {
    case LF_DTYPE_F32: e = go(head_forward_kernel<float>); break;
    case LF_DTYPE_BF16: e = go(head_forward_kernel<__nv_bfloat16>); break;
    case LF_DTYPE_F16: e = go(head_forward_kernel<__half>); break;
    default:
      return set_error(LF_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (e != cudaSuccess) return cuda_error(e, "launch head_forward");
  count_launch();
  return LF_OK;
}


int run_pooler(int dtype, const PoolerParams& p, cudaStream_t s) {
  const size_t smem = size_t(kPoolRows) * p.H * sizeof(float);
  if (smem > 220 * 1024) return set_error(LF_ERR_UNSUPPORTED, "head_forward_rows: hidden %d too large", p.H);
  const dim3 grid((p.H + kPoolCols - 1) / kPoolCols, (p.batch + kPoolRows - 1) / kPoolRows);
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    return launch_pdl(kern, grid, dim3(256), smem, s, p);
  };
  cudaError_t e;
  switch (dtype) {
    case LF_DTYPE_F32: e = go(pooler_rows_kernel<float>); break;
    case LF_DTYPE_BF16: e = go(pooler_rows_kernel<__nv_bfloat16>); break;
    case LF_DTYPE_F16: e = go(pooler_rows_kernel<__half>); break;
    default:
      return set_error(LF_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (e != cudaSuccess) return cuda_error(e, "launch pooler_rows");
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
  p.row_index = nullptr;
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

extern "C" int lf_head_forward_rows(void* stream, int dtype, const void* hidden, int64_t ld,
                                    const int32_t* row_index, int batch, int hidden_size,
                                    const void* pooler_w, const void* pooler_b, void* pooled_out,
                                    void* normed_out, const void* coef, const void* bias, int64_t head_rows,
                                    const int32_t* head_off, const int32_t* head_n, int n_max,
                                    void* logits_out, float* probs_out, int32_t* status) {
  using namespace lf;
  if (dtype != LF_DTYPE_F32 && dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_INVALID, "lf_head_forward_rows: unknown dtype %d", dtype);
  if (hidden == nullptr || batch < 0 || hidden_size <= 0 || ld < hidden_size)
    return set_error(LF_ERR_INVALID, "lf_head_forward_rows: bad hidden/batch/hidden_size/ld");
  if (coef != nullptr && (bias == nullptr || head_off == nullptr || head_n == nullptr || n_max <= 0))
    return set_error(LF_ERR_INVALID, "lf_head_forward_rows: head needs bias, head_off, head_n and n_max > 0");
  if (pooler_w != nullptr) {
    const size_t esz = dtype == LF_DTYPE_F32 ? 4 : 2;
    if (pooled_out == nullptr)
      return set_error(LF_ERR_INVALID, "lf_head_forward_rows: the pooler writes its rows to pooled_out");
    if (hidden_size % 8 != 0 || (reinterpret_cast<uintptr_t>(pooler_w) & 15u) != 0 || (hidden_size * esz) % 16 != 0)
      return set_error(LF_ERR_UNSUPPORTED, "lf_head_forward_rows: pooler needs hidden %% 8 == 0 and a 16-byte "
                       "aligned weight");
  }
  if (batch == 0) return LF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  HeadParams p{};
  if (pooler_w != nullptr) {
    PoolerParams q{hidden, ld, row_index, batch, hidden_size, pooler_w, pooler_b, pooled_out};
    int rc = run_pooler(dtype, q, s);
    if (rc != LF_OK) return rc;
    if (normed_out == nullptr && coef == nullptr) return LF_OK;  // the pooled rows were all that was asked
    p.hidden = pooled_out;  // the head reads the pooled rows in order
    p.row_index = nullptr;
    p.ld_batch = hidden_size;
    p.pooled_out = nullptr;
  } else {
    p.hidden = hidden;
    p.row_index = row_index;
    p.ld_batch = ld;
    p.pooled_out = pooled_out;
  }
  p.ld_seq = 0;
  p.mask = nullptr;
  p.batch = batch;
  p.seq = 1;
  p.H = hidden_size;
  p.pooling = LF_POOL_NONE;
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
  return run_head_forward(dtype, p, s);
}
