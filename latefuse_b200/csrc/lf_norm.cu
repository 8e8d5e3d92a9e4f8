// Encoder elementwise kernels: residual add + LayerNorm, and the exact GELU.
//
// add + LayerNorm (the encoder's "LayerNorm(sublayer_out + residual)",
// src/latefuse/model/encoder.py:137,141, and the embeddings' LayerNorm at :275
// with no residual):
//     s   = round_T(a + b)                       the add materialises in T first
// or, with a row vector v instead of b (a projection bias, when the GEMM has
// already added the residual), s = round_T(a + v);
//     out = round_T((s - mean) * rsqrt(var + eps) * gamma + beta)
// mean and biased variance in f32 over the row (two passes over registers).
// One warp per row: lane l holds elements [256 c + 8 l, 256 c + 8 l + 8) of
// chunk c, read and written as 16-byte vectors, so a row is one pass over HBM.
//
// GELU (ACT2FN["gelu"], src/latefuse/model/encoder.py:122,139):
//     out = round_T(x * 0.5 * (1 + erf(x / sqrt(2))))       in f32
// For bf16 and f16 the input has only 65,536 values, so the function is a
// table: each device computes it once (every input bit pattern through the f32
// formula above, then rounded), and the kernel copies the 128 KB table into
// shared memory and looks every element up.  The results are the formula's,
// bit for bit, and the kernel runs at the speed of its HBM traffic instead of
// the erf arithmetic.
#include <mutex>
#include <type_traits>

#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

namespace {

// 8 consecutive elements of T as floats, and back (16-byte vectors for 2-byte T).
template <typename T>
struct Vec8 {
  static __device__ __forceinline__ void load(const T* p, float (&v)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Pack2<T>::unpack(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(T* p, const float (&v)[8]) {
    uint4 raw;
    raw.x = Pack2<T>::pack(v[0], v[1]);
    raw.y = Pack2<T>::pack(v[2], v[3]);
    raw.z = Pack2<T>::pack(v[4], v[5]);
    raw.w = Pack2<T>::pack(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = raw;
  }
};

template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// 8 consecutive elements of T kept as raw bytes (one or two 16-byte words)
// until they are needed: half the registers of 8 floats for 2-byte T.
template <typename T>
struct Raw8 {
  uint4 w[sizeof(T) / 2];
  __device__ __forceinline__ void load(const T* p) {
#pragma unroll
    for (int i = 0; i < int(sizeof(T) / 2); ++i) w[i] = reinterpret_cast<const uint4*>(p)[i];
  }
  __device__ __forceinline__ void unpack(float (&v)[8]) const {
    if constexpr (sizeof(T) == 2) {
      const uint32_t u[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = Pack2<T>::unpack(u[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const uint32_t u[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(u[i]);
    }
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kNormWarps = 8;

// MODE 0: a alone; 1: a + b (a second matrix); 2: a + v (one row vector); 3: the
// embeddings, round(round(a[ia] + c[ic]) + b[ib]) of gathered table rows (the
// encoder's word + token type, then + position, each sum rounded as torch rounds it).
template <typename T, int NC, int MODE>
__global__ void __launch_bounds__(32 * kNormWarps)
add_layernorm_kernel(const NormParams p, int full) {
  constexpr bool HAS_B = MODE != 0;
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (row >= p.n_rows) return;
  int64_t ra_row = row, rb_row = row, rc_row = 0;
  if constexpr (MODE == 3) {
    ra_row = __ldg(p.ia + row);
    rb_row = __ldg(p.ib + row);
    rc_row = p.ic != nullptr ? __ldg(p.ic + row) : 0;
    const bool bad = ra_row < 0 || ra_row >= p.n_a || rb_row < 0 || rb_row >= p.n_b || rc_row < 0 || rc_row >= p.n_c;
    if (bad) {
      if (lane == 0) set_status(p.status, LF_STATUS_BAD_SLOT);
      ra_row = (ra_row < 0 || ra_row >= p.n_a) ? 0 : ra_row;
      rb_row = (rb_row < 0 || rb_row >= p.n_b) ? 0 : rb_row;
      rc_row = (rc_row < 0 || rc_row >= p.n_c) ? 0 : rc_row;
    }
  }
  const T* a = reinterpret_cast<const T*>(p.a) + ra_row * p.lda;
  const T* b = MODE == 1 || MODE == 3 ? reinterpret_cast<const T*>(p.b) + rb_row * p.ldb
               : MODE == 2 ? reinterpret_cast<const T*>(p.vec) : nullptr;
  const T* cc = MODE == 3 ? reinterpret_cast<const T*>(p.c) + rc_row * p.ldc : nullptr;
  const T* gamma = reinterpret_cast<const T*>(p.gamma);
  const T* beta = reinterpret_cast<const T*>(p.beta);
  T* out = reinterpret_cast<T*>(p.out) + row * p.ldo;
  const int H = p.hidden;

  // every load of the row (and gamma / beta) is issued before any arithmetic
  Raw8<T> ra[NC], rb[NC], rc[MODE == 3 ? NC : 1];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = c * 256 + lane * 8;
    if (full || col < H) {
      ra[c].load(a + col);
      if (HAS_B) rb[c].load(b + col);
      if constexpr (MODE == 3) rc[c].load(cc + col);
    }
  }
  // gamma and beta too, so that their latency overlaps the reductions instead
  // of following them (rows up to 2048 wide; wider rows load them at the end,
  // where the registers are free)
  constexpr bool kEarly = NC <= 8;
  Raw8<T> g[kEarly ? NC : 1], bt[kEarly ? NC : 1];
  if constexpr (kEarly) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = c * 256 + lane * 8;
      if (full || col < H) {
        g[c].load(gamma + col);
        bt[c].load(beta + col);
      }
    }
  }
  float v[NC][8];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = c * 256 + lane * 8;
    if (full || col < H) {
      ra[c].unpack(v[c]);
      if constexpr (MODE == 3) {
        float w[8];
        rc[c].unpack(w);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = round_through<T>(v[c][i] + w[i]);
      }
      if (HAS_B) {
        float w[8];
        rb[c].unpack(w);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = round_through<T>(v[c][i] + w[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[c][i];
    }
  }
  const float mean = warp_sum(sum) / float(H);
  float sq = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (full || c * 256 + lane * 8 < H) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / float(H) + p.eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = c * 256 + lane * 8;
    if (full || col < H) {
      float gf[8], bf[8], o[8];
      if constexpr (kEarly) {
        g[c].unpack(gf);
        bt[c].unpack(bf);
      } else {
        Vec8<T>::load(gamma + col, gf);
        Vec8<T>::load(beta + col, bf);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * rstd * gf[i] + bf[i];
      Vec8<T>::store(out + col, o);
    }
  }
}

// One table per 2-byte dtype and device: entry i is GELU of the value whose bits are i.
__device__ uint16_t g_gelu_table[2][65536];

template <typename T>
__global__ void __launch_bounds__(256) gelu_table_init_kernel(int which) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536) return;
  const uint16_t bits = uint16_t(i);
  const T v = *reinterpret_cast<const T*>(&bits);
  const T r = DT<T>::from_f(gelu_f32(DT<T>::to_f(v)));
  g_gelu_table[which][i] = *reinterpret_cast<const uint16_t*>(&r);
}

constexpr int kLutThreads = 1024;

// x and out as 16-byte vectors of 8 elements; the table goes to shared memory first.
__global__ void __launch_bounds__(kLutThreads, 1)
gelu_lut_kernel(const uint4* __restrict__ x, uint4* __restrict__ out, int64_t n8, int which) {
  extern __shared__ uint4 s_tab4[];
  const uint4* tab = reinterpret_cast<const uint4*>(g_gelu_table[which]);
  for (int i = threadIdx.x; i < 65536 / 8; i += kLutThreads) s_tab4[i] = tab[i];
  __syncthreads();
  pdl_wait();  // the table was built long before; x comes from the previous kernel
  pdl_launch_dependents();
  const uint16_t* s_tab = reinterpret_cast<const uint16_t*>(s_tab4);
  auto map = [&](uint32_t w) {
    return uint32_t(s_tab[w & 0xffffu]) | (uint32_t(s_tab[w >> 16]) << 16);
  };
  const int64_t stride = int64_t(gridDim.x) * kLutThreads;
  int64_t i = int64_t(blockIdx.x) * kLutThreads + threadIdx.x;
  for (; i + stride < n8; i += 2 * stride) {  // two vectors in flight per thread
    const uint4 a = x[i], b = x[i + stride];
    out[i] = make_uint4(map(a.x), map(a.y), map(a.z), map(a.w));
    out[i + stride] = make_uint4(map(b.x), map(b.y), map(b.z), map(b.w));
  }
  if (i < n8) {
    const uint4 a = x[i];
    out[i] = make_uint4(map(a.x), map(a.y), map(a.z), map(a.w));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) gelu_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t n8) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    float v[8];
    Vec8<T>::load(x + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = gelu_f32(v[k]);
    Vec8<T>::store(out + i * 8, v);
  }
}

template <typename T>
int launch_norm(const NormParams& p, cudaStream_t s) {
  const int nc = (p.hidden + 255) / 256;
  const int full = p.hidden == nc * 256;  // every lane holds NC whole 8-element chunks
  cudaError_t e = cudaSuccess;
  const unsigned blocks = unsigned((p.n_rows + kNormWarps - 1) / kNormWarps);
  const dim3 grid{blocks}, block{32 * kNormWarps};
  switch (nc) {
#define LF_NORM_CASE(N)                                                                  \
  case N:                                                                                \
    e = launch_pdl(p.ia != nullptr ? add_layernorm_kernel<T, N, 3>                       \
                   : p.b != nullptr ? add_layernorm_kernel<T, N, 1>                      \
                   : p.vec != nullptr ? add_layernorm_kernel<T, N, 2> : add_layernorm_kernel<T, N, 0>, \
                   grid, block, 0, s, p, full);                                          \
    break;
    LF_NORM_CASE(1) LF_NORM_CASE(2) LF_NORM_CASE(3) LF_NORM_CASE(4) LF_NORM_CASE(5) LF_NORM_CASE(6)
    LF_NORM_CASE(7) LF_NORM_CASE(8) LF_NORM_CASE(9) LF_NORM_CASE(10) LF_NORM_CASE(11) LF_NORM_CASE(12)
    LF_NORM_CASE(13) LF_NORM_CASE(14) LF_NORM_CASE(15) LF_NORM_CASE(16)
#undef LF_NORM_CASE
    default: return set_error(LF_ERR_UNSUPPORTED, "lf_add_layernorm: hidden %d above 4096", p.hidden);
  }
  if (e != cudaSuccess) return cuda_error(e, "launch add_layernorm");
  count_launch();
  return LF_OK;
}

constexpr int kMaxDevices = 64;
std::mutex g_table_mu;
bool g_table_ready[kMaxDevices][2];

// The device's table for this dtype, built on first use (on `s`, then waited for).
template <typename T>
int ensure_gelu_table(int dev, int which, cudaStream_t s) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(LF_ERR_UNSUPPORTED, "lf_gelu: device %d", dev);
  std::lock_guard<std::mutex> lock(g_table_mu);
  if (g_table_ready[dev][which]) return LF_OK;
  gelu_table_init_kernel<T><<<65536 / 256, 256, 0, s>>>(which);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch gelu table");
  count_launch();
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(e, "gelu table");
  e = cudaFuncSetAttribute(gelu_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536 * 2);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gelu_lut)");
  g_table_ready[dev][which] = true;
  return LF_OK;
}

template <typename T>
int launch_gelu(const void* x, void* out, int64_t n, cudaStream_t s) {
  const int64_t n8 = n / 8;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cap);
  const int which = std::is_same<T, __half>::value ? 1 : 0;
  bool ready = false;
  if (sizeof(T) == 2 && dev >= 0 && dev < kMaxDevices) {
    std::lock_guard<std::mutex> lock(g_table_mu);
    ready = g_table_ready[dev][which];
  }
  // the table is built (and waited for) outside a stream capture; a captured
  // call before that computes the formula directly, with the same results
  if (sizeof(T) == 2 && (ready || cap == cudaStreamCaptureStatusNone)) {
    if (n8 == 0) return LF_OK;
    int rc = ensure_gelu_table<T>(dev, which, s);
    if (rc) return rc;
    int64_t blocks = (n8 + kLutThreads - 1) / kLutThreads;
    if (blocks > sms) blocks = sms;
    const cudaError_t e = launch_pdl(gelu_lut_kernel, dim3(unsigned(blocks)), dim3(kLutThreads), 65536 * 2, s,
                                     static_cast<const uint4*>(x), static_cast<uint4*>(out), n8, which);
    if (e != cudaSuccess) return cuda_error(e, "launch gelu_lut");
    count_launch();
    return LF_OK;
  }
  int64_t blocks = (n8 + 255) / 256;
  if (blocks > int64_t(sms) * 8) blocks = int64_t(sms) * 8;
  if (blocks == 0) return LF_OK;
  gelu_kernel<T><<<unsigned(blocks), 256, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(out), n8);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch gelu");
  count_launch();
  return LF_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

}  // namespace lf

using namespace lf;

extern "C" int lf_add_layernorm(void* stream, int dtype, const void* a, int64_t lda, const void* b, int64_t ldb,
                                const void* vec, const void* gamma, const void* beta, float eps, int64_t n_rows,
                                int hidden, void* out, int64_t ldo) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16 && dtype != LF_DTYPE_F32)
    return set_error(LF_ERR_INVALID, "lf_add_layernorm: unknown dtype %d", dtype);
  if (a == nullptr || gamma == nullptr || beta == nullptr || out == nullptr)
    return set_error(LF_ERR_INVALID, "lf_add_layernorm: null a, gamma, beta or out");
  if (b != nullptr && vec != nullptr) return set_error(LF_ERR_INVALID, "lf_add_layernorm: b and vec together");
  if (n_rows < 0 || hidden <= 0 || hidden % 8 != 0)
    return set_error(LF_ERR_INVALID, "lf_add_layernorm: hidden %d must be a positive multiple of 8", hidden);
  if (hidden > 4096) return set_error(LF_ERR_UNSUPPORTED, "lf_add_layernorm: hidden %d above 4096", hidden);
  if (lda < hidden || ldo < hidden || (b != nullptr && ldb < hidden))
    return set_error(LF_ERR_INVALID, "lf_add_layernorm: a row stride is below hidden %d", hidden);
  const int es = dtype == LF_DTYPE_F32 ? 4 : 2;
  if (!aligned16(a) || !aligned16(out) || !aligned16(gamma) || !aligned16(beta) || (b != nullptr && !aligned16(b)) ||
      (vec != nullptr && !aligned16(vec)) ||
      (lda * es) % 16 != 0 || (ldo * es) % 16 != 0 || (b != nullptr && (ldb * es) % 16 != 0))
    return set_error(LF_ERR_INVALID, "lf_add_layernorm: pointers and row strides must be 16-byte aligned");
  if (n_rows == 0) return LF_OK;
  NormParams p = {};
  p.a = a;
  p.b = b;
  p.lda = lda;
  p.ldb = ldb;
  p.vec = vec;
  p.gamma = gamma;
  p.beta = beta;
  p.eps = eps;
  p.n_rows = n_rows;
  p.hidden = hidden;
  p.out = out;
  p.ldo = ldo;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LF_DTYPE_BF16) return launch_norm<__nv_bfloat16>(p, s);
  if (dtype == LF_DTYPE_F16) return launch_norm<__half>(p, s);
  return launch_norm<float>(p, s);
}

extern "C" int lf_embed_layernorm(void* stream, int dtype, const void* word, int64_t ld_word, int64_t n_word,
                                  const int32_t* ids, const void* pos, int64_t ld_pos, int64_t n_pos,
                                  const int32_t* positions, const void* type, int64_t ld_type, int64_t n_type,
                                  const int32_t* types, const void* gamma, const void* beta, float eps,
                                  int64_t n_rows, int hidden, void* out, int64_t ldo, int32_t* status) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16 && dtype != LF_DTYPE_F32)
    return set_error(LF_ERR_INVALID, "lf_embed_layernorm: unknown dtype %d", dtype);
  if (word == nullptr || pos == nullptr || type == nullptr || ids == nullptr || positions == nullptr ||
      gamma == nullptr || beta == nullptr || out == nullptr)
    return set_error(LF_ERR_INVALID, "lf_embed_layernorm: null table, index, gamma, beta or out");
  if (n_rows < 0 || hidden <= 0 || hidden % 8 != 0 || n_word <= 0 || n_pos <= 0 || n_type <= 0)
    return set_error(LF_ERR_INVALID, "lf_embed_layernorm: hidden %d must be a positive multiple of 8", hidden);
  if (hidden > 4096) return set_error(LF_ERR_UNSUPPORTED, "lf_embed_layernorm: hidden %d above 4096", hidden);
  if (ld_word < hidden || ld_pos < hidden || ld_type < hidden || ldo < hidden)
    return set_error(LF_ERR_INVALID, "lf_embed_layernorm: a row stride is below hidden %d", hidden);
  const int es = dtype == LF_DTYPE_F32 ? 4 : 2;
  if (!aligned16(word) || !aligned16(pos) || !aligned16(type) || !aligned16(out) || !aligned16(gamma) ||
      !aligned16(beta) || (ld_word * es) % 16 || (ld_pos * es) % 16 || (ld_type * es) % 16 || (ldo * es) % 16)
    return set_error(LF_ERR_INVALID, "lf_embed_layernorm: pointers and row strides must be 16-byte aligned");
  if (n_rows == 0) return LF_OK;
  NormParams p = {};
  p.a = word;
  p.lda = ld_word;
  p.n_a = n_word;
  p.ia = ids;
  p.b = pos;
  p.ldb = ld_pos;
  p.n_b = n_pos;
  p.ib = positions;
  p.c = type;
  p.ldc = ld_type;
  p.n_c = n_type;
  p.ic = types;  // null: every row takes type row 0
  p.gamma = gamma;
  p.beta = beta;
  p.eps = eps;
  p.n_rows = n_rows;
  p.hidden = hidden;
  p.out = out;
  p.ldo = ldo;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LF_DTYPE_BF16) return launch_norm<__nv_bfloat16>(p, s);
  if (dtype == LF_DTYPE_F16) return launch_norm<__half>(p, s);
  return launch_norm<float>(p, s);
}

extern "C" int lf_gelu(void* stream, int dtype, const void* x, void* out, int64_t n) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16 && dtype != LF_DTYPE_F32)
    return set_error(LF_ERR_INVALID, "lf_gelu: unknown dtype %d", dtype);
  if (n < 0 || n % 8 != 0) return set_error(LF_ERR_INVALID, "lf_gelu: n %lld must be a multiple of 8", (long long)n);
  if (n > 0 && (x == nullptr || out == nullptr)) return set_error(LF_ERR_INVALID, "lf_gelu: null x or out");
  if (!aligned16(x) || !aligned16(out)) return set_error(LF_ERR_INVALID, "lf_gelu: x and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LF_DTYPE_BF16) return launch_gelu<__nv_bfloat16>(x, out, n, s);
  if (dtype == LF_DTYPE_F16) return launch_gelu<__half>(x, out, n, s);
  return launch_gelu<float>(x, out, n, s);
}
