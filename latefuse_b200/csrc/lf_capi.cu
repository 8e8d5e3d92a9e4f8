// C ABI of the LoRA path: argument validation, kernel selection (tcgen05 or
// CUDA-core), TMA descriptor encoding, error reporting and options.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "lf_common.cuh"
#include "lf_internal.h"

#define LF_VERSION_STRING "latefuse_b200 0.1.0 (sm_100a)"

namespace lf {

static thread_local char g_err[512] = "";
static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_force_simt{0};
static std::atomic<int> g_shrink_cluster{0};
static std::atomic<int> g_require_tc{0};
static std::atomic<int> g_persistent{1};
static std::atomic<int> g_fused_apply{1};
static std::atomic<int> g_fused_split{0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(LF_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int option_force_simt() { return g_force_simt.load(); }
int option_shrink_cluster() { return g_shrink_cluster.load(); }

void* get_driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return fn;
}

PFN_encodeTiled get_encode_tiled() {
  static PFN_encodeTiled fn = reinterpret_cast<PFN_encodeTiled>(get_driver_fn("cuTensorMapEncodeTiled"));
  return fn;
}

static int elem_size(int dtype) { return dtype == LF_DTYPE_F32 ? 4 : 2; }

static CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == LF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int encode(CUtensorMap* map, int dtype, int rank, const void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz,
                  const char* what) {
  PFN_encodeTiled fn = get_encode_tiled();
  if (fn == nullptr) return set_error(LF_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, tma_dtype(dtype), cuuint32_t(rank), const_cast<void*>(base), dims, strides_bytes, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LF_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed: %d", what, int(r));
  return LF_OK;
}

// ---------------------------------------------------------------------------
// argument checks shared by shrink / expand / apply
// ---------------------------------------------------------------------------
static int check_common(const char* fn, int dtype, int64_t n_tokens, int hidden, int rank, int n_slots,
                        int n_modules, const int32_t* modules, const int32_t* seg_start,
                        const int32_t* seg_len, const int32_t* seg_slot, int n_segs) {
  if (dtype != LF_DTYPE_F32 && dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_INVALID, "%s: unknown dtype %d", fn, dtype);
  if (n_tokens < 0 || n_tokens > INT32_MAX) return set_error(LF_ERR_INVALID, "%s: n_tokens %lld out of range", fn, (long long)n_tokens);
  if (hidden <= 0 || rank <= 0) return set_error(LF_ERR_INVALID, "%s: hidden %d / rank %d must be positive", fn, hidden, rank);
  if (n_slots <= 0) return set_error(LF_ERR_INVALID, "%s: n_slots must be positive", fn);
  if (n_modules < 1 || n_modules > kMaxModules)
    return set_error(LF_ERR_INVALID, "%s: n_modules %d not in [1, %d]", fn, n_modules, kMaxModules);
  if (modules == nullptr) return set_error(LF_ERR_INVALID, "%s: modules is NULL", fn);
  for (int m = 0; m < n_modules; ++m)
    if (modules[m] < 0) return set_error(LF_ERR_INVALID, "%s: negative module index", fn);
  if (n_segs < 0) return set_error(LF_ERR_INVALID, "%s: n_segs < 0", fn);
  if (n_segs > 0 && (seg_start == nullptr || seg_len == nullptr || seg_slot == nullptr))
    return set_error(LF_ERR_INVALID, "%s: segment arrays are NULL", fn);
  const int64_t all_tiles = (n_tokens + LF_TILE_TOKENS - 1) / LF_TILE_TOKENS;
  if (all_tiles > 65535) return set_error(LF_ERR_UNSUPPORTED, "%s: more than 65535 token tiles", fn);
  return LF_OK;
}

static int check_tiles(const char* fn, const int32_t* tiles, int n_tiles, int n_multi, int64_t n_tokens) {
  const int64_t all_tiles = (n_tokens + LF_TILE_TOKENS - 1) / LF_TILE_TOKENS;
  if (n_multi < 0 || n_multi > n_tiles)
    return set_error(LF_ERR_INVALID, "%s: n_multi %d not in [0, n_tiles]", fn, n_multi);
  if (n_tiles < 0 || n_tiles > all_tiles || (tiles == nullptr && n_tiles != 0))
    return set_error(LF_ERR_INVALID, "%s: tile list of %d entries for %lld tiles", fn, n_tiles, (long long)all_tiles);
  if (tiles != nullptr && (reinterpret_cast<uintptr_t>(tiles) & 15u) != 0)
    return set_error(LF_ERR_INVALID, "%s: tile records must be 16-byte aligned", fn);
  return LF_OK;
}

static bool tc_rank(int r) { return r == 8 || r == 16 || r == 32 || r == 64; }

// ---------------------------------------------------------------------------
// shrink
// ---------------------------------------------------------------------------
static int choose_cluster(int64_t n_tokens, int hidden, int rank, int n_mod) {
  const int forced = option_shrink_cluster();
  const int nkb = hidden / 64;
  if (forced > 0) return (forced <= 8 && nkb % forced == 0) ? forced : -1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n_rt = (n_tokens + 127) / 128;
  int best = -1;
  for (int c = 1; c <= 8; c <<= 1) {
    if (nkb % c != 0) continue;
    const size_t smem = shrink_tc_smem(LF_DTYPE_BF16, rank, hidden / c, n_mod);
    if (smem > 100 * 1024) continue;
    best = c;
    if (n_rt * c >= 2 * sms) return c;
  }
  if (best > 0) return best;
  for (int c = 1; c <= 8; c <<= 1) {
    if (nkb % c != 0) continue;
    if (shrink_tc_smem(LF_DTYPE_BF16, rank, hidden / c, n_mod) <= 220 * 1024) return c;
  }
  return -1;
}

static int shrink_impl(cudaStream_t stream, int dtype, const void* x, int64_t ldx, int64_t n_tokens,
                       int hidden, int rank, const void* cache_a, int64_t a_slot_stride,
                       int64_t a_module_stride, int n_slots, int n_modules, const int32_t* modules,
                       const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                       int n_segs, const int32_t* tiles, int n_tiles, int n_multi, void* u, int32_t* status,
                       bool blocked = false) {
  const int es = elem_size(dtype);
  const bool tc = !option_force_simt() && dtype != LF_DTYPE_F32 && tc_rank(rank) && hidden % 64 == 0 &&
                  aligned16(x) && aligned16(cache_a) && aligned16(u) && (ldx * es) % 16 == 0 &&
                  (a_slot_stride * es) % 16 == 0 && (a_module_stride * es) % 16 == 0 && ldx >= hidden &&
                  (n_slots == 1 || a_slot_stride >= int64_t(hidden) * rank);
  if (blocked && !(tc && rank >= 16 && tiles != nullptr && n_tiles > 0 && g_persistent.load()))
    return set_error(LF_ERR_UNSUPPORTED,
                     "lf_lora_shrink_blocked: needs bf16/f16, rank 16/32/64, hidden %% 64 == 0, tile records, "
                     "16-byte aligned buffers and the persistent tcgen05 path");
  if (!tc && g_require_tc.load())
    return set_error(LF_ERR_UNSUPPORTED, "lf_lora_shrink: tcgen05 path required but not applicable");
  if (!tc) {
    SimtParams p{};
    p.x = x;
    p.ldx = ldx;
    p.n_tokens = n_tokens;
    p.hidden = hidden;
    p.rank = rank;
    for (int m = 0; m < n_modules; ++m)
      p.cache_a[m] = static_cast<const uint8_t*>(cache_a) + int64_t(modules[m]) * a_module_stride * es;
    p.a_slot_stride = a_slot_stride;
    p.n_modules = n_modules;
    p.n_slots = n_slots;
    p.seg_start = seg_start;
    p.seg_len = seg_len;
    p.seg_slot = seg_slot;
    p.n_segs = n_segs;
    p.u = u;
    p.status = status;
    return run_shrink_simt(dtype, p, stream);
  }
  // tcgen05 path: the persistent kernel (all modules in one pass over x) when
  // there are tile records, else the per-tile cluster kernel.
  const int rp = rank < 16 ? 16 : rank;
  (void)n_multi;
  if (tiles != nullptr && g_persistent.load() && n_tiles > 0) {
    ShrinkPersistParams q;
    memset(&q, 0, sizeof(q));
    {
      cuuint64_t dims[2] = {cuuint64_t(hidden), cuuint64_t(n_tokens)};
      cuuint64_t strides[1] = {cuuint64_t(ldx) * es};
      cuuint32_t box[2] = {64, 128};
      int rc = encode(&q.x_map, dtype, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "x");
      if (rc) return rc;
    }
    for (int m = 0; m < n_modules; ++m) {
      const void* a = static_cast<const uint8_t*>(cache_a) + int64_t(modules[m]) * a_module_stride * es;
      const int64_t ss = n_slots == 1 ? int64_t(hidden) * rank : a_slot_stride;
      cuuint64_t dims[3] = {cuuint64_t(rank), cuuint64_t(hidden), cuuint64_t(n_slots)};
      cuuint64_t strides[2] = {cuuint64_t(rank) * es, cuuint64_t(ss) * es};
      cuuint32_t box[3] = {cuuint32_t(rank), 64, 1};
      int rc = encode(&q.a_map[m], dtype, 3, a, dims, strides, box, a_tma_swizzle(rank), "a");
      if (rc) return rc;
    }
    // modules whose cache indices step evenly (q/k/v as 0, 1, 2), or a single
    // module, share one 4D map: module i's A is d * a_module_stride elements after
    // module i - 1's
    int d = n_modules > 1 ? modules[1] - modules[0] : 1;
    for (int m = 2; m < n_modules && d > 0; ++m)
      if (modules[m] - modules[m - 1] != d) d = 0;
    const int64_t mstride = n_modules == 1 ? int64_t(hidden) * rank * es : int64_t(d) * a_module_stride * es;
    if (d > 0 && mstride >= int64_t(hidden) * rank * es && mstride % 16 == 0) {
      const void* a = static_cast<const uint8_t*>(cache_a) + int64_t(modules[0]) * a_module_stride * es;
      const int64_t ss = n_slots == 1 ? int64_t(hidden) * rank : a_slot_stride;
      cuuint64_t dims[4] = {cuuint64_t(rank), cuuint64_t(hidden), cuuint64_t(n_modules), cuuint64_t(n_slots)};
      cuuint64_t strides[3] = {cuuint64_t(rank) * es, cuuint64_t(mstride), cuuint64_t(ss) * es};
      cuuint32_t box[4] = {cuuint32_t(rank), 64, cuuint32_t(n_modules), 1};
      int rc = encode(&q.a_modules_map, dtype, 4, a, dims, strides, box, a_tma_swizzle(rank), "a (modules)");
      if (rc) return rc;
      q.a_one_box = 1;
    }
    q.n_tokens = n_tokens;
    q.hidden = hidden;
    q.n_modules = n_modules;
    q.n_slots = n_slots;
    q.n_tiles = n_tiles;
    q.tiles = tiles;
    q.seg_start = seg_start;
    q.seg_len = seg_len;
    q.seg_slot = seg_slot;
    q.n_segs = n_segs;
    q.u = u;
    q.status = status;
    q.u_blocked = blocked ? 1 : 0;
    return run_shrink_persist(dtype, q, rank, stream);
  }
  // per-tile cluster kernel; modules in groups whose fp32 partials fit on chip
  const int group = rp * n_modules <= 64 ? n_modules : (64 / rp > 0 ? 64 / rp : 1);
  for (int m0 = 0; m0 < n_modules; m0 += group) {
    const int gm = (n_modules - m0) < group ? (n_modules - m0) : group;
    const int csize = choose_cluster(n_tokens, hidden, rank, gm);
    if (csize <= 0) return set_error(LF_ERR_UNSUPPORTED, "lf_lora_shrink: no cluster split fits hidden %d rank %d", hidden, rank);
    ShrinkTcParams p;
    memset(&p, 0, sizeof(p));
    {
      cuuint64_t dims[2] = {cuuint64_t(hidden), cuuint64_t(n_tokens)};
      cuuint64_t strides[1] = {cuuint64_t(ldx) * es};
      cuuint32_t box[2] = {64, 128};
      int rc = encode(&p.x_map, dtype, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "x");
      if (rc) return rc;
    }
    for (int m = 0; m < gm; ++m) {
      const void* a = static_cast<const uint8_t*>(cache_a) + int64_t(modules[m0 + m]) * a_module_stride * es;
      const int64_t ss = n_slots == 1 ? int64_t(hidden) * rank : a_slot_stride;
      cuuint64_t dims[3] = {cuuint64_t(rank), cuuint64_t(hidden), cuuint64_t(n_slots)};
      cuuint64_t strides[2] = {cuuint64_t(rank) * es, cuuint64_t(ss) * es};
      cuuint32_t box[3] = {cuuint32_t(rank), 64, 1};
      int rc = encode(&p.a_map[m], dtype, 3, a, dims, strides, box, a_tma_swizzle(rank), "a");
      if (rc) return rc;
    }
    p.n_tokens = n_tokens;
    p.hidden = hidden;
    p.kchunk = hidden / csize;
    p.n_modules = gm;
    p.n_slots = n_slots;
    p.tmem_cols = shrink_tc_tmem_cols(rank, gm);
    p.seg_start = seg_start;
    p.seg_len = seg_len;
    p.seg_slot = seg_slot;
    p.n_segs = n_segs;
    p.tiles = tiles;
    p.u = static_cast<uint8_t*>(u) + int64_t(m0) * n_tokens * rank * es;
    p.status = status;
    const int grid_tiles = tiles != nullptr ? n_tiles : int((n_tokens + LF_TILE_TOKENS - 1) / LF_TILE_TOKENS);
    if (grid_tiles == 0) return LF_OK;
    int rc = run_shrink_tc(dtype, p, rank, csize, grid_tiles, stream);
    if (rc) return rc;
  }
  return LF_OK;
}

// ---------------------------------------------------------------------------
// expand
// ---------------------------------------------------------------------------
static int expand_impl(cudaStream_t stream, int dtype, const void* u, void* y, int64_t ldy, int64_t n_tokens,
                       int hidden, int rank, const void* cache_b, int64_t b_slot_stride,
                       int64_t b_module_stride, int n_slots, int n_modules, const int32_t* modules,
                       const int64_t* y_col_offsets, const int32_t* seg_start, const int32_t* seg_len,
                       const int32_t* seg_slot, int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                       int accumulate, bool after_shrink, int32_t* status, const void* into_r = nullptr,
                       int64_t ldr = 0, const void* into_bias = nullptr, bool into = false) {
  const int es = elem_size(dtype);
  int64_t y_cols = 0;
  bool offs_aligned = true;
  for (int m = 0; m < n_modules; ++m) {
    if (y_col_offsets[m] < 0) return set_error(LF_ERR_INVALID, "lf_lora_expand: negative y column offset");
    if (y_col_offsets[m] + hidden > y_cols) y_cols = y_col_offsets[m] + hidden;
    if (y_col_offsets[m] % 8 != 0) offs_aligned = false;
  }
  if (ldy < y_cols) return set_error(LF_ERR_INVALID, "lf_lora_expand: ldy %lld < output columns %lld", (long long)ldy, (long long)y_cols);
  if (into) {
    // into mode runs on the persistent tcgen05 expand only
    const bool ok = !option_force_simt() && g_persistent.load() && dtype != LF_DTYPE_F32 && tc_rank(rank) &&
                    hidden % 128 == 0 && offs_aligned && tiles != nullptr && n_tiles > 0 && aligned16(y) &&
                    aligned16(cache_b) && aligned16(u) && (ldy * es) % 16 == 0 &&
                    (b_slot_stride * es) % 16 == 0 && (b_module_stride * es) % 16 == 0 &&
                    (n_slots == 1 || b_slot_stride >= int64_t(hidden) * rank) &&
                    (into_r == nullptr || (aligned16(into_r) && (ldr * es) % 16 == 0)) &&
                    (into_bias == nullptr || aligned16(into_bias));
    if (!ok)
      return set_error(LF_ERR_UNSUPPORTED,
                       "lf_lora_apply_into: needs bf16/f16, rank 8/16/32/64, hidden %% 128 == 0, tile records, "
                       "16-byte aligned buffers and strides, and the persistent tcgen05 path");
    if (into_r != nullptr && ldr < y_cols)
      return set_error(LF_ERR_INVALID, "lf_lora_apply_into: ldr %lld < output columns %lld", (long long)ldr,
                       (long long)y_cols);
  }
  const bool tc = !option_force_simt() && dtype != LF_DTYPE_F32 && tc_rank(rank) && hidden % 64 == 0 &&
                  offs_aligned && aligned16(y) && aligned16(cache_b) && aligned16(u) && (ldy * es) % 16 == 0 &&
                  (hidden * es) % 16 == 0 && (b_slot_stride * es) % 16 == 0 && (b_module_stride * es) % 16 == 0 &&
                  (n_slots == 1 || b_slot_stride >= int64_t(hidden) * rank);
  if (!tc && g_require_tc.load())
    return set_error(LF_ERR_UNSUPPORTED, "lf_lora_expand: tcgen05 path required but not applicable");
  if (!tc) {
    SimtParams p{};
    p.y = y;
    p.ldy = ldy;
    p.n_tokens = n_tokens;
    p.hidden = hidden;
    p.rank = rank;
    for (int m = 0; m < n_modules; ++m) {
      p.cache_b[m] = static_cast<const uint8_t*>(cache_b) + int64_t(modules[m]) * b_module_stride * es;
      p.y_col_off[m] = y_col_offsets[m];
    }
    p.b_slot_stride = b_slot_stride;
    p.n_modules = n_modules;
    p.n_slots = n_slots;
    p.seg_start = seg_start;
    p.seg_len = seg_len;
    p.seg_slot = seg_slot;
    p.n_segs = n_segs;
    p.u = const_cast<void*>(u);
    p.accumulate = accumulate;
    p.status = status;
    return run_expand_simt(dtype, p, stream);
  }
  ExpandTcParams p;
  memset(&p, 0, sizeof(p));
  {
    cuuint64_t dims[2] = {cuuint64_t(y_cols), cuuint64_t(n_tokens)};
    cuuint64_t strides[1] = {cuuint64_t(ldy) * es};
    cuuint32_t box[2] = {64, 128};
    int rc = encode(&p.y_map, dtype, 2, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "y");
    if (rc) return rc;
  }
  for (int m = 0; m < n_modules; ++m) {
    const void* b = static_cast<const uint8_t*>(cache_b) + int64_t(modules[m]) * b_module_stride * es;
    const int64_t ss = n_slots == 1 ? int64_t(hidden) * rank : b_slot_stride;
    cuuint64_t dims[3] = {cuuint64_t(hidden), cuuint64_t(rank), cuuint64_t(n_slots)};
    cuuint64_t strides[2] = {cuuint64_t(hidden) * es, cuuint64_t(ss) * es};
    cuuint32_t box[3] = {64, cuuint32_t(rank), 1};
    int rc = encode(&p.b_map[m], dtype, 3, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "b");
    if (rc) return rc;
    p.y_col_off[m] = y_col_offsets[m];
  }
  p.n_tokens = n_tokens;
  p.hidden = hidden;
  p.n_modules = n_modules;
  p.n_slots = n_slots;
  p.accumulate = accumulate;
  p.seg_start = seg_start;
  p.seg_len = seg_len;
  p.seg_slot = seg_slot;
  p.n_segs = n_segs;
  p.u = u;
  p.status = status;
  const int nt = hidden % 128 == 0 ? 128 : 64;
  if (!accumulate || tiles == nullptr) {
    // with accumulate == 0 every tile must be written (rows outside segments become 0)
    p.tiles = accumulate ? tiles : nullptr;
    p.n_tiles = (accumulate && tiles != nullptr) ? n_tiles : int((n_tokens + LF_TILE_TOKENS - 1) / LF_TILE_TOKENS);
    if (p.n_tiles == 0) return LF_OK;
    return run_expand_tc(dtype, p, rank, nt, stream);
  }
  (void)n_multi;  // the persistent expand takes tiles with any number of segments
  if (g_persistent.load() && nt == 128 && n_tiles > 0) {
    ExpandPersistParams q;
    memset(&q, 0, sizeof(q));
    q.y_map = p.y_map;
    if (into) {
      q.into = 1;
      q.bias = into_bias;
      if (into_r != nullptr) {
        cuuint64_t dims[2] = {cuuint64_t(y_cols), cuuint64_t(n_tokens)};
        cuuint64_t strides[1] = {cuuint64_t(ldr) * es};
        cuuint32_t box[2] = {64, 128};
        int rc = encode(&q.r_map, dtype, 2, const_cast<void*>(into_r), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                        "r");
        if (rc) return rc;
        q.has_r = 1;
      }
    }
    for (int m = 0; m < n_modules; ++m) {
      q.b_map[m] = p.b_map[m];
      q.y_col_off[m] = p.y_col_off[m];
    }
    {
      cuuint64_t dims[2] = {cuuint64_t(rank), cuuint64_t(n_modules) * cuuint64_t(n_tokens)};
      cuuint64_t strides[1] = {cuuint64_t(rank) * es};
      cuuint32_t box[2] = {cuuint32_t(rank), 128};
      int rc = encode(&q.u_map, dtype, 2, u, dims, strides, box, a_tma_swizzle(rank), "u");
      if (rc) return rc;
    }
    q.n_tokens = n_tokens;
    q.n_modules = n_modules;
    q.n_col_blocks = hidden / 128;
    q.n_slots = n_slots;
    q.n_tiles = n_tiles;
    q.tiles = tiles;
    q.seg_start = seg_start;
    q.seg_len = seg_len;
    q.seg_slot = seg_slot;
    q.n_segs = n_segs;
    q.status = status;
    return run_expand_persist(dtype, q, rank, 128, after_shrink, stream);
  }
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  return run_expand_tc(dtype, p, rank, nt, stream);
}

// ---------------------------------------------------------------------------
// one-launch apply
// ---------------------------------------------------------------------------
static bool ranges_overlap(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + nb && b0 < a0 + na;
}

// Column chunks per tile record: doubled while the items still fit on the SMs at one
// each (a split item reads the record's x again, from L2), each chunk a multiple of 128
// columns; or the LF_OPT_FUSED_SPLIT choice.  At 128 records of
// the isolated op one chunk measured 29 us, two 33.
static int fused_chunks(int hidden, int n_tiles) {
  const int forced = g_fused_split.load();
  if (forced > 0) return (hidden % (128 * forced) == 0) ? forced : -1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int c = 1;
  while (int64_t(n_tiles) * c * 2 <= sms && hidden % (128 * 2 * c) == 0) c *= 2;
  return c;
}

// Launches lf_lora_apply's one-launch kernel and returns LF_OK, an error code if the
// launch failed, or -1 (nothing launched) where the two-launch path must run.
static int fused_apply(cudaStream_t stream, int dtype, const void* x, int64_t ldx, void* y, int64_t ldy,
                       int64_t n_tokens, int hidden, int rank, const void* cache_a, int64_t a_slot_stride,
                       int64_t a_module_stride, const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                       int n_slots, int n_modules, const int32_t* modules, const int64_t* y_col_offsets,
                       const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot, int n_segs,
                       const int32_t* tiles, int n_tiles, int32_t* status) {
  if (!g_fused_apply.load() || !g_persistent.load() || option_force_simt()) return -1;
  if (dtype == LF_DTYPE_F32 || !tc_rank(rank) || hidden % 128 != 0 || tiles == nullptr || n_tiles <= 0) return -1;
  // one module per call (the hf engine's hooks, the isolated op): with three modules
  // sharing x (q/k/v, 17,369 tokens) the shrink + expand launches measured faster
  // (68.6 vs 82.0 us), the expand's 128-column items draining y faster than the
  // one-launch kernel's 64-column boxes
  if (n_modules != 1 && g_fused_apply.load() != 2) return -1;
  const int es = elem_size(dtype);
  int64_t y_cols = 0;
  for (int m = 0; m < n_modules; ++m) {
    if (y_col_offsets[m] < 0 || y_col_offsets[m] % 8 != 0) return -1;
    if (y_col_offsets[m] + hidden > y_cols) y_cols = y_col_offsets[m] + hidden;
  }
  if (ldy < y_cols) return -1;  // the two-launch path reports it
  if (!aligned16(x) || !aligned16(y) || !aligned16(cache_a) || !aligned16(cache_b) || (ldx * es) % 16 != 0 ||
      (ldy * es) % 16 != 0 || (a_slot_stride * es) % 16 != 0 || (a_module_stride * es) % 16 != 0 ||
      (b_slot_stride * es) % 16 != 0 || (b_module_stride * es) % 16 != 0)
    return -1;
  if (n_slots > 1 && (a_slot_stride < int64_t(hidden) * rank || b_slot_stride < int64_t(hidden) * rank)) return -1;
  // y is written while other items still read x: they must not share memory
  if (ranges_overlap(x, size_t(((n_tokens - 1) * ldx + hidden) * es), y, size_t(((n_tokens - 1) * ldy + y_cols) * es)))
    return -1;
  const int chunks = fused_chunks(hidden, n_tiles);
  if (chunks <= 0) return -1;
  FusedApplyParams p;
  memset(&p, 0, sizeof(p));
  {
    cuuint64_t dims[2] = {cuuint64_t(hidden), cuuint64_t(n_tokens)};
    cuuint64_t strides[1] = {cuuint64_t(ldx) * es};
    cuuint32_t box[2] = {64, 128};
    int rc = encode(&p.x_map, dtype, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "x");
    if (rc) return rc;
  }
  {
    cuuint64_t dims[2] = {cuuint64_t(y_cols), cuuint64_t(n_tokens)};
    cuuint64_t strides[1] = {cuuint64_t(ldy) * es};
    cuuint32_t sbox[2] = {64, 32};
    int rc = encode(&p.ys_map, dtype, 2, y, dims, strides, sbox, CU_TENSOR_MAP_SWIZZLE_128B, "y (reductions)");
    if (rc) return rc;
  }
  const int64_t a_ss = n_slots == 1 ? int64_t(hidden) * rank : a_slot_stride;
  const int64_t b_ss = n_slots == 1 ? int64_t(hidden) * rank : b_slot_stride;
  for (int m = 0; m < n_modules; ++m) {
    const void* a = static_cast<const uint8_t*>(cache_a) + int64_t(modules[m]) * a_module_stride * es;
    cuuint64_t adims[3] = {cuuint64_t(rank), cuuint64_t(hidden), cuuint64_t(n_slots)};
    cuuint64_t astrides[2] = {cuuint64_t(rank) * es, cuuint64_t(a_ss) * es};
    cuuint32_t abox[3] = {cuuint32_t(rank), 64, 1};
    int rc = encode(&p.a_map[m], dtype, 3, a, adims, astrides, abox, a_tma_swizzle(rank), "a");
    if (rc) return rc;
    const void* b = static_cast<const uint8_t*>(cache_b) + int64_t(modules[m]) * b_module_stride * es;
    cuuint64_t bdims[3] = {cuuint64_t(hidden), cuuint64_t(rank), cuuint64_t(n_slots)};
    cuuint64_t bstrides[2] = {cuuint64_t(hidden) * es, cuuint64_t(b_ss) * es};
    cuuint32_t bbox[3] = {64, cuuint32_t(rank), 1};
    rc = encode(&p.b_map[m], dtype, 3, b, bdims, bstrides, bbox, CU_TENSOR_MAP_SWIZZLE_128B, "b");
    if (rc) return rc;
    p.y_col_off[m] = y_col_offsets[m];
  }
  // modules whose cache indices step evenly share one 4D map of A (as the shrink does)
  int d = n_modules > 1 ? modules[1] - modules[0] : 1;
  for (int m = 2; m < n_modules && d > 0; ++m)
    if (modules[m] - modules[m - 1] != d) d = 0;
  const int64_t mstride = n_modules == 1 ? int64_t(hidden) * rank * es : int64_t(d) * a_module_stride * es;
  if (d > 0 && mstride >= int64_t(hidden) * rank * es && mstride % 16 == 0) {
    const void* a = static_cast<const uint8_t*>(cache_a) + int64_t(modules[0]) * a_module_stride * es;
    cuuint64_t dims[4] = {cuuint64_t(rank), cuuint64_t(hidden), cuuint64_t(n_modules), cuuint64_t(n_slots)};
    cuuint64_t strides[3] = {cuuint64_t(rank) * es, cuuint64_t(mstride), cuuint64_t(a_ss) * es};
    cuuint32_t box[4] = {cuuint32_t(rank), 64, cuuint32_t(n_modules), 1};
    int rc = encode(&p.a_modules_map, dtype, 4, a, dims, strides, box, a_tma_swizzle(rank), "a (modules)");
    if (rc) return rc;
    p.a_one_box = 1;
  }
  p.n_tokens = n_tokens;
  p.hidden = hidden;
  p.n_modules = n_modules;
  p.n_slots = n_slots;
  p.n_tiles = n_tiles;
  p.n_chunks = chunks;
  p.chunk_cols = hidden / chunks;
  p.tiles = tiles;
  p.seg_start = seg_start;
  p.seg_len = seg_len;
  p.seg_slot = seg_slot;
  p.n_segs = n_segs;
  p.status = status;
  const int rc = run_lora_fused(dtype, p, rank, stream);
  if (rc == LF_ERR_UNSUPPORTED) {  // no size fits: the two launches run, and the call does not fail
    g_err[0] = '\0';
    return -1;
  }
  return rc;
}

// lf_lora_apply as a shrink launch into `workspace` and an expand launch that reads it.
static int apply_two_launch(cudaStream_t s, int dtype, const void* x, int64_t ldx, void* y, int64_t ldy,
                            int64_t n_tokens, int hidden, int rank, const void* cache_a, int64_t a_slot_stride,
                            int64_t a_module_stride, const void* cache_b, int64_t b_slot_stride,
                            int64_t b_module_stride, int n_slots, int n_modules, const int32_t* modules,
                            const int64_t* y_col_offsets, const int32_t* seg_start, const int32_t* seg_len,
                            const int32_t* seg_slot, int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                            void* workspace, int32_t* status) {
  int rc = shrink_impl(s, dtype, x, ldx, n_tokens, hidden, rank, cache_a, a_slot_stride, a_module_stride, n_slots,
                       n_modules, modules, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles, n_multi, workspace,
                       status);
  if (rc) return rc;
  return expand_impl(s, dtype, workspace, y, ldy, n_tokens, hidden, rank, cache_b, b_slot_stride, b_module_stride,
                     n_slots, n_modules, modules, y_col_offsets, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles,
                     n_multi, 1, true, status);
}

int apply_entry(bool allow_fused, void* stream, int dtype, const void* x, int64_t ldx, void* y, int64_t ldy,
                int64_t n_tokens, int hidden, int rank, const void* cache_a, int64_t a_slot_stride,
                int64_t a_module_stride, const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                int n_slots, int n_modules, const int32_t* modules, const int64_t* y_col_offsets,
                const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot, int n_segs,
                const int32_t* tiles, int n_tiles, int n_multi, void* workspace, size_t workspace_bytes,
                int32_t* status) {
  int rc = check_common("lf_lora_apply", dtype, n_tokens, hidden, rank, n_slots, n_modules, modules, seg_start,
                        seg_len, seg_slot, n_segs);
  if (rc) return rc;
  if ((rc = check_tiles("lf_lora_apply", tiles, n_tiles, n_multi, n_tokens))) return rc;
  if (x == nullptr || y == nullptr || cache_a == nullptr || cache_b == nullptr || y_col_offsets == nullptr)
    return set_error(LF_ERR_INVALID, "lf_lora_apply: NULL buffer");
  if (ldx < hidden) return set_error(LF_ERR_INVALID, "lf_lora_apply: ldx < hidden");
  if (n_tokens == 0) return LF_OK;
  const size_t need = lf_lora_workspace_bytes(dtype, n_tokens, rank, n_modules);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(LF_ERR_WORKSPACE, "lf_lora_apply: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (allow_fused) {
    rc = fused_apply(s, dtype, x, ldx, y, ldy, n_tokens, hidden, rank, cache_a, a_slot_stride, a_module_stride,
                     cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules, y_col_offsets, seg_start,
                     seg_len, seg_slot, n_segs, tiles, n_tiles, status);
    if (rc >= 0) return rc;
  }
  return apply_two_launch(s, dtype, x, ldx, y, ldy, n_tokens, hidden, rank, cache_a, a_slot_stride, a_module_stride,
                          cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules, y_col_offsets,
                          seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles, n_multi, workspace, status);
}

}  // namespace lf

using namespace lf;

extern "C" {

const char* lf_version(void) { return LF_VERSION_STRING; }

const char* lf_last_error(void) { return g_err; }

int lf_device_supported(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
  return prop.major == 10 && prop.minor == 0 ? 1 : 0;
}

int lf_set_option(int key, int value) {
  switch (key) {
    case LF_OPT_FORCE_SIMT: g_force_simt.store(value ? 1 : 0); return LF_OK;
    case LF_OPT_REQUIRE_TC: g_require_tc.store(value ? 1 : 0); return LF_OK;
    case LF_OPT_PERSISTENT: g_persistent.store(value ? 1 : 0); return LF_OK;
    case LF_OPT_FUSED_APPLY:
      if (value < 0 || value > 2) return set_error(LF_ERR_INVALID, "LF_OPT_FUSED_APPLY must be 0, 1 or 2");
      g_fused_apply.store(value);
      return LF_OK;
    case LF_OPT_FUSED_SPLIT:
      if (value < 0 || value > 16) return set_error(LF_ERR_INVALID, "LF_OPT_FUSED_SPLIT must be in [0, 16]");
      g_fused_split.store(value);
      return LF_OK;
    case LF_OPT_SHRINK_CLUSTER:
      if (value < 0 || value > 8 || (value & (value - 1)) != 0)
        return set_error(LF_ERR_INVALID, "LF_OPT_SHRINK_CLUSTER must be 0 or a power of two <= 8");
      g_shrink_cluster.store(value);
      return LF_OK;
  }
  return set_error(LF_ERR_INVALID, "unknown option %d", key);
}

uint64_t lf_launch_count(void) { return g_launches.load(); }

size_t lf_lora_workspace_bytes(int dtype, int64_t n_tokens, int rank, int n_modules) {
  if (n_tokens <= 0 || rank <= 0 || n_modules <= 0) return 0;
  const size_t b = size_t(n_modules) * size_t(n_tokens) * size_t(rank) * size_t(elem_size(dtype));
  return (b + 255) / 256 * 256;
}

int lf_lora_shrink(void* stream, int dtype, const void* x, int64_t ldx, int64_t n_tokens, int hidden, int rank,
                   const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride, int n_slots,
                   int n_modules, const int32_t* modules, const int32_t* seg_start, const int32_t* seg_len,
                   const int32_t* seg_slot, int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                   void* u, int32_t* status) {
  int rc = check_common("lf_lora_shrink", dtype, n_tokens, hidden, rank, n_slots, n_modules, modules, seg_start,
                        seg_len, seg_slot, n_segs);
  if (rc) return rc;
  if ((rc = check_tiles("lf_lora_shrink", tiles, n_tiles, n_multi, n_tokens))) return rc;
  if (x == nullptr || cache_a == nullptr || u == nullptr) return set_error(LF_ERR_INVALID, "lf_lora_shrink: NULL buffer");
  if (ldx < hidden) return set_error(LF_ERR_INVALID, "lf_lora_shrink: ldx < hidden");
  if (n_tokens == 0) return LF_OK;
  return shrink_impl(static_cast<cudaStream_t>(stream), dtype, x, ldx, n_tokens, hidden, rank, cache_a,
                     a_slot_stride, a_module_stride, n_slots, n_modules, modules, seg_start, seg_len, seg_slot,
                     n_segs, tiles, n_tiles, n_multi, u, status);
}

int lf_lora_shrink_blocked(void* stream, int dtype, const void* x, int64_t ldx, int64_t n_tokens, int hidden,
                           int rank, const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                           int n_slots, int n_modules, const int32_t* modules, const int32_t* seg_start,
                           const int32_t* seg_len, const int32_t* seg_slot, int n_segs, const int32_t* tiles,
                           int n_tiles, int n_multi, void* u, int32_t* status) {
  int rc = check_common("lf_lora_shrink_blocked", dtype, n_tokens, hidden, rank, n_slots, n_modules, modules,
                        seg_start, seg_len, seg_slot, n_segs);
  if (rc) return rc;
  if ((rc = check_tiles("lf_lora_shrink_blocked", tiles, n_tiles, n_multi, n_tokens))) return rc;
  if (x == nullptr || cache_a == nullptr || u == nullptr)
    return set_error(LF_ERR_INVALID, "lf_lora_shrink_blocked: NULL buffer");
  if (ldx < hidden) return set_error(LF_ERR_INVALID, "lf_lora_shrink_blocked: ldx < hidden");
  if (n_tokens == 0) return LF_OK;
  return shrink_impl(static_cast<cudaStream_t>(stream), dtype, x, ldx, n_tokens, hidden, rank, cache_a,
                     a_slot_stride, a_module_stride, n_slots, n_modules, modules, seg_start, seg_len, seg_slot,
                     n_segs, tiles, n_tiles, n_multi, u, status, true);
}

int lf_lora_expand(void* stream, int dtype, const void* u, void* y, int64_t ldy, int64_t n_tokens, int hidden,
                   int rank, const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride, int n_slots,
                   int n_modules, const int32_t* modules, const int64_t* y_col_offsets, const int32_t* seg_start,
                   const int32_t* seg_len, const int32_t* seg_slot, int n_segs, const int32_t* tiles, int n_tiles,
                   int n_multi, int accumulate, int32_t* status) {
  int rc = check_common("lf_lora_expand", dtype, n_tokens, hidden, rank, n_slots, n_modules, modules, seg_start,
                        seg_len, seg_slot, n_segs);
  if (rc) return rc;
  if ((rc = check_tiles("lf_lora_expand", tiles, n_tiles, n_multi, n_tokens))) return rc;
  if (u == nullptr || y == nullptr || cache_b == nullptr || y_col_offsets == nullptr)
    return set_error(LF_ERR_INVALID, "lf_lora_expand: NULL buffer");
  if (n_tokens == 0) return LF_OK;
  return expand_impl(static_cast<cudaStream_t>(stream), dtype, u, y, ldy, n_tokens, hidden, rank, cache_b,
                     b_slot_stride, b_module_stride, n_slots, n_modules, modules, y_col_offsets, seg_start, seg_len,
                     seg_slot, n_segs, tiles, n_tiles, n_multi, accumulate, false, status);
}

int lf_lora_apply(void* stream, int dtype, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t n_tokens,
                  int hidden, int rank, const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                  const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride, int n_slots, int n_modules,
                  const int32_t* modules, const int64_t* y_col_offsets, const int32_t* seg_start,
                  const int32_t* seg_len, const int32_t* seg_slot, int n_segs, const int32_t* tiles, int n_tiles,
                  int n_multi, void* workspace, size_t workspace_bytes, int32_t* status) {
  return apply_entry(true, stream, dtype, x, ldx, y, ldy, n_tokens, hidden, rank, cache_a, a_slot_stride,
                     a_module_stride, cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules,
                     y_col_offsets, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles, n_multi, workspace,
                     workspace_bytes, status);
}

int lf_lora_apply_into(void* stream, int dtype, const void* x, int64_t ldx, const void* r, int64_t ldr,
                       const void* bias, void* y, int64_t ldy, int64_t n_tokens, int hidden, int rank,
                       const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride, const void* cache_b,
                       int64_t b_slot_stride, int64_t b_module_stride, int n_slots, int n_modules,
                       const int32_t* modules, const int64_t* y_col_offsets, const int32_t* seg_start,
                       const int32_t* seg_len, const int32_t* seg_slot, int n_segs, const int32_t* tiles,
                       int n_tiles, int n_multi, void* workspace, size_t workspace_bytes, int32_t* status) {
  int rc = check_common("lf_lora_apply_into", dtype, n_tokens, hidden, rank, n_slots, n_modules, modules, seg_start,
                        seg_len, seg_slot, n_segs);
  if (rc) return rc;
  if ((rc = check_tiles("lf_lora_apply_into", tiles, n_tiles, n_multi, n_tokens))) return rc;
  if (x == nullptr || y == nullptr || cache_a == nullptr || cache_b == nullptr || y_col_offsets == nullptr)
    return set_error(LF_ERR_INVALID, "lf_lora_apply_into: NULL buffer");
  if (ldx < hidden) return set_error(LF_ERR_INVALID, "lf_lora_apply_into: ldx < hidden");
  if (r != nullptr && r == y) return set_error(LF_ERR_INVALID, "lf_lora_apply_into: r and y must not alias");
  if (n_tokens == 0) return LF_OK;
  if (tiles == nullptr || n_tiles == 0)
    return set_error(LF_ERR_UNSUPPORTED, "lf_lora_apply_into: tile records are required");
  const size_t need = lf_lora_workspace_bytes(dtype, n_tokens, rank, n_modules);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(LF_ERR_WORKSPACE, "lf_lora_apply_into: workspace of %zu bytes needed, %zu given", need,
                     workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = shrink_impl(s, dtype, x, ldx, n_tokens, hidden, rank, cache_a, a_slot_stride, a_module_stride, n_slots,
                   n_modules, modules, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles, n_multi, workspace,
                   status);
  if (rc) return rc;
  return expand_impl(s, dtype, workspace, y, ldy, n_tokens, hidden, rank, cache_b, b_slot_stride, b_module_stride,
                     n_slots, n_modules, modules, y_col_offsets, seg_start, seg_len, seg_slot, n_segs, tiles, n_tiles,
                     n_multi, 1, true, status, r, ldr, bias, true);
}

}  // extern "C"
