// Variable-length self-attention of packed sequences, head_dim 64, on tcgen05.
//
// Replaces the encoder's masked attention (src/latefuse/model/encoder.py:82-98:
// scores = q k^T * scale, padded keys masked, softmax in f32, probs @ v) for a
// batch whose padding has been removed: every sequence attends to itself only.
//
// Work unit = (query tile of 128 rows of one sequence, head).  One persistent
// CTA per SM loops over units with four roles:
//   warp 0      producer: Q tile (double-buffered) and the sequence's K/V tiles
//               (128 keys each, a 3-stage ring) by TMA straight from the fused
//               QKV activation buffer (SW128, 128-byte rows of 64 head dims);
//   warp 1      MMA issuer: S_j = Q K_j^T (M=128, N=128, K=64) into one of two
//               TMEM S buffers, then O += P_j V_j (M=128, N=64, K=128) into the
//               TMEM O accumulator, S_{j+1} issued before O += P_j V_j so the
//               tensor core works while the softmax warps do;
//   warps 2-9   softmax, two warps per TMEM lane quadrant (a query row's 128
//               key columns split 64/64, the pair exchanging row maxima through
//               shared memory): online softmax in the log2 domain with the
//               running max raised only when a tile's max exceeds it by more
//               than 2^8 (the final division keeps the result exact), P rounded
//               to the model dtype into shared memory (the canonical K-major
//               SW128 layout the MMA reads), O rescaled in TMEM when the max
//               moves, and at the end O / l rounded and stored.
// Keys past the sequence end (the next sequence's rows, or TMA zero fill past
// the buffer) are masked; query rows past it are computed and not stored.
// Every wait is bounded: a timeout sets LF_STATUS_TIMEOUT and the roles unwind.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

namespace {

constexpr int kRows = 128;                   // query / key tile rows
constexpr int kHd = 64;                      // head dim: one 128-byte swizzle atom
constexpr int kTileBytes = kRows * kHd * 2;  // 16 KB
constexpr int kKvStages = 3;
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 64 + 32 * kSoftmaxWarps;
constexpr int kSmemBytes = 1024 + 2 * kTileBytes + kKvStages * 2 * kTileBytes + 2 * 2 * kTileBytes + 1024 + 3072;
constexpr float kMaxSlack = 8.f;             // log2 units the running max may lag a tile's max

__device__ __forceinline__ bool aborted(const int32_t* flag) {
  return *reinterpret_cast<const volatile int32_t*>(flag) != 0;
}

// 2^x by the SFU's approximate base-2 exponential (results below 2^-126 flush
// to 0, which a softmax probability can take).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) attention_varlen_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const uint32_t sQ = base;                                   // 2 x 16 KB
  const uint32_t sKV = sQ + 2 * kTileBytes;                   // stages x (K 16 KB | V 16 KB)
  const uint32_t sP = sKV + kKvStages * 2 * kTileBytes;       // 2 x 32 KB (two 64-key SW128 blocks)
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (sP + 4 * kTileBytes - base));
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int Q_FULL = 0, Q_EMPTY = 2, KV_FULL = 4, KV_EMPTY = 4 + kKvStages, S_FULL = 4 + 2 * kKvStages,
            S_EMPTY = S_FULL + 2, P_FULL = S_EMPTY + 2, P_EMPTY = P_FULL + 2, O_FULL = P_EMPTY + 2,
            O_EMPTY = O_FULL + 2, DRAIN = O_EMPTY + 2, N_BARS = DRAIN + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[N_BARS]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);
  float* s_max = reinterpret_cast<float*>(gbase + (sP + 4 * kTileBytes + 1024 - base));  // [2][2][128]
  float* s_lsum = s_max + 512;                                                          // [2][128]

  const int64_t n_units = int64_t(p.n_items) * p.n_heads;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(Q_FULL + i), 1);
      mbar_init(bar(Q_EMPTY + i), 1);
      mbar_init(bar(S_FULL + i), 1);
      mbar_init(bar(S_EMPTY + i), kSoftmaxWarps);
      mbar_init(bar(P_FULL + i), kSoftmaxWarps);
      mbar_init(bar(P_EMPTY + i), 1);
    }
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(bar(KV_FULL + i), 1);
      mbar_init(bar(KV_EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(O_FULL + i), 1);
      mbar_init(bar(O_EMPTY + i), kSoftmaxWarps);
    }
    mbar_init(bar(DRAIN), 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), 512);  // S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384)
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };
  // {row_start, len, q_tile, 0}; a zero length is read as 1 so that every role
  // walks the same tiles (nothing of such an item is stored)
  auto unit_item = [&](int64_t unit) {
    if (unit >= n_units) return make_int4(0, 1, 0, 0);
    int4 it = __ldg(p.items + unit / p.n_heads);
    it.y = max(it.y, 1);
    return it;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int u = 0, g = 0, nq = 0;
      bool stop = false;
      int4 nxt = unit_item(blockIdx.x);
      for (int64_t unit = blockIdx.x; unit < n_units && !stop; unit += gridDim.x, ++u) {
        const int4 it = nxt;
        nxt = unit_item(unit + gridDim.x);  // the next unit's item loads while this one issues
        const int h = int(unit % p.n_heads);
        const int n_kv = (it.y + kRows - 1) / kRows;
        const int qb = u & 1;
        if (aborted(s_abort) || !mbar_wait(bar(Q_EMPTY + qb), ((u >> 1) & 1) ^ 1)) {
          if (!aborted(s_abort)) fail();
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(bar(Q_FULL + qb), kTileBytes);
        tma_load_2d(sQ + qb * kTileBytes, &p.qkv_map, bar(Q_FULL + qb), p.q_col + h * kHd,
                    it.x + it.z * kRows);
        ++nq;
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int s = g % kKvStages;
          if (aborted(s_abort) || !mbar_wait(bar(KV_EMPTY + s), ((g / kKvStages) & 1) ^ 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          const uint32_t sk = sKV + s * 2 * kTileBytes;
          mbar_arrive_expect_tx(bar(KV_FULL + s), 2 * kTileBytes);
          tma_load_2d(sk, &p.qkv_map, bar(KV_FULL + s), p.k_col + h * kHd, it.x + j * kRows);
          tma_load_2d(sk + kTileBytes, &p.qkv_map, bar(KV_FULL + s), p.v_col + h * kHd, it.x + j * kRows);
        }
      }
      if (aborted(s_abort)) {  // loads nobody consumed must land before the CTA exits (bounded)
        for (int q = (g > kKvStages ? g - kKvStages : 0); q < g; ++q)
          mbar_wait(bar(KV_FULL + q % kKvStages), (q / kKvStages) & 1);
        for (int q = (nq > 2 ? nq - 2 : 0); q < nq; ++q) mbar_wait(bar(Q_FULL + (q & 1)), (q >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // One flat sequence over the CTA's tiles: S of a tile is issued before the
    // previous tile's O += P V, across unit boundaries too, so the next unit's
    // first scores are ready when the softmax warps finish the last tile.
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(DT<T>::umma_fmt, kRows, kRows, /*a_mn=*/0, /*b_mn=*/0);
      constexpr uint32_t idesc_o = umma_idesc_f16(DT<T>::umma_fmt, kRows, kHd, /*a_mn=*/0, /*b_mn=*/1);
      int u = 0, g = 0;
      bool stop = false;
      // O_uu += P_gp V_gp; the first of a unit overwrites O buffer uu&1 once unit
      // uu-2's O was read from it; the last of a unit publishes O
      auto pv = [&](int gp, bool first, bool last, int uu) -> bool {
        const int bp = gp & 1, sp = gp % kKvStages;
        if (!mbar_wait(bar(P_FULL + bp), (gp >> 1) & 1)) return false;
        if (first && !mbar_wait(bar(O_EMPTY + (uu & 1)), ((uu >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t pb = sP + bp * 2 * kTileBytes;
        const uint32_t vb = sKV + sp * 2 * kTileBytes + kTileBytes;
#pragma unroll
        for (int t = 0; t < kRows / 16; ++t) {
          const uint64_t ad = smem_desc(pb + (t >> 2) * kTileBytes + (t & 3) * 32, 16, 1024, 2);
          const uint64_t bd = smem_desc(vb + t * 2048, kTileBytes, 1024, 2);
          umma_f16(tmem + 256 + (uu & 1) * kHd, ad, bd, idesc_o, (first && t == 0) ? 0u : 1u);
        }
        umma_commit(bar(P_EMPTY + bp));
        umma_commit(bar(KV_EMPTY + sp));
        if (last) umma_commit(bar(O_FULL + (uu & 1)));
        return true;
      };
      bool have_prev = false, prev_first = false, prev_last = false;
      int prev_g = 0, prev_u = 0;
      int4 nxt = unit_item(blockIdx.x);
      for (int64_t unit = blockIdx.x; unit < n_units && !stop; unit += gridDim.x, ++u) {
        const int4 it = nxt;
        nxt = unit_item(unit + gridDim.x);
        const int n_kv = (it.y + kRows - 1) / kRows;
        const int qb = u & 1;
        if (aborted(s_abort) || !mbar_wait(bar(Q_FULL + qb), (u >> 1) & 1)) {
          if (!aborted(s_abort)) fail();
          stop = true;
          break;
        }
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int s = g % kKvStages, b = g & 1;
          if (aborted(s_abort) || !mbar_wait(bar(KV_FULL + s), (g / kKvStages) & 1) ||
              !mbar_wait(bar(S_EMPTY + b), ((g >> 1) & 1) ^ 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t qa = sQ + qb * kTileBytes, kb = sKV + s * 2 * kTileBytes;
#pragma unroll
          for (int t = 0; t < kHd / 16; ++t)
            umma_f16(tmem + b * kRows, smem_desc(qa + t * 32, 16, 1024, 2), smem_desc(kb + t * 32, 16, 1024, 2),
                     idesc_s, t > 0 ? 1u : 0u);
          umma_commit(bar(S_FULL + b));
          if (j == n_kv - 1) umma_commit(bar(Q_EMPTY + qb));
          if (have_prev && !pv(prev_g, prev_first, prev_last, prev_u)) {
            fail();
            stop = true;
            break;
          }
          have_prev = true;
          prev_g = g;
          prev_first = j == 0;
          prev_last = j == n_kv - 1;
          prev_u = u;
        }
      }
      if (!stop && have_prev && !pv(prev_g, prev_first, prev_last, prev_u)) fail();
      if (aborted(s_abort)) {  // every issued MMA must finish before TMEM is released (bounded)
        umma_commit(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + output (warps 2..9)
    // Both warps of a quadrant take every tile and every pair barrier, whatever
    // happens, so that neither can be left waiting at bar.sync.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // key columns [64 half, +64) of S, O columns [32 half, +32)
    const int row = quad * 32 + lane;
    const uint32_t pair_bar = 1 + quad;  // named barrier of this quadrant's two warps
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const uint32_t prow = (row >> 3) * 1024 + (row & 7) * 128;  // this row in a SW128 block
    // O / l of a finished unit: the pair adds its two shares of the row sum,
    // normalises and stores this half's 32 columns, and frees O buffer uu&1
    auto epilogue = [&](const int4& eit, int eh, int uu, float el) {
      s_lsum[half * 128 + row] = el;
      named_barrier_sync(pair_bar, 64);
      const float l_row = el + s_lsum[(half ^ 1) * 128 + row];
      bool ok = !aborted(s_abort);
      if (ok && !mbar_wait(bar(O_FULL + (uu & 1)), (uu >> 1) & 1)) {
        fail();
        ok = false;
      }
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        uint32_t ov[32];
        tmem_ld32(tmem + lane_addr + 256 + (uu & 1) * kHd + half * 32, ov);
        const int qr = eit.z * kRows + row;
        if (qr < eit.y) {
          const float inv = 1.f / l_row;
          T* dst = reinterpret_cast<T*>(p.out) + int64_t(eit.x + qr) * p.ldo + eh * kHd + half * 32;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 w;
            w.x = Pack2<T>::pack(__uint_as_float(ov[8 * c + 0]) * inv, __uint_as_float(ov[8 * c + 1]) * inv);
            w.y = Pack2<T>::pack(__uint_as_float(ov[8 * c + 2]) * inv, __uint_as_float(ov[8 * c + 3]) * inv);
            w.z = Pack2<T>::pack(__uint_as_float(ov[8 * c + 4]) * inv, __uint_as_float(ov[8 * c + 5]) * inv);
            w.w = Pack2<T>::pack(__uint_as_float(ov[8 * c + 6]) * inv, __uint_as_float(ov[8 * c + 7]) * inv);
            reinterpret_cast<uint4*>(dst)[c] = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(O_EMPTY + (uu & 1)));
    };
    bool have_pending = false;
    int4 pend_it = make_int4(0, 1, 0, 0);
    int pend_h = 0, pend_u = 0;
    float pend_l = 0.f;
    int u = 0, g = 0;
    int4 nxt = unit_item(blockIdx.x);
    for (int64_t unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++u) {
      const int4 it = nxt;
      nxt = unit_item(unit + gridDim.x);
      const int h = int(unit % p.n_heads);
      const int n_kv = (it.y + kRows - 1) / kRows;
      float m = -INFINITY, l = 0.f;         // l: this half's share of the row sum
      for (int j = 0; j < n_kv; ++j, ++g) {
        const int b = g & 1;
        bool ok = !aborted(s_abort);
        if (ok && !mbar_wait(bar(S_FULL + b), (g >> 1) & 1)) {
          fail();
          ok = false;
        }
        const bool work = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        const int nvalid = min(kRows, it.y - j * kRows) - half * 64;  // valid keys in this half
        uint32_t sv[64];
        float mx = -INFINITY;
        if (work) {
          tmem_ld64(tmem + lane_addr + b * kRows + half * 64, sv);
          float mxs[8];  // eight independent chains instead of one 64-long one
#pragma unroll
          for (int q = 0; q < 8; ++q) mxs[q] = -INFINITY;
          if (nvalid >= 64) {  // warp-uniform: a full half tile needs no mask
#pragma unroll
            for (int c = 0; c < 64; ++c) mxs[c & 7] = fmaxf(mxs[c & 7], __uint_as_float(sv[c]));
          } else {
#pragma unroll
            for (int c = 0; c < 64; ++c)
              if (c < nvalid) mxs[c & 7] = fmaxf(mxs[c & 7], __uint_as_float(sv[c]));
          }
          const float raw_max = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                                      fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
          mx = raw_max * p.scale_log2;  // the scale is positive: max commutes with it
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(S_EMPTY + b));  // this half of S_j is in registers
        // the row max over both halves
        float* smx = s_max + (g & 1) * 256;
        smx[half * 128 + row] = mx;
        named_barrier_sync(pair_bar, 64);
        mx = fmaxf(mx, smx[(half ^ 1) * 128 + row]);
        const float m_new = (j == 0 || mx > m + kMaxSlack) ? mx : m;
        const float alpha = (j == 0) ? 1.f : ex2(m - m_new);
        // P_j goes into buffer b once the MMA that read it two tiles ago has finished
        ok = work && !aborted(s_abort);
        if (ok && !mbar_wait(bar(P_EMPTY + b), ((g >> 1) & 1) ^ 1)) {
          fail();
          ok = false;
        }
        float sums[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains
        if (__all_sync(0xffffffffu, ok)) {
          const uint32_t pb = sP + b * 2 * kTileBytes + half * kTileBytes - base;
          const float sl2 = p.scale_log2, neg_m = -m_new;
          const bool full = nvalid >= 64;  // warp-uniform
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {  // 16-byte chunks = 8 keys
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int c = c8 * 8 + 2 * i;
              float p0 = ex2(fmaf(__uint_as_float(sv[c]), sl2, neg_m));
              float p1 = ex2(fmaf(__uint_as_float(sv[c + 1]), sl2, neg_m));
              if (!full) {
                p0 = c < nvalid ? p0 : 0.f;
                p1 = c + 1 < nvalid ? p1 : 0.f;
              }
              sums[i] += p0 + p1;
              w[i] = Pack2<T>::pack(p0, p1);
            }
            *reinterpret_cast<uint4*>(gbase + pb + prow + ((c8 ^ (row & 7)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        l = l * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
        m = m_new;
        // the max moved: rescale this half's O columns once the previous O += P V has finished
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
          bool ok2 = !aborted(s_abort);
          if (ok2 && !mbar_wait(bar(P_EMPTY + ((g - 1) & 1)), ((g - 1) >> 1) & 1)) {
            fail();
            ok2 = false;
          }
          if (__all_sync(0xffffffffu, ok2)) {
            tc_fence_after();
            uint32_t ov[32];
            tmem_ld32(tmem + lane_addr + 256 + (u & 1) * kHd + half * 32, ov);
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st32(tmem + lane_addr + 256 + (u & 1) * kHd + half * 32, ov);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(P_FULL + b));
        // the previous unit's output, now that its last O += P V has long finished
        if (j == 0 && have_pending) {
          epilogue(pend_it, pend_h, pend_u, pend_l);
          have_pending = false;
        }
      }
      pend_it = it;
      pend_h = h;
      pend_u = u;
      pend_l = l;
      have_pending = true;
    }
    if (have_pending) epilogue(pend_it, pend_h, pend_u, pend_l);
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

}  // namespace lf

using namespace lf;

extern "C" int lf_attention_varlen(void* stream, int dtype, const void* qkv, int64_t ld_qkv, int64_t n_tokens,
                                   int64_t q_col, int64_t k_col, int64_t v_col, int n_heads, int head_dim,
                                   const int32_t* items, int n_items, float scale, void* out, int64_t ld_out,
                                   int32_t* status) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_UNSUPPORTED, "lf_attention_varlen: dtype %d (bf16 or f16 only)", dtype);
  if (head_dim != kHd) return set_error(LF_ERR_UNSUPPORTED, "lf_attention_varlen: head_dim %d (64 only)", head_dim);
  if (n_heads <= 0 || n_items < 0 || n_tokens < 0 || (n_items > 0 && (items == nullptr || qkv == nullptr || out == nullptr)))
    return set_error(LF_ERR_INVALID, "lf_attention_varlen: bad sizes or null pointers");
  const int64_t width = int64_t(n_heads) * head_dim;
  if (q_col < 0 || k_col < 0 || v_col < 0 || q_col % 64 || k_col % 64 || v_col % 64 || q_col + width > ld_qkv ||
      k_col + width > ld_qkv || v_col + width > ld_qkv)
    return set_error(LF_ERR_INVALID, "lf_attention_varlen: q/k/v column offsets must be multiples of 64 inside a row");
  if (ld_out < width || !aligned16(qkv) || !aligned16(out) || !aligned16(items) || (ld_qkv * 2) % 16 || (ld_out * 2) % 16)
    return set_error(LF_ERR_INVALID, "lf_attention_varlen: pointers and row strides must be 16-byte aligned");
  if (n_items == 0 || n_tokens == 0) return LF_OK;
  AttnParams p;
  memset(&p, 0, sizeof(p));
  PFN_encodeTiled enc = get_encode_tiled();
  if (enc == nullptr) return set_error(LF_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cuuint64_t(ld_qkv), cuuint64_t(n_tokens)};
  const cuuint64_t strides[1] = {cuuint64_t(ld_qkv) * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&p.qkv_map, dtype == LF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(qkv), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LF_ERR_CUDA, "cuTensorMapEncodeTiled(qkv) failed: %d", int(r));
  p.items = reinterpret_cast<const int4*>(items);
  p.n_items = n_items;
  p.n_heads = n_heads;
  p.q_col = int32_t(q_col);
  p.k_col = int32_t(k_col);
  p.v_col = int32_t(v_col);
  p.out = out;
  p.ldo = ld_out;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n_units = int64_t(n_items) * n_heads;
  const int grid = int(n_units < sms ? n_units : sms);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = dtype == LF_DTYPE_BF16 ? attention_varlen_kernel<__nv_bfloat16> : attention_varlen_kernel<__half>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(attention)");
  kern<<<grid, kThreads, kSmemBytes, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch attention_varlen");
  count_launch();
  return LF_OK;
}
