// Projection GEMM on tcgen05: Y = act(X W^T + bias), bf16 / f16 in, f32 accumulate.
//
// Replaces the encoder's nn.Linear projections (src/latefuse/model/encoder.py:
// the fused q/k/v, attention-output, FFN up and down projections) with an
// sm_100a kernel of this library, so that work around a projection can be
// fused into it (the FFN's GELU in the epilogue: ACT2FN["gelu"] of
// encoder.py:122,139).  Rounding follows torch: round(acc + bias) to the dtype,
// then for GELU round(gelu_f32(that)).
//
// Persistent, one CTA per SM, 128 x 256 output tiles in m-major order (the CTAs
// working at one time share the rows of X and all of W through L2):
//   warp 0      TMA producer: per 64-wide K block an X box {64, 128} and a W box
//               {64, 256} (both K-major, SW128) into a 4-stage ring of 48 KB;
//   warp 1      MMA issuer: four tcgen05.mma (M=128, N=256, K=16) per K block
//               into one of two TMEM accumulators (256 columns each), so the
//               epilogue of one tile overlaps the main loop of the next;
//   warps 2-9   epilogue, two warps per TMEM lane quadrant (128 columns each),
//               one output row per thread: 32 columns per tcgen05.ld, bias and
//               activation in f32, rounded, staged per warp in a 32 x 32 SW64
//               tile and written by TMA (rows past M are clipped by
//               the tensor map).
// With LoRA (lf_linear_lora) the per-row delta joins the same accumulator: after
// a tile's K blocks come one "delta block" per adapter segment overlapping the
// tile's rows, staged through the same ring: the (tile, segment) block of the
// shrink output u (written by lf_lora_shrink_blocked: the tile's rows of that
// segment, other rows 0, in the no-swizzle K-major operand layout, so one bulk
// copy stages it) and the segment's B factor columns (MN-major SW128, four
// 64-column blocks in one copy straight from the slot cache, prefetched into L2
// one tile ahead), multiplied with K = R, so every row gets its own adapter's delta:
// y = act(round(x W^T + bias + u B)).
// Every wait is bounded: a timeout sets LF_STATUS_TIMEOUT and the roles unwind.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kABytes = kBM * kBK * 2;           // 16 KB
constexpr int kBBytes = kBN * kBK * 2;           // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;   // 48 KB
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;                    // two per TMEM lane quadrant, 128 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kOutCols = 32;                     // output columns per epilogue store
constexpr int kOutBuf = 32 * kOutCols * 2;       // one warp's 32 x 32 staging tile: 2 KB
constexpr int kDeltaBuf = 16384;                 // one delta block (rank 16) loaded at the tile's start
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiWarps * kOutBuf + kDeltaBuf + 1024;

struct alignas(64) LinearParams {
  CUtensorMap x_map;  // 2D {K, M}, box {64, 128}, SW128
  CUtensorMap w_map;  // 2D {K, N}, box {64, 256}, SW128
  CUtensorMap y_map;  // 2D {N, M}, box {32, 32}, SW64
  CUtensorMap b_map[kMaxModules];     // LoRA: 4D {64, R, module_cols / 64, n_slots}, box {64, R, 4, 1}, SW128
  const void* u;                      // LoRA: blocked shrink output (lf_lora_shrink_blocked)
  const void* b_ptr[kMaxModules];     // LoRA: (slot 0, module i) B factors, for L2 prefetch
  int64_t b_slot_stride;              // elements
  int32_t n_slots;
  const void* bias;   // N entries or null
  const int32_t* tile_pairs;          // LoRA: tile b's (segment, slot) pairs are entries
  const int32_t* pairs;               //   tile_pairs[b] .. tile_pairs[b + 1] of pairs; null: no delta
  int32_t n_segs;
  int32_t rank;
  int32_t n_mod;                      // output column block i (module_cols wide) takes module i's delta
  int32_t module_cols;
  int64_t m_rows;
  int64_t n_tiles;
  int32_t n_tiles_n;
  int32_t n_kb;
  int32_t act;        // LF_ACT_*
  int32_t* status;
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Entries [q0, q1) of the pair table for 128-row tile b.  A range that is not
// ascending or holds more pairs than there are segments reads as empty, and
// `bad` says so, so that every role walks the same (no) pairs.
__device__ __forceinline__ int2 pair_range(const int32_t* tile_pairs, int b, int n_segs, bool* bad = nullptr) {
  const int q0 = __ldg(tile_pairs + b), q1 = __ldg(tile_pairs + b + 1);
  const bool ok = q0 >= 0 && q1 >= q0 && q1 - q0 <= n_segs;
  if (bad != nullptr) *bad = !ok;
  return ok ? make_int2(q0, q1) : make_int2(0, 0);
}

__device__ __forceinline__ bool aborted_flag(const int32_t* f) {
  return *reinterpret_cast<const volatile int32_t*>(f) != 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) linear_kernel(const __grid_constant__ LinearParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const uint32_t s_stage0 = base;
  const uint32_t s_out0 = base + kStages * kStageBytes;  // [warp] 2 KB staging tiles
  const uint32_t s_delta = s_out0 + kEpiWarps * kOutBuf;  // the tile's first delta block (rank 16)
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (s_delta + kDeltaBuf - base));
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int FULL = 0, EMPTY = kStages, ACC_FULL = 2 * kStages, ACC_EMPTY = 2 * kStages + 2,
            DRAIN = 2 * kStages + 4, DFULL = DRAIN + 1, DEMPTY = DRAIN + 2, N_BARS = DRAIN + 3;
  // a tile's first delta block goes to its own buffer, loaded before the tile's K
  // blocks, so it has landed when the MMA reaches it (later ones use the ring)
  const bool dbuf = p.pairs != nullptr && 768 * p.rank <= kDeltaBuf;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[N_BARS]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), kEpiWarps);
    }
    mbar_init(bar(DRAIN), 1);
    mbar_init(bar(DFULL), 1);
    mbar_init(bar(DEMPTY), 1);
    *s_abort = 0;
    fence_mbar_init();
    prefetch_tmap(&p.x_map);
    prefetch_tmap(&p.w_map);
    prefetch_tmap(&p.y_map);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), 2 * kBN);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_launch_dependents();

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int kk = 0, dk = 0;
      bool stop = false;
      // the B factors of a tile's segments, into L2 (whole rank x module_cols block)
      auto prefetch_b = [&](int64_t tt) {
        if (p.pairs == nullptr || tt >= p.n_tiles) return;
        const int pmod = int32_t(tt % p.n_tiles_n) * kBN / p.module_cols;
        if (pmod >= p.n_mod) return;
        const int mb = int32_t(tt / p.n_tiles_n);
        const int2 qr = pair_range(p.tile_pairs, mb, p.n_segs);
        for (int q = qr.x; q < qr.y; ++q) {
          const int32_t slot = __ldg(p.pairs + 2 * q + 1);
          if (slot >= 0 && slot < p.n_slots)
            prefetch_l2(static_cast<const T*>(p.b_ptr[pmod]) + int64_t(slot) * p.b_slot_stride,
                        uint32_t(p.rank) * uint32_t(p.module_cols) * 2u);
        }
      };
      prefetch_b(blockIdx.x);
      for (int64_t t = blockIdx.x; t < p.n_tiles && !stop; t += gridDim.x) {
        const int32_t m0 = int32_t(t / p.n_tiles_n) * kBM, n0 = int32_t(t % p.n_tiles_n) * kBN;
        const int mod = p.pairs != nullptr ? n0 / p.module_cols : p.n_mod;
        int q0 = 0, q1 = 0;
        if (mod < p.n_mod) {  // loaded now, used after the K blocks
          bool bad = false;
          const int2 qr = pair_range(p.tile_pairs, m0 / kBM, p.n_segs, &bad);
          if (bad) set_status(p.status, LF_STATUS_BAD_SEGMENT);
          q0 = qr.x;
          q1 = qr.y;
        }
        const int32_t n_loc = mod < p.n_mod ? n0 - mod * p.module_cols : 0;
        const int64_t n_blk = (p.m_rows + kBM - 1) / kBM + p.n_segs;
        // u block of pair q (tile rows of its segment, others 0) and the segment's B columns
        auto load_delta = [&](uint32_t dst, uint32_t b_dst, uint32_t full, int q) {
          int j = __ldg(p.pairs + 2 * q);
          const int32_t slot = __ldg(p.pairs + 2 * q + 1);  // out of range: zero fill, no delta, reported
          if (j < 0 || j >= p.n_segs) {  // a segment outside the table: read block j = 0, reported
            set_status(p.status, LF_STATUS_BAD_SEGMENT);
            j = 0;
          }
          if (slot < 0 || slot >= p.n_slots) set_status(p.status, LF_STATUS_BAD_SLOT);
          mbar_arrive_expect_tx(full, 768 * p.rank);        // u 128 x R + B R x 256
          bulk_load(dst, static_cast<const T*>(p.u) + (int64_t(mod) * n_blk + m0 / kBM + j) * kBM * p.rank,
                    256 * p.rank, full);
          // the tile's 256 B columns as four 64-column blocks of R rows, block b at
          // b_dst + b * R * 128, in one copy (a copy costs about as much to issue as
          // it takes to move 2 KB)
          tma_load_4d(b_dst, &p.b_map[mod], full, 0, 0, n_loc / 64, slot);
        };
        // The first pair goes to the delta buffer once the MMA has started this tile
        // (after K block kStages of it has been issued, the previous tile's delta is
        // done): it then has the rest of the tile's K blocks to land.
        const bool use_dbuf = dbuf && q1 > q0;
        const int d_after = (p.n_kb < kStages ? p.n_kb : kStages) - 1;
        for (int kb = 0; kb < p.n_kb; ++kb, ++kk) {
          const int s = kk % kStages;
          if (aborted_flag(s_abort) || !mbar_wait(bar(EMPTY + s), ((kk / kStages) & 1) ^ 1)) {
            if (!aborted_flag(s_abort)) fail();
            stop = true;
            break;
          }
          const uint32_t st = s_stage0 + s * kStageBytes;
          mbar_arrive_expect_tx(bar(FULL + s), kStageBytes);
          tma_load_2d(st, &p.x_map, bar(FULL + s), kb * kBK, m0);
          tma_load_2d(st + kABytes, &p.w_map, bar(FULL + s), kb * kBK, n0);
          if (use_dbuf && kb == d_after) {
            if (aborted_flag(s_abort) || !mbar_wait(bar(DEMPTY), (dk & 1) ^ 1)) {
              if (!aborted_flag(s_abort)) fail();
              stop = true;
              ++kk;
              break;
            }
            // the delta buffer holds u at its start and B right after it (1 KB-aligned)
            load_delta(s_delta, s_delta + 256 * p.rank, bar(DFULL), q0);
            ++dk;
          }
        }
        if (use_dbuf) ++q0;
        if (!stop) prefetch_b(t + gridDim.x);  // the ring is full here: the producer has time
        if (stop || mod >= p.n_mod) continue;
        for (int q = q0; q < q1; ++q) {
          const int s = kk % kStages;
          if (aborted_flag(s_abort) || !mbar_wait(bar(EMPTY + s), ((kk / kStages) & 1) ^ 1)) {
            if (!aborted_flag(s_abort)) fail();
            stop = true;
            break;
          }
          load_delta(s_stage0 + s * kStageBytes, s_stage0 + s * kStageBytes + kABytes, bar(FULL + s), q);
          ++kk;
        }
      }
      if (aborted_flag(s_abort)) {  // loads nobody consumed land before the CTA exits (bounded)
        for (int q = (kk > kStages ? kk - kStages : 0); q < kk; ++q)
          mbar_wait(bar(FULL + q % kStages), (q / kStages) & 1);
        if (dk > 0) mbar_wait(bar(DFULL), (dk - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kBM, kBN, 0, 0);
      const uint32_t idesc_d = umma_idesc_f16(DT<T>::umma_fmt, kBM, kBN, 0, 1);
      int kk = 0, it = 0, dk = 0;
      bool stop = false;
      auto wait = [&](uint32_t b, uint32_t parity) {
        if (aborted_flag(s_abort)) return false;
        if (mbar_wait(b, parity)) return true;
        if (!aborted_flag(s_abort)) fail();
        return false;
      };
      for (int64_t t = blockIdx.x; t < p.n_tiles && !stop; t += gridDim.x, ++it) {
        const int a = it & 1;
        const int32_t m0 = int32_t(t / p.n_tiles_n) * kBM, n0 = int32_t(t % p.n_tiles_n) * kBN;
        const int mod = p.pairs != nullptr ? n0 / p.module_cols : p.n_mod;
        int n_delta = 0;
        if (mod < p.n_mod) {  // loaded now, used after the K blocks
          const int2 qr = pair_range(p.tile_pairs, m0 / kBM, p.n_segs);
          n_delta = qr.y - qr.x;
        }
        if (!wait(bar(ACC_EMPTY + a), ((it >> 1) & 1) ^ 1)) break;
        for (int kb = 0; kb < p.n_kb; ++kb, ++kk) {
          const int s = kk % kStages;
          if (!wait(bar(FULL + s), (kk / kStages) & 1)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t st = s_stage0 + s * kStageBytes;
#pragma unroll
          for (int q = 0; q < kBK / 16; ++q)
            umma_f16(tmem + a * kBN, smem_desc(st + q * 32, 16, 1024, 2), smem_desc(st + kABytes + q * 32, 16, 1024, 2),
                     idesc, (kb | q) != 0 ? 1u : 0u);
          umma_commit(bar(EMPTY + s));
        }
        if (!stop && n_delta > 0) {
          const int nq = p.rank / 8;  // 16-byte chunks of a u row
          auto delta_mma = [&](uint32_t ua, uint32_t ba) {
            tc_fence_after();
            for (int q = 0; q < p.rank / 16; ++q)
              umma_f16(tmem + a * kBN, smem_desc(ua + q * 256, 128, uint32_t(nq) * 128, 0),
                       smem_desc(ba + q * 2048, p.rank * 128, 1024, 2), idesc_d, 1u);
          };
          int d = 0;
          if (dbuf) {  // the first pair, from the delta buffer
            if (!wait(bar(DFULL), dk & 1)) {
              stop = true;
            } else {
              delta_mma(s_delta, s_delta + 256 * p.rank);
              umma_commit(bar(DEMPTY));
              ++dk;
              d = 1;
            }
          }
          for (; d < n_delta && !stop; ++d) {
            const int s = kk % kStages;
            if (!wait(bar(FULL + s), (kk / kStages) & 1)) {
              stop = true;
              break;
            }
            const uint32_t st = s_stage0 + s * kStageBytes;
            delta_mma(st, st + kABytes);
            umma_commit(bar(EMPTY + s));
            ++kk;
          }
        }
        if (!stop) umma_commit(bar(ACC_FULL + a));
      }
      if (aborted_flag(s_abort)) {  // every issued MMA finishes before TMEM is released (bounded)
        umma_commit(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [128 half, 128 half + 128) of the tile
    const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t my_out = s_out0 + (warp - 2) * kOutBuf;
    const T* bias = static_cast<const T*>(p.bias);
    int it = 0;
    for (int64_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++it) {
      const int a = it & 1;
      const int32_t m0 = int32_t(t / p.n_tiles_n) * kBM, n0 = int32_t(t % p.n_tiles_n) * kBN;
      bool ok = !aborted_flag(s_abort);
      if (ok && !mbar_wait(bar(ACC_FULL + a), (it >> 1) & 1)) {
        fail();
        ok = false;
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      for (int c = half * (kBN / kOutCols / 2); c < (half + 1) * (kBN / kOutCols / 2); ++c) {
        uint32_t v[32];
        tmem_ld32(taddr + a * kBN + c * kOutCols, v);
        const int col0 = n0 + c * kOutCols;
        float bf[32];
        if (bias != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + col0) + q);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = Pack2<T>::unpack(ws[i]);
              bf[q * 8 + 2 * i] = f.x;
              bf[q * 8 + 2 * i + 1] = f.y;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) bf[i] = 0.f;
        }
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float y0 = __uint_as_float(v[2 * i]) + bf[2 * i];
          float y1 = __uint_as_float(v[2 * i + 1]) + bf[2 * i + 1];
          if (p.act == LF_ACT_GELU) {
            y0 = gelu_f32(round_through<T>(y0));
            y1 = gelu_f32(round_through<T>(y1));
          }
          packed[i] = Pack2<T>::pack(y0, y1);
        }
        // the store that last read this staging tile must be done with it
        if (lane == 0) tma_store_wait_read_all();
        __syncwarp();
        const uint32_t buf = my_out;
#pragma unroll
        for (int q = 0; q < 4; ++q)  // SW64: 16-byte chunk q of row `lane` at q ^ ((lane >> 1) & 3)
          *reinterpret_cast<uint4*>(gbase + (buf - base) + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&p.y_map, buf, col0, m0 + quad * 32);
          tma_store_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_EMPTY + a));  // this warp's TMEM reads of the tile are done
    }
    if (lane == 0) tma_store_wait_all();
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 2 * kBN);
  }
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

}  // namespace lf

using namespace lf;

// Shared by lf_linear and lf_linear_lora; `lora` null for the plain GEMM.
struct LoraArgs {
  const void* u;
  int rank;
  const void* cache_b;
  int64_t b_slot_stride, b_module_stride;
  int n_slots, n_modules;
  const int32_t* modules;
  int module_cols;
  int n_segs;
  const int32_t *tile_pairs, *pairs;
};

static int linear_impl(const char* fn, void* stream, int dtype, const void* x, int64_t ldx, const void* w,
                       int64_t ldw, const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                       const LoraArgs* lora, int32_t* status) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_UNSUPPORTED, "%s: dtype %d (bf16 or f16 only)", fn, dtype);
  if (act != LF_ACT_NONE && act != LF_ACT_GELU) return set_error(LF_ERR_INVALID, "%s: unknown act %d", fn, act);
  if (m < 0 || m > INT32_MAX || n <= 0 || k <= 0 || n % kBN != 0 || k % kBK != 0)
    return set_error(LF_ERR_UNSUPPORTED, "%s: n %d must be a multiple of 256 and k %d of 64", fn, n, k);
  if (x == nullptr || w == nullptr || y == nullptr) return set_error(LF_ERR_INVALID, "%s: null x, w or y", fn);
  if (ldx < k || ldw < k || ldy < n) return set_error(LF_ERR_INVALID, "%s: a row stride is below its row", fn);
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (bias != nullptr && !aligned16(bias)) || (ldx * 2) % 16 ||
      (ldw * 2) % 16 || (ldy * 2) % 16)
    return set_error(LF_ERR_INVALID, "%s: pointers and row strides must be 16-byte aligned", fn);
  if (lora != nullptr) {
    const LoraArgs& L = *lora;
    if (L.rank != 16 && L.rank != 32 && L.rank != 64)
      return set_error(LF_ERR_UNSUPPORTED, "%s: rank %d (16, 32 or 64)", fn, L.rank);
    if (L.n_modules < 1 || L.n_modules > kMaxModules || L.modules == nullptr)
      return set_error(LF_ERR_INVALID, "%s: n_modules %d not in [1, %d]", fn, L.n_modules, kMaxModules);
    if (L.module_cols <= 0 || L.module_cols % kBN != 0 || n % L.module_cols != 0)
      return set_error(LF_ERR_UNSUPPORTED, "%s: module_cols %d must be a multiple of 256 dividing n %d", fn,
                       L.module_cols, n);
    if (L.u == nullptr || L.cache_b == nullptr || L.n_slots <= 0 || L.n_segs < 0 || L.tile_pairs == nullptr ||
        L.pairs == nullptr)
      return set_error(LF_ERR_INVALID, "%s: null u, cache_b or pair table", fn);
    for (int i = 0; i < L.n_modules; ++i)
      if (L.modules[i] < 0) return set_error(LF_ERR_INVALID, "%s: negative module index", fn);
    if (!aligned16(L.u) || !aligned16(L.cache_b) || (L.b_slot_stride * 2) % 16 || (L.b_module_stride * 2) % 16 ||
        (L.n_slots > 1 && L.b_slot_stride < int64_t(L.module_cols) * L.rank))
      return set_error(LF_ERR_INVALID, "%s: u / cache_b alignment or slot stride", fn);
  }
  if (m == 0) return LF_OK;
  PFN_encodeTiled enc = get_encode_tiled();
  if (enc == nullptr) return set_error(LF_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
  LinearParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType dt = dtype == LF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  auto tmap = [&](CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                  const cuuint32_t* box, CUtensorMapSwizzle swz, const char* what) {
    if (enc(map, dt, cuuint32_t(rank), const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return set_error(LF_ERR_CUDA, "%s: cuTensorMapEncodeTiled(%s) failed", fn, what);
    return int(LF_OK);
  };
  int rc;
  {
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
    const cuuint32_t box[2] = {kBK, kBM};
    if ((rc = tmap(&p.x_map, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "x"))) return rc;
  }
  {
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(ldw) * 2};
    const cuuint32_t box[2] = {kBK, kBN};
    if ((rc = tmap(&p.w_map, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "w"))) return rc;
  }
  {
    const cuuint64_t dims[2] = {cuuint64_t(n), cuuint64_t(m)};
    const cuuint64_t strides[1] = {cuuint64_t(ldy) * 2};
    const cuuint32_t box[2] = {kOutCols, 32};
    if ((rc = tmap(&p.y_map, 2, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B, "y"))) return rc;
  }
  if (lora != nullptr) {
    const LoraArgs& L = *lora;
    const cuuint32_t R = cuuint32_t(L.rank);
    p.u = L.u;
    for (int i = 0; i < L.n_modules; ++i) {
      const void* b = static_cast<const uint8_t*>(L.cache_b) + int64_t(L.modules[i]) * L.b_module_stride * 2;
      const int64_t ss = L.n_slots == 1 ? int64_t(L.module_cols) * L.rank : L.b_slot_stride;
      p.b_ptr[i] = b;
      p.b_slot_stride = ss;
      // (64 columns, R rows, column block, slot): one box holds a tile's four blocks
      const cuuint64_t dims[4] = {64, R, cuuint64_t(L.module_cols / 64), cuuint64_t(L.n_slots)};
      const cuuint64_t strides[3] = {cuuint64_t(L.module_cols) * 2, 128, cuuint64_t(ss) * 2};
      const cuuint32_t box[4] = {64, R, kBN / 64, 1};
      if ((rc = tmap(&p.b_map[i], 4, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "b"))) return rc;
    }
    p.tile_pairs = L.tile_pairs;
    p.pairs = L.pairs;
    p.n_segs = L.n_segs;
    p.rank = L.rank;
    p.n_slots = L.n_slots;
    p.n_mod = L.n_modules;
    p.module_cols = L.module_cols;
  }
  p.bias = bias;
  p.m_rows = m;
  p.n_tiles_n = n / kBN;
  p.n_tiles = ((m + kBM - 1) / kBM) * p.n_tiles_n;
  p.n_kb = k / kBK;
  p.act = act;
  p.status = status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(p.n_tiles < sms ? p.n_tiles : sms);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = dtype == LF_DTYPE_BF16 ? linear_kernel<__nv_bfloat16> : linear_kernel<__half>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(linear)");
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), kSmemBytes, s, p);
  if (e != cudaSuccess) return cuda_error(e, "launch linear");
  count_launch();
  return LF_OK;
}

extern "C" int lf_linear(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                         const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                         int32_t* status) {
  return linear_impl("lf_linear", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, act, nullptr, status);
}

extern "C" int lf_linear_lora(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                              const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                              const void* u, int rank, const void* cache_b, int64_t b_slot_stride,
                              int64_t b_module_stride, int n_slots, int n_modules, const int32_t* modules,
                              int module_cols, int n_segs, const int32_t* tile_pairs, const int32_t* pairs,
                              int32_t* status) {
  LoraArgs L{u, rank, cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules, module_cols,
             n_segs, tile_pairs, pairs};
  return linear_impl("lf_linear_lora", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, act, &L, status);
}
