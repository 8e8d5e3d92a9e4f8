// Persistent, warp-specialised LoRA kernels over the tile records.
//
// Both kernels run one CTA per SM that loops over work items, with three roles:
//   warp 0      producer: streams the item's operands by TMA into a ring of
//               shared-memory stages (mbarrier "full"/"empty" per stage);
//   warp 1      MMA issuer: tcgen05.mma into one of two TMEM accumulators;
//   epilogue    drains the accumulator (a warp may only read the 32 TMEM lanes
//               = tile rows of its quadrant) while the next item's loads and
//               MMAs are already in flight: 4 warps in the shrink, 8 in the
//               expand (two per quadrant, 64 columns each).
//
// Shrink  (item = 128-token tile):  u[m][t] = round(x[t] . A(slot(t), m)) for
//         every module, the hidden dimension streamed in 64-wide K blocks; the
//         epilogue writes u (0 for tile rows outside every segment).  A tile
//         with several segments multiplies each x K-block by every segment's
//         A (up to kmax at once, more in further passes).
// Expand  (item = tile x module x 128 columns):  y += round(u . B(slot, m)); the
//         y tile, the B factor tile and the u tile (canonical K-major layout,
//         straight from the shrink output) arrive by TMA; the epilogue adds in
//         f32, rounds, writes a separate double-buffered output tile and stores
//         it by TMA, so an input stage is free as soon as it has been read.
//         A tile that holds k segments is k sub-items, one per segment, run
//         back to back by the same CTA: each multiplies the tile's u by its
//         segment's B and folds that segment's rows into the one output tile,
//         which is stored once, after the last sub-item.  Segments are sorted
//         by start and do not overlap (the segment-table contract).
//
// Every wait is bounded; a timeout sets LF_STATUS_TIMEOUT and the roles unwind
// without leaving a warp at a hardware barrier.
#include "lf_common.cuh"
#include "lf_internal.h"
#include "lf_records.cuh"

namespace lf {

namespace {

using namespace rec;
constexpr int kYBox = kTile * 64 * 2;  // one 128 x 64 bf16 box, 16 KB
constexpr int kSmemBudget = 220 * 1024;

template <int R>
struct UOperand {  // K-major u tile: 128 rows of R elements
  static constexpr uint32_t kLayout = (R == 8) ? 0u : (R == 16) ? 6u : (R == 32) ? 4u : 2u;
  static constexpr uint32_t kSbo = (R == 8) ? 128u : 8u * R * 2u;  // 8-row group stride
};

template <int R>
struct AOperand {  // MN-major A factor box: 64 K rows of R elements
  static constexpr uint32_t kRowBytes = R * 2;
  static constexpr uint32_t kLayout = (R == 8) ? 0u : (R == 16) ? 6u : (R == 32) ? 4u : 2u;
  static constexpr uint32_t kSbo = 8 * kRowBytes;
};

// ------------------------------------------------------------------ expand
template <int R, int NT>
struct ExpandCfg {
  static constexpr int kNBox = NT / 64;
  static constexpr int kYBytes = kNBox * kYBox;
  static constexpr int kBBox = R * 64 * 2;
  static constexpr int kBBytes = kNBox * kBBox;
  static constexpr int kUBytes = kTile * R * 2;
  static constexpr int kStageBytes = kYBytes + kBBytes + kUBytes;  // multiple of 1024
  static constexpr int kOutBytes = 2 * kYBytes;                     // double-buffered output tile
  static constexpr int kZeroB = (R == 8) ? kNBox * 1024 : 0;
  static constexpr int kZeroU = (R == 8) ? kTile * 16 : 0;
  static constexpr int kRP = R < 16 ? 16 : R;
  static constexpr int kMeta = 1024;
  static constexpr int kStages = (kSmemBudget - 1024 - kOutBytes - kZeroB - kZeroU - kMeta) / kStageBytes;
  static_assert(kStages >= 2, "expand stage ring does not fit");
  static constexpr int kST = kStages > 4 ? 4 : kStages;
  static constexpr size_t kSmem = 1024 + size_t(kST) * kStageBytes + kOutBytes + kZeroB + kZeroU + kMeta;
};

constexpr int kExpandEpiWarps = 8;
constexpr int kExpandThreads = 64 + 32 * kExpandEpiWarps;

}  // namespace

template <typename T, int R, int NT>
__global__ void __launch_bounds__(kExpandThreads, 1)
lora_expand_persist_kernel(const __grid_constant__ ExpandPersistParams p) {
  static_assert(NT == 128, "two epilogue warps per quadrant, 64 columns each");
  using C = ExpandCfg<R, NT>;
  constexpr int ST = C::kST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t s_stage0 = base;
  const uint32_t s_out0 = base + ST * C::kStageBytes;
  const uint32_t s_zero_b = s_out0 + C::kOutBytes;
  const uint32_t s_zero_u = s_zero_b + C::kZeroB;
  uint8_t* meta_base = gbase + (s_zero_u + C::kZeroU - base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(meta_base);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int FULL = 0, EMPTY = ST, ACC_FULL = 2 * ST, ACC_EMPTY = 2 * ST + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[2 * ST + 4]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);
  int4* s_meta = reinterpret_cast<int4*>(&bars[2 * ST + 6]);  // per stage: {row0, col0}

  const int ncb = p.n_col_blocks;
  const int64_t per_tile = int64_t(p.n_modules) * ncb;
  const int64_t total = int64_t(p.n_tiles) * per_tile;
  const int4* recs = reinterpret_cast<const int4*>(p.tiles);
  auto rec_at = [&](int64_t i) { return i < total ? __ldg(recs + i / per_tile) : int4{}; };

  if (tid == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 2);  // the MMA's commit + the epilogue's release
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), kExpandEpiWarps);  // one arrive per epilogue warp
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (R == 8) {
    uint4* z = reinterpret_cast<uint4*>(gbase + (s_zero_b - base));
    for (int i = tid; i < (C::kZeroB + C::kZeroU) / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), 2 * NT);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool stop = false;
      // When launched as a programmatic dependent of the shrink, u may not be
      // written yet: the first ST stages get their y and B loads at once and
      // their u loads after griddepcontrol.wait (which returns at once when
      // there is nothing to wait for).
      bool dep_done = false;
      int n_pend = 0;
      int4 pend[ST];  // {stage, u row, 0, 0}
      auto flush = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int q = 0; q < n_pend; ++q) {
          const uint32_t su = s_stage0 + pend[q].x * C::kStageBytes + C::kYBytes + C::kBBytes;
          tma_load_2d(su, &p.u_map, bar(FULL + pend[q].x), 0, pend[q].y);
        }
        n_pend = 0;
        dep_done = true;
      };
      int64_t item = blockIdx.x;
      int4 rnext = rec_at(item);
      for (; item < total && !stop; item += gridDim.x) {
        const int rem = int(item % per_tile);
        const int m = rem / ncb, cb = rem % ncb;
        const int4 cur = rnext;
        rnext = rec_at(item + gridDim.x);  // the next item's record loads while this one issues
        const int k = sub_items(cur, p.n_segs);
        const int32_t row0 = cur.x * kTile;
        const int32_t col0 = int32_t(p.y_col_off[m]) + cb * NT;
        for (int j = 0; j < k; ++j, ++it) {
          const int s = it % ST;
          const uint32_t ph = (it / ST) & 1;
          if (aborted(s_abort)) { stop = true; break; }
          if (!mbar_wait(bar(EMPTY + s), ph ^ 1)) { fail(); stop = true; break; }
          const uint32_t st = s_stage0 + s * C::kStageBytes;
          const uint32_t sy = st, sb = st + C::kYBytes, su = sb + C::kBBytes;
          // an out-of-range slot reads zeros (TMA fill); the epilogue also adds nothing for it
          const int32_t slot = sub_slot(cur, j, p.seg_slot, p.n_segs);
          if (j == 0) {
            s_meta[s] = make_int4(row0, col0, 0, 0);
            if (!p.into || p.has_r) {  // the tile's y (in place) or r (into mode)
              mbar_arrive_expect_tx(bar(FULL + s), C::kStageBytes);
              const CUtensorMap* src = p.into ? &p.r_map : &p.y_map;
              for (int b = 0; b < C::kNBox; ++b) tma_load_2d(sy + b * kYBox, src, bar(FULL + s), col0 + b * 64, row0);
            } else {
              mbar_arrive_expect_tx(bar(FULL + s), C::kBBytes + C::kUBytes);
            }
          } else {
            mbar_arrive_expect_tx(bar(FULL + s), C::kBBytes + C::kUBytes);
          }
          for (int b = 0; b < C::kNBox; ++b)
            tma_load_3d(sb + b * C::kBBox, &p.b_map[m], bar(FULL + s), cb * NT + b * 64, 0, slot);
          const int32_t urow = int32_t(int64_t(m) * p.n_tokens + row0);
          if (dep_done) {
            tma_load_2d(su, &p.u_map, bar(FULL + s), 0, urow);
          } else {
            pend[n_pend++] = make_int4(s, urow, 0, 0);
            if (n_pend == ST) flush();  // every stage is waiting for its u
          }
        }
      }
      if (!dep_done) flush();
      if (aborted(s_abort)) {  // loads nobody consumed must land before the CTA exits (bounded)
        for (int q = (it > ST ? it - ST : 0); q < it; ++q) mbar_wait(bar(FULL + q % ST), (q / ST) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kTile, NT, /*a_mn=*/0, /*b_mn=*/1);
      using U = UOperand<R>;
      int it = 0;
      bool stop = false;
      int64_t item = blockIdx.x;
      int4 rnext = rec_at(item);
      for (; item < total && !stop; item += gridDim.x) {
        const int4 rec = rnext;
        rnext = rec_at(item + gridDim.x);
        const int k = sub_items(rec, p.n_segs);
        for (int j = 0; j < k; ++j, ++it) {
          const int s = it % ST;
          const uint32_t ph = (it / ST) & 1;
          const int a = it & 1;
          const uint32_t aph = (it >> 1) & 1;
          if (aborted(s_abort)) { stop = true; break; }
          if (!mbar_wait(bar(FULL + s), ph) || !mbar_wait(bar(ACC_EMPTY + a), aph ^ 1)) {
            fail();
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t st = s_stage0 + s * C::kStageBytes;
          const uint32_t sb = st + C::kYBytes, su = sb + C::kBBytes;
#pragma unroll
          for (int kk = 0; kk < C::kRP / 16; ++kk) {
            uint64_t ad, bd;
            if (R == 8) {
              ad = smem_desc(su, s_zero_u - su, U::kSbo, 0);  // K elements 8..15 read zeros
              bd = smem_desc(sb, C::kBBox, s_zero_b - sb, 2);
            } else {
              ad = smem_desc(su + kk * 32, 16, U::kSbo, U::kLayout);
              bd = smem_desc(sb + kk * 2048, C::kBBox, 1024, 2);
            }
            umma_f16(tmem + a * NT, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(bar(ACC_FULL + a));
          umma_commit(bar(EMPTY + s));
        }
      }
      if (it > 0 && aborted(s_abort))  // MMAs in flight must finish before TMEM is released (bounded)
        mbar_wait(bar(ACC_FULL + ((it - 1) & 1)), ((it - 1) >> 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    // All eight warps take every item, sub-item and named barrier, whatever
    // happens, so that no warp can be left waiting at bar.sync.
    constexpr int kEpi = 32 * kExpandEpiWarps;
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;       // output columns [64 * half, 64 * half + 64)
    const int row = quad * 32 + lane;       // tile row
    const bool leader = (warp == 2 && lane == 0);
    const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + half * 64;
    const uint32_t rbase = half * kYBox + (row >> 3) * 1024 + (row & 7) * 128;  // this row in a SW128 box
    int it = 0, n_items = 0;
    int4 meta = make_int4(0, 0, 0, 0);  // leader: the item's {row0, col0}
    // records two items ahead and the next item's first segment, so that no
    // dependent global load sits between two items
    int64_t item = blockIdx.x;
    int4 r1 = rec_at(item), r2 = rec_at(item + gridDim.x);
    int4 g1 = first_seg(r1, p.seg_start, p.seg_len, p.seg_slot, p.n_segs);
    for (; item < total; item += gridDim.x, ++n_items) {
      const int4 rec = r1, seg0 = g1;
      r1 = r2;
      g1 = first_seg(r1, p.seg_start, p.seg_len, p.seg_slot, p.n_segs);
      r2 = rec_at(item + 2 * int64_t(gridDim.x));
      const int k = sub_items(rec, p.n_segs);
      const int64_t row0 = int64_t(rec.x) * kTile;
      const int ob = n_items & 1;
      const uint32_t so = s_out0 + ob * C::kYBytes;
      // (B) the leader has seen the store that last read out[ob] finish (end of the previous item)
      named_barrier_sync(1, kEpi);
      for (int j = 0; j < k; ++j, ++it) {
        const int s = it % ST;
        const uint32_t ph = (it / ST) & 1;
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        const SubRows sr = rows_of(rec, j, seg0, row0, p.n_tokens, p.seg_start, p.seg_len, p.seg_slot, p.n_segs,
                                   p.n_slots, p.status, leader && (item % per_tile) == 0);
        const bool in_seg = row >= sr.lo && row < sr.hi;
        if (j > 0 && leader) mbar_arrive(bar(EMPTY + s));  // nothing here reads a later sub-item's stage
        bool ok = !aborted(s_abort);
        if (ok && !(mbar_wait(bar(ACC_FULL + a), aph) && (j > 0 || mbar_wait(bar(FULL + s), ph)))) {
          fail();
          ok = false;
        }
        const bool work = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is collective
        tc_fence_after();
        if (work) {
          uint32_t acc[64];
          tmem_ld64(taddr + a * NT, acc);
          if (j == 0 || in_seg) {
            // sub-item 0 copies the y tile (its segment's rows with the delta);
            // later sub-items add their segment's rows to the output tile.  In
            // into mode sub-item 0 starts from round(r + bias) instead of y.
            const uint32_t src = (j == 0 ? s_stage0 + s * C::kStageBytes : so) - base;
            uint4 yv[8];
            if (j > 0 || !p.into || p.has_r) {
#pragma unroll
              for (int c = 0; c < 8; ++c)
                yv[c] = *reinterpret_cast<const uint4*>(gbase + src + rbase + ((c ^ (row & 7)) << 4));
            } else {
#pragma unroll
              for (int c = 0; c < 8; ++c) yv[c] = make_uint4(0, 0, 0, 0);
            }
            if (j == 0 && p.into && p.bias != nullptr) {
              const int rem = int(item % per_tile);
              const int64_t col = p.y_col_off[rem / ncb] + (rem % ncb) * NT + half * 64;
              const uint4* bv = reinterpret_cast<const uint4*>(static_cast<const T*>(p.bias) + col);
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const uint4 braw = __ldg(bv + c);
                const uint32_t bw[4] = {braw.x, braw.y, braw.z, braw.w};
                uint32_t* w = reinterpret_cast<uint32_t*>(&yv[c]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 yf = Pack2<T>::unpack(w[i]);
                  const float2 bf = Pack2<T>::unpack(bw[i]);
                  w[i] = Pack2<T>::pack(yf.x + bf.x, yf.y + bf.y);
                }
              }
            }
            if (in_seg) {
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                uint32_t* w = reinterpret_cast<uint32_t*>(&yv[c]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  // y + round(delta), rounded: the reference's two rounding points
                  const float2 yf = Pack2<T>::unpack(w[i]);
                  const float2 d = Pack2<T>::unpack(Pack2<T>::pack(__uint_as_float(acc[c * 8 + 2 * i]),
                                                                   __uint_as_float(acc[c * 8 + 2 * i + 1])));
                  w[i] = Pack2<T>::pack(yf.x + d.x, yf.y + d.y);
                }
              }
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(gbase + (so - base) + rbase + ((c ^ (row & 7)) << 4)) = yv[c];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(ACC_EMPTY + a));  // this warp's TMEM reads are done
        if (j == 0) {
          // (C) every warp has read its rows of the y stage
          named_barrier_sync(1, kEpi);
          if (leader) {
            meta = s_meta[s];             // read before the stage (and its metadata) is handed back
            mbar_arrive(bar(EMPTY + s));  // the input stage may be refilled now
          }
        }
      }
      fence_proxy_async_smem();
      // (D) every warp has written its rows of out[ob]
      named_barrier_sync(1, kEpi);
      if (leader) {
        if (!aborted(s_abort)) {
          for (int b = 0; b < NT / 64; ++b) tma_store_2d(&p.y_map, so + b * kYBox, meta.y + b * 64, meta.x);
          tma_store_commit();
        }
        tma_store_wait_read_le1();  // the store that read the other output buffer has finished
      }
    }
    if (leader) tma_store_wait_all();
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 2 * NT);
  }
}

// ------------------------------------------------------------------ shrink
// One item per tile record.  A record with k segments takes ceil(k / kmax)
// passes over the tile's x; a pass multiplies each x K-block by the A factors
// of up to kmax segments at once (one TMEM accumulator set per segment), and
// its epilogue writes the rows that pass owns: each row gets the product with
// its own segment's A, rows in no segment get 0.
template <typename T, int R>
__global__ void __launch_bounds__(192, 1)
lora_shrink_persist_kernel(const __grid_constant__ ShrinkPersistParams p, int stages, int stage_bytes) {
  constexpr int RP = R < 16 ? 16 : R;
  constexpr int kABox = 64 * R * 2;
  using A = AOperand<R>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);


  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ST = stages;
  const int n_mod = p.n_modules;
  const int KM = p.kmax;
  const int nkb = p.hidden / 64;
  const uint32_t s_stage0 = base;
  const uint32_t s_zero = base + ST * stage_bytes;  // 1 KB of zeros (rank 8 only)
  uint8_t* meta_base = gbase + (s_zero + 1024 - base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(meta_base);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int FULL = 0, EMPTY = ST, ACC_FULL = 2 * ST, ACC_EMPTY = 2 * ST + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[2 * ST + 4]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);
  const uint32_t acc_cols = p.acc_cols;  // one accumulator set: kmax * n_mod * RP columns
  uint32_t alloc_cols = 32;
  while (alloc_cols < 2 * acc_cols) alloc_cols <<= 1;
  const int4* recs = reinterpret_cast<const int4*>(p.tiles);
  auto rec_at = [&](int i) { return i < p.n_tiles ? __ldg(recs + i) : int4{}; };

  if (tid == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);  // the MMA's commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (R == 8) {
    uint4* z = reinterpret_cast<uint4*>(gbase + (s_zero - base));
    for (int i = tid; i < 1024 / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), alloc_cols);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // x comes from the previous kernel; then the next kernel (the expand, or the
  // GEMM that reads u) may be scheduled on SMs this grid leaves free
  pdl_wait();
  pdl_launch_dependents();

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int kk = 0;
      int ti = blockIdx.x;
      int4 rnext = rec_at(ti);
      bool stop = false;
      for (; ti < p.n_tiles && !stop; ti += gridDim.x) {
        const int4 cur = rnext;
        rnext = rec_at(ti + gridDim.x);
        const int32_t row0 = cur.x * kTile;
        const int k = sub_items(cur, p.n_segs);
        for (int j0 = 0; j0 < k && !stop; j0 += KM) {
          const int kp = min(KM, k - j0);
          for (int kb = 0; kb < nkb; ++kb, ++kk) {
            const int s = kk % ST;
            const uint32_t ph = (kk / ST) & 1;
            if (aborted(s_abort) || !mbar_wait(bar(EMPTY + s), ph ^ 1)) {
              if (!aborted(s_abort)) fail();
              stop = true;
              break;
            }
            const uint32_t st = s_stage0 + s * stage_bytes;
            mbar_arrive_expect_tx(bar(FULL + s), kYBox + kp * n_mod * kABox);
            tma_load_2d(st, &p.x_map, bar(FULL + s), kb * 64, row0);
            for (int jj = 0; jj < kp; ++jj) {
              const int32_t slot = sub_slot(cur, j0 + jj, p.seg_slot, p.n_segs);
              // a copy costs about as much to issue as it takes to move 2 KB, so
              // the modules' boxes go in one copy where the cache layout allows
              if (p.a_one_box)
                tma_load_4d(st + kYBox + jj * n_mod * kABox, &p.a_modules_map, bar(FULL + s), 0, kb * 64, 0, slot);
              else
                for (int m = 0; m < n_mod; ++m)
                  tma_load_3d(st + kYBox + (jj * n_mod + m) * kABox, &p.a_map[m], bar(FULL + s), 0, kb * 64, slot);
            }
          }
        }
      }
      if (aborted(s_abort)) {
        for (int q = (kk > ST ? kk - ST : 0); q < kk; ++q) mbar_wait(bar(FULL + q % ST), (q / ST) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc16 = umma_idesc_f16(DT<T>::umma_fmt, kTile, RP, /*a_mn=*/0, /*b_mn=*/1);
      int kk = 0, it = 0;
      bool stop = false;
      int ti = blockIdx.x;
      int4 rnext = rec_at(ti);
      for (; ti < p.n_tiles && !stop; ti += gridDim.x) {
        const int4 rec = rnext;
        rnext = rec_at(ti + gridDim.x);
        const int k = sub_items(rec, p.n_segs);
        for (int j0 = 0; j0 < k && !stop; j0 += KM, ++it) {
          const int kp = min(KM, k - j0);
          const int a = it & 1;
          const uint32_t aph = (it >> 1) & 1;
          if (aborted(s_abort) || !mbar_wait(bar(ACC_EMPTY + a), aph ^ 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          for (int kb = 0; kb < nkb; ++kb, ++kk) {
            const int s = kk % ST;
            const uint32_t ph = (kk / ST) & 1;
            if (!mbar_wait(bar(FULL + s), ph)) { fail(); stop = true; break; }
            tc_fence_after();
            const uint32_t st = s_stage0 + s * stage_bytes;
            if (R == 8) {
              // 8 columns per box, padded to N=16 with a zero block: one MMA per box
              for (int jm = 0; jm < kp * n_mod; ++jm) {
                const uint32_t ab = st + kYBox + jm * kABox;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint64_t ad = smem_desc(st + q * 32, 16, 1024, 2);
                  const uint32_t bstart = ab + q * 16 * A::kRowBytes;
                  const uint64_t bd = smem_desc(bstart, 128, s_zero + q * 256 - bstart, 0);
                  umma_f16(tmem + a * acc_cols + jm * RP, ad, bd, idesc16, (kb | q) != 0 ? 1u : 0u);
                }
              }
            } else {
              // the pass's A boxes lie kABox apart, one swizzle atom of R columns
              // each: a single MMA with N = kp * n_mod * R reads them all as
              // consecutive MN atoms (leading byte offset = kABox)
              const uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kTile, uint32_t(kp * n_mod * R), 0, 1);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint64_t ad = smem_desc(st + q * 32, 16, 1024, 2);
                const uint64_t bd = smem_desc(st + kYBox + q * 16 * A::kRowBytes, kABox, A::kSbo, A::kLayout);
                umma_f16(tmem + a * acc_cols, ad, bd, idesc, (kb | q) != 0 ? 1u : 0u);
              }
            }
            umma_commit(bar(EMPTY + s));
          }
          if (!stop) umma_commit(bar(ACC_FULL + a));
        }
      }
      if (it > 0 && aborted(s_abort)) mbar_wait(bar(ACC_FULL + ((it - 1) & 1)), ((it - 1) >> 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int it = 0;
    int ti = blockIdx.x;
    int4 r1 = rec_at(ti), r2 = rec_at(ti + int(gridDim.x));
    int4 g1 = first_seg(r1, p.seg_start, p.seg_len, p.seg_slot, p.n_segs);
    for (; ti < p.n_tiles; ti += gridDim.x) {
      // records two tiles ahead, the next tile's first segment one ahead
      const int4 rec = r1, seg0 = g1;
      r1 = r2;
      g1 = first_seg(r1, p.seg_start, p.seg_len, p.seg_slot, p.n_segs);
      r2 = rec_at(ti + 2 * int(gridDim.x));
      const int64_t row0 = int64_t(rec.x) * kTile;
      const int64_t t = row0 + row;
      const int k = sub_items(rec, p.n_segs);
      // a record whose tile lies outside the tokens or whose first segment is not
      // in the table writes nothing (every u address below is then in range)
      const bool rec_ok = rec.x >= 0 && row0 < p.n_tokens && rec.y >= 0 && rec.y < p.n_segs;
      if (!rec_ok && row == 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
      int own_lo = 0;  // rows below were written by an earlier pass
      for (int j0 = 0; j0 < k; j0 += KM, ++it) {
        const int kp = min(KM, k - j0);
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        int j_row = -1, hi_last = 0;
        for (int jj = 0; jj < kp; ++jj) {
          const SubRows sr = rows_of(rec, j0 + jj, seg0, row0, p.n_tokens, p.seg_start, p.seg_len, p.seg_slot,
                                     p.n_segs, p.n_slots, p.status, row == 0 && quad == 0);
          if (row >= sr.lo && row < sr.hi) j_row = jj;
          if (sr.hi > hi_last) hi_last = sr.hi;
        }
        const int own_hi = (j0 + kp >= k) ? kTile : max(own_lo, hi_last);
        const bool mine = row >= own_lo && row < own_hi && t < p.n_tokens;
        own_lo = own_hi;
        bool ok = !aborted(s_abort);
        if (ok && !mbar_wait(bar(ACC_FULL + a), aph)) {
          fail();
          ok = false;
        }
        const bool work = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        if (work && rec_ok) {
          for (int m = 0; m < n_mod; ++m) {
            T* dst = reinterpret_cast<T*>(p.u) + (int64_t(m) * p.n_tokens + t) * R;
            // blocked: one 128 x R block per (tile, segment) pair, index tile + segment
            const int64_t n_blk = (p.n_tokens + kTile - 1) / kTile + p.n_segs;
            for (int jj = 0; jj < kp; ++jj) {
#pragma unroll
              for (int c = 0; c < RP / 16; ++c) {
                float v[16];
                tmem_ld16(tmem + (uint32_t(quad * 32) << 16) + a * acc_cols + (jj * n_mod + m) * RP + c * 16, v);
                if (p.u_blocked) {
                  // every row of the tile: its product if it lies in this segment, else 0
                  T* blk = reinterpret_cast<T*>(p.u) +
                           (int64_t(m) * n_blk + rec.x + rec.y + j0 + jj) * (kTile * R);
                  const bool in = j_row == jj && t < p.n_tokens;
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    if (c * 16 + h * 8 < R) {
                      uint4 pk;
                      pk.x = Pack2<T>::pack(in ? v[h * 8 + 0] : 0.f, in ? v[h * 8 + 1] : 0.f);
                      pk.y = Pack2<T>::pack(in ? v[h * 8 + 2] : 0.f, in ? v[h * 8 + 3] : 0.f);
                      pk.z = Pack2<T>::pack(in ? v[h * 8 + 4] : 0.f, in ? v[h * 8 + 5] : 0.f);
                      pk.w = Pack2<T>::pack(in ? v[h * 8 + 6] : 0.f, in ? v[h * 8 + 7] : 0.f);
                      // 8-element chunk q of tile row r in core matrix (r / 8, q)
                      const int q = c * 2 + h;
                      *reinterpret_cast<uint4*>(blk + ((row >> 3) * (R / 8) + q) * 64 + (row & 7) * 8) = pk;
                    }
                  }
                  continue;
                }
                // a row in no segment of this pass writes zeros once (with jj == 0)
                if (mine && (j_row == jj || (j_row < 0 && jj == 0))) {
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    if (c * 16 + h * 8 < R) {
                      uint4 pk;
                      pk.x = Pack2<T>::pack(j_row < 0 ? 0.f : v[h * 8 + 0], j_row < 0 ? 0.f : v[h * 8 + 1]);
                      pk.y = Pack2<T>::pack(j_row < 0 ? 0.f : v[h * 8 + 2], j_row < 0 ? 0.f : v[h * 8 + 3]);
                      pk.z = Pack2<T>::pack(j_row < 0 ? 0.f : v[h * 8 + 4], j_row < 0 ? 0.f : v[h * 8 + 5]);
                      pk.w = Pack2<T>::pack(j_row < 0 ? 0.f : v[h * 8 + 6], j_row < 0 ? 0.f : v[h * 8 + 7]);
                      const int64_t off = (c * 2 + h) * 8;
                      *reinterpret_cast<uint4*>(dst + off) = pk;
                    }
                  }
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(ACC_EMPTY + a));
      }
    }
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, alloc_cols);
  }
}

// ------------------------------------------------------------------ launchers
namespace {

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <typename T, int R, int NT>
int launch_expand(const ExpandPersistParams& p, bool after_shrink, cudaStream_t stream) {
  using C = ExpandCfg<R, NT>;
  auto kern = lora_expand_persist_kernel<T, R, NT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::kSmem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(expand_persist)");
  const int64_t total = int64_t(p.n_tiles) * p.n_modules * p.n_col_blocks;
  const int sms = sm_count();
  const int grid = int(total < sms ? total : sms);
  if (grid == 0) return LF_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kExpandThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (after_shrink) {  // may start while the shrink that writes u still runs
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return cuda_error(e, "launch lora_expand_persist");
  count_launch();
  return LF_OK;
}

template <typename T, int R>
int launch_shrink(ShrinkPersistParams p, cudaStream_t stream) {
  constexpr int RP = R < 16 ? 16 : R;
  const int fixed = 1024 + 1024 + 1024;  // alignment, zeros, barriers
  // segments per pass: one MMA covers every segment and module of a pass
  // (N = kmax * n_modules * RP <= 256, which also keeps two accumulator sets
  // inside TMEM's 512 columns), and the ring keeps at least 5 stages
  int kmax = 256 / (p.n_modules * RP);
  if (kmax > 4) kmax = 4;
  if (kmax < 1) return set_error(LF_ERR_UNSUPPORTED, "persistent shrink: %d modules of rank %d", p.n_modules, R);
  auto stage_of = [&](int km) { return kYBox + km * p.n_modules * 64 * R * 2; };  // multiple of 1024
  while (kmax > 1 && (kSmemBudget - fixed) / stage_of(kmax) < 5) --kmax;
  const int stage_bytes = stage_of(kmax);
  int stages = (kSmemBudget - fixed) / stage_bytes;
  if (stages > 8) stages = 8;
  if (stages < 2) return set_error(LF_ERR_UNSUPPORTED, "persistent shrink: %d modules of rank %d do not fit", p.n_modules, R);
  p.kmax = kmax;
  p.acc_cols = uint32_t(kmax * p.n_modules * RP);
  const size_t smem = size_t(fixed) + size_t(stages) * stage_bytes;
  auto kern = lora_shrink_persist_kernel<T, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(shrink_persist)");
  const int sms = sm_count();
  const int grid = p.n_tiles < sms ? p.n_tiles : sms;
  if (grid == 0) return LF_OK;
  e = launch_pdl(kern, dim3(grid), dim3(192), smem, stream, p, stages, stage_bytes);
  if (e != cudaSuccess) return cuda_error(e, "launch lora_shrink_persist");
  count_launch();
  return LF_OK;
}

template <typename T>
int expand_rank(const ExpandPersistParams& p, int rank, bool after_shrink, cudaStream_t s) {
  switch (rank) {
    case 8: return launch_expand<T, 8, 128>(p, after_shrink, s);
    case 16: return launch_expand<T, 16, 128>(p, after_shrink, s);
    case 32: return launch_expand<T, 32, 128>(p, after_shrink, s);
    case 64: return launch_expand<T, 64, 128>(p, after_shrink, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "persistent expand: rank %d", rank);
}

template <typename T>
int shrink_rank(const ShrinkPersistParams& p, int rank, cudaStream_t s) {
  switch (rank) {
    case 8: return launch_shrink<T, 8>(p, s);
    case 16: return launch_shrink<T, 16>(p, s);
    case 32: return launch_shrink<T, 32>(p, s);
    case 64: return launch_shrink<T, 64>(p, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "persistent shrink: rank %d", rank);
}

}  // namespace

int run_expand_persist(int dtype, const ExpandPersistParams& p, int rank, int nt, bool after_shrink,
                       cudaStream_t s) {
  if (nt != 128) return set_error(LF_ERR_UNSUPPORTED, "persistent expand: column tile %d", nt);
  if (dtype == LF_DTYPE_BF16) return expand_rank<__nv_bfloat16>(p, rank, after_shrink, s);
  return expand_rank<__half>(p, rank, after_shrink, s);
}

int run_shrink_persist(int dtype, const ShrinkPersistParams& p, int rank, cudaStream_t s) {
  if (dtype == LF_DTYPE_BF16) return shrink_rank<__nv_bfloat16>(p, rank, s);
  return shrink_rank<__half>(p, rank, s);
}

}  // namespace lf
