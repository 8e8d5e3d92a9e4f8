// The late-fusion delta in one launch (lf_lora_apply's tcgen05 path over tile records):
//
//     u_m[t]        = round(x[t] . A(slot(t), m))
//     y[t, off_m+n] = round(y[t, off_m+n] + round(u_m[t] . B(slot(t), m)[:, n]))
//
// for every token t of a segment and every module m, with u kept on chip.
//
// An item is one tile record (128 tokens) times one column chunk (chunk_cols of
// every module's hidden columns).  One persistent CTA per SM runs items one after
// another with four roles around two rings of shared-memory stages:
//   warp 0      x producer: for each item, the x K-blocks with the A boxes of the
//               round's segments, by TMA, through a ring of at least 4 x stages;
//   warp 14     B producer: for each 128-column step of y the matching B boxes,
//               through a separate, deeper ring of small stages (freed by the
//               epilogue group that drains the step), from the start of the item:
//               the B factors (scattered 2 KB boxes of the slot cache, whose latency
//               set the pace when they shared the x ring) are in shared memory by the
//               time the shrink is done;
//   warp 1      MMA issuer: u = x A into a TMEM accumulator (one MMA per K step,
//               N = segments x modules x rank), then for each 128-column step of y
//               the delta u B (K = rank, N = 128: two 64-column boxes per MMA, which
//               halves this thread's waits, MMAs and commits, whose latency set the
//               pace at one box per step) into one of up to three TMEM accumulators;
//               an x stage is free as soon as its MMAs complete;
//   warps 2..13 epilogue, three groups of four warps (a warp per TMEM lane quadrant,
//               a thread per tile row).  The groups round u and write each (segment,
//               module) block into shared memory as the delta MMA's K-major operand
//               (the product for rows of that segment, 0 for the others); then the y
//               steps go round-robin to the groups: for each 64-column half of a step
//               each warp rounds its 32 rows of the delta, stages them (in one or two
//               staging boxes per warp; with two, two reductions are in flight) and
//               adds them to y in L2 with one TMA reduction
//               (cp.reduce.async.bulk.tensor .add), which computes round(y + delta)
//               element by element as the reference's add does.
// y never passes through the SM: x is read once per item (the items of one record
// run side by side, so their x comes from L2 after the first), y is read and written
// once by L2, u never leaves the SM, and there is no second launch.  Rows of a
// staged box outside the round's segments add -0, which leaves every value as it was
// (-0 included); a warp whose 32 rows hold none of them adds nothing.
//
// A record with more than kmax segments takes several rounds, each a shrink pass
// and a delta pass over the record's boxes; their reductions touch disjoint rows
// with non-zero values, so the rounds need no ordering between them.
#include "lf_common.cuh"
#include "lf_internal.h"
#include "lf_records.cuh"

namespace lf {

namespace {

using namespace rec;

constexpr int kBoxBytes = kTile * 64 * 2;  // one 128 x 64 box of x or y, 16 KB
constexpr int kGroups = 3;                 // epilogue groups: y boxes go round-robin to them
constexpr int kMaxDBufs = 3;               // 128-column TMEM delta accumulators (fewer where u needs the room)
constexpr int kEpiWarps = 4 * kGroups;       // warps 2 .. 2 + kEpiWarps - 1
constexpr int kBWarp = 2 + kEpiWarps;         // the B producer
constexpr int kFusedThreads = 32 * (kBWarp + 1);
constexpr int kSmemMax = 227 * 1024;       // dynamic shared memory per CTA on sm_100
constexpr int kFixedBytes = 2048;          // alignment slack + barriers
constexpr int kStageOut = 32 * 128;        // one warp's 32 rows x 64 columns of the delta (SW128)

template <int R>
struct FusedOps {
  static constexpr int RP = R < 16 ? 16 : R;    // TMEM columns per (segment, module) of u
  static constexpr int kABox = 64 * R * 2;      // A box: 64 K rows of R (MN-major)
  static constexpr int kBBox = R * 64 * 2;      // B box: R rows of 64 columns (SW128)
  static constexpr int kUBlk = kTile * R * 2;   // u block: 128 rows of R (K-major, no swizzle)
  static constexpr uint32_t kALayout = (R == 8) ? 0u : (R == 16) ? 6u : (R == 32) ? 4u : 2u;
  // rank 8 pads K or N to 16 with zero operands: [0, 1 KB) the shrink's A columns
  // 8..15, [1, 3 KB) the delta's B rows 8..15 (two 64-column atoms), [3, 5 KB) the u
  // blocks' columns 8..15
  static constexpr int kZeroBytes = (R == 8) ? 5120 : 0;
};

}  // namespace

template <typename T, int R>
__global__ void __launch_bounds__(kFusedThreads, 1)
lora_fused_kernel(const __grid_constant__ FusedApplyParams p) {
  using F = FusedOps<R>;
  constexpr int RP = F::RP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.stages, KM = p.kmax, n_mod = p.n_modules;
  const int nkb = p.hidden / 64;
  const int nys = p.chunk_cols / 128;  // 128-column steps of y per module
  const int NB = p.b_stages;
  const uint32_t s_ring = base;
  const uint32_t s_bring = s_ring + uint32_t(NS * p.stage_bytes);
  const uint32_t s_u = s_bring + uint32_t(NB * p.b_stage_bytes);
  const uint32_t s_out = s_u + uint32_t(KM * n_mod * F::kUBlk);  // a staging box per epilogue warp
  const uint32_t s_zero = s_out + uint32_t(kEpiWarps * p.out_bufs * kStageOut);
  const uint32_t s_meta = s_zero + F::kZeroBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (s_meta - base));
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int FULL = 0, EMPTY = NS, BFULL = 2 * NS, BEMPTY = BFULL + NB, DFULL = BEMPTY + NB,
            DEMPTY = DFULL + kMaxDBufs, UFULL = DEMPTY + kMaxDBufs, UEMPTY = UFULL + 1, UREADY = UEMPTY + 1,
            USFREE = UREADY + 1, DRAIN = USFREE + 1, NBAR = DRAIN + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[NBAR]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);
  auto stage = [&](int k) { return s_ring + uint32_t((k % NS) * p.stage_bytes); };
  auto bstage = [&](int k) { return s_bring + uint32_t((k % NB) * p.b_stage_bytes); };
  const int ND = p.d_bufs;

  const int C = p.n_chunks;
  const int n_items = p.n_tiles * C;
  const int4* recs = reinterpret_cast<const int4*>(p.tiles);

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);  // the commit of the MMAs that read the stage
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(bar(BFULL + i), 1);
      // the four warps of the epilogue group that saw the step's delta complete (the MMAs
      // that read the stage are done then), so the MMA thread commits once per step
      mbar_init(bar(BEMPTY + i), 4);
    }
    for (int i = 0; i < ND; ++i) {
      mbar_init(bar(DFULL + i), 1);
      mbar_init(bar(DEMPTY + i), 4);  // the four warps of the group that drained it
    }
    mbar_init(bar(UFULL), 1);
    mbar_init(bar(UEMPTY), 4 * kGroups);
    mbar_init(bar(UREADY), 4 * kGroups);
    mbar_init(bar(USFREE), 1);
    mbar_init(bar(DRAIN), 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (R == 8) {
    uint4* z = reinterpret_cast<uint4*>(gbase + (s_zero - base));
    for (int i = tid; i < F::kZeroBytes / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (tid == 0) {
    prefetch_tmap(&p.x_map);
    prefetch_tmap(&p.ys_map);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), p.tmem_alloc);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // x, y and the tables come from earlier work on the stream; the next kernel may
  // set up on SMs this grid leaves free
  pdl_wait();
  pdl_launch_dependents();

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };
  // a record whose tile lies outside the tokens or whose first segment lies outside
  // the table is skipped by every role (and reported by the epilogue)
  auto rec_valid = [&](const int4& r) {
    return r.x >= 0 && int64_t(r.x) * kTile < p.n_tokens && r.y >= 0 && r.y < p.n_segs;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ x producer
    if (lane == 0) {
      int k = 0;  // ring position
      bool stop = false;
      auto acquire = [&](int kk) {  // the stage at ring position kk is free
        if (aborted(s_abort) || !mbar_wait(bar(EMPTY + kk % NS), ((kk / NS) & 1) ^ 1)) {
          if (!aborted(s_abort)) fail();
          return false;
        }
        return true;
      };
      for (int item = blockIdx.x; item < n_items && !stop; item += gridDim.x) {
        const int4 rc = __ldg(recs + item / C);
        if (!rec_valid(rc)) continue;
        const int ns = sub_items(rc, p.n_segs);
        const int32_t row0 = rc.x * kTile;
        for (int j0 = 0; j0 < ns && !stop; j0 += KM) {
          const int kp = min(KM, ns - j0);
          for (int kb = 0; kb < nkb; ++kb, ++k) {
            if (!acquire(k)) {
              stop = true;
              break;
            }
            const uint32_t st = stage(k);
            const uint32_t full = bar(FULL + k % NS);
            mbar_arrive_expect_tx(full, uint32_t(kBoxBytes + kp * n_mod * F::kABox));
            tma_load_2d(st, &p.x_map, full, kb * 64, row0);
            for (int jj = 0; jj < kp; ++jj) {
              // an out-of-range slot reads zeros (TMA fill); its rows get no delta
              const int32_t slot = sub_slot(rc, j0 + jj, p.seg_slot, p.n_segs);
              const uint32_t ab = st + kBoxBytes + uint32_t(jj * n_mod * F::kABox);
              if (p.a_one_box)
                tma_load_4d(ab, &p.a_modules_map, full, 0, kb * 64, 0, slot);
              else
                for (int m = 0; m < n_mod; ++m) tma_load_3d(ab + m * F::kABox, &p.a_map[m], full, 0, kb * 64, slot);
            }
          }
        }
      }
      if (aborted(s_abort)) {  // copies nobody consumed land before the CTA exits (bounded)
        for (int q = (k > NS ? k - NS : 0); q < k; ++q) mbar_wait(bar(FULL + q % NS), (q / NS) & 1);
      }
    }
  } else if (warp == kBWarp) {
    // ------------------------------------------------------------ B producer
    if (lane == 0) {
      int kb = 0;  // B ring position
      bool stop = false;
      for (int item = blockIdx.x; item < n_items && !stop; item += gridDim.x) {
        const int4 rc = __ldg(recs + item / C);
        const int ch = item % C;
        if (!rec_valid(rc)) continue;
        const int ns = sub_items(rc, p.n_segs);
        for (int j0 = 0; j0 < ns && !stop; j0 += KM) {
          const int kp = min(KM, ns - j0);
          for (int m = 0; m < n_mod && !stop; ++m) {
            for (int b = 0; b < nys; ++b, ++kb) {
              if (aborted(s_abort) || !mbar_wait(bar(BEMPTY + kb % NB), ((kb / NB) & 1) ^ 1)) {
                if (!aborted(s_abort)) fail();
                stop = true;
                break;
              }
              const uint32_t st = bstage(kb);
              const uint32_t full = bar(BFULL + kb % NB);
              const int32_t hcol = ch * p.chunk_cols + b * 128;
              mbar_arrive_expect_tx(full, uint32_t(kp * 2 * F::kBBox));
              // an out-of-range slot reads zeros (TMA fill); its rows get no delta
              for (int jj = 0; jj < kp; ++jj) {
                const int32_t slot = sub_slot(rc, j0 + jj, p.seg_slot, p.n_segs);
                for (int h = 0; h < 2; ++h)  // the step's two 64-column atoms, kBBox apart
                  tma_load_3d(st + uint32_t((jj * 2 + h) * F::kBBox), &p.b_map[m], full, hcol + h * 64, 0, slot);
              }
            }
          }
        }
      }
      if (aborted(s_abort)) {  // copies nobody consumed land before the CTA exits (bounded)
        for (int q = (kb > NB ? kb - NB : 0); q < kb; ++q) mbar_wait(bar(BFULL + q % NB), (q / NB) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_d = umma_idesc_f16(DT<T>::umma_fmt, kTile, 128, /*a_mn=*/0, /*b_mn=*/1);
      constexpr uint32_t idesc16 = umma_idesc_f16(DT<T>::umma_fmt, kTile, RP, /*a_mn=*/0, /*b_mn=*/1);
      const uint32_t s_zero_s = s_zero, s_zero_b = s_zero + 1024, s_zero_u = s_zero + 3072;
      int k = 0, kb = 0, rk = 0, dk = 0;  // x ring position, B ring position, round, y step
      bool stop = false, issued = false;
      auto full_wait = [&](int kk) {
        if (aborted(s_abort) || !mbar_wait(bar(FULL + kk % NS), (kk / NS) & 1)) {
          if (!aborted(s_abort)) fail();
          return false;
        }
        return true;
      };
      for (int item = blockIdx.x; item < n_items && !stop; item += gridDim.x) {
        const int4 rc = __ldg(recs + item / C);
        if (!rec_valid(rc)) continue;
        const int ns = sub_items(rc, p.n_segs);
        for (int j0 = 0; j0 < ns && !stop; j0 += KM, ++rk) {
          const int kp = min(KM, ns - j0);
          // the epilogue has read the previous round's u out of TMEM
          if (aborted(s_abort) || !mbar_wait(bar(UEMPTY), (rk & 1) ^ 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          for (int kx = 0; kx < nkb; ++kx, ++k) {
            if (!full_wait(k)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t st = stage(k);
            if (R == 8) {
              // 8 columns per box, padded to N = 16 with zero columns: one MMA per box
              for (int jm = 0; jm < kp * n_mod; ++jm) {
                const uint32_t ab = st + kBoxBytes + uint32_t(jm * F::kABox);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint64_t ad = smem_desc(st + q * 32, 16, 1024, 2);
                  const uint32_t bstart = ab + q * 16 * (R * 2);
                  const uint64_t bd = smem_desc(bstart, 128, s_zero_s + q * 256 - bstart, 0);
                  umma_f16(tmem + jm * RP, ad, bd, idesc16, (kx | q) != 0 ? 1u : 0u);
                }
              }
            } else {
              // the round's A boxes lie kABox apart, one swizzle atom of R columns each:
              // one MMA with N = kp * n_mod * R reads them as consecutive MN atoms
              const uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kTile, uint32_t(kp * n_mod * R), 0, 1);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint64_t ad = smem_desc(st + q * 32, 16, 1024, 2);
                const uint64_t bd = smem_desc(st + kBoxBytes + q * 16 * (R * 2), F::kABox, 8 * R * 2, F::kALayout);
                umma_f16(tmem, ad, bd, idesc, (kx | q) != 0 ? 1u : 0u);
              }
            }
            issued = true;
            umma_commit(bar(EMPTY + k % NS));  // the stage is free once these MMAs have read it
          }
          if (stop) break;
          umma_commit(bar(UFULL));
          // the epilogue has written this round's u blocks into shared memory
          if (aborted(s_abort) || !mbar_wait(bar(UREADY), rk & 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          tc_fence_after();
          for (int m = 0; m < n_mod && !stop; ++m) {
            for (int b = 0; b < nys; ++b, ++kb, ++dk) {
              const int a = dk % ND;
              if (aborted(s_abort) || !mbar_wait(bar(BFULL + kb % NB), (kb / NB) & 1) ||
                  !mbar_wait(bar(DEMPTY + a), ((dk / ND) & 1) ^ 1)) {
                if (!aborted(s_abort)) fail();
                stop = true;
                break;
              }
              tc_fence_after();
              const uint32_t st = bstage(kb);
              const uint32_t d = tmem + p.d_col + uint32_t(a * 128);
              for (int jj = 0; jj < kp; ++jj) {
                const uint32_t ub = s_u + uint32_t((jj * n_mod + m) * F::kUBlk);
                const uint32_t bb = st + uint32_t(jj * 2 * F::kBBox);
                if (R == 8) {
                  const uint64_t ad = smem_desc(ub, s_zero_u - ub, 128, 0);  // K 8..15 read zeros
                  const uint64_t bd = smem_desc(bb, F::kBBox, s_zero_b - bb, 2);
                  umma_f16(d, ad, bd, idesc_d, jj > 0 ? 1u : 0u);
                } else {
#pragma unroll
                  for (int q = 0; q < R / 16; ++q) {
                    const uint64_t ad = smem_desc(ub + q * 256, 128, uint32_t(R / 8) * 128, 0);
                    const uint64_t bd = smem_desc(bb + q * 2048, F::kBBox, 1024, 2);
                    umma_f16(d, ad, bd, idesc_d, (jj | q) != 0 ? 1u : 0u);
                  }
                }
              }
              issued = true;
              umma_commit(bar(DFULL + a));
            }
          }
          if (!stop) umma_commit(bar(USFREE));  // the u blocks may be rewritten once these MMAs finish
        }
      }
      if (issued && aborted(s_abort)) {  // every issued MMA finishes before TMEM is released (bounded)
        umma_commit(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..)
    // kGroups groups of four warps, one warp per TMEM lane quadrant in each; group g
    // takes every kGroups-th y step (and every kGroups-th u block), so that several
    // steps are drained and reduced into y at once.
    const int eg = (warp - 2) >> 2;
    const int quad = warp & 3;  // the TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    const uint32_t s_mine = s_out + uint32_t((warp - 2) * p.out_bufs * kStageOut);  // this warp's staging boxes
    int nbox = 0;  // reductions this warp has issued
    const bool reporter = row == 0 && eg == 0;
    int rk = 0, dk = 0;
    bool stop = false;
    for (int item = blockIdx.x; item < n_items && !stop; item += gridDim.x) {
      const int4 rc = __ldg(recs + item / C);
      const int ch = item % C;
      if (!rec_valid(rc)) {
        if (reporter && ch == 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
        continue;
      }
      const int ns = sub_items(rc, p.n_segs);
      const int64_t row0 = int64_t(rc.x) * kTile;
      const int64_t r0 = row0 + quad * 32;  // this warp's first row
      const int4 seg0 = first_seg(rc, p.seg_start, p.seg_len, p.seg_slot, p.n_segs);
      for (int j0 = 0; j0 < ns && !stop; j0 += KM, ++rk) {
        const int kp = min(KM, ns - j0);
        int j_row = -1;  // this row's segment within the round
        for (int jj = 0; jj < kp; ++jj) {
          const SubRows sr = rows_of(rc, j0 + jj, seg0, row0, p.n_tokens, p.seg_start, p.seg_len, p.seg_slot,
                                     p.n_segs, p.n_slots, p.status, reporter && ch == 0);
          if (row >= sr.lo && row < sr.hi) j_row = jj;
        }
        // a warp with none of the round's rows adds nothing to y
        const bool warp_rows = __any_sync(0xffffffffu, j_row >= 0) && r0 < p.n_tokens;
        // (1) u, rounded: the row's product in its own segment's blocks, 0 in the others
        bool ok = !aborted(s_abort);
        if (ok && !(mbar_wait(bar(UFULL), rk & 1) && mbar_wait(bar(USFREE), (rk & 1) ^ 1))) {
          fail();
          ok = false;
        }
        if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: tcgen05.ld is collective
          stop = true;
          break;
        }
        tc_fence_after();
        for (int q = eg; q < kp * n_mod; q += kGroups) {
          const int jj = q / n_mod;
          const bool in = j_row == jj;
          uint8_t* blk = gbase + (s_u - base) + q * F::kUBlk;
#pragma unroll
          for (int c = 0; c < RP / 16; ++c) {
            float v[16];
            tmem_ld16(tmem + lane_base + uint32_t(q * RP + c * 16), v);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (c * 16 + h * 8 < R) {
                uint4 pk;
                pk.x = Pack2<T>::pack(in ? v[h * 8 + 0] : 0.f, in ? v[h * 8 + 1] : 0.f);
                pk.y = Pack2<T>::pack(in ? v[h * 8 + 2] : 0.f, in ? v[h * 8 + 3] : 0.f);
                pk.z = Pack2<T>::pack(in ? v[h * 8 + 4] : 0.f, in ? v[h * 8 + 5] : 0.f);
                pk.w = Pack2<T>::pack(in ? v[h * 8 + 6] : 0.f, in ? v[h * 8 + 7] : 0.f);
                // 8-element chunk q of row r sits in core matrix (r / 8, q)
                *reinterpret_cast<uint4*>(blk + ((row >> 3) * (R / 8) + c * 2 + h) * 128 + (row & 7) * 16) = pk;
              }
            }
          }
        }
        tc_fence_before();
        fence_proxy_async_smem();  // the u blocks are read by the MMA (async proxy)
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(UEMPTY));
          mbar_arrive(bar(UREADY));
        }
        // (2) the delta, one 128-column step of y at a time, the steps dealt round-robin
        for (int m = 0; m < n_mod && !stop; ++m) {
          for (int b = 0; b < nys; ++b, ++dk) {
            if (dk % kGroups != eg) continue;
            const int a = dk % ND;
            bool ok2 = !aborted(s_abort);
            if (ok2 && !mbar_wait(bar(DFULL + a), (dk / ND) & 1)) {
              fail();
              ok2 = false;
            }
            if (!__all_sync(0xffffffffu, ok2)) {
              stop = true;
              break;
            }
            tc_fence_after();
            // the step's MMAs are done: its B stage (ring position = step index) is free
            if (lane == 0) mbar_arrive(bar(BEMPTY + dk % NB));
            for (int h = 0; h < 2; ++h) {  // the step's two 64-column halves
              uint32_t acc[64];
              tmem_ld64(tmem + lane_base + p.d_col + uint32_t(a * 128 + h * 64), acc);
              if (h == 1) {  // both halves are in registers: the accumulator is free
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(DEMPTY + a));
              }
              if (!warp_rows) continue;
              const uint32_t sbox = s_mine + uint32_t((nbox % p.out_bufs) * kStageOut);
              uint8_t* my_line = gbase + (sbox - base) + lane * 128;  // this row in the SW128 staging box
              // with two staging boxes two reductions are in flight per warp: the one issued
              // two boxes ago has read this box; with one, the previous one has
              if (lane == 0) {
                if (p.out_bufs == 2)
                  tma_store_wait_read_le1();
                else
                  tma_store_wait_read_all();
              }
              __syncwarp();
              // round(delta) for the round's rows, -0 for the others (y + -0 is y).  The box
              // is SW128: chunk c of row r sits at 16 * (c ^ (r % 8)) in its 128-byte line.
              const bool in = j_row >= 0;
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                uint4 pk = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
                if (in) {
                  pk.x = Pack2<T>::pack(__uint_as_float(acc[c * 8 + 0]), __uint_as_float(acc[c * 8 + 1]));
                  pk.y = Pack2<T>::pack(__uint_as_float(acc[c * 8 + 2]), __uint_as_float(acc[c * 8 + 3]));
                  pk.z = Pack2<T>::pack(__uint_as_float(acc[c * 8 + 4]), __uint_as_float(acc[c * 8 + 5]));
                  pk.w = Pack2<T>::pack(__uint_as_float(acc[c * 8 + 6]), __uint_as_float(acc[c * 8 + 7]));
                }
                *reinterpret_cast<uint4*>(my_line + ((c ^ (lane & 7)) << 4)) = pk;
              }
              fence_proxy_async_smem();  // the rows are read by the TMA reduction (async proxy)
              __syncwarp();
              if (lane == 0) {
                // rows past the end of the tokens are clipped
                tma_reduce_add_2d(&p.ys_map, sbox,
                                  int32_t(p.y_col_off[m]) + ch * p.chunk_cols + b * 128 + h * 64, int32_t(r0));
                tma_store_commit();
              }
              ++nbox;
            }
          }
        }
      }
    }
    if (lane == 0) tma_store_wait_all();  // every reduction has completed
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, p.tmem_alloc);
  }
}

// ------------------------------------------------------------------ launcher
namespace {

template <typename T, int R>
int launch_fused(FusedApplyParams& p, cudaStream_t stream) {
  using F = FusedOps<R>;
  constexpr int RP = F::RP;
  // Sizes, in order of preference: two segments per round (u for all of them, kmax *
  // n_modules * RP TMEM columns, and at least two 128-column delta accumulators fit in
  // TMEM), the deepest B ring, two staging boxes per epilogue warp, with at least 4 x
  // stages (4 stages of 16 KB per SM already stream x at the full HBM rate).  Where
  // nothing gives 4 (three or four modules of rank 64) the call takes the two launches:
  // sizes with 2 x stages and 2 B stages timed out in a test (the status word reported
  // it; the cause was not found), so they are not used.
  int chosen = 0, stages = 0, sb = 0, fixed = 0, bufs = 0, nbs = 0;
  for (int pass = 0; pass < 1 && chosen == 0; ++pass) {
    const int need = 4;
    for (int km = 2; km >= 1 && chosen == 0; --km) {
      if (km * p.n_modules * RP > 256) continue;
      for (int nb : {16, 12, 8, 6, 4, 2}) {
        for (int ob = 2; ob >= 1; --ob) {
          sb = kBoxBytes + km * p.n_modules * F::kABox;
          fixed = kFixedBytes + F::kZeroBytes + km * p.n_modules * F::kUBlk + kEpiWarps * ob * kStageOut +
                  nb * km * 2 * F::kBBox;
          const int st = (kSmemMax - fixed) / sb;
          if (st >= need) {
            chosen = km;
            bufs = ob;
            nbs = nb;
            stages = st > 12 ? 12 : st;
            break;
          }
        }
        if (chosen) break;
      }
    }
  }
  if (chosen == 0)
    return set_error(LF_ERR_UNSUPPORTED, "fused LoRA: %d modules of rank %d do not fit", p.n_modules, R);
  p.kmax = chosen;
  p.out_bufs = bufs;
  p.stages = stages;
  p.stage_bytes = sb;
  p.b_stages = nbs;
  p.b_stage_bytes = chosen * 2 * F::kBBox;
  p.u_cols = uint32_t(chosen * p.n_modules * RP);
  p.d_col = (p.u_cols + 63u) & ~63u;
  p.d_bufs = int((512u - p.d_col) / 128u);  // 2 or 3 (u takes at most 256 columns)
  if (p.d_bufs > kMaxDBufs) p.d_bufs = kMaxDBufs;
  p.tmem_alloc = 512;
  // one CTA per SM: the request stays above half of the SM's shared memory, so a
  // second CTA of this kernel can never wait on TMEM the first one holds
  size_t smem = size_t(fixed) + size_t(stages) * size_t(sb);
  if (smem < 120 * 1024) smem = 120 * 1024;
  auto kern = lora_fused_kernel<T, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(lora_fused)");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = int64_t(p.n_tiles) * p.n_chunks;
  const int grid = int(items < sms ? items : sms);
  if (grid == 0) return LF_OK;
  e = launch_pdl(kern, dim3(unsigned(grid)), dim3(kFusedThreads), smem, stream, p);
  if (e != cudaSuccess) return cuda_error(e, "launch lora_fused");
  count_launch();
  return LF_OK;
}

template <typename T>
int fused_rank(FusedApplyParams& p, int rank, cudaStream_t s) {
  switch (rank) {
    case 8: return launch_fused<T, 8>(p, s);
    case 16: return launch_fused<T, 16>(p, s);
    case 32: return launch_fused<T, 32>(p, s);
    case 64: return launch_fused<T, 64>(p, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "fused LoRA: rank %d", rank);
}

}  // namespace

int run_lora_fused(int dtype, FusedApplyParams& p, int rank, cudaStream_t s) {
  if (dtype == LF_DTYPE_BF16) return fused_rank<__nv_bfloat16>(p, rank, s);
  if (dtype == LF_DTYPE_F16) return fused_rank<__half>(p, rank, s);
  return set_error(LF_ERR_UNSUPPORTED, "fused LoRA: dtype %d", dtype);
}

}  // namespace lf
