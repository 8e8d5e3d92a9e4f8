// tcgen05 (5th-generation tensor core) LoRA kernels for bf16 / f16.
//
// Shrink  u[m][t] = x[t] . A(slot(t), m)          (M=128 tokens x N=rank per MMA)
// Expand  y[t, off_m + n] (+)= u[m][t] . B(slot(t), m)   (M=128 tokens x N=128..256 cols)
//
// Both are HBM-streaming kernels: the big operands (x tiles for the shrink, y
// tiles for the expand) move by TMA with 128-byte swizzle straight into the
// canonical UMMA shared-memory layout; the per-tenant factors A and B are read
// in place from the slot cache by TMA (MN-major operands, so the cache keeps
// the reference's (hidden x rank) / (rank x hidden) layouts); accumulators
// live in TMEM.  The shrink splits the hidden (K) dimension over a thread-block
// cluster and reduces the fp32 partials through distributed shared memory in a
// fixed order, so results are deterministic.
//
// Tiles of 128 tokens are "segmented": a tile may hold rows of several
// adapter slots (short or packed sequences).  The MMA is issued once per slot
// present and each row keeps only its own slot's result, so any segment
// layout is handled; the padded (B, S) serving layout with S % 128 == 0 has
// exactly one segment per tile.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

constexpr int kTileM = 128;     // tokens per tile (MMA M)
constexpr int kKBlock = 64;     // hidden elements per 128-byte swizzled K block
constexpr int kMaxSegPerTile = kTileM;

// ---------------------------------------------------------------------------
// Segment list of one 128-token tile, computed by one thread into smem.
// ---------------------------------------------------------------------------
struct TileSegs {
  int32_t n;
  int32_t slot[kMaxSegPerTile];
  int16_t lo[kMaxSegPerTile];
  int16_t hi[kMaxSegPerTile];
};

// Where a CTA's 128-token tile starts, and (with a caller-built tile record)
// which segments overlap it and the slot of the first one, so that every load
// of the tile can be issued after a single 16-byte read.
struct TileInfo {
  int64_t row0;
  int32_t first;  // first overlapping segment (record path), -1 otherwise
  int32_t count;  // number of overlapping segments (record path)
  int32_t slot0;  // slot of the first overlapping segment (record path)
};

__device__ __forceinline__ TileInfo load_tile_info(const int32_t* __restrict__ tiles) {
  if (tiles != nullptr) {
    const int4 r = __ldg(reinterpret_cast<const int4*>(tiles) + blockIdx.y);
    return {int64_t(r.x) * kTileM, r.y, r.z, r.w};
  }
  return {int64_t(blockIdx.y) * kTileM, -1, 0, -1};
}

__device__ __forceinline__ void add_segment(TileSegs* ts, int& cnt, int64_t s, int64_t l, int32_t slot,
                                            int64_t row0, int64_t row_end, int64_t n_tokens, int n_slots,
                                            int32_t* status) {
  if (l <= 0) {
    if (l < 0) set_status(status, LF_STATUS_BAD_SEGMENT);
    return;
  }
  if (s < 0 || s + l > n_tokens) set_status(status, LF_STATUS_BAD_SEGMENT);
  const int64_t lo = max(s, row0), hi = min(s + l, row_end);
  if (lo >= hi) return;
  if (slot < 0 || slot >= n_slots) {
    set_status(status, LF_STATUS_BAD_SLOT);
    return;
  }
  if (cnt < kMaxSegPerTile) {
    ts->slot[cnt] = slot;
    ts->lo[cnt] = static_cast<int16_t>(lo - row0);
    ts->hi[cnt] = static_cast<int16_t>(hi - row0);
    ++cnt;
  }
}

// Segments overlapping the tile, into smem.  With a tile record the overlapping
// segments are named directly (their loads issue together); without one, a
// binary search over the sorted segment starts finds the first.
__device__ void build_tile_segments(TileSegs* ts, const TileInfo& ti, int64_t n_tokens,
                                    const int32_t* __restrict__ seg_start,
                                    const int32_t* __restrict__ seg_len,
                                    const int32_t* __restrict__ seg_slot, int n_segs, int n_slots,
                                    int32_t* status) {
  const int64_t row0 = ti.row0;
  const int64_t row_end = min(row0 + kTileM, n_tokens);
  int cnt = 0;
  if (ti.first >= 0) {
    if (ti.count < 0 || int64_t(ti.first) + ti.count > n_segs) {
      set_status(status, LF_STATUS_BAD_SEGMENT);
      ts->n = 0;
      return;
    }
    for (int g = ti.first; g < ti.first + ti.count; ++g)
      add_segment(ts, cnt, seg_start[g], seg_len[g], seg_slot[g], row0, row_end, n_tokens, n_slots, status);
  } else {
    for (int g = first_seg_ending_after(seg_start, seg_len, n_segs, row0); g < n_segs; ++g) {
      const int64_t st = seg_start[g];
      if (st >= row_end) break;
      add_segment(ts, cnt, st, seg_len[g], seg_slot[g], row0, row_end, n_tokens, n_slots, status);
    }
  }
  ts->n = cnt;
}

// Layout constants of the MN-major operand holding `rows` x R elements where
// R is the contiguous (MN) dimension: 16 B (R=8, no swizzle) .. 128 B (R=64, SW128).
template <int R>
struct MnOperand {
  static constexpr int kRowBytes = R * 2;
  static constexpr uint32_t kLayout = (R == 8) ? 0u : (R == 16) ? 6u : (R == 32) ? 4u : 2u;
  static constexpr CUtensorMapSwizzle kTmaSwizzle =
      (R == 8)    ? CU_TENSOR_MAP_SWIZZLE_NONE
      : (R == 16) ? CU_TENSOR_MAP_SWIZZLE_32B
      : (R == 32) ? CU_TENSOR_MAP_SWIZZLE_64B
                  : CU_TENSOR_MAP_SWIZZLE_128B;
  // byte stride between 8-row K groups (the swizzle atom height is 8 rows)
  static constexpr uint32_t kSbo = 8 * kRowBytes;
};

// ===========================================================================
// Shrink
// ===========================================================================
template <typename T, int R>
struct ShrinkTc {
  static constexpr int kRPad = R < 16 ? 16 : R;
  static constexpr int kABox = kKBlock * R * 2;  // one (64 x R) A box
  static constexpr int kXBox = kTileM * kKBlock * 2;  // one (128 x 64) X box = 16 KB

  static size_t smem_bytes(int kchunk, int n_mod) {
    const int nkb = kchunk / kKBlock;
    size_t b = 1024;  // alignment slack
    b += size_t(nkb) * kXBox;
    b += size_t(n_mod) * nkb * kABox;
    b += (R == 8) ? 1024 : 0;
    b += size_t(kTileM) * n_mod * kRPad * 4;  // fp32 partials
    b += sizeof(TileSegs) + 64;
    return b;
  }
};

template <typename T, int R>
__global__ void __launch_bounds__(128, 1)
lora_shrink_tc_kernel(const __grid_constant__ ShrinkTcParams p) {
  using S = ShrinkTc<T, R>;
  constexpr int RP = S::kRPad;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int csize = gridDim.x;                 // cluster size (split-K factor)
  const int crank = blockIdx.x;                // == %cluster_ctarank for cluster dims (csize,1,1)
  const int kchunk = p.kchunk;
  const int nkb = kchunk / kKBlock;
  const int k0 = crank * kchunk;
  const int n_mod = p.n_modules;

  // ---- carve shared memory ----
  uint32_t off = 0;
  const uint32_t s_x = base + off;            off += nkb * S::kXBox;
  const uint32_t s_a = base + off;            off += n_mod * nkb * S::kABox;
  const uint32_t s_z = base + off;            off += (R == 8) ? 1024 : 0;
  float* s_part = reinterpret_cast<float*>(gbase + off);
  const uint32_t s_part_u32 = base + off;     off += kTileM * n_mod * RP * 4;
  TileSegs* segs = reinterpret_cast<TileSegs*>(gbase + off);
  off += (sizeof(TileSegs) + 15) & ~15;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + off);  // [0]=x, [1]=a, [2]=mma
  const uint32_t bar_x = smem_u32(&bars[0]), bar_a = smem_u32(&bars[1]), bar_mma = smem_u32(&bars[2]);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[3]);

  const uint32_t tmem_cols = p.tmem_cols;
  bool ok = true;
  int32_t* s_pref = reinterpret_cast<int32_t*>(&bars[4]);  // 1 if the first A was prefetched
  const TileInfo ti = load_tile_info(p.tiles);
  const int64_t row0 = ti.row0;

  auto issue_a = [&](int32_t slot) {
    mbar_arrive_expect_tx(bar_a, n_mod * nkb * S::kABox);
    for (int m = 0; m < n_mod; ++m)
      for (int kb = 0; kb < nkb; ++kb)
        tma_load_3d(s_a + (m * nkb + kb) * S::kABox, &p.a_map[m], bar_a, 0, k0 + kb * kKBlock, slot);
  };

  if (tid == 0) {
    mbar_init(bar_x, 1);
    mbar_init(bar_a, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    // x chunk: rows [row0, row0+128) x cols [k0, k0+kchunk); rows past n_tokens read as 0
    mbar_arrive_expect_tx(bar_x, nkb * S::kXBox);
    for (int kb = 0; kb < nkb; ++kb)
      tma_load_2d(s_x + kb * S::kXBox, &p.x_map, bar_x, k0 + kb * kKBlock, int32_t(row0));
    // the record names the first segment's slot: start its A factor now
    const bool pref = ti.first >= 0 && ti.count > 0 && ti.slot0 >= 0 && ti.slot0 < p.n_slots;
    if (pref) issue_a(ti.slot0);
    build_tile_segments(segs, ti, p.n_tokens, p.seg_start, p.seg_len, p.seg_slot, p.n_segs,
                        p.n_slots, p.status);
    if (pref && (segs->n == 0 || segs->slot[0] != ti.slot0)) {
      // the record disagrees with the segment table: no delta for this tile
      if (segs->n != 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
      segs->n = 0;
    }
    *s_pref = pref ? 1 : 0;
  }
  // zero the fp32 partials (rows in no segment contribute 0) and the R=8 pad
  for (int i = tid; i < kTileM * n_mod * RP; i += blockDim.x) s_part[i] = 0.f;
  if (R == 8) {
    uint4* z = reinterpret_cast<uint4*>(gbase + (s_z - base));
    for (int i = tid; i < 1024 / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), tmem_cols);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  const int nseg = segs->n;
  const bool prefetched = *s_pref != 0;

  constexpr uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kTileM, RP, /*a_mn=*/0, /*b_mn=*/1);
  using A = MnOperand<R>;

  for (int g = 0; g < nseg; ++g) {
    if (tid == 0) {
      if (g > 0 || !prefetched) issue_a(segs->slot[g]);
      bool w = mbar_wait(bar_a, g & 1);
      if (g == 0) w = w && mbar_wait(bar_x, 0);
      if (!w) {
        set_status(p.status, LF_STATUS_TIMEOUT);
        ok = false;
      }
      tc_fence_after();
      if (ok) {
        for (int m = 0; m < n_mod; ++m) {
          for (int kb = 0; kb < nkb; ++kb) {
            const uint32_t xb = s_x + kb * S::kXBox;
            const uint32_t ab = s_a + (m * nkb + kb) * S::kABox;
#pragma unroll
            for (int k = 0; k < kKBlock / 16; ++k) {
              // A operand: x box, K-major SW128; a K step of 16 elements is +32 bytes.
              const uint64_t ad = smem_desc(xb + k * 32, 16, 1024, 2);
              // B operand: A factor box (64 K rows x R), MN-major; a K step is 16 rows.
              const uint32_t bstart = ab + k * 16 * A::kRowBytes;
              uint64_t bd;
              if (R == 8) {
                // no swizzle: K groups (8 rows x 16 B) at LBO = 128; the padded
                // MN group (columns 8..15) reads the zero block.
                bd = smem_desc(bstart, 128, s_z + k * 256 - bstart, 0);
              } else {
                bd = smem_desc(bstart, A::kSbo, A::kSbo, A::kLayout);
              }
              umma_f16(taddr + m * RP, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
        }
      }
      umma_commit(bar_mma);
    }
    __syncthreads();  // ok flag of thread 0 is only advisory for the others
    if (!mbar_wait(bar_mma, g & 1)) {
      set_status(p.status, LF_STATUS_TIMEOUT);
      ok = false;
    }
    tc_fence_after();
    __syncwarp();
    // Each warp reads its 32 TMEM lanes (= tile rows); rows of this segment keep the values.
    const int row = warp * 32 + lane;
    const bool mine = row >= segs->lo[g] && row < segs->hi[g];
    for (int m = 0; m < n_mod; ++m) {
#pragma unroll
      for (int c = 0; c < RP / 16; ++c) {
        float v[16];
        tmem_ld16(taddr + (uint32_t(warp * 32) << 16) + m * RP + c * 16, v);
        if (mine) {
          float* dst = s_part + (row * n_mod + m) * RP + c * 16;
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[i] = v[i];
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }

  if (nseg == 0 && tid == 0) {
    // loads that nothing consumed must land before the CTA exits
    if (!mbar_wait(bar_x, 0)) set_status(p.status, LF_STATUS_TIMEOUT);
    if (prefetched && !mbar_wait(bar_a, 0)) set_status(p.status, LF_STATUS_TIMEOUT);
  }
  __syncthreads();

  // ---- split-K reduction over the cluster, fixed order -> deterministic ----
  if (csize > 1) cluster_sync();
  {
    const int rows_per = kTileM / csize;
    const int r_begin = crank * rows_per;
    const int w4 = n_mod * RP / 4;  // float4 per row
    for (int it = tid; it < rows_per * w4; it += blockDim.x) {
      const int row = r_begin + it / w4;
      const int q = it % w4;
      const uint32_t local = s_part_u32 + uint32_t((row * n_mod * RP + q * 4) * 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < csize; ++c) {
        float4 v;
        if (csize == 1) v = *reinterpret_cast<const float4*>(gbase + (local - base));
        else v = ld_dsmem_f4(mapa_shared(local, uint32_t(c)));
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      const int64_t t = row0 + row;
      const int m = (q * 4) / RP;
      const int j = (q * 4) % RP;
      if (t < p.n_tokens && j < R && ok) {
        T* dst = reinterpret_cast<T*>(p.u) + (int64_t(m) * p.n_tokens + t) * R + j;
        dst[0] = DT<T>::from_f(acc.x);
        dst[1] = DT<T>::from_f(acc.y);
        dst[2] = DT<T>::from_f(acc.z);
        dst[3] = DT<T>::from_f(acc.w);
      }
    }
  }
  if (csize > 1) cluster_sync();  // peers may still read this CTA's partials until here

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(taddr, tmem_cols);
  }
}

// ===========================================================================
// Expand (+ add into y)
// ===========================================================================
template <typename T, int R, int NT>
struct ExpandTc {
  static constexpr int kRPad = R < 16 ? 16 : R;
  static constexpr int kYBox = kTileM * 64 * 2;      // 16 KB
  static constexpr int kBBox = R * 64 * 2;           // (R rows x 64 cols)
  static constexpr int kNBox = NT / 64;
  static constexpr int kUBytes = kTileM * kRPad * 2;
  static constexpr int kZBytes = (R == 8) ? kNBox * 1024 : 0;

  static size_t smem_bytes() {
    size_t b = 1024;
    b += size_t(kNBox) * kYBox;
    b += size_t(kNBox) * kBBox + kZBytes;
    b += kUBytes;
    b += sizeof(TileSegs) + 64;
    return b;
  }
};

template <typename T, int R, int NT>
__global__ void __launch_bounds__(128, 1)
lora_expand_tc_kernel(const __grid_constant__ ExpandTcParams p) {
  using E = ExpandTc<T, R, NT>;
  constexpr int RP = E::kRPad;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ct = blockIdx.x;
  const TileInfo ti = load_tile_info(p.tiles);  // every thread: row0 is needed for the U loads
  const int64_t row0 = ti.row0;
  const int m = blockIdx.z;
  const int32_t col0 = int32_t(p.y_col_off[m] + int64_t(ct) * NT);
  const bool acc_y = p.accumulate != 0;

  uint32_t off = 0;
  const uint32_t s_y = base + off;  off += E::kNBox * E::kYBox;
  const uint32_t s_b = base + off;  off += E::kNBox * E::kBBox;
  const uint32_t s_z = base + off;  off += E::kZBytes;
  const uint32_t s_u = base + off;  off += E::kUBytes;
  TileSegs* segs = reinterpret_cast<TileSegs*>(gbase + off);
  off += (sizeof(TileSegs) + 15) & ~15;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + off);  // [0]=y, [1]=b, [2]=mma
  const uint32_t bar_y = smem_u32(&bars[0]), bar_b = smem_u32(&bars[1]), bar_mma = smem_u32(&bars[2]);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[3]);
  int32_t* s_fail = reinterpret_cast<int32_t*>(&bars[4]);
  int32_t* s_pref = reinterpret_cast<int32_t*>(&bars[4]) + 1;  // 1 if the first B was prefetched

  auto issue_b = [&](int32_t slot) {
    mbar_arrive_expect_tx(bar_b, E::kNBox * E::kBBox);
    for (int j = 0; j < E::kNBox; ++j)
      tma_load_3d(s_b + j * E::kBBox, &p.b_map[m], bar_b, ct * NT + j * 64, 0, slot);
  };

  if (tid == 0) {
    *s_fail = 0;
    mbar_init(bar_y, 1);
    mbar_init(bar_b, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    if (acc_y) {
      // the y tile does not depend on anything: start streaming it first
      mbar_arrive_expect_tx(bar_y, E::kNBox * E::kYBox);
      for (int j = 0; j < E::kNBox; ++j)
        tma_load_2d(s_y + j * E::kYBox, &p.y_map, bar_y, col0 + j * 64, int32_t(row0));
    }
    // the record names the first segment's slot: start its B factor now
    const bool pref = ti.first >= 0 && ti.count > 0 && ti.slot0 >= 0 && ti.slot0 < p.n_slots;
    if (pref) issue_b(ti.slot0);
    build_tile_segments(segs, ti, p.n_tokens, p.seg_start, p.seg_len, p.seg_slot, p.n_segs,
                        p.n_slots, p.status);
    if (pref && (segs->n == 0 || segs->slot[0] != ti.slot0)) {
      // the record disagrees with the segment table: no delta for this tile
      if (segs->n != 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
      segs->n = 0;
    }
    *s_pref = pref ? 1 : 0;
  }
  // This thread's U row, read now (in parallel with the y / B loads).  Every row
  // of a launched tile was written by the shrink (0 for rows in no segment).
  const int row = warp * 32 + lane;     // this thread's tile row (U operand and epilogue)
  const int64_t t = row0 + row;
  uint4 u_reg[RP / 8];
  {
    const T* __restrict__ u_row = reinterpret_cast<const T*>(p.u) + (int64_t(m) * p.n_tokens + t) * R;
#pragma unroll
    for (int kc = 0; kc < RP / 8; ++kc)
      u_reg[kc] = (t < p.n_tokens && kc * 8 < R) ? *reinterpret_cast<const uint4*>(u_row + kc * 8)
                                                 : make_uint4(0, 0, 0, 0);
  }
  if (R == 8) {
    uint4* z = reinterpret_cast<uint4*>(gbase + (s_z - base));
    for (int i = tid; i < E::kZBytes / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), NT);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  const int nseg = segs->n;
  const bool prefetched = *s_pref != 0;

  constexpr uint32_t idesc = umma_idesc_f16(DT<T>::umma_fmt, kTileM, NT, /*a_mn=*/0, /*b_mn=*/1);

  for (int g = 0; g < nseg; ++g) {
    if (g > 0) {
      // the previous MMA must have finished reading the U and B buffers
      if (!mbar_wait(bar_mma, (g - 1) & 1)) atomicOr(s_fail, 1);
    }
    if (tid == 0 && (g > 0 || !prefetched)) issue_b(segs->slot[g]);
    // U operand, K-major without swizzle: core matrices of 8 rows x 16 bytes;
    // K chunks (8 elements) are LBO = 128 B apart, 8-row groups SBO = RP*16 B apart.
    {
      const bool mine = row >= segs->lo[g] && row < segs->hi[g];
      uint8_t* ub = gbase + (s_u - base) + (row >> 3) * (RP * 16) + (row & 7) * 16;
#pragma unroll
      for (int kc = 0; kc < RP / 8; ++kc)
        *reinterpret_cast<uint4*>(ub + kc * 128) = mine ? u_reg[kc] : make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      if (!mbar_wait(bar_b, g & 1)) atomicOr(s_fail, 1);
      tc_fence_after();
      if (*s_fail == 0) {
#pragma unroll
        for (int k = 0; k < RP / 16; ++k) {
          const uint64_t ad = smem_desc(s_u + k * 256, 128, RP * 16, 0);
          uint64_t bd;
          if (R == 8) {
            // B: one 8-row K group per 64-col box; the second K group (rows 8..15) is zeros
            bd = smem_desc(s_b, E::kBBox, s_z - s_b, 2);
          } else {
            // B: MN-major SW128, 64-col boxes LBO = kBBox apart, 8-row K groups SBO = 1024 apart
            bd = smem_desc(s_b + k * 2048, E::kBBox, 1024, 2);
          }
          umma_f16(taddr, ad, bd, idesc, (g > 0 || k > 0) ? 1u : 0u);
        }
      }
      umma_commit(bar_mma);
    }
  }

  if (nseg > 0) {
    if (!mbar_wait(bar_mma, (nseg - 1) & 1)) atomicOr(s_fail, 1);
  }
  if (acc_y) {
    if (!mbar_wait(bar_y, 0)) atomicOr(s_fail, 1);
  }
  __syncthreads();
  const bool failed = *s_fail != 0;
  if (failed && tid == 0) {
    set_status(p.status, LF_STATUS_TIMEOUT);
    // give copies still in flight one more bounded chance to land before teardown
    if (nseg > 0) mbar_wait(bar_mma, (nseg - 1) & 1);
    if (acc_y) mbar_wait(bar_y, 0);
  }
  if (nseg == 0 && prefetched && tid == 0) {
    // a prefetched B that no MMA consumed must land before the CTA exits
    if (!mbar_wait(bar_b, 0)) set_status(p.status, LF_STATUS_TIMEOUT);
  }
  tc_fence_after();
  __syncwarp();

  // A tile with no segment leaves y unchanged when accumulating: skip the store.
  const bool store = !failed && (nseg > 0 || !acc_y);
  if (store) {
    // epilogue: row `row`, 32 columns at a time; y tile is SW128 (128 rows x 64 cols per box)
    for (int q = 0; q < NT / 32; ++q) {
      float v[32];
      if (nseg > 0) {
        float a[16], b[16];
        tmem_ld16(taddr + (uint32_t(warp * 32) << 16) + q * 32, a);
        tmem_ld16(taddr + (uint32_t(warp * 32) << 16) + q * 32 + 16, b);
#pragma unroll
        for (int i = 0; i < 16; ++i) { v[i] = a[i]; v[16 + i] = b[i]; }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      uint8_t* yb = gbase + (s_y - base) + (q >> 1) * E::kYBox + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        const int chunk = (q & 1) * 4 + c4;
        uint4* ptr = reinterpret_cast<uint4*>(yb + ((chunk ^ (row & 7)) << 4));
        uint4 raw16 = acc_y ? *ptr : make_uint4(0, 0, 0, 0);
        T* e = reinterpret_cast<T*>(&raw16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = round_through<T>(v[c4 * 8 + i]);
          e[i] = acc_y ? DT<T>::from_f(DT<T>::to_f(e[i]) + d) : DT<T>::from_f(d);
        }
        *ptr = raw16;
      }
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (tid == 0 && store) {
    for (int j = 0; j < E::kNBox; ++j)
      tma_store_2d(&p.y_map, s_y + j * E::kYBox, col0 + j * 64, int32_t(row0));
    tma_store_commit();
    tma_store_wait_read_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(taddr, NT);
  }
}

// ===========================================================================
// host-side launchers
// ===========================================================================
static uint32_t pow2_cols(int n) {
  uint32_t c = 32;
  while (c < uint32_t(n)) c <<= 1;
  return c;
}

// Smallest dynamic smem request that keeps at most `cap` CTAs on one SM, so the
// CTAs resident on an SM never ask for more than its 512 TMEM columns.
static size_t occupancy_capped_smem(size_t need, int cap) {
  const size_t per_sm = 233472;  // 228 KB shared memory per SM
  const size_t reserve = 1024;   // per-CTA system reservation
  const size_t floor_bytes = per_sm / size_t(cap + 1) + 1 - reserve;
  return need > floor_bytes ? need : floor_bytes;
}

template <typename T, int R>
static int launch_shrink_tc(const ShrinkTcParams& p, int csize, int n_tiles, cudaStream_t stream) {
  const size_t need = ShrinkTc<T, R>::smem_bytes(p.kchunk, p.n_modules);
  const int cap = 512 / int(p.tmem_cols);
  const size_t smem = occupancy_capped_smem(need, cap);
  if (smem > 232448) return set_error(LF_ERR_UNSUPPORTED, "shrink tile needs %zu B of shared memory", smem);
  auto kern = lora_shrink_tc_kernel<T, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(shrink)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(csize, unsigned(n_tiles), 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return cuda_error(e, "launch lora_shrink_tc");
  count_launch();
  return LF_OK;
}

template <typename T, int R, int NT>
static int launch_expand_tc(const ExpandTcParams& p, cudaStream_t stream) {
  const size_t need = ExpandTc<T, R, NT>::smem_bytes();
  const size_t smem = occupancy_capped_smem(need, 512 / NT);
  auto kern = lora_expand_tc_kernel<T, R, NT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(expand)");
  dim3 grid(unsigned(p.hidden / NT), unsigned(p.n_tiles), unsigned(p.n_modules));
  kern<<<grid, 128, smem, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "launch lora_expand_tc");
  count_launch();
  return LF_OK;
}

size_t shrink_tc_smem(int dtype, int rank, int kchunk, int n_mod) {
  (void)dtype;
  switch (rank) {
    case 8: return ShrinkTc<__nv_bfloat16, 8>::smem_bytes(kchunk, n_mod);
    case 16: return ShrinkTc<__nv_bfloat16, 16>::smem_bytes(kchunk, n_mod);
    case 32: return ShrinkTc<__nv_bfloat16, 32>::smem_bytes(kchunk, n_mod);
    default: return ShrinkTc<__nv_bfloat16, 64>::smem_bytes(kchunk, n_mod);
  }
}

uint32_t shrink_tc_tmem_cols(int rank, int n_mod) {
  const int rp = rank < 16 ? 16 : rank;
  return pow2_cols(rp * n_mod);
}

CUtensorMapSwizzle a_tma_swizzle(int rank) {
  switch (rank) {
    case 8: return MnOperand<8>::kTmaSwizzle;
    case 16: return MnOperand<16>::kTmaSwizzle;
    case 32: return MnOperand<32>::kTmaSwizzle;
    default: return MnOperand<64>::kTmaSwizzle;
  }
}

template <typename T>
static int dispatch_shrink_rank(const ShrinkTcParams& p, int rank, int csize, int n_tiles, cudaStream_t s) {
  switch (rank) {
    case 8: return launch_shrink_tc<T, 8>(p, csize, n_tiles, s);
    case 16: return launch_shrink_tc<T, 16>(p, csize, n_tiles, s);
    case 32: return launch_shrink_tc<T, 32>(p, csize, n_tiles, s);
    case 64: return launch_shrink_tc<T, 64>(p, csize, n_tiles, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "tcgen05 shrink: rank %d", rank);
}

int run_shrink_tc(int dtype, const ShrinkTcParams& p, int rank, int csize, int n_tiles, cudaStream_t s) {
  if (dtype == LF_DTYPE_BF16) return dispatch_shrink_rank<__nv_bfloat16>(p, rank, csize, n_tiles, s);
  return dispatch_shrink_rank<__half>(p, rank, csize, n_tiles, s);
}

template <typename T, int R>
static int dispatch_expand_nt(const ExpandTcParams& p, int nt, cudaStream_t s) {
  switch (nt) {
    case 64: return launch_expand_tc<T, R, 64>(p, s);
    case 128: return launch_expand_tc<T, R, 128>(p, s);
    case 256: return launch_expand_tc<T, R, 256>(p, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "tcgen05 expand: column tile %d", nt);
}

template <typename T>
static int dispatch_expand_rank(const ExpandTcParams& p, int rank, int nt, cudaStream_t s) {
  switch (rank) {
    case 8: return dispatch_expand_nt<T, 8>(p, nt, s);
    case 16: return dispatch_expand_nt<T, 16>(p, nt, s);
    case 32: return dispatch_expand_nt<T, 32>(p, nt, s);
    case 64: return dispatch_expand_nt<T, 64>(p, nt, s);
  }
  return set_error(LF_ERR_UNSUPPORTED, "tcgen05 expand: rank %d", rank);
}

int run_expand_tc(int dtype, const ExpandTcParams& p, int rank, int nt, cudaStream_t s) {
  if (dtype == LF_DTYPE_BF16) return dispatch_expand_rank<__nv_bfloat16>(p, rank, nt, s);
  return dispatch_expand_rank<__half>(p, rank, nt, s);
}

}  // namespace lf
