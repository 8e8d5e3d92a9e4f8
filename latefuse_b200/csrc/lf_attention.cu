// Variable-length self-attention of packed sequences, head_dim 64, on tcgen05.
//
// Replaces the encoder's masked attention (src/latefuse/model/encoder.py:82-98:
// scores = q k^T * scale, padded keys masked, softmax in f32, probs @ v) for a
// batch whose padding has been removed: every sequence attends to itself only.
//
// Work unit = (query tile of 128 rows of one sequence, head).  One persistent
// CTA per SM takes every gridDim-th unit and splits them over two softmax
// groups that run in ping-pong, so that one group's exponentials overlap the
// other group's row-max phase and the tensor core works for both:
//   warp 0      producer: each group's Q tile, and the K and V tiles of the
//               units' sequences (128 keys each; K in a 3-stage ring, freed once
//               S is computed; V in a 4-stage ring, freed once O += P V is), by
//               TMA straight from the fused QKV activation buffer (SW128, 128-
//               byte rows of 64 head dims), in the order the MMA warp uses them;
//   warp 1      MMA issuer, alternating between the groups: for a group's next
//               tile S = Q K^T (M=128, N=128, K=64) into one of three TMEM S
//               buffers the groups share round-robin (so the next S is computed
//               while the group's softmax still reads the current one), then
//               O += P V (M=128, N=64, K=128) for its previous tile into the
//               group's TMEM O accumulator;
//   warps 2-5,  softmax groups 0 and 1, one thread per query row (its TMEM
//   6-9         lane): online softmax in the log2 domain with the running max
//               raised only when a tile's max exceeds it by more than 2^8 (the
//               final division keeps the result exact), P rounded to the model
//               dtype into the group's shared-memory P tile (the MMA's K-major
//               SW128 layout), O rescaled in TMEM when the max moves, and after
//               a unit's last tile O / l rounded and stored.  The softmax loops
//               run 64 columns per iteration without unrolling the iterations:
//               the smaller loop body measured faster than the unrolled one
//               (instruction-fetch stalls), and the paired f32x2 FMA / add and
//               three-input max cut the instruction count per score.
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
constexpr int kKStages = 3;
constexpr int kVStages = 4;
constexpr int kGroups = 2;
constexpr int kSBufs = 3;                    // TMEM S buffers shared by the groups
constexpr int kOCol = kSBufs * kRows;        // group g's O at TMEM column kOCol + 64 g
constexpr int kSoftmaxWarps = 4 * kGroups;
constexpr int kThreads = 64 + 32 * kSoftmaxWarps;
// Q per group, K and V rings, P per group, barriers
constexpr int kSmemBytes =
    1024 + kGroups * kTileBytes + (kKStages + kVStages) * kTileBytes + kGroups * 2 * kTileBytes + 1024;
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

// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two lanes of a * b + c (each rounded once, as fmaf) in one paired instruction.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "mov.b64 pc, {%6, %7};\n\tfma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Two lanes of a + b in one paired instruction.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pd;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "add.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// A group's walk over its units and their key tiles.
struct Cursor {
  int64_t unit;  // global unit index, or >= n_units when done
  int4 it;       // {row_start, len, q_tile, 0}
  int j, n_kv;   // key tile within the unit
  int u;         // units this group has started (for buffer parities)
  int t;         // tiles this group has started
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) attention_varlen_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const uint32_t sQ = base;                              // kGroups x 16 KB
  const uint32_t sK = sQ + kGroups * kTileBytes;         // kKStages x 16 KB
  const uint32_t sV = sK + kKStages * kTileBytes;        // kVStages x 16 KB
  const uint32_t sP = sV + kVStages * kTileBytes;        // kGroups x 32 KB (two 64-key SW128 blocks)
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (sP + kGroups * 2 * kTileBytes - base));
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // per-group barriers at index (kind * kGroups + group)
  const int Q_FULL = 0, Q_EMPTY = 1, P_FULL = 2, P_EMPTY = 3, O_FULL = 4, O_EMPTY = 5;
  auto gbar = [&](int kind, int grp) { return bar(kind * kGroups + grp); };
  const int S_FULL = 6 * kGroups, S_EMPTY = S_FULL + kSBufs, K_FULL = S_EMPTY + kSBufs,
            K_EMPTY = K_FULL + kKStages, V_FULL = K_EMPTY + kKStages, V_EMPTY = V_FULL + kVStages,
            DRAIN = V_EMPTY + kVStages, N_BARS = DRAIN + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[N_BARS]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);

  const int64_t n_units = int64_t(p.n_items) * p.n_heads;

  if (tid == 0) {
    for (int grp = 0; grp < kGroups; ++grp) {
      mbar_init(gbar(Q_FULL, grp), 1);
      mbar_init(gbar(Q_EMPTY, grp), 1);
      mbar_init(gbar(P_FULL, grp), 4);
      mbar_init(gbar(P_EMPTY, grp), 1);
      mbar_init(gbar(O_FULL, grp), 1);
      mbar_init(gbar(O_EMPTY, grp), 4);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(bar(S_FULL + i), 1);
      mbar_init(bar(S_EMPTY + i), 4);
    }
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(bar(K_FULL + i), 1);
      mbar_init(bar(K_EMPTY + i), 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(bar(V_FULL + i), 1);
      mbar_init(bar(V_EMPTY + i), 1);
    }
    mbar_init(bar(DRAIN), 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), 512);  // S buffers at 0, 128, 256; group g's O at 384 + 64 g
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
  // {row_start, len, q_tile, 0}.  Every role reads a record through here, so
  // all walk the same tiles.  A zero length is read as one key with w = 1
  // (nothing stored); a record outside the batch (row_start < 0, len < 0,
  // row_start + len > n_tokens, or a q_tile past its length) is flagged
  // LF_STATUS_BAD_SEGMENT and read as one key of row 0 with nothing stored, so
  // no store leaves out's rows.
  auto item_of = [&](int64_t unit) {
    int4 it = __ldg(p.items + unit / p.n_heads);
    const bool in_batch = it.x >= 0 && it.y >= 0 && int64_t(it.x) + it.y <= p.n_tokens && it.z >= 0 &&
                          (it.y == 0 || int64_t(it.z) * kRows < it.y);
    if (!in_batch) {
      set_status(p.status, LF_STATUS_BAD_SEGMENT);
      return make_int4(0, 1, 0, 1);
    }
    if (it.y == 0) return make_int4(it.x, 1, 0, 1);
    it.w = 0;
    return it;
  };
  // group grp takes the CTA's units 2k + grp
  auto start = [&](Cursor& c, int grp) {
    c.unit = blockIdx.x + int64_t(grp) * gridDim.x;
    c.u = 0;
    c.t = 0;
    c.j = 0;
    if (c.unit < n_units) {
      c.it = item_of(c.unit);
      c.n_kv = (c.it.y + kRows - 1) / kRows;
    }
  };
  auto advance = [&](Cursor& c) {
    ++c.t;
    if (++c.j < c.n_kv) return;
    c.unit += int64_t(kGroups) * gridDim.x;
    ++c.u;
    c.j = 0;
    if (c.unit < n_units) {
      c.it = item_of(c.unit);
      c.n_kv = (c.it.y + kRows - 1) / kRows;
    }
  };
  auto live = [&](const Cursor& c) { return c.unit < n_units; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      Cursor c[kGroups];
      for (int grp = 0; grp < kGroups; ++grp) start(c[grp], grp);
      int kc = 0, nq[kGroups] = {0, 0};
      bool stop = false;
      while (!stop && (live(c[0]) || live(c[1]))) {
        for (int grp = 0; grp < kGroups && !stop; ++grp) {
          Cursor& cg = c[grp];
          if (!live(cg)) continue;
          const int h = int(cg.unit % p.n_heads);
          if (cg.j == 0) {  // the unit's Q tile, once the group's previous unit has no S left to issue
            if (aborted(s_abort) || !mbar_wait(gbar(Q_EMPTY, grp), (cg.u & 1) ^ 1)) {
              if (!aborted(s_abort)) fail();
              stop = true;
              break;
            }
            mbar_arrive_expect_tx(gbar(Q_FULL, grp), kTileBytes);
            tma_load_2d(sQ + grp * kTileBytes, &p.qkv_map, gbar(Q_FULL, grp), p.q_col + h * kHd,
                        cg.it.x + cg.it.z * kRows);
            ++nq[grp];
          }
          const int sk = kc % kKStages, sv = kc % kVStages;
          if (aborted(s_abort) || !mbar_wait(bar(K_EMPTY + sk), ((kc / kKStages) & 1) ^ 1) ||
              !mbar_wait(bar(V_EMPTY + sv), ((kc / kVStages) & 1) ^ 1)) {
            if (!aborted(s_abort)) fail();
            stop = true;
            break;
          }
          const int32_t krow = cg.it.x + cg.j * kRows;
          mbar_arrive_expect_tx(bar(K_FULL + sk), kTileBytes);
          tma_load_2d(sK + sk * kTileBytes, &p.qkv_map, bar(K_FULL + sk), p.k_col + h * kHd, krow);
          mbar_arrive_expect_tx(bar(V_FULL + sv), kTileBytes);
          tma_load_2d(sV + sv * kTileBytes, &p.qkv_map, bar(V_FULL + sv), p.v_col + h * kHd, krow);
          ++kc;
          advance(cg);
        }
      }
      if (aborted(s_abort)) {  // loads nobody consumed must land before the CTA exits (bounded)
        for (int q = (kc > kKStages ? kc - kKStages : 0); q < kc; ++q)
          mbar_wait(bar(K_FULL + q % kKStages), (q / kKStages) & 1);
        for (int q = (kc > kVStages ? kc - kVStages : 0); q < kc; ++q)
          mbar_wait(bar(V_FULL + q % kVStages), (q / kVStages) & 1);
        for (int grp = 0; grp < kGroups; ++grp)  // only a group's latest Q can be unconsumed
          if (nq[grp] > 0) mbar_wait(gbar(Q_FULL, grp), (nq[grp] - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(DT<T>::umma_fmt, kRows, kRows, /*a_mn=*/0, /*b_mn=*/0);
      // a key tile with at most 64 keys of its sequence: S over those 64 only
      constexpr uint32_t idesc_s64 = umma_idesc_f16(DT<T>::umma_fmt, kRows, kRows / 2, /*a_mn=*/0, /*b_mn=*/0);
      constexpr uint32_t idesc_o = umma_idesc_f16(DT<T>::umma_fmt, kRows, kHd, /*a_mn=*/0, /*b_mn=*/1);
      struct Prev { bool valid, first, last; int t, u, kv, nk; };  // nk: 16-key steps of O += P V
      Cursor c[kGroups];
      Prev prev[kGroups];
      for (int grp = 0; grp < kGroups; ++grp) {
        start(c[grp], grp);
        prev[grp].valid = false;
      }
      int kc = 0;
      bool stop = false;
      // O_grp += P V for the group's previous tile
      auto pv = [&](int grp, const Prev& e) -> bool {
        const int sv = e.kv % kVStages;
        if (!mbar_wait(gbar(P_FULL, grp), e.t & 1)) return false;
        if (!mbar_wait(bar(V_FULL + sv), (e.kv / kVStages) & 1)) return false;
        if (e.first && !mbar_wait(gbar(O_EMPTY, grp), (e.u & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t pb = sP + grp * 2 * kTileBytes;
        const uint32_t vb = sV + sv * kTileBytes;
        // keys past the sequence end stop at the last 16-key step that holds one
        // (that step's other keys have p = 0)
#pragma unroll
        for (int t = 0; t < kRows / 16; ++t) {
          if (t >= e.nk) break;
          const uint64_t ad = smem_desc(pb + (t >> 2) * kTileBytes + (t & 3) * 32, 16, 1024, 2);
          const uint64_t bd = smem_desc(vb + t * 2048, kTileBytes, 1024, 2);
          umma_f16(tmem + kOCol + kHd * grp, ad, bd, idesc_o, (e.first && t == 0) ? 0u : 1u);
        }
        umma_commit(gbar(P_EMPTY, grp));
        umma_commit(bar(V_EMPTY + sv));
        if (e.last) umma_commit(gbar(O_FULL, grp));
        return true;
      };
      // S for tile kc goes to buffer kc % kSBufs once that buffer's previous
      // tile (kc - kSBufs, of either group) has been read
      while (!stop && (live(c[0]) || live(c[1]) || prev[0].valid || prev[1].valid)) {
        for (int grp = 0; grp < kGroups && !stop; ++grp) {
          Cursor& cg = c[grp];
          Prev cur{false, false, false, 0, 0, 0, 0};
          if (live(cg)) {
            const int sk = kc % kKStages, sb = kc % kSBufs;
            if (aborted(s_abort) || (cg.j == 0 && !mbar_wait(gbar(Q_FULL, grp), cg.u & 1)) ||
                !mbar_wait(bar(K_FULL + sk), (kc / kKStages) & 1) ||
                !mbar_wait(bar(S_EMPTY + sb), ((kc / kSBufs) & 1) ^ 1)) {
              if (!aborted(s_abort)) fail();
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t qa = sQ + grp * kTileBytes, kb = sK + sk * kTileBytes;
            const int nvalid = min(kRows, cg.it.y - cg.j * kRows);
            const uint32_t idesc = nvalid > kRows / 2 ? idesc_s : idesc_s64;
#pragma unroll
            for (int t = 0; t < kHd / 16; ++t)
              umma_f16(tmem + kRows * sb, smem_desc(qa + t * 32, 16, 1024, 2), smem_desc(kb + t * 32, 16, 1024, 2),
                       idesc, t > 0 ? 1u : 0u);
            umma_commit(bar(S_FULL + sb));
            umma_commit(bar(K_EMPTY + sk));
            if (cg.j == cg.n_kv - 1) umma_commit(gbar(Q_EMPTY, grp));
            cur = Prev{true, cg.j == 0, cg.j == cg.n_kv - 1, cg.t, cg.u, kc, (nvalid + 15) / 16};
            ++kc;
            advance(cg);
          }
          if (prev[grp].valid && !pv(grp, prev[grp])) {
            fail();
            stop = true;
            break;
          }
          prev[grp] = cur;
        }
      }
      if (aborted(s_abort)) {  // every issued MMA must finish before TMEM is released (bounded)
        umma_commit(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax groups (warps 2..9)
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t o_addr = lane_addr + kOCol + kHd * grp;  // this row of the group's O
    const uint32_t prow = (row >> 3) * 1024 + (row & 7) * 128;  // this row in a SW128 block
    const uint32_t pb = sP + grp * 2 * kTileBytes - base;
    const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
    // The MMA warp issues the groups' S tiles round-robin (group 0 first), so
    // this group's n-th tile is global tile n + min(n + grp, tiles of the other group).
    int other_tiles = 0;
    {
      Cursor o;
      start(o, grp ^ 1);
      while (live(o)) {
        other_tiles += o.n_kv;
        o.t += o.n_kv - 1;
        o.j = o.n_kv - 1;
        advance(o);
      }
    }
    Cursor c;
    start(c, grp);
    float m = -INFINITY, l = 0.f;
    while (live(c)) {
      const int t = c.t, j = c.j;
      const int kc = t + min(t + grp, other_tiles);
      const int sb = kc % kSBufs;
      const uint32_t s_addr = lane_addr + kRows * sb;
      const int4 it = c.it;
      const int64_t unit = c.unit;
      const int uu = c.u;
      const bool last = j == c.n_kv - 1;
      const int nvalid = min(kRows, it.y - j * kRows);
      // warp-uniform skips of what the sequence does not reach: a warp whose 32 query
      // rows all lie past its end does no softmax (its P rows only feed O rows that
      // are never stored), and a key tile with at most 64 keys reads one 64-column
      // half of S (the MMA computed only that half, and O += P V stops there)
      const bool rows_live = quad * 32 < it.y - it.z * kRows;
      const int n_half = nvalid > kRows / 2 ? 2 : 1;
      bool ok = !aborted(s_abort);
      if (ok && !mbar_wait(bar(S_FULL + sb), (kc / kSBufs) & 1)) {
        fail();
        ok = false;
      }
      const bool work = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      // pass 1: the row max over the valid keys, 64 columns at a time
      float mx = -INFINITY;
      if (work && rows_live) {
#pragma unroll 1
        for (int hh = 0; hh < n_half; ++hh) {
          uint32_t sv[64];
          tmem_ld64(s_addr + hh * 64, sv);
          if (nvalid < hh * 64 + 64) {  // warp-uniform: keys past the end do not count
#pragma unroll
            for (int q = 0; q < 64; ++q)
              if (hh * 64 + q >= nvalid) sv[q] = __float_as_uint(-INFINITY);
          }
          float mxs[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int q = 0; q < 64; q += 8) {
            mxs[(q >> 3) & 3] = max3(mxs[(q >> 3) & 3], __uint_as_float(sv[q]), __uint_as_float(sv[q + 1]));
            mxs[(q >> 3) & 3] = max3(mxs[(q >> 3) & 3], __uint_as_float(sv[q + 2]), __uint_as_float(sv[q + 3]));
            mxs[((q >> 3) + 2) & 3] =
                max3(mxs[((q >> 3) + 2) & 3], __uint_as_float(sv[q + 4]), __uint_as_float(sv[q + 5]));
            mxs[((q >> 3) + 2) & 3] =
                max3(mxs[((q >> 3) + 2) & 3], __uint_as_float(sv[q + 6]), __uint_as_float(sv[q + 7]));
          }
          mx = max3(mx, fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3]));
        }
        mx *= sl2.x;  // the scale is positive: max commutes with it
      }
      const float m_new = (j == 0 || mx > m + kMaxSlack) ? mx : m;
      const float alpha = (j == 0) ? 1.f : ex2(m - m_new);
      // the previous tile's O += P V has finished: P may be overwritten, O rescaled
      ok = work && !aborted(s_abort);
      if (ok && !mbar_wait(gbar(P_EMPTY, grp), (t & 1) ^ 1)) {
        fail();
        ok = false;
      }
      const bool go = __all_sync(0xffffffffu, ok);
      if (go && rows_live && j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        tc_fence_after();
        uint32_t ov[64];
        tmem_ld64(o_addr, ov);
#pragma unroll
        for (int q = 0; q < 64; ++q) ov[q] = __float_as_uint(__uint_as_float(ov[q]) * alpha);
        tmem_st64(o_addr, ov);
      }
      // pass 2: p = 2^(s - max), rounded to T into the group's SW128 K-major P tile
      float2 sums[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      if (go && rows_live) {
        const float2 neg_m = make_float2(-m_new, -m_new);
#pragma unroll 1
        for (int hh = 0; hh < n_half; ++hh) {
          uint32_t sv[64];
          tmem_ld64(s_addr + hh * 64, sv);
          if (nvalid < hh * 64 + 64) {  // warp-uniform: keys past the end score -inf, so p = 0
#pragma unroll
            for (int q = 0; q < 64; ++q)
              if (hh * 64 + q >= nvalid) sv[q] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {  // 16-byte chunks = 8 keys
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int col = c8 * 8 + 2 * i;
              const float2 x = fma2(make_float2(__uint_as_float(sv[col]), __uint_as_float(sv[col + 1])), sl2, neg_m);
              const float2 pr = make_float2(ex2(x.x), ex2(x.y));
              sums[i & 1] = add2(sums[i & 1], pr);
              w[i] = Pack2<T>::pack(pr.x, pr.y);
            }
            *reinterpret_cast<uint4*>(gbase + pb + hh * kTileBytes + prow + ((c8 ^ (row & 7)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(S_EMPTY + sb));  // S has been read: the buffer may take the next S
      const float sum = (sums[0].x + sums[0].y) + (sums[1].x + sums[1].y);
      l = (j == 0) ? sum : l * alpha + sum;
      m = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(gbar(P_FULL, grp));
      advance(c);
      if (last) {
        // the unit's output: O / l, once its last O += P V has finished
        ok = !aborted(s_abort);
        if (ok && !mbar_wait(gbar(O_FULL, grp), uu & 1)) {
          fail();
          ok = false;
        }
        if (__all_sync(0xffffffffu, ok) && rows_live) {
          tc_fence_after();
          uint32_t ov[64];
          tmem_ld64(o_addr, ov);
          const int qr = it.z * kRows + row;
          if (qr < it.y && it.w == 0) {
            const float inv = 1.f / l;
            T* dst = reinterpret_cast<T*>(p.out) + int64_t(it.x + qr) * p.ldo + int(unit % p.n_heads) * kHd;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              uint4 w;
              w.x = Pack2<T>::pack(__uint_as_float(ov[8 * q + 0]) * inv, __uint_as_float(ov[8 * q + 1]) * inv);
              w.y = Pack2<T>::pack(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv);
              w.z = Pack2<T>::pack(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv);
              w.w = Pack2<T>::pack(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv);
              reinterpret_cast<uint4*>(dst)[q] = w;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(gbar(O_EMPTY, grp));
      }
    }
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
  p.n_tokens = n_tokens;
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
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), kSmemBytes, s, p);
  if (e != cudaSuccess) return cuda_error(e, "launch attention_varlen");
  count_launch();
  return LF_OK;
}
