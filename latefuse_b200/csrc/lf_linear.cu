// Projection GEMM on tcgen05 CTA pairs: Y = act(X W^T + bias), bf16 / f16 in, f32 accumulate.
//
// Replaces the encoder's nn.Linear projections (src/latefuse/model/encoder.py:
// the fused q/k/v, attention-output, FFN up and down projections) with an
// sm_100a kernel of this library, so that work around a projection can be
// fused into it (the FFN's GELU in the epilogue: ACT2FN["gelu"] of
// encoder.py:122,139).  Rounding follows torch: round(acc + bias) to the dtype,
// then for GELU round(gelu_f32(that)).
//
// Persistent, one cluster of two CTAs per SM pair, 256 x 256 output tiles in
// m-major order (the pairs working at one time share the rows of X and all of
// W through L2).  The MMAs are tcgen05.mma.cta_group::2 with M = 256: CTA r of
// the pair stages its own 128 rows of X and W rows [n0 + 128 r, n0 + 128 r + 128)
// per 64-wide K block, and the leader's MMA reads both CTAs' shared memory, so
// each SM stages 32 KB per K block instead of the 48 KB of a 128 x 256 tile on
// one SM (less L2 -> SM traffic and fewer shared-memory writes per FLOP: more
// work per joule, which is what the 1000 W cap rations).  Each CTA's TMEM holds
// its 128 rows x 256 columns, twice (the epilogue of one tile overlaps the main
// loop of the next).
//   warp 0      TMA producer (both CTAs): an X box {64, 128} and a W box {64, 128}
//               (K-major, SW128) per K block into a 6-stage ring of 32 KB; every
//               copy completes on the leader's "full" barrier, which the leader's
//               producer arms with both CTAs' bytes;
//   warp 1      MMA issuer (leader only): four tcgen05.mma (M=256, N=256, K=16) per
//               K block; each commit arrives on both CTAs' barriers (multicast);
//   warps 2-9   epilogue (both CTAs), two warps per TMEM lane quadrant (128 columns
//               each), one output row per thread: 32 columns per tcgen05.ld, bias
//               and activation in f32, rounded, staged per warp in a 32 x 32 SW64
//               tile and written by TMA (rows past M are clipped by the tensor map);
//               each warp then arrives on the leader's "accumulator empty" barrier.
// With LoRA (lf_linear_lora) the per-row delta joins the same accumulator: after
// a tile's K blocks come one "delta block" per adapter segment with tokens in the
// tile's 256 rows: each CTA stages its 128 rows of the segment's shrink output u
// (written by lf_lora_shrink_blocked in the no-swizzle K-major operand layout: the
// block of (128-row tile, segment), or zeros when the segment has no token in this
// CTA's rows, fetched from past the end of u) and its 128 columns of the segment's
// B factor (MN-major SW128, straight from the slot cache, prefetched into L2 one
// tile ahead), and the leader multiplies them with K = R, so every row gets its
// own adapter's delta: y = act(round(x W^T + bias + u B)).
// With the shrink in the same launch (lf_linear_lora_shrink) each pair owns whole
// 256-row blocks: before a block's column tiles it runs one or more shrink passes,
// u = round(x A_slot(t)) for every segment and module of the block, as an MMA of the
// block's x against the segments' A factors (MN-major, all modules of a segment in one
// copy from the slot cache, each CTA staging half of the segments); the epilogue
// writes u in the blocked layout (every row of a (128-row tile, segment) block: its
// product if it lies in the segment, else 0), fences it for the async proxy and
// signals the producer, which then stages the blocks for the tiles' delta MMAs from L2.
// u never leaves the launch except through L2, and x is read in the same launch.
// Every wait is bounded: a timeout sets LF_STATUS_TIMEOUT and the roles unwind.
// No load uses cluster multicast: each CTA loads only its own operands.
#include "lf_common.cuh"
#include "lf_internal.h"

namespace lf {

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;     // kBM rows per CTA, 2 kBM per pair
constexpr int kABytes = kBM * kBK * 2;            // 16 KB: this CTA's X rows
constexpr int kBBytes = (kBN / 2) * kBK * 2;      // 16 KB: this CTA's half of the W rows
constexpr int kStageBytes = kABytes + kBBytes;    // 32 KB
constexpr int kStages = 6;
constexpr int kEpiWarps = 8;                      // two per TMEM lane quadrant, 128 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kOutCols = 32;                      // output columns per epilogue store
constexpr int kOutBuf = 32 * kOutCols * 2;        // one warp's 32 x 32 staging tile: 2 KB
constexpr int kDeltaBuf = 16384;                  // a tile's first delta blocks: two at rank 16 (u 4 KB + B 4 KB each), one at 32
constexpr int kDeltaBufs = 1;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiWarps * kOutBuf + kDeltaBufs * kDeltaBuf + 1024;
static_assert(kSmemBytes <= 232448, "above the 227 KB of shared memory a CTA may use");

struct alignas(64) LinearParams {
  CUtensorMap x_map;  // 2D {K, M}, box {64, 128}, SW128
  CUtensorMap w_map;  // 2D {K, N}, box {64, 128}, SW128; w_kn: 3D {64, K, N / 64}, box {64, 64, 2}, SW128
  CUtensorMap y_map;  // 2D {N, M}, box {32, 32}, SW64
  CUtensorMap u_map;  // LoRA: 3D {256, R / 2, n_mod * n_blk}, box {256, R / 2, 1}: one 128 x R block
  CUtensorMap b_map[kMaxModules];     // LoRA: 4D {64, R, module_cols / 64, n_slots}, box {64, R, 2, 1}, SW128
  const void* b_ptr[kMaxModules];     // LoRA: (slot 0, module i) B factors, for L2 prefetch
  int64_t b_slot_stride;              // elements
  int32_t n_slots;
  const void* bias;   // N entries or null
  const int32_t* tile_pairs;          // LoRA: 256-row tile q's delta blocks are entries
  const int32_t* pairs;               //   tile_pairs[q] .. tile_pairs[q + 1] of pairs (3 each); null: no delta
  CUtensorMap a_map;                  // shrink: 4D {R, K, n_mod, n_slots}, box {R, 64, n_mod, 1}, MN-major
  void* u_out;                        // shrink: the blocked u this launch writes (u_map reads it back)
  const int32_t* seg_start;           // shrink: segment starts and lengths (tokens)
  const int32_t* seg_len;
  int32_t shrink;                     // 1: u is computed in this launch
  int32_t s_epc;                      // shrink: segments per CTA per pass (n_mod * R * s_epc <= 128)
  int32_t n_rb;                       // 256-row blocks
  int64_t tiles_per_pair;             // shrink: each pair's contiguous range of tiles
  int32_t n_segs;
  int32_t n_blk;                      // LoRA: u blocks per module (128-row tiles + segments)
  int32_t rank;
  int32_t n_mod;                      // output column block i (module_cols wide) takes module i's delta
  int32_t module_cols;
  int64_t m_rows;
  int64_t n_tiles;
  int32_t n_tiles_n;
  int32_t n_kb;
  int32_t act;        // LF_ACT_*
  int32_t w_kn;       // 1: w is (K, N) (the transposed nn.Linear weight), read MN-major
  int32_t* status;
  const void* y_in;   // accumulate: y's current values (the output itself), row stride ldy
  int64_t ldy;
};

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// D[tmem] (+)= A * B over the CTA pair (M = 256: each CTA supplies 128 rows of A and
// half of B's columns from the same shared-memory offsets).
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at offset `bar` in both CTAs of the pair once every MMA
// issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(both)
      : "memory");
}

__device__ __forceinline__ void umma_commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Entries [q0, q1) of the pair table for 256-row tile q.  A range that is not
// ascending or holds more entries than there are segments reads as empty, and
// `bad` says so, so that every role walks the same (no) entries.
__device__ __forceinline__ int2 pair_range(const int32_t* tile_pairs, int q, int n_segs, bool* bad = nullptr) {
  const int q0 = __ldg(tile_pairs + q), q1 = __ldg(tile_pairs + q + 1);
  const bool ok = q0 >= 0 && q1 >= q0 && q1 - q0 <= n_segs;
  if (bad != nullptr) *bad = !ok;
  return ok ? make_int2(q0, q1) : make_int2(0, 0);
}

// A tile's pair-table range loaded ahead of its use: the loads are issued one work item
// early and checked (as pair_range does) only when the item starts, so their latency
// overlaps the previous item instead of stalling the thread that issues copies or MMAs.
struct RangeAhead {
  int32_t q0, q1;
  __device__ __forceinline__ void load(const int32_t* tile_pairs, int q) {
    q0 = __ldg(tile_pairs + q);
    q1 = __ldg(tile_pairs + q + 1);
  }
  __device__ __forceinline__ int2 get(int n_segs, bool* bad = nullptr) const {
    const bool ok = q0 >= 0 && q1 >= q0 && q1 - q0 <= n_segs;
    if (bad != nullptr) *bad = !ok;
    return ok ? make_int2(q0, q1) : make_int2(0, 0);
  }
};

__device__ __forceinline__ bool aborted_flag(const int32_t* f) {
  return *reinterpret_cast<const volatile int32_t*>(f) != 0;
}

// One work item of a CTA pair: a 256 x 256 output tile (rb, c), or shrink pass `pass`
// of row block rb.  Every role walks the same sequence: round robin over all tiles
// without the shrink; with it, a contiguous range of tiles in row-block order
// (p.tiles_per_pair of them), each row block the range touches preceded by its shrink
// passes.  A range that shares a row block with its neighbour computes that block's u
// too: both write identical values, and each pair reads only after its own writes.
struct Item {
  int32_t rb, c, pass;
  bool shrink;
  bool first;  // the first tile after its row block's shrink passes
};

template <bool kShrinkable>
struct Sched {
  int64_t t;       // next tile
  int64_t t_end;   // shrink: end of this pair's range
  int32_t rb;      // shrink: the row block whose passes were emitted last (-1: none)
  int32_t pass, n_pass;
  int32_t n_pairs;
  bool fresh;      // shrink: the next tile is the first after its block's passes

  __device__ __forceinline__ static int32_t passes(const LinearParams& p, int32_t rb) {
    const int2 qr = pair_range(p.tile_pairs, rb, p.n_segs);
    const int32_t per = 2 * p.s_epc;
    return (qr.y - qr.x + per - 1) / per;
  }
  __device__ __forceinline__ Sched(const LinearParams& p, int pair, int n_pairs_)
      : t(pair), t_end(0), rb(-1), pass(0), n_pass(0), n_pairs(n_pairs_), fresh(false) {
    if (kShrinkable && p.shrink) {
      t = int64_t(pair) * p.tiles_per_pair;
      t_end = t + p.tiles_per_pair < p.n_tiles ? t + p.tiles_per_pair : p.n_tiles;
    }
  }
  __device__ __forceinline__ bool next(const LinearParams& p, Item& it) {
    if (!kShrinkable || !p.shrink) {
      if (t >= p.n_tiles) return false;
      it = Item{int32_t(t / p.n_tiles_n), int32_t(t % p.n_tiles_n), 0, false, false};
      t += n_pairs;
      return true;
    }
    if (t >= t_end) return false;
    const int32_t trb = int32_t(t / p.n_tiles_n);
    if (trb != rb) {  // entering a row block: its shrink passes first
      rb = trb;
      pass = 0;
      n_pass = passes(p, rb);
      fresh = true;
    }
    if (pass < n_pass) {
      it = Item{rb, 0, pass++, true, false};
      return true;
    }
    it = Item{trb, int32_t(t % p.n_tiles_n), 0, false, fresh};
    fresh = false;
    ++t;
    return true;
  }
};

// The MN-major operand layout of an A-factor box (64 K rows of R elements), as the
// slot cache's TMA copy lands it: (swizzle, stride between 8-row groups).
__device__ __forceinline__ uint32_t a_box_layout(int R) { return R == 16 ? 6u : R == 32 ? 4u : 2u; }

// kLora: the LoRA delta blocks (and the shrink passes when p.shrink) are compiled in;
// the plain projection GEMM is its own instantiation without them.  kAcc: the epilogue
// adds y's current values (y += x W^T + bias, rounded once).  kAct: the activation
// (LF_ACT_NONE / LF_ACT_GELU).
template <typename T, bool kLora, bool kAcc, int kAct>
__global__ void __launch_bounds__(kThreads, 1) linear_kernel(const __grid_constant__ LinearParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();          // 0: the leader, which issues the MMAs
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

  const uint32_t s_stage0 = base;
  const uint32_t s_out0 = base + kStages * kStageBytes;  // [warp] 2 KB staging tiles
  const uint32_t s_delta = s_out0 + kEpiWarps * kOutBuf;  // a tile's first delta blocks
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (s_delta + kDeltaBufs * kDeltaBuf - base));
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int FULL = 0, EMPTY = kStages, ACC_FULL = 2 * kStages, ACC_EMPTY = 2 * kStages + 2,
            DRAIN = 2 * kStages + 4, DFULL = DRAIN + 1, DEMPTY = DFULL + kDeltaBufs, U_READY = DEMPTY + kDeltaBufs,
            N_BARS = U_READY + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[N_BARS]);
  int32_t* s_abort = reinterpret_cast<int32_t*>(tmem_slot + 1);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(FULL + i), 1);   // the leader's arrive, with both CTAs' bytes
      mbar_init(bar(EMPTY + i), 1);  // the leader's MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 2 * kEpiWarps);  // both CTAs' epilogue warps
    }
    mbar_init(bar(DRAIN), 1);
    for (int i = 0; i < kDeltaBufs; ++i) {
      mbar_init(bar(DFULL + i), 1);   // the leader's arrive, with both CTAs' bytes
      mbar_init(bar(DEMPTY + i), 1);  // the leader's MMA commit
    }
    mbar_init(bar(U_READY), kEpiWarps);  // this CTA's epilogue warps: a shrink pass's u is written
    *s_abort = 0;
    fence_mbar_init();
    prefetch_tmap(&p.x_map);
    prefetch_tmap(&p.w_map);
    prefetch_tmap(&p.y_map);
    if (kLora) {  // the delta blocks' u and B maps, and the shrink's A map
      prefetch_tmap(&p.u_map);
      for (int i = 0; i < p.n_mod; ++i) prefetch_tmap(&p.b_map[i]);
      if (p.shrink) prefetch_tmap(&p.a_map);
    }
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's TMEM
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_launch_dependents();

  auto fail = [&]() {
    set_status(p.status, LF_STATUS_TIMEOUT);
    atomicExch(s_abort, 1);
  };
  constexpr bool lora = kLora;
  // a tile's first delta blocks (as many as the delta buffer holds: 512 * rank bytes
  // each per CTA) go to their own buffer, loaded while the tile's K blocks stream, so
  // they have landed when the MMA reaches them; later ones use the ring, where a block
  // in a stage carries a sixteenth of a K block's work and the ring's lead shrinks
  const int n_dslots = lora ? kDeltaBuf / (512 * p.rank) : 0;
  const bool dbuf = n_dslots > 0;
  auto dbuf_tile = [&](const Item& it) { return !(kLora && p.shrink && it.first); };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int kk = 0, dk = 0, u_wait = 0, u_ph = 0;
      bool stop = false;
      const int32_t half_cols = int32_t(rank) * (kBN / 2);
      // the stage of K block kb is free: arm it (leader) and return its address
      auto take = [&](uint32_t bytes, uint32_t& st, uint32_t& full) {
        const int s = kk % kStages;
        if (aborted_flag(s_abort) || !mbar_wait(bar(EMPTY + s), ((kk / kStages) & 1) ^ 1)) {
          if (!aborted_flag(s_abort)) fail();
          return false;
        }
        st = s_stage0 + s * kStageBytes;
        full = mapa_shared(bar(FULL + s), 0);
        if (rank == 0) mbar_arrive_expect_tx(bar(FULL + s), bytes);
        return true;
      };
      // u written in this launch must be there before its blocks are staged: one phase of
      // U_READY per row block with shrink passes, waited before that block's first delta
      // copy, or before the next block's passes when the range had no delta for it, so no
      // more than one phase is ever pending
      auto wait_u = [&]() {
        for (; u_wait > 0; --u_wait, u_ph ^= 1)
          if (aborted_flag(s_abort) || !mbar_wait(bar(U_READY), u_ph)) {
            if (!aborted_flag(s_abort)) fail();
            return false;
          }
        return true;
      };
      Sched<kLora> sched(p, pair, n_pairs);
      Item it, nit;
      bool more = sched.next(p, nit);
      RangeAhead ahead_r{0, 0};
      if (lora && more) ahead_r.load(p.tile_pairs, nit.rb);
      while (!stop && more) {
        it = nit;
        const RangeAhead cur_r = ahead_r;
        more = sched.next(p, nit);
        if (lora && more) ahead_r.load(p.tile_pairs, nit.rb);  // in flight while this item runs
        const int32_t m0 = it.rb * (2 * kBM) + int32_t(rank) * kBM;
        int q0 = 0, q1 = 0;
        if (lora) {
          bool bad = false;
          const int2 qr = cur_r.get(p.n_segs, &bad);
          if (bad && rank == 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
          q0 = qr.x;
          q1 = qr.y;
        }
        if (it.shrink) {
          // pass `it.pass`: this CTA stages the x rows and the A factors (all modules of a
          // segment in one copy) of its half of the pass's segments; the other half's
          // columns come from the peer; a missing segment reads zeros (slot past the cache)
          const int32_t e0 = it.pass * 2 * p.s_epc;
          const int32_t ne_p = min(2 * p.s_epc, q1 - q0 - e0);
          const int32_t ne_h = (ne_p + 1) / 2;
          const uint32_t box = uint32_t(p.n_mod) * 128u * uint32_t(p.rank);  // one segment's modules
          if (it.pass == 0 && !wait_u()) {
            stop = true;
            break;
          }
          for (int kb = 0; kb < p.n_kb; ++kb, ++kk) {
            uint32_t st, full;
            if (!take(2 * (kABytes + ne_h * box), st, full)) {
              stop = true;
              break;
            }
            tma_load_2d_pair(st, &p.x_map, full, kb * kBK, m0);
            for (int i = 0; i < ne_h; ++i) {
              const int32_t e = e0 + int32_t(rank) * ne_h + i;
              const int32_t slot = e < ne_p + e0 ? __ldg(p.pairs + 3 * (q0 + e) + 1) : p.n_slots;
              tma_load_4d_pair(st + kABytes + i * box, &p.a_map, full, 0, kb * kBK, 0, slot);
            }
          }
          u_wait = 1;  // the epilogue arrives once per block, after its last pass
          continue;
        }
        const int32_t n0 = it.c * kBN;
        const int mod = lora ? n0 / p.module_cols : p.n_mod;
        if (mod >= p.n_mod) q0 = q1 = 0;
        const int32_t n_loc = mod < p.n_mod ? n0 - mod * p.module_cols : 0;
        const int32_t zero_blk = p.n_mod * p.n_blk;  // past the last block: the copy reads zeros
        // delta block q: this CTA's 128 rows of u (its block of (128-row tile, segment), or
        // zeros) and its 128 columns of the segment's B, completing on the leader's `full`
        // entry q's {segment, slot, halves}, loaded ahead where the caller can
        struct Entry { int32_t j, slot, mask; };
        auto entry = [&](int q) {
          return Entry{__ldg(p.pairs + 3 * q), __ldg(p.pairs + 3 * q + 1), __ldg(p.pairs + 3 * q + 2)};
        };
        auto load_delta = [&](uint32_t dst_u, uint32_t dst_b, uint32_t full_local, Entry e, uint32_t arm_bytes) {
          int j = e.j;
          const int32_t slot = e.slot;  // out of range: zero fill, no delta, reported
          const int32_t mask = e.mask;
          if (j < 0 || j >= p.n_segs) {  // a segment outside the table: treated as absent, reported
            if (rank == 0) set_status(p.status, LF_STATUS_BAD_SEGMENT);
            j = -1;
          }
          if ((slot < 0 || slot >= p.n_slots) && rank == 0) set_status(p.status, LF_STATUS_BAD_SLOT);
          const int32_t blk = (j >= 0 && ((mask >> rank) & 1)) ? mod * p.n_blk + 2 * it.rb + int32_t(rank) + j
                                                               : zero_blk;
          const uint32_t full = mapa_shared(full_local, 0);
          if (rank == 0 && arm_bytes) mbar_arrive_expect_tx(full_local, arm_bytes);  // every block's bytes, both CTAs
          tma_load_3d_pair(dst_u, &p.u_map, full, 0, 0, blk);
          tma_load_4d_pair(dst_b, &p.b_map[mod], full, 0, 0, (n_loc + half_cols) / 64, slot);
        };
        // the first blocks go to the delta buffer half way through the tile's K blocks:
        // the copies issue about kStages K blocks ahead of the MMA, so the previous
        // tile's blocks were multiplied by then and these land before the MMA needs
        // them; not for a block's first tile when this launch writes u (its delta
        // blocks wait for the shrink's epilogue)
        const bool use_dbuf = dbuf && q1 > q0 && dbuf_tile(it);
        const int n_in = use_dbuf ? min(q1 - q0, n_dslots) : 0;
        const int d_after = p.n_kb / 2;
        // the tile's first two delta entries, in flight while its K blocks stream
        Entry e_first{0, 0, 0}, e_second{0, 0, 0};
        if (q1 > q0) e_first = entry(q0);
        if (q1 > q0 + 1) e_second = entry(q0 + 1);
        for (int kb = 0; kb < p.n_kb; ++kb, ++kk) {
          uint32_t st, full;
          if (!take(2 * kStageBytes, st, full)) {
            stop = true;
            break;
          }
          tma_load_2d_pair(st, &p.x_map, full, kb * kBK, m0);
          if (p.w_kn)
            tma_load_3d_pair(st + kABytes, &p.w_map, full, 0, kb * kBK, (n0 + half_cols) / 64);
          else
            tma_load_2d_pair(st + kABytes, &p.w_map, full, kb * kBK, n0 + half_cols);
          if (use_dbuf && kb == d_after) {
            const int db = dk % kDeltaBufs;
            if (aborted_flag(s_abort) || !mbar_wait(bar(DEMPTY + db), ((dk / kDeltaBufs) & 1) ^ 1)) {
              if (!aborted_flag(s_abort)) fail();
              stop = true;
              ++kk;
              break;
            }
            const uint32_t blk_bytes = 512u * uint32_t(p.rank);
            for (int i = 0; i < n_in; ++i) {
              const uint32_t dst = s_delta + db * kDeltaBuf + i * blk_bytes;
              load_delta(dst, dst + 256 * p.rank, bar(DFULL + db), i == 0 ? e_first : i == 1 ? e_second : entry(q0 + i),
                         i == 0 ? 2u * blk_bytes * uint32_t(n_in) : 0u);
            }
            ++dk;
          }
        }
        q0 += n_in;
        if (stop || q1 <= q0) continue;
        if (!wait_u()) {
          stop = true;
          break;
        }
        for (int q = q0; q < q1; ++q, ++kk) {
          const int s = kk % kStages;
          if (aborted_flag(s_abort) || !mbar_wait(bar(EMPTY + s), ((kk / kStages) & 1) ^ 1)) {
            if (!aborted_flag(s_abort)) fail();
            stop = true;
            break;
          }
          const uint32_t st = s_stage0 + s * kStageBytes;
          const int q_first = q0 - n_in;  // the tile's first entry
          load_delta(st, st + kABytes, bar(FULL + s),
                     q == q_first ? e_first : q == q_first + 1 ? e_second : entry(q), 2u * 512u * uint32_t(p.rank));
        }
      }
      if (aborted_flag(s_abort)) {  // loads nobody consumed land before the CTA exits (bounded)
        if (rank == 0) {
          for (int q = (kk > kStages ? kk - kStages : 0); q < kk; ++q)
            mbar_wait(bar(FULL + q % kStages), (q / kStages) & 1);
          for (int q = (dk > kDeltaBufs ? dk - kDeltaBufs : 0); q < dk; ++q)
            mbar_wait(bar(DFULL + q % kDeltaBufs), (q / kDeltaBufs) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the leader's lane 0)
    if (lane == 0 && rank == 0) {
      // the delta blocks' B is MN-major (the cache's (R, cols) rows); with w (K, N) the main
      // loop's B is MN-major too, and every MMA of a tile has one instruction descriptor
      constexpr uint32_t idesc_d = umma_idesc_f16(DT<T>::umma_fmt, 2 * kBM, kBN, 0, 1);
      const uint32_t idesc = p.w_kn ? idesc_d : umma_idesc_f16(DT<T>::umma_fmt, 2 * kBM, kBN, 0, 0);
      int kk = 0, n_it = 0, dk = 0;
      bool stop = false;
      auto wait = [&](uint32_t b, uint32_t parity) {
        if (aborted_flag(s_abort)) return false;
        if (mbar_wait(b, parity)) return true;
        if (!aborted_flag(s_abort)) fail();
        return false;
      };
      Sched<kLora> sched(p, pair, n_pairs);
      Item it, nit;
      bool more = sched.next(p, nit);
      RangeAhead ahead_r{0, 0};
      if (lora && more) ahead_r.load(p.tile_pairs, nit.rb);
      for (; !stop && more; ++n_it) {
        it = nit;
        const RangeAhead cur_r = ahead_r;
        more = sched.next(p, nit);
        if (lora && more) ahead_r.load(p.tile_pairs, nit.rb);  // in flight while this item runs
        const int a = n_it & 1;
        int n_delta = 0, ne_p = 0;
        if (lora) {
          const int2 qr = cur_r.get(p.n_segs);
          if (it.shrink) {
            ne_p = min(2 * p.s_epc, qr.y - qr.x - it.pass * 2 * p.s_epc);
          } else if (it.c * kBN / p.module_cols < p.n_mod) {
            n_delta = qr.y - qr.x;
          }
        }
        if (!wait(bar(ACC_EMPTY + a), ((n_it >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        if (it.shrink) {
          // u = x A over the pass's segments: N = both halves' A boxes (MN-major atoms of
          // R columns, one box of R x 64 per segment and module, box bytes apart)
          const int ne_h = (ne_p + 1) / 2;
          const uint32_t n_cols = uint32_t(2 * ne_h * p.n_mod * p.rank);
          const uint32_t idesc_s = umma_idesc_f16(DT<T>::umma_fmt, 2 * kBM, n_cols, 0, 1);
          const uint32_t abox = 128u * uint32_t(p.rank), row_b = 2u * uint32_t(p.rank);
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
              umma_pair(tmem + a * kBN, smem_desc(st + q * 32, 16, 1024, 2),
                        smem_desc(st + kABytes + q * 16 * row_b, abox, 8 * row_b, a_box_layout(p.rank)), idesc_s,
                        (kb | q) != 0 ? 1u : 0u);
            umma_commit_pair(bar(EMPTY + s));
          }
          if (!stop) umma_commit_pair(bar(ACC_FULL + a));
          continue;
        }
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
            umma_pair(tmem + a * kBN, smem_desc(st + q * 32, 16, 1024, 2),
                      p.w_kn ? smem_desc(st + kABytes + q * 2048, 8192, 1024, 2)   // [N/64][K][64] MN-major
                             : smem_desc(st + kABytes + q * 32, 16, 1024, 2),
                      idesc, (kb | q) != 0 ? 1u : 0u);
          umma_commit_pair(bar(EMPTY + s));
        }
        const int nq = p.rank / 8;  // 16-byte chunks of a u row
        auto delta_mma = [&](uint32_t ua, uint32_t ba) {
          tc_fence_after();
          for (int q = 0; q < p.rank / 16; ++q)
            umma_pair(tmem + a * kBN, smem_desc(ua + q * 256, 128, uint32_t(nq) * 128, 0),
                      smem_desc(ba + q * 2048, p.rank * 128, 1024, 2), idesc_d, 1u);
        };
        int d = 0;
        if (!stop && dbuf && n_delta > 0 && dbuf_tile(it)) {  // the first blocks, from the delta buffer
          const int db = dk % kDeltaBufs;
          const int n_in = min(n_delta, n_dslots);
          if (!wait(bar(DFULL + db), (dk / kDeltaBufs) & 1)) {
            stop = true;
          } else {
            for (int i = 0; i < n_in; ++i) {
              const uint32_t src = s_delta + db * kDeltaBuf + i * 512u * uint32_t(p.rank);
              delta_mma(src, src + 256 * p.rank);
            }
            umma_commit_pair(bar(DEMPTY + db));
            ++dk;
            d = n_in;
          }
        }
        for (; d < n_delta && !stop; ++d, ++kk) {
          const int s = kk % kStages;
          if (!wait(bar(FULL + s), (kk / kStages) & 1)) {
            stop = true;
            break;
          }
          const uint32_t ua = s_stage0 + s * kStageBytes;
          delta_mma(ua, ua + kABytes);
          umma_commit_pair(bar(EMPTY + s));
        }
        if (!stop) umma_commit_pair(bar(ACC_FULL + a));
      }
      if (aborted_flag(s_abort)) {  // every issued MMA finishes before TMEM is released (bounded)
        umma_commit_pair_local(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [128 half, 128 half + 128) of the tile
    const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t my_out = s_out0 + (warp - 2) * kOutBuf;
    const uint32_t acc_empty = mapa_shared(bar(ACC_EMPTY), 0);  // the leader's
    // A shrink pass's u: for each segment of the pass with tokens in this CTA's 128 rows
    // and each module, its (128-row tile, segment) block, every row of it (the product
    // for rows in the segment, else 0), in the no-swizzle K-major operand layout the
    // delta MMA reads (8-element chunk q of row r at core matrix (r / 8, q)).  The two
    // warps of a lane quadrant take alternate boxes.  The writes are fenced for the
    // async proxy before the producer's copies read them.
    auto write_u = [&](const Item& it, int a, int32_t m0, int quad_, int half_) {
      const int2 qr = pair_range(p.tile_pairs, it.rb, p.n_segs);
      const int32_t e0 = it.pass * 2 * p.s_epc;
      const int32_t ne_p = min(2 * p.s_epc, qr.y - qr.x - e0);
      const int32_t ne_h = (ne_p + 1) / 2;
      const int R = p.rank;
      const int row = quad_ * 32 + lane;
      const int64_t t = int64_t(m0) + row;
      T* u = static_cast<T*>(p.u_out);
      // the pass's entries (at most 2 * s_epc <= 16), lane e holding entry e, fetched in
      // one round of loads and handed out by shuffles
      int ej = -1, emask = 0;
      int64_t es0 = 0, es1 = 0;
      if (lane < ne_p) {
        const int q = qr.x + e0 + lane;
        ej = __ldg(p.pairs + 3 * q);
        emask = __ldg(p.pairs + 3 * q + 2);
        if (ej >= 0 && ej < p.n_segs) {
          es0 = __ldg(p.seg_start + ej);
          es1 = es0 + __ldg(p.seg_len + ej);
        }
      }
      int box = 0;
      for (int owner = 0; owner < 2; ++owner) {
        for (int i = 0; i < ne_h; ++i) {
          const int32_t e = owner * ne_h + i;  // entry within the pass
          for (int m = 0; m < p.n_mod; ++m, ++box) {
            if ((box & 1) != half_ || e >= ne_p) continue;
            const int j = __shfl_sync(0xffffffffu, ej, e);
            const int mask = __shfl_sync(0xffffffffu, emask, e);
            if (j < 0 || j >= p.n_segs || !((mask >> rank) & 1)) continue;  // no block of this CTA's tile
            const int64_t s0 = __shfl_sync(0xffffffffu, es0, e), s1 = __shfl_sync(0xffffffffu, es1, e);
            const bool in = t >= s0 && t < s1 && t < p.m_rows;
            T* blk = u + (int64_t(m) * p.n_blk + 2 * it.rb + int32_t(rank) + j) * (int64_t(kBM) * R);
            const uint32_t col = uint32_t(owner) * uint32_t(ne_h * p.n_mod * R) + uint32_t((i * p.n_mod + m) * R);
            for (int c = 0; c < R / 16; ++c) {
              float v[16];
              tmem_ld16(taddr + a * kBN + col + c * 16, v);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint4 pk;
                pk.x = Pack2<T>::pack(in ? v[h * 8 + 0] : 0.f, in ? v[h * 8 + 1] : 0.f);
                pk.y = Pack2<T>::pack(in ? v[h * 8 + 2] : 0.f, in ? v[h * 8 + 3] : 0.f);
                pk.z = Pack2<T>::pack(in ? v[h * 8 + 4] : 0.f, in ? v[h * 8 + 5] : 0.f);
                pk.w = Pack2<T>::pack(in ? v[h * 8 + 6] : 0.f, in ? v[h * 8 + 7] : 0.f);
                *reinterpret_cast<uint4*>(blk + ((row >> 3) * (R / 8) + c * 2 + h) * 64 + (row & 7) * 8) = pk;
              }
            }
          }
        }
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
    };
    // LoRA: the B factors of every delta block this pair will stage, prefetched into L2
    // once by the epilogue warps after their first item (a shrink pass's u must not wait
    // for it), each warp taking every kEpiWarps-th tile of the pair's sequence, so the
    // copy-issuing thread never waits on the table reads behind these addresses
    auto prefetch_walk = [&]() {
      if (!kLora || lane != 0) return;
      Sched<kLora> walk(p, pair, n_pairs);
      Item w;
      for (int i = 0; walk.next(p, w);) {
        if (w.shrink) continue;
        if (i++ % kEpiWarps != warp - 2) continue;
        const int pmod = w.c * kBN / p.module_cols;
        if (pmod >= p.n_mod) continue;
        const int2 qr = pair_range(p.tile_pairs, w.rb, p.n_segs);
        for (int q = qr.x; q < qr.y; ++q) {
          const int32_t slot = __ldg(p.pairs + 3 * q + 1);
          if (slot >= 0 && slot < p.n_slots)
            prefetch_l2(static_cast<const T*>(p.b_ptr[pmod]) + int64_t(slot) * p.b_slot_stride,
                        uint32_t(p.rank) * uint32_t(p.module_cols) * 2u);
        }
      }
    };
    const T* bias = static_cast<const T*>(p.bias);
    Sched<kLora> sched(p, pair, n_pairs);
    Item item;
    // accumulate: this lane's row of y at a chunk's 32 columns, loaded one chunk ahead
    // (the tile's first chunk before its accumulator is waited for); rows past m read
    // as 0 and are stored nowhere
    const int c_begin = half * (kBN / kOutCols / 2), c_end = c_begin + kBN / kOutCols / 2;
    auto load_y = [&](uint4 (&dst)[4], int32_t m0_, int col0_) {
      const int64_t r = int64_t(m0_) + quad * 32 + lane;
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.y_in) + r * p.ldy + col0_);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = r < p.m_rows ? src[q] : make_uint4(0u, 0u, 0u, 0u);
    };
    uint4 y_next[4];
    for (int n_it = 0; sched.next(p, item); ++n_it) {
      if (n_it == 1) prefetch_walk();
      const int a = n_it & 1;
      const int32_t m0 = item.rb * (2 * kBM) + int32_t(rank) * kBM;
      const int32_t n0 = item.c * kBN;
      if constexpr (kAcc) load_y(y_next, m0, n0 + c_begin * kOutCols);
      bool ok = !aborted_flag(s_abort);
      if (ok && !mbar_wait(bar(ACC_FULL + a), (n_it >> 1) & 1)) {
        fail();
        ok = false;
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      if (item.shrink) {
        write_u(item, a, m0, quad, half);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (item.pass == sched.n_pass - 1) mbar_arrive(bar(U_READY));  // the block's u is complete
          mbar_arrive_cluster(acc_empty + a * 8);
        }
        continue;
      }
      for (int c = c_begin; c < c_end; ++c) {
        const int col0 = n0 + c * kOutCols;
        uint4 yq[4];
        if constexpr (kAcc) {
#pragma unroll
          for (int q = 0; q < 4; ++q) yq[q] = y_next[q];
          if (c + 1 < c_end) load_y(y_next, m0, col0 + kOutCols);
        }
        uint32_t v[32];
        tmem_ld32(taddr + a * kBN + c * kOutCols, v);
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
        if constexpr (kAcc) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t ws[4] = {yq[q].x, yq[q].y, yq[q].z, yq[q].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = Pack2<T>::unpack(ws[i]);
              bf[q * 8 + 2 * i] += f.x;
              bf[q * 8 + 2 * i + 1] += f.y;
            }
          }
        }
        uint32_t packed[16];
        if constexpr (kAct == LF_ACT_GELU) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 y = f2_add(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                                    make_float2(bf[2 * i], bf[2 * i + 1]));
            const float2 g = gelu2_fast(make_float2(round_through<T>(y.x), round_through<T>(y.y)));
            packed[i] = Pack2<T>::pack(g.x, g.y);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[i] = Pack2<T>::pack(__uint_as_float(v[2 * i]) + bf[2 * i], __uint_as_float(v[2 * i + 1]) + bf[2 * i + 1]);
        }
        // the store that last read this staging tile must be done with it
        if (lane == 0) tma_store_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q)  // SW64: 16-byte chunk q of row `lane` at q ^ ((lane >> 1) & 3)
          *reinterpret_cast<uint4*>(gbase + (my_out - base) + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&p.y_map, my_out, col0, m0 + quad * 32);
          tma_store_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty + a * 8);  // this warp's TMEM reads of the tile are done
    }
    if (lane == 0) tma_store_wait_all();
  }

  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its operands
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kBN) : "memory");
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
  // the shrink in the same launch (cache_a null: u was written before the launch)
  const void* cache_a;
  int64_t a_slot_stride, a_module_stride;
  const int32_t *seg_start, *seg_len;
};

static int linear_impl(const char* fn, void* stream, int dtype, const void* x, int64_t ldx, const void* w,
                       int64_t ldw, const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                       const LoraArgs* lora, int32_t* status, bool accumulate = false, bool w_kn = false) {
  if (dtype != LF_DTYPE_BF16 && dtype != LF_DTYPE_F16)
    return set_error(LF_ERR_UNSUPPORTED, "%s: dtype %d (bf16 or f16 only)", fn, dtype);
  if (act != LF_ACT_NONE && act != LF_ACT_GELU) return set_error(LF_ERR_INVALID, "%s: unknown act %d", fn, act);
  if (accumulate && (act != LF_ACT_NONE || lora != nullptr))
    return set_error(LF_ERR_INVALID, "%s: accumulation takes no activation and no LoRA", fn);
  if (m < 0 || m > INT32_MAX || n <= 0 || k <= 0 || n % kBN != 0 || k % kBK != 0)
    return set_error(LF_ERR_UNSUPPORTED, "%s: n %d must be a multiple of 256 and k %d of 64", fn, n, k);
  if (x == nullptr || w == nullptr || y == nullptr) return set_error(LF_ERR_INVALID, "%s: null x, w or y", fn);
  if (ldx < k || ldw < (w_kn ? n : k) || ldy < n)
    return set_error(LF_ERR_INVALID, "%s: a row stride is below its row", fn);
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
    if (L.cache_a != nullptr) {
      if (L.n_modules * L.rank > 128)
        return set_error(LF_ERR_UNSUPPORTED, "%s: n_modules * rank %d above 128; run lf_lora_shrink_blocked and "
                         "lf_linear_lora instead", fn, L.n_modules * L.rank);
      if (L.seg_start == nullptr || L.seg_len == nullptr || !aligned16(L.cache_a) || (L.a_slot_stride * 2) % 16 ||
          (L.a_module_stride * 2) % 16 || (L.n_slots > 1 && L.a_slot_stride < int64_t(k) * L.rank))
        return set_error(LF_ERR_INVALID, "%s: null segment arrays, or cache_a alignment or slot stride", fn);
    }
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
  if (w_kn) {  // w (k, n): blocks of 64 output columns, each K rows of 128 bytes
    const cuuint64_t dims[3] = {64, cuuint64_t(k), cuuint64_t(n / 64)};
    const cuuint64_t strides[2] = {cuuint64_t(ldw) * 2, 128};
    const cuuint32_t box[3] = {64, kBK, kBN / 128};
    if ((rc = tmap(&p.w_map, 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "w"))) return rc;
  } else {
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(ldw) * 2};
    const cuuint32_t box[2] = {kBK, kBN / 2};
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
    // u: n_modules x n_blk blocks of 128 x R, each viewed as R/2 rows of 256 elements
    p.n_blk = int32_t((m + kBM - 1) / kBM + L.n_segs);
    {
      const cuuint64_t dims[3] = {256, R / 2, cuuint64_t(L.n_modules) * cuuint64_t(p.n_blk)};
      const cuuint64_t strides[2] = {512, cuuint64_t(kBM) * R * 2};
      const cuuint32_t box[3] = {256, R / 2, 1};
      if ((rc = tmap(&p.u_map, 3, L.u, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE, "u"))) return rc;
    }
    for (int i = 0; i < L.n_modules; ++i) {
      const void* b = static_cast<const uint8_t*>(L.cache_b) + int64_t(L.modules[i]) * L.b_module_stride * 2;
      const int64_t ss = L.n_slots == 1 ? int64_t(L.module_cols) * L.rank : L.b_slot_stride;
      p.b_ptr[i] = b;
      p.b_slot_stride = ss;
      // (64 columns, R rows, column block, slot): one box holds a CTA's two blocks
      const cuuint64_t dims[4] = {64, R, cuuint64_t(L.module_cols / 64), cuuint64_t(L.n_slots)};
      const cuuint64_t strides[3] = {cuuint64_t(L.module_cols) * 2, 128, cuuint64_t(ss) * 2};
      const cuuint32_t box[4] = {64, R, kBN / 128, 1};
      if ((rc = tmap(&p.b_map[i], 4, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "b"))) return rc;
    }
    if (L.cache_a != nullptr) {
      // every module's A box of a segment in one copy: the modules' A factors must lie
      // evenly spaced in the cache (q/k/v as 0, 1, 2), or there is one module
      const int64_t es = 2;
      int d = L.n_modules > 1 ? L.modules[1] - L.modules[0] : 1;
      for (int i = 2; i < L.n_modules && d > 0; ++i)
        if (L.modules[i] - L.modules[i - 1] != d) d = 0;
      const int64_t mstride = L.n_modules == 1 ? int64_t(k) * L.rank * es : int64_t(d) * L.a_module_stride * es;
      if (d <= 0 || mstride < int64_t(k) * L.rank * es || mstride % 16 != 0)
        return set_error(LF_ERR_UNSUPPORTED, "%s: the modules' A factors are not evenly spaced in the cache; "
                         "run lf_lora_shrink_blocked and lf_linear_lora instead", fn);
      const void* a = static_cast<const uint8_t*>(L.cache_a) + int64_t(L.modules[0]) * L.a_module_stride * es;
      const int64_t ss = L.n_slots == 1 ? int64_t(k) * L.rank : L.a_slot_stride;
      const cuuint64_t dims[4] = {R, cuuint64_t(k), cuuint64_t(L.n_modules), cuuint64_t(L.n_slots)};
      const cuuint64_t strides[3] = {cuuint64_t(R) * es, cuuint64_t(mstride), cuuint64_t(ss) * es};
      const cuuint32_t box[4] = {R, 64, cuuint32_t(L.n_modules), 1};
      if ((rc = tmap(&p.a_map, 4, a, dims, strides, box, a_tma_swizzle(L.rank), "a"))) return rc;
      p.shrink = 1;
      p.s_epc = 128 / (L.n_modules * L.rank);
      p.u_out = const_cast<void*>(L.u);
      p.seg_start = L.seg_start;
      p.seg_len = L.seg_len;
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
  p.n_rb = int32_t((m + 2 * kBM - 1) / (2 * kBM));
  p.n_tiles = int64_t(p.n_rb) * p.n_tiles_n;
  p.n_kb = k / kBK;
  p.act = act;
  p.w_kn = w_kn ? 1 : 0;
  p.status = status;
  p.y_in = accumulate ? y : nullptr;
  p.ldy = ldy;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == LF_DTYPE_BF16;
  const int mode = lora != nullptr ? 1 : accumulate ? 2 : 0;
  const bool gelu = act == LF_ACT_GELU;
  auto kern = mode == 1   ? (gelu ? (bf ? linear_kernel<__nv_bfloat16, true, false, LF_ACT_GELU>
                                         : linear_kernel<__half, true, false, LF_ACT_GELU>)
                                  : (bf ? linear_kernel<__nv_bfloat16, true, false, LF_ACT_NONE>
                                        : linear_kernel<__half, true, false, LF_ACT_NONE>))
              : mode == 2 ? (bf ? linear_kernel<__nv_bfloat16, false, true, LF_ACT_NONE>
                                : linear_kernel<__half, false, true, LF_ACT_NONE>)
              : gelu      ? (bf ? linear_kernel<__nv_bfloat16, false, false, LF_ACT_GELU>
                                : linear_kernel<__half, false, false, LF_ACT_GELU>)
                          : (bf ? linear_kernel<__nv_bfloat16, false, false, LF_ACT_NONE>
                                : linear_kernel<__half, false, false, LF_ACT_NONE>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(linear)");
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  // as many pairs as can be resident at once (a GPC with an odd SM count leaves one idle)
  static int resident_pairs[64][6] = {};
  int pairs = sms / 2;
  if (dev >= 0 && dev < 64) {
    int& resident = resident_pairs[dev][2 * mode + (gelu ? 1 : 0)];
    if (resident == 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(unsigned(sms & ~1));
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = kSmemBytes;
      q.attrs = attr;
      q.numAttrs = 1;
      int nc = 0;
      resident = (cudaOccupancyMaxActiveClusters(&nc, kern, &q) == cudaSuccess && nc > 0) ? nc : sms / 2;
    }
    pairs = resident < sms / 2 ? resident : sms / 2;
  }
  if (p.n_tiles < pairs) pairs = int(p.n_tiles);
  if (p.shrink) {  // each pair takes a contiguous range of tiles (and its blocks' shrink passes)
    p.tiles_per_pair = (p.n_tiles + pairs - 1) / pairs;
    pairs = int((p.n_tiles + p.tiles_per_pair - 1) / p.tiles_per_pair);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return cuda_error(e, "launch linear");
  count_launch();
  return LF_OK;
}

extern "C" int lf_linear(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                         const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                         int32_t* status) {
  return linear_impl("lf_linear", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, act, nullptr, status);
}

extern "C" int lf_linear_accumulate(void* stream, int dtype, const void* x, int64_t ldx, const void* w,
                                    int64_t ldw, const void* bias, void* y, int64_t ldy, int64_t m, int n, int k,
                                    int32_t* status) {
  return linear_impl("lf_linear_accumulate", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, LF_ACT_NONE,
                     nullptr, status, true);
}

extern "C" int lf_linear_lora(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                              int w_kn, const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                              const void* u, int rank, const void* cache_b, int64_t b_slot_stride,
                              int64_t b_module_stride, int n_slots, int n_modules, const int32_t* modules,
                              int module_cols, int n_segs, const int32_t* tile_pairs, const int32_t* pairs,
                              int32_t* status) {
  LoraArgs L{u, rank, cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules, module_cols,
             n_segs, tile_pairs, pairs, nullptr, 0, 0, nullptr, nullptr};
  return linear_impl("lf_linear_lora", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, act, &L, status, false,
                     w_kn != 0);
}

extern "C" int lf_linear_lora_shrink(void* stream, int dtype, const void* x, int64_t ldx, const void* w,
                                     int64_t ldw, int w_kn, const void* bias, void* y, int64_t ldy, int64_t m, int n,
                                     int k,
                                     int act, void* u, int rank, const void* cache_a, int64_t a_slot_stride,
                                     int64_t a_module_stride, const void* cache_b, int64_t b_slot_stride,
                                     int64_t b_module_stride, int n_slots, int n_modules, const int32_t* modules,
                                     int module_cols, const int32_t* seg_start, const int32_t* seg_len, int n_segs,
                                     const int32_t* tile_pairs, const int32_t* pairs, int32_t* status) {
  if (cache_a == nullptr) return set_error(LF_ERR_INVALID, "lf_linear_lora_shrink: null cache_a");
  LoraArgs L{u, rank, cache_b, b_slot_stride, b_module_stride, n_slots, n_modules, modules, module_cols,
             n_segs, tile_pairs, pairs, cache_a, a_slot_stride, a_module_stride, seg_start, seg_len};
  return linear_impl("lf_linear_lora_shrink", stream, dtype, x, ldx, w, ldw, bias, y, ldy, m, n, k, act, &L, status,
                     false, w_kn != 0);
}
