// Internal declarations shared by the LateFuse-B200 translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/latefuse_b200.h"

namespace lf {

constexpr int kMaxModules = 4;

// Kernel parameter blocks (passed as __grid_constant__, so the TMA descriptors
// live in parameter space as cp.async.bulk.tensor requires).
struct alignas(64) ShrinkTcParams {
  CUtensorMap x_map;                 // 2D {hidden, n_tokens}, box {64, 128}, SW128
  CUtensorMap a_map[kMaxModules];    // 3D {rank, hidden, n_slots}, box {rank, 64, 1}
  int64_t n_tokens;
  int32_t hidden;
  int32_t kchunk;                    // hidden columns handled by one CTA of the cluster
  int32_t n_modules;
  int32_t n_slots;
  uint32_t tmem_cols;
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  const int32_t* tiles;              // row tiles to process (NULL: all)
  void* u;                           // (n_modules, n_tokens, rank)
  int32_t* status;
};

struct alignas(64) ExpandTcParams {
  CUtensorMap y_map;                 // 2D {y_cols, n_tokens}, box {64, 128}, SW128
  CUtensorMap b_map[kMaxModules];    // 3D {hidden, rank, n_slots}, box {64, rank, 1}, SW128
  int64_t n_tokens;
  int64_t y_col_off[kMaxModules];
  int32_t hidden;
  int32_t n_modules;
  int32_t n_slots;
  int32_t accumulate;
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  const int32_t* tiles;              // row tiles to process (NULL: all)
  int32_t n_tiles;                   // grid rows (tiles listed, or all tiles)
  const void* u;                     // (n_modules, n_tokens, rank)
  int32_t* status;
};

// Persistent expand over single-segment tiles (see lf_lora_persist.cu).
struct alignas(64) ExpandPersistParams {
  CUtensorMap y_map;                 // 2D {y_cols, n_tokens}, box {64, 128}, SW128
  CUtensorMap r_map;                 // into mode with a residual: like y_map, over r
  CUtensorMap b_map[kMaxModules];    // 3D {hidden, rank, n_slots}, box {64, rank, 1}, SW128
  CUtensorMap u_map;                 // 2D {rank, n_modules * n_tokens}, box {rank, 128}, swizzle by rank
  int64_t n_tokens;
  int64_t y_col_off[kMaxModules];
  int32_t n_modules;
  int32_t n_col_blocks;              // hidden / NT
  int32_t n_slots;
  int32_t n_tiles;                   // tile records
  const int32_t* tiles;              // records {tile, first segment, segment count, first slot}
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  int32_t* status;
  // into mode: y = round(round(r + bias) + delta) written to every row of every
  // record's tiles (r and bias each optional), instead of y += delta in place
  int32_t into;
  int32_t has_r;
  const void* bias;                  // y_cols entries, or null
};

// Persistent shrink over the tile records (see lf_lora_persist.cu).
struct alignas(64) ShrinkPersistParams {
  CUtensorMap x_map;                 // 2D {hidden, n_tokens}, box {64, 128}, SW128
  CUtensorMap a_map[kMaxModules];    // 3D {rank, hidden, n_slots}, box {rank, 64, 1}
  // a_modules_map: 4D {rank, hidden, n_modules, n_slots}, box {rank, 64, n_modules, 1},
  // set (a_one_box = 1) when the modules' A factors lie equally spaced in the cache,
  // so that one copy per segment and K block stages every module's box
  CUtensorMap a_modules_map;
  int32_t a_one_box;
  int64_t n_tokens;
  int32_t hidden;
  int32_t n_modules;
  int32_t n_slots;
  int32_t n_tiles;                   // tile records
  int32_t kmax;                      // segments multiplied per pass over a tile's x
  uint32_t acc_cols;                 // TMEM columns of one accumulator set (kmax * n_modules * rank, padded)
  const int32_t* tiles;              // records {tile, first segment, segment count, first slot}
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  void* u;                           // (n_modules, n_tokens, rank), or blocked (u_blocked)
  int32_t* status;
  // u_blocked: u as (n_modules, ceil(n_tokens / 128) + n_segs) blocks of 128 rows
  // x rank, block (tile + segment) holding the tile's rows of that segment (other
  // rows 0), each in the canonical no-swizzle K-major layout of a tcgen05 operand
  // (8-row x 16-byte core matrices, K direction 128 bytes apart, row groups
  // 16 * rank bytes apart), so that one bulk copy stages a (tile, segment) pair
  int32_t u_blocked;
};

// One-launch late-fusion delta over the tile records (see lf_lora_fused.cu).
struct alignas(64) FusedApplyParams {
  CUtensorMap x_map;                 // 2D {hidden, n_tokens}, box {64, 128}, SW128
  CUtensorMap a_map[kMaxModules];    // 3D {rank, hidden, n_slots}, box {rank, 64, 1}
  CUtensorMap a_modules_map;         // 4D, as ShrinkPersistParams (a_one_box = 1)
  CUtensorMap ys_map;                // 2D {y_cols, n_tokens}, box {64, 32}, SW128: one warp's rows (reductions)
  CUtensorMap b_map[kMaxModules];    // 3D {hidden, rank, n_slots}, box {64, rank, 1}, SW128
  int32_t a_one_box;
  int64_t n_tokens;
  int64_t y_col_off[kMaxModules];
  int32_t hidden;
  int32_t n_modules;
  int32_t n_slots;
  int32_t n_tiles;                   // tile records
  int32_t n_chunks;                  // column chunks per record (items = n_tiles * n_chunks)
  int32_t chunk_cols;                // hidden / n_chunks, a multiple of 128
  int32_t kmax;                      // segments per round (one shrink pass + one expand pass)
  int32_t stages;                    // x ring stages (each an x box with the round's A boxes)
  int32_t stage_bytes;
  int32_t b_stages;                  // B ring stages (each the round's B boxes of one 128-column step)
  int32_t b_stage_bytes;
  int32_t out_bufs;                  // staging boxes per epilogue warp (1 or 2)
  uint32_t u_cols;                   // TMEM columns of the u accumulator (kmax * n_modules * rank, padded)
  uint32_t d_col;                    // first TMEM column of the 128-column delta accumulators
  int32_t d_bufs;                    // delta accumulators (2 or 3)
  uint32_t tmem_alloc;               // TMEM columns allocated
  const int32_t* tiles;              // records {tile, first segment, segment count, first slot}
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  int32_t* status;
};

// Packed varlen attention, head_dim 64 (see lf_attention.cu).
struct alignas(64) AttnParams {
  CUtensorMap qkv_map;               // 2D {ld_qkv, n_tokens}, box {64, 128}, SW128
  const int4* items;                 // {row_start, len, q_tile, 0} per (sequence, 128-query tile)
  int32_t n_items;
  int64_t n_tokens;                  // rows of qkv and out: records must lie inside
  int32_t n_heads;
  int32_t q_col, k_col, v_col;       // column of head 0's q / k / v in a qkv row
  void* out;                         // (n_tokens, ld_out): head h at columns [64 h, 64 h + 64)
  int64_t ldo;
  float scale_log2;                  // softmax scale * log2(e)
  int32_t* status;
};

struct NormParams {
  const void* a;
  const void* b;       // may be null
  int64_t lda, ldb;
  const void* vec;     // row vector added to every row, may be null (not with b)
  const void* gamma;
  const void* beta;
  float eps;
  int64_t n_rows;
  int32_t hidden;
  void* out;
  int64_t ldo;
  // embeddings (MODE 3): row r is LN(round(round(a[ia[r]] + c[ic[r]]) + b[ib[r]])),
  // tables a / b / c with n_a / n_b / n_c rows; an index outside its table reads row 0
  // and sets LF_STATUS_BAD_SLOT
  const int32_t* ia;
  const int32_t* ib;
  const int32_t* ic;
  const void* c;
  int64_t ldc;
  int64_t n_a, n_b, n_c;
  int32_t* status;
};

struct SimtParams {
  const void* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
  int64_t n_tokens;
  int32_t hidden;
  int32_t rank;
  const void* cache_a[kMaxModules];  // per-module base for slot 0
  const void* cache_b[kMaxModules];
  int64_t a_slot_stride;
  int64_t b_slot_stride;
  int64_t y_col_off[kMaxModules];
  int32_t n_modules;
  int32_t n_slots;
  const int32_t* seg_start;
  const int32_t* seg_len;
  const int32_t* seg_slot;
  int32_t n_segs;
  void* u;
  int32_t accumulate;
  int32_t* status;
};

// error reporting (thread-local message, see lf_last_error)
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
void count_launch();

// tcgen05 path
int run_shrink_tc(int dtype, const ShrinkTcParams& p, int rank, int csize, int n_tiles, cudaStream_t s);
int run_expand_tc(int dtype, const ExpandTcParams& p, int rank, int nt, cudaStream_t s);
size_t shrink_tc_smem(int dtype, int rank, int kchunk, int n_mod);
uint32_t shrink_tc_tmem_cols(int rank, int n_mod);
CUtensorMapSwizzle a_tma_swizzle(int rank);

// after_shrink: launched right behind the persistent shrink that writes u, as
// its programmatic dependent (the expand starts early and waits for u).
int run_expand_persist(int dtype, const ExpandPersistParams& p, int rank, int nt, bool after_shrink,
                       cudaStream_t s);
int run_shrink_persist(int dtype, const ShrinkPersistParams& p, int rank, cudaStream_t s);
// Fills p's ring and round sizes for this rank and launches; LF_ERR_UNSUPPORTED
// (nothing launched) when no configuration fits.
int run_lora_fused(int dtype, FusedApplyParams& p, int rank, cudaStream_t s);
// lf_lora_apply with its argument checks; allow_fused = false keeps it on the shrink
// and expand launches, whose u goes through `workspace`.
int apply_entry(bool allow_fused, void* stream, int dtype, const void* x, int64_t ldx, void* y, int64_t ldy,
                int64_t n_tokens, int hidden, int rank, const void* cache_a, int64_t a_slot_stride,
                int64_t a_module_stride, const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                int n_slots, int n_modules, const int32_t* modules, const int64_t* y_col_offsets,
                const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot, int n_segs,
                const int32_t* tiles, int n_tiles, int n_multi, void* workspace, size_t workspace_bytes,
                int32_t* status);

// CUDA-core path
int run_shrink_simt(int dtype, const SimtParams& p, cudaStream_t s);
int run_expand_simt(int dtype, const SimtParams& p, cudaStream_t s);

// driver entry points
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled get_encode_tiled();
void* get_driver_fn(const char* name);

// options
int option_force_simt();
int option_shrink_cluster();

}  // namespace lf
