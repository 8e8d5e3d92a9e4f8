/*
 * latefuse_b200.h -- C ABI of the B200-native late-fusion LoRA serving path.
 *
 * LateFuse serves many LoRA-adapted encoders in one mixed-tenant forward pass:
 * every row (sequence) of a batch carries its own tenant, whose low-rank delta
 *     y = W0 x + B_t (A_t x)
 * is added to each targeted projection output, and whose classification head is
 * applied to the pooled output.  The reference library does this in pure
 * PyTorch (torch.bmm shrink/expand plus an index_select gather of per-tenant
 * factors, and a zero-padded head bmm).  This library replaces those ops with
 * hand-written sm_100a kernels reached through the plain C entry points below:
 * plain pointers, sizes and a cudaStream_t passed as void*; no exceptions cross
 * the boundary; every function returns LF_OK (0) or an LF_ERR_* code, with a
 * message available from lf_last_error().
 *
 * Memory ownership: the caller owns every buffer passed in (inputs, outputs,
 * workspaces, the adapter cache).  The LoRA, head and gather entry points
 * allocate nothing; only the lf_arena_* functions allocate (they back the
 * adapter cache with CUDA virtual memory so it can grow without moving).
 *
 * Layout conventions
 *   dtype            LF_DTYPE_F32 / LF_DTYPE_BF16 / LF_DTYPE_F16 for every
 *                    floating-point buffer of one call.
 *   tokens           a batch is n_tokens rows; row t of x starts at x + t*ldx
 *                    (elements).  A padded (B, S) batch is n_tokens = B*S.
 *   segments         seg_start/seg_len/seg_slot (device int32 arrays, n_segs
 *                    entries) name runs of consecutive tokens that share one
 *                    adapter slot.  Segments are sorted by start and do not
 *                    overlap; tokens covered by no segment get no delta.  For a
 *                    padded (B, S) batch, segment b is {b*S, S, slot of row b}.
 *   adapter cache    for slot s and op-module m the shrink factor A is the
 *                    (hidden x rank) row-major matrix at
 *                        cache_a + s*a_slot_stride + modules[m]*a_module_stride
 *                    and the expand factor B is the (rank x hidden) row-major
 *                    matrix at
 *                        cache_b + s*b_slot_stride + modules[m]*b_module_stride
 *                    (strides in elements).  These are the reference's
 *                    LoraWeight.wa[m][layer] / wb[m][layer] layouts
 *                    (src/latefuse/weights/store.py:22-39), so a per-tenant
 *                    adapter is addressed in place, never gathered.
 *   tiles            optional device array of n_tiles tile records, 16-byte
 *                    aligned, one per row tile (tokens [i*LF_TILE_TOKENS,
 *                    (i+1)*LF_TILE_TOKENS)) that holds any segment token:
 *                    int32 {i, index of the first segment overlapping the
 *                    tile, number of segments overlapping it, slot of that
 *                    first segment}.  Tiles of pure padding are then never
 *                    launched and each tile's loads issue after one read.
 *                    Records of tiles with exactly one segment come first;
 *                    the last n_multi records are the tiles with several.
 *                    NULL (n_tiles = 0) means every tile (segments found by
 *                    binary search).  A record that disagrees with the
 *                    segment arrays gives its tile no delta and sets
 *                    LF_STATUS_BAD_SEGMENT.
 *   status           optional device int32; kernels OR LF_STATUS_* bits into
 *                    it instead of faulting on a bad slot id, a bad segment or
 *                    a wait that timed out.
 */
#ifndef LATEFUSE_B200_H
#define LATEFUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define LF_OK 0
#define LF_ERR_INVALID 1     /* an argument is out of range or inconsistent */
#define LF_ERR_UNSUPPORTED 2 /* valid, but not a configuration this build handles */
#define LF_ERR_CUDA 3        /* a CUDA runtime or driver call failed */
#define LF_ERR_WORKSPACE 4   /* the workspace passed is smaller than required */
#define LF_ERR_DRIVER 5      /* a driver entry point could not be resolved */

/* dtypes */
#define LF_DTYPE_F32 0
#define LF_DTYPE_BF16 1
#define LF_DTYPE_F16 2

/* tokens per row tile of the LoRA kernels (the unit of the optional tile list) */
#define LF_TILE_TOKENS 128

/* device status bits (written by kernels into *status) */
#define LF_STATUS_BAD_SLOT 1    /* a segment named a slot outside [0, n_slots) */
#define LF_STATUS_BAD_SEGMENT 2 /* a segment lies outside [0, n_tokens) or has len < 0 */
#define LF_STATUS_TIMEOUT 4     /* an on-chip wait exceeded its time limit; output invalid */
#define LF_STATUS_BAD_HEAD 8    /* a head row range lies outside [0, head_rows) */

/* pooling modes of lf_head_forward (src/latefuse/ops/pooling.py:23) */
#define LF_POOL_CLS 0    /* hidden[b, 0, :] */
#define LF_POOL_MEAN 1   /* mask-weighted mean over the sequence, count clamped at 1e-9 */
#define LF_POOL_NONE 2   /* hidden is already pooled: (B, H) */

/* options for lf_set_option */
#define LF_OPT_FORCE_SIMT 1     /* 1: run the CUDA-core LoRA kernels even where the
                                   tcgen05 kernels apply (cross-checking) */
#define LF_OPT_SHRINK_CLUSTER 2 /* 0 = automatic, else the shrink's split-K cluster size */
#define LF_OPT_REQUIRE_TC 3     /* 1: fail with LF_ERR_UNSUPPORTED instead of running the
                                   CUDA-core kernels where the tcgen05 kernels do not apply */
#define LF_OPT_PERSISTENT 4     /* 0: do not use the persistent expand kernel (default 1) */
#define LF_OPT_FUSED_APPLY 5    /* 1 (default): lf_lora_apply runs as one launch (shrink and
                                   expand in one kernel, u kept on chip) where that kernel
                                   applies and the call has one module; 2: also with several
                                   modules; 0: a shrink launch and an expand launch */
#define LF_OPT_FUSED_SPLIT 6    /* 0 = automatic, else the column chunks each tile record of
                                   the one-launch lf_lora_apply is split into */

/* ------------------------------------------------------------------------ */
/* library                                                                   */
/* ------------------------------------------------------------------------ */

/* Version string of this build. */
const char* lf_version(void);

/* Message describing the last failing call on this host thread ("" if none). */
const char* lf_last_error(void);

/* 1 if `device` is an sm_100 GPU this build has kernels for, else 0. */
int lf_device_supported(int device);

/* Set a process-wide option (LF_OPT_*).  Returns LF_ERR_INVALID for an unknown key. */
int lf_set_option(int key, int value);

/* Number of kernels this library has launched in this process. */
uint64_t lf_launch_count(void);

/* ------------------------------------------------------------------------ */
/* LoRA delta (replaces LoraOps.shrink / expand / output,                   */
/* src/latefuse/ops/lora.py:29-80, the hook body                            */
/* src/latefuse/model/hf_wrapper.py:212-217 and the "bert" engine block     */
/* src/latefuse/model/encoder.py:70-80)                                     */
/* ------------------------------------------------------------------------ */

/* Shrink: u[m][t][:] = x[t] . A(slot(t), m) for every token t of a segment
 * (0 for tokens in no segment), rounded to dtype.  u is a dense
 * (n_modules, n_tokens, rank) device buffer.  Replaces LoraOps.shrink
 * (src/latefuse/ops/lora.py:29-57, torch.bmm(x, a_weights, out=_out_A)) and the
 * per-layer torch.cat / index_select gather of A that feeds it
 * (src/latefuse/weights/batch.py:186-220): A is read in place from the cache.
 * n_modules <= 4; `modules` is a host array of n_modules cache module indices. */
int lf_lora_shrink(void* stream, int dtype,
                   const void* x, int64_t ldx,
                   int64_t n_tokens, int hidden, int rank,
                   const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                   int n_slots, int n_modules, const int32_t* modules,
                   const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                   int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                   void* u, int32_t* status);

/* lf_lora_shrink writing u in the blocked layout lf_linear_lora reads: one
 * block of 128 * rank elements per (128-token tile b, segment g) pair, at
 * (m * (ceil(n_tokens / 128) + n_segs) + b + g) * 128 * rank for module m,
 * holding the tile's rows that lie in segment g (other rows 0).  Inside a block
 * the 8 elements [8q, 8q + 8) of tile row r sit at
 * ((r / 8) * (rank / 8) + q) * 64 + (r % 8) * 8 (the canonical no-swizzle
 * K-major operand layout of tcgen05.mma, so one bulk copy stages a block).
 * u holds n_modules * (ceil(n_tokens / 128) + n_segs) * 128 * rank elements;
 * blocks of pairs without shared tokens are not written.  Needs tile records,
 * rank 16/32/64, bf16/f16 (LF_ERR_UNSUPPORTED otherwise). */
int lf_lora_shrink_blocked(void* stream, int dtype,
                           const void* x, int64_t ldx,
                           int64_t n_tokens, int hidden, int rank,
                           const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                           int n_slots, int n_modules, const int32_t* modules,
                           const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                           int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                           void* u, int32_t* status);

/* Expand: for every token t and op-module m,
 *     delta = round(u[m][t] . B(slot(t), m))
 *     y[t, y_col_offsets[m] + n] = accumulate ? round(y + delta) : delta     (n < hidden)
 * where round() rounds to dtype (the reference materialises the delta in the
 * model dtype before adding it).  Tokens in no segment get delta = 0.  Replaces
 * LoraOps.expand (src/latefuse/ops/lora.py:59-75, torch.bmm(out_A, b_weights,
 * out=_out_B)) plus `output + owner.lora_ops.output`
 * (src/latefuse/model/hf_wrapper.py:217; src/latefuse/model/encoder.py:80).
 * `modules` and `y_col_offsets` are host arrays of n_modules entries. */
int lf_lora_expand(void* stream, int dtype,
                   const void* u,
                   void* y, int64_t ldy,
                   int64_t n_tokens, int hidden, int rank,
                   const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                   int n_slots, int n_modules, const int32_t* modules,
                   const int64_t* y_col_offsets,
                   const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                   int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                   int accumulate, int32_t* status);

/* Device workspace bytes lf_lora_apply needs for these sizes. */
size_t lf_lora_workspace_bytes(int dtype, int64_t n_tokens, int rank, int n_modules);

/* Fused late-fusion delta: shrink into `workspace`, then expand-accumulate into
 * y, i.e. y[t, off_m + :] += B(slot(t), m)^T (A(slot(t), m)^T x[t]) for up to 4
 * modules that share the input x (query/key/value of one layer share one read of
 * x).  One call replaces, per layer, the reference's cat -> bmm -> bmm -> add
 * sequence of every hook (src/latefuse/model/hf_wrapper.py:213-217).  With one
 * module, tile records, bf16/f16, rank 8/16/32/64, hidden a multiple of 128,
 * 16-byte aligned buffers and x not overlapping y, it runs as ONE kernel that keeps u on chip
 * (the workspace is then unused; LF_OPT_FUSED_APPLY = 0 selects the shrink and
 * expand launches, which give the same bits); otherwise as a shrink launch into
 * `workspace` and an expand launch. */
int lf_lora_apply(void* stream, int dtype,
                  const void* x, int64_t ldx,
                  void* y, int64_t ldy,
                  int64_t n_tokens, int hidden, int rank,
                  const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                  const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                  int n_slots, int n_modules, const int32_t* modules,
                  const int64_t* y_col_offsets,
                  const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                  int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                  void* workspace, size_t workspace_bytes, int32_t* status);

/* Bytes of the static device scratch behind lf_lora_apply_noalloc (8 MiB). */
#define LF_NOALLOC_SCRATCH_BYTES (8u << 20)

/* lf_lora_apply without a caller-provided workspace, for callers that cannot
 * allocate device memory (a host framework that owns every allocation, or code
 * that must not call cudaMalloc while serving).  It has no counterpart in the
 * reference.  Same arguments, contract and results as lf_lora_apply minus the
 * workspace.  It always runs lf_lora_apply's shrink launch and expand launch
 * (never the one-launch kernel), and the shrink output lives in a file-scope device array of
 * LF_NOALLOC_SCRATCH_BYTES that every GPU using the library holds until the
 * process exits.  Batches needing more scratch than that
 * (lf_lora_workspace_bytes) are rejected with LF_ERR_WORKSPACE.  The first call
 * on each device, with that device current, resolves the array's device
 * address (cudaGetSymbolAddress); make it before any stream capture.  All calls
 * share the array, so calls whose kernels can overlap on the GPU race; order
 * them on one stream.  It allocates nothing. */
int lf_lora_apply_noalloc(void* stream, int dtype,
                          const void* x, int64_t ldx,
                          void* y, int64_t ldy,
                          int64_t n_tokens, int hidden, int rank,
                          const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                          const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                          int n_slots, int n_modules, const int32_t* modules,
                          const int64_t* y_col_offsets,
                          const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                          int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                          int32_t* status);

/* The delta written into a fresh output for a GEMM to accumulate onto:
 *     y[t, off_m + n] = round(round(r[t, off_m + n] + bias[off_m + n]) + delta)
 * for every token of every tile the records name (r and bias may each be NULL,
 * read as 0; rows of a record's tile in no segment get round(r + bias)).  A
 * caller then adds the projection with a beta = 1 GEMM (y += x W^T), so the
 * projection output is written once and never re-read for the delta, and a
 * residual r that a LayerNorm would add is already in y.  Same shrink, factor
 * layout and segment rules as lf_lora_apply; it needs tile records whose tiles
 * cover every token (segments covering [0, n_tokens)), bf16 or f16, rank 8, 16,
 * 32 or 64, hidden a multiple of 128, and 16-byte aligned buffers and strides
 * (LF_ERR_UNSUPPORTED otherwise); r must not alias y.  It fuses, per layer, the
 * reference's projection bias, `output + owner.lora_ops.output`
 * (src/latefuse/model/hf_wrapper.py:217; src/latefuse/model/encoder.py:80) and,
 * with r, the residual add before LayerNorm (src/latefuse/model/encoder.py:137). */
int lf_lora_apply_into(void* stream, int dtype,
                       const void* x, int64_t ldx,
                       const void* r, int64_t ldr,
                       const void* bias,
                       void* y, int64_t ldy,
                       int64_t n_tokens, int hidden, int rank,
                       const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                       const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                       int n_slots, int n_modules, const int32_t* modules,
                       const int64_t* y_col_offsets,
                       const int32_t* seg_start, const int32_t* seg_len, const int32_t* seg_slot,
                       int n_segs, const int32_t* tiles, int n_tiles, int n_multi,
                       void* workspace, size_t workspace_bytes, int32_t* status);

/* ------------------------------------------------------------------------ */
/* Adapter cache                                                            */
/* ------------------------------------------------------------------------ */

/* Gather: dst[i][:] = src + slots[i]*slot_stride + offset, n_elems elements of
 * elem_bytes each, for i < n.  Bit-exact materialisation of per-row adapter
 * factors, the equivalent of IndexSelectBatchAssembler.assemble_lora's
 * wa[m].index_select(0, idx) (src/latefuse/weights/batch.py:186-203); the
 * serving path never needs it (kernels read the cache by slot). */
int lf_cache_gather(void* stream, const void* src, int64_t slot_stride, int64_t offset,
                    int64_t n_elems, int elem_bytes, int n_slots,
                    const int32_t* slots, int n, void* dst, int32_t* status);

/* Copy nbytes from src (host or device) into slot `slot` of a cache whose slots
 * are slot_stride_bytes apart, at byte offset `offset` within the slot, on
 * `stream`.  Registration of a pre-packed adapter
 * (src/latefuse/weights/store.py:158-167 AdapterStore.insert). */
int lf_cache_write_slot(void* stream, void* cache_base, int64_t slot_stride_bytes, int slot,
                        int n_slots, size_t offset, const void* src, size_t nbytes);

/* Growable device arena backing the slot cache: reserves reserve_bytes of
 * device virtual address space and maps physical memory on demand, so the cache
 * grows without moving (views handed out earlier stay valid).  The reference
 * instead repacks the whole store after every registration
 * (src/latefuse/tasks/base.py:181-190, src/latefuse/weights/batch.py:163-170). */
int lf_arena_create(int device, size_t reserve_bytes, void** handle);
int lf_arena_grow(void* handle, size_t mapped_bytes);   /* ensure >= mapped_bytes are mapped */
void* lf_arena_base(void* handle);
size_t lf_arena_mapped_bytes(void* handle);
int lf_arena_destroy(void* handle);

/* ------------------------------------------------------------------------ */
/* Pooling, normalisation and per-tenant heads                              */
/* ------------------------------------------------------------------------ */

/* One kernel per batch: pooling (pool_tokens, src/latefuse/ops/pooling.py:36-73)
 * -> optional L2 normalisation (F.normalize(p=2, eps=1e-12),
 * src/latefuse/tasks/embedding.py:69-70) -> optional per-tenant head, a
 * gather-GEMV over a packed head cache: for row b the head is rows
 * [head_off[b], head_off[b] + head_n[b]) of coef (head_rows x hidden) and bias,
 *     logits[b][j] = round(round(pooled[b] . coef[off+j]) + bias[off+j])   j < n
 *     logits[b][j] = 0                                                      n <= j < n_max
 * which is the zero-padded bmm + add of LRHeadOps.predict_proba
 * (src/latefuse/ops/head.py:50-51) after HeadStore.assemble
 * (src/latefuse/tasks/heads.py:125-158) without materialising the padding; and
 * probs[b][:n] = softmax over the row's own n logits (max-shifted), or the
 * sigmoid when n == 1 (src/latefuse/tasks/classification.py:72-84,109-119),
 * 0 in padded lanes.
 *
 *   hidden     (B, S, H) with row strides (ld_batch, ld_seq) for CLS/MEAN, or
 *              (B, H) with row stride ld_batch for LF_POOL_NONE
 *   mask       (B, S) int64 attention mask (1 = real token); may be NULL for
 *              CLS/NONE and for MEAN when there is no padding
 *   pooled_out (B, H) dtype or NULL: the pooled rows, before normalisation
 *   normed_out (B, H) dtype or NULL: the L2-normalised pooled rows
 *   coef/bias  NULL to skip the head; else head_off/head_n device int32 (B,)
 *   logits_out (B, n_max) dtype, probs_out (B, n_max) float32 (either may be NULL)
 */
int lf_head_forward(void* stream, int dtype,
                    const void* hidden, int64_t ld_batch, int64_t ld_seq,
                    const int64_t* mask, int batch, int seq, int hidden_size,
                    int pooling,
                    void* pooled_out, void* normed_out,
                    const void* coef, const void* bias, int64_t head_rows,
                    const int32_t* head_off, const int32_t* head_n, int n_max,
                    void* logits_out, float* probs_out,
                    int32_t* status);

/* The same heads for the padding-free forward, whose hidden states are packed
 * (n_tokens, H) with row stride ld: row b is token row_index[b] (its first, CLS,
 * token; NULL: row b).  With pooler_w (H x H) and pooler_b the rows first go
 * through the encoder's pooler,
 *     pooled[b] = round(tanh(round(hidden[row_index[b]] . pooler_w^T + pooler_b)))
 * (the HF pooler the reference's "auto" pooling returns,
 * src/latefuse/model/hf_wrapper.py:337-342, src/latefuse/model/encoder.py:281:
 * nn.Linear then tanh), written to
 * pooled_out, which is then required; then normalisation / head / softmax as
 * lf_head_forward with LF_POOL_NONE.  This fuses the reference classifier's CLS
 * gather, pooler and padded head bmm (src/latefuse/tasks/classification.py:42-119,
 * src/latefuse/ops/head.py:50-51) into one call of two launches (the head
 * kernel is a programmatic dependent of the pooler). */
int lf_head_forward_rows(void* stream, int dtype,
                         const void* hidden, int64_t ld, const int32_t* row_index,
                         int batch, int hidden_size,
                         const void* pooler_w, const void* pooler_b,
                         void* pooled_out, void* normed_out,
                         const void* coef, const void* bias, int64_t head_rows,
                         const int32_t* head_off, const int32_t* head_n, int n_max,
                         void* logits_out, float* probs_out,
                         int32_t* status);

/* ------------------------------------------------------------------------
 * Projection GEMM
 * ------------------------------------------------------------------------ */

#define LF_ACT_NONE 0
#define LF_ACT_GELU 1   /* exact erf GELU, ACT2FN["gelu"] */

/* y = act(x w^T + bias) for x (m, k), w (n, k) (an nn.Linear weight), y (m, n),
 * row-major with row strides ldx / ldw / ldy (elements); bias has n entries or
 * is NULL.  bf16 or f16, f32 accumulation; the sum is rounded to dtype, then for
 * LF_ACT_GELU gelu_f32 of that rounded value is rounded again (torch's
 * F.linear followed by F.gelu).  Replaces the encoder's projections
 * (src/latefuse/model/encoder.py: q/k/v, attention output, FFN up with its GELU
 * at :122,139, FFN down).  n % 256 == 0, k % 64 == 0, pointers and strides
 * 16-byte aligned (LF_ERR_UNSUPPORTED / LF_ERR_INVALID otherwise). */
int lf_linear(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
              const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act, int32_t* status);

/* y = y + x w^T + bias, in place: the projection accumulated onto y's current
 * values (cuBLAS's beta = 1), summed in f32 and rounded once; bias may be NULL.
 * Shapes, dtypes and alignment as lf_linear.  Replaces the encoder's FFN output
 * projection onto its residual (src/latefuse/model/encoder.py:139-141,
 * `output(intermediate) + h`, with the bias added where the caller chooses). */
int lf_linear_accumulate(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                         const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int32_t* status);

/* lf_linear with the late-fusion LoRA delta in the same accumulator:
 *     y[t, c] = act(round(x[t] . w[c] + bias[c] + u[i][t] . B(slot(t), i)[:, c - i * module_cols]))
 * for output column block i = c / module_cols < n_modules (columns of blocks
 * past n_modules get no delta), with u the shrink output in the blocked layout
 * of lf_lora_shrink_blocked (n_segs as there) and B read in place from the slot
 * cache (cache module modules[i], (rank, module_cols) row-major per slot, as
 * lf_lora_expand reads it).  tile_pairs / pairs (device int32) list, for each
 * 256-token tile q (the rows one CTA pair computes), the segments with tokens in
 * it: entries tile_pairs[q] .. tile_pairs[q + 1] - 1 of pairs, each
 * {segment, slot, halves} with bit r of halves set when the segment has tokens in
 * the tile's 128-token half r, in segment order (latefuse_b200.lora.SegmentTable
 * builds them).  The delta is not rounded
 * separately: the result is rounded once, where the reference rounds the
 * projection and the delta apart and then their sum
 * (src/latefuse/model/hf_wrapper.py:217, `output + lora_ops.output`; the fused
 * q/k/v and attention-output projections of src/latefuse/model/encoder.py:70-80).
 * Tokens in no segment, or in a segment whose slot is out of range, get no
 * delta.  rank 16, 32 or 64; module_cols a multiple of 256 dividing n.
 * w_kn = 0: w is (n, k), the nn.Linear weight, as for lf_linear.  w_kn = 1: w is
 * (k, n) row-major (its transpose, ldw >= n), read in the same operand form as the
 * cache's B factors (results agree to the dtype's rounding; the speed is the same). */
int lf_linear_lora(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw, int w_kn,
                   const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                   const void* u, int rank, const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                   int n_slots, int n_modules, const int32_t* modules, int module_cols, int n_segs,
                   const int32_t* tile_pairs, const int32_t* pairs, int32_t* status);

/* lf_linear_lora with the shrink in the same launch: u = round(x A(slot(t), i)) for
 * every segment and module i is computed by the GEMM's own CTA pairs (a pass over each
 * 256-token block's x against its segments' A factors, read in place from the slot
 * cache like lf_lora_shrink_blocked reads them: cache module modules[i], (hidden, rank)
 * row-major per slot, hidden = k) and written to u, the caller's buffer in the blocked
 * layout of lf_lora_shrink_blocked, before the block's projection tiles add
 * u B in their accumulators.  Replaces the two calls lf_lora_shrink_blocked +
 * lf_linear_lora (the reference's hook body, src/latefuse/model/hf_wrapper.py:212-217,
 * around the projection): one launch, x read once per block pass.  seg_start /
 * seg_len (device int32, n_segs) are the segment table; the other arguments are
 * lf_linear_lora's.  Needs n_modules * rank <= 128 and the modules' A factors evenly
 * spaced in the cache (or one module); LF_ERR_UNSUPPORTED otherwise. */
int lf_linear_lora_shrink(void* stream, int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw, int w_kn,
                          const void* bias, void* y, int64_t ldy, int64_t m, int n, int k, int act,
                          void* u, int rank, const void* cache_a, int64_t a_slot_stride, int64_t a_module_stride,
                          const void* cache_b, int64_t b_slot_stride, int64_t b_module_stride,
                          int n_slots, int n_modules, const int32_t* modules, int module_cols,
                          const int32_t* seg_start, const int32_t* seg_len, int n_segs,
                          const int32_t* tile_pairs, const int32_t* pairs, int32_t* status);

/* ------------------------------------------------------------------------
 * Encoder elementwise ops around the projections
 * ------------------------------------------------------------------------ */

/* out = LayerNorm(round(a + b)) * gamma + beta over rows of `hidden` elements
 * (b may be NULL: plain LayerNorm).  Replaces the encoder's
 * `LayerNorm(sublayer_out + residual)` (src/latefuse/model/encoder.py:137,141)
 * and the embeddings' LayerNorm (:275), i.e. torch's add followed by
 * nn.LayerNorm: the sum is rounded to dtype, mean and biased variance are
 * taken in f32, the result is rounded to dtype.  Instead of b, `vec` (hidden
 * entries, may be NULL, not together with b) is one row added to every row:
 * LayerNorm(round(a + vec)), for a projection whose GEMM has already
 * accumulated onto the residual and whose bias is still to be added.
 * hidden % 8 == 0, hidden <= 4096; pointers and row strides (elements)
 * 16-byte aligned; gamma/beta/vec in dtype.  out may alias a or b. */
int lf_add_layernorm(void* stream, int dtype, const void* a, int64_t lda, const void* b, int64_t ldb,
                     const void* vec, const void* gamma, const void* beta, float eps, int64_t n_rows,
                     int hidden, void* out, int64_t ldo);

/* The encoder's embeddings and their LayerNorm in one pass over gathered rows:
 *     e = round(round(word[ids[r]] + type[types[r]]) + pos[positions[r]])
 *     out[r] = LayerNorm(e) with gamma, beta, eps
 * (each sum rounded to dtype as torch rounds it: src/latefuse/model/encoder.py:270-282,
 * the HF embeddings `inputs_embeds + token_type_embeddings`, `+ position_embeddings`,
 * `LayerNorm`).  ids / positions / types are device int32 (types may be NULL: row 0);
 * an index outside its table reads row 0 and sets LF_STATUS_BAD_SLOT in status.
 * Layout rules as lf_add_layernorm. */
int lf_embed_layernorm(void* stream, int dtype, const void* word, int64_t ld_word, int64_t n_word,
                       const int32_t* ids, const void* pos, int64_t ld_pos, int64_t n_pos,
                       const int32_t* positions, const void* type, int64_t ld_type, int64_t n_type,
                       const int32_t* types, const void* gamma, const void* beta, float eps,
                       int64_t n_rows, int hidden, void* out, int64_t ldo, int32_t* status);

/* out = x * 0.5 * (1 + erf(x / sqrt(2))) in f32, rounded to dtype: the exact
 * GELU of the FFN (ACT2FN["gelu"], src/latefuse/model/encoder.py:122,139).
 * n % 8 == 0; x and out 16-byte aligned; out may alias x. */
int lf_gelu(void* stream, int dtype, const void* x, void* out, int64_t n);

/* Self-attention of packed sequences (no padding): for every sequence, head h
 * and query row i,  out[i][h] = softmax(scale * q_i . k_j over the sequence's
 * keys j) @ v.  Replaces the encoder's masked attention
 * (src/latefuse/model/encoder.py:82-98: scores, additive padding mask, f32
 * softmax, probs @ v) on a padding-free batch.  q, k and v of token t, head h
 * are the 64 elements at columns q_col + 64 h (k_col, v_col) of row t of qkv
 * (row stride ld_qkv elements; the fused projection output).  `items` is a
 * device int32 array of n_items records {row_start, len, q_tile, 0}, one per
 * (sequence, 128-query tile), 16-byte aligned; ordering them longest sequence
 * first balances the work.  head_dim must be 64; dtype bf16 or f16; column
 * offsets multiples of 64.  out row t, head h at columns [64 h, 64 h + 64).
 * A record outside [0, n_tokens) (or with len < 0, or a q_tile past its length)
 * sets LF_STATUS_BAD_SEGMENT and stores nothing; a zero length stores nothing. */
int lf_attention_varlen(void* stream, int dtype, const void* qkv, int64_t ld_qkv, int64_t n_tokens,
                        int64_t q_col, int64_t k_col, int64_t v_col, int n_heads, int head_dim,
                        const int32_t* items, int n_items, float scale, void* out, int64_t ld_out,
                        int32_t* status);

#ifdef __cplusplus
}
#endif

#endif /* LATEFUSE_B200_H */
