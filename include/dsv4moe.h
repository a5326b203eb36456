/*
 * dsv4moe — C ABI of the B200 (sm_100a) routed-expert MoE library.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream passed as
 * `void*` (a cudaStream_t; NULL = legacy default stream), returns 0 or a
 * negative DSV4_E* code, and never throws.  Device buffers are owned by the
 * caller.  Work is enqueued asynchronously on the given stream; a kernel that
 * detects bad input or a timed-out wait records the code in a device status
 * word that the host reads with dsv4_moe_status().  dsv4_last_error_string()
 * describes the last failure of the calling thread.
 *
 * Each declaration names the reference interface it replaces
 * (ErnestW2019/deepseek-v4-flash-offload, file:line).
 */
#ifndef DSV4MOE_H
#define DSV4MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV4_ABI_VERSION 2

#define DSV4_OK 0
#define DSV4_EINVAL (-1)      /* bad shape, pointer or argument */
#define DSV4_ENOMEM (-2)      /* workspace / pool / slot budget too small */
#define DSV4_ECUDA (-3)       /* CUDA runtime or driver error */
#define DSV4_ETIMEOUT (-4)    /* a bounded device-side wait ran out */
#define DSV4_ENCCL (-5)       /* collective failure (expert parallel) */
#define DSV4_ENOTFOUND (-6)   /* expert not registered or not resident */
#define DSV4_EUNSUPPORTED (-7)

/* router score functions (deepseek_v4.py:126-131) */
#define DSV4_SCORE_SOFTMAX 0
#define DSV4_SCORE_SIGMOID 1
#define DSV4_SCORE_SQRTSOFTPLUS 2

/* expert compute profiles: PROFILE=bf16|a4w4, DSV4_MXFP4_GMM (deepseek_v4.py:28-32) */
#define DSV4_PROFILE_BF16 0
#define DSV4_PROFILE_A4W4 1

/* token row formats of the expert-parallel dispatch (no counterpart in the
 * reference, which sends bf16 through its all-to-all):
 *   BF16: H bf16 values (2H bytes);
 *   FP8:  H E4M3 bytes, then H/128 scale exponent bytes (e + 127, scale 2^e),
 *         the bf16 profile's activation quantisation;
 *   MXFP4: H/2 bytes of E2M1 codes (low nibble = even column), then H/32
 *         E8M0 scale bytes, the a4w4 profile's;
 * each row padded to a multiple of 16 bytes (dsv4_ep_row_bytes). */
#define DSV4_ROWS_BF16 0
#define DSV4_ROWS_FP8 1
#define DSV4_ROWS_MXFP4 2

const char* dsv4_last_error_string(void);
int dsv4_abi_version(void);

/* ------------------------------------------------------------------------ *
 * Packed expert slot layout.
 * One expert = w1/w3 [I, H/2] + w2 [H, I/2] packed E2M1 (low nibble = even k)
 * and E8M0 per-32 scales, stored as ONE contiguous slot:
 *   [w13 packed (w1 rows then w3 rows) | w2 packed | w13 scales | w2 scales]
 * The packed weights are tiled into contiguous 16 KiB blocks of 256 rows x
 * 128 elements (one TMA box each): for w13 a block holds 128 rows of w1 and
 * the same 128 rows of w3, for w2 two consecutive 128-row tiles.  The scales
 * are re-tiled into 512-byte atoms (128 rows x 4 scale bytes, row r at
 * (r%32)*16 + (r/32)*4), two per block, that the tensor cores read directly.
 * Replaces the six per-expert host tensors of ExpertBank.register
 * (offload.py:59-68) and their per-call stacking (deepseek_v4.py:218-223).
 * ------------------------------------------------------------------------ */
int64_t dsv4_expert_slot_bytes(int32_t hidden, int32_t inter);
/* host-side pack of the checkpoint tensors into one slot (CPU memory) */
int dsv4_pack_expert_host(const uint8_t* w1p, const uint8_t* w1s, const uint8_t* w2p, const uint8_t* w2s,
                          const uint8_t* w3p, const uint8_t* w3s, int32_t hidden, int32_t inter,
                          uint8_t* slot_out);
/* inverse of dsv4_pack_expert_host (CPU memory); used by get_packed views */
int dsv4_unpack_expert_host(const uint8_t* slot, int32_t hidden, int32_t inter, uint8_t* w1p, uint8_t* w1s,
                            uint8_t* w2p, uint8_t* w2s, uint8_t* w3p, uint8_t* w3s);

/* ------------------------------------------------------------------------ *
 * Element-wise ops.
 * ------------------------------------------------------------------------ */
/* dequant_fp4_weight (npu_ops.py:142-158): [rows, k/2] packed E2M1 +
 * [rows, k/32] E8M0 -> [rows, k] bf16, bit-exact. */
int dsv4_dequant_mxfp4(const uint8_t* w_packed, const uint8_t* scale, void* out_bf16, int64_t rows, int64_t k,
                       void* stream);
/* ExpertBank._dequant_on_device (offload.py:77-84) from a packed slot:
 * w1/w3 -> [I, H] bf16, w2 -> [H, I] bf16. */
int dsv4_slot_dequant(const uint8_t* slot, int32_t hidden, int32_t inter, void* w1_bf16, void* w2_bf16,
                      void* w3_bf16, void* stream);
/* act_quant(x, 128, "ue8m0", None, inplace=True) (npu_ops.py:73-98):
 * in-place FP8-E4M3 round trip of bf16 [rows, cols], bit-exact. */
int dsv4_act_quant_fp8_rt(void* x_bf16, int64_t rows, int64_t cols, void* stream);
/* npu_dynamic_mx_quant(x, dst_type=F4) (deepseek_v4.py:212, 240): bf16
 * [rows, cols] -> packed E2M1 [rows, cols/2] + E8M0 [rows, cols/32];
 * scale = floor(log2(amax/6)), elements round-to-nearest-even, saturating. */
int dsv4_act_quant_mxfp4(const void* x_bf16, int64_t rows, int64_t cols, uint8_t* q_packed, uint8_t* scale,
                         void* stream);

/* ------------------------------------------------------------------------ *
 * Router: OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148).
 * logits = float(x) @ gate_w^T; scores by score_func; experts = top-k of
 * scores + bias (or tid2eid[input_ids] when tid2eid != NULL, the table
 * [vocab_size, topk]; a token id outside [0, vocab_size) gets expert id
 * n_experts for every pick, which the layer's align rejects); weights =
 * unbiased scores, renormalised when renormalize != 0, times route_scale.
 * Indices come out in descending biased-score order (ties: lower id first).
 * The logits are fp32: decode batches on the FP32 pipes; from 256 tokens
 * (with n_experts >= 128) on the tensor cores, the gate split into three
 * bf16 terms that sum to it exactly (DSV4_ROUTE_TC=0 keeps the FP32 pipes).
 * If a device-side wait of the tensor-core kernel runs out, every index is
 * written as n_experts (out of range) so that the layer's align rejects it.
 * dsv4_route_workspace_bytes covers both paths: the fp32 partial logits, and
 * from 256 tokens also the three bf16 gate terms (6 * n_experts * hidden B).
 * ------------------------------------------------------------------------ */
int64_t dsv4_route_workspace_bytes(int64_t n_tokens, int32_t hidden, int32_t n_experts);
int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                    const int64_t* input_ids, int64_t vocab_size, int64_t n_tokens, int32_t hidden,
                    int32_t n_experts, int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                    float* weights_out, int32_t* indices_out, void* workspace, int64_t workspace_bytes,
                    void* stream);

/* Router that allocates nothing; it has no counterpart in the reference.
 * For callers that cannot allocate device memory at routing time (a serving
 * engine whose cache pool already holds nearly all free HBM, or a C caller
 * without a device allocator).  Same arguments as dsv4_route_topk minus
 * the workspace.  Its results equal dsv4_route_topk's up to the fp32
 * summation order of the logits (it adds 4 partial sums of H/4 each, the
 * workspace router H/128 of them, or uses the tensor cores from 256
 * tokens), so an expert pair whose biased scores tie to within rounding
 * may be picked differently.  The logits scratch is a fixed 1 MiB device
 * array inside the library, so n_tokens * n_experts must not exceed
 * DSV4_ROUTE_NOALLOC_MAX_LOGITS (larger calls return DSV4_EINVAL).
 * The first call on a device resolves the array's address on that device;
 * make it before any stream capture.  All calls share the array: calls that
 * overlap on the GPU race on it. */
#define DSV4_ROUTE_NOALLOC_MAX_LOGITS 65536
int dsv4_route_topk_noalloc(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                            const int64_t* input_ids, int64_t vocab_size, int64_t n_tokens, int32_t hidden,
                            int32_t n_experts, int32_t topk, int32_t score_func, int32_t renormalize,
                            float route_scale, float* weights_out, int32_t* indices_out, void* stream);

/* Tensor-core rate of the grouped GEMM's MMA kinds on `device` (no
 * counterpart in the reference, which quotes no tensor peak): kind 0 =
 * tcgen05 kind::mxf4 block-scaled (the a4w4 profile), 1 = kind::mxf8f6f4
 * with E2M1 x E4M3 (the bf16 profile); M = 128, N = n, `iters` k-tiles of 128
 * per SM, back to back from shared memory.  Synchronous; writes dense TFLOP/s
 * and the timed milliseconds. */
int dsv4_mma_peak(int32_t kind, int32_t n, int64_t iters, int32_t device, double* tflops_out, double* ms_out);

/* ------------------------------------------------------------------------ *
 * moe_align (deepseek_v4.py:154-164): stable counting sort of the T*k
 * (token, slot) assignments by expert id.  sorted_flat[pos] = t*k + j,
 * inv[t*k + j] = pos, offsets = exclusive prefix of counts (E+1 entries),
 * active = ascending ids with count > 0, *n_active their number.  An index
 * of -1 is an empty assignment (inv = -1, no error: the padding rows of the
 * expert-parallel exchange); any other index outside [0, n_experts) sets
 * DSV4_EINVAL in *status (device word).
 * ------------------------------------------------------------------------ */
int dsv4_moe_align(const int32_t* indices, int64_t n_tokens, int32_t topk, int32_t n_experts, int32_t* counts,
                   int32_t* offsets, int32_t* sorted_flat, int32_t* inv, int32_t* active, int32_t* n_active,
                   int* status, void* stream);

/* ------------------------------------------------------------------------ *
 * Routed-expert layer: _routed / _routed_mxfp4 (deepseek_v4.py:150-245).
 * A plan binds the layer dims, the HBM slot arena (n_slots packed slots of
 * dsv4_expert_slot_bytes each, 256-byte aligned) and a workspace, and builds
 * the TMA descriptors once.  dsv4_moe_forward then runs, on `stream`:
 * align -> activation quant + gather -> fused gate/up GEMM with SwiGLU,
 * route weight and activation re-quant -> down GEMM -> deterministic
 * combine (ascending expert order per token, fp32) -> y bf16 [T, H].
 * route_weights/route_indices are the router outputs [T, k];
 * slot_of_expert[e] is the arena slot holding expert e (or -1).  A token
 * whose k indices are all -1 (empty assignments) gets no output row: its
 * row of y is left as it was.
 * ------------------------------------------------------------------------ */
typedef struct dsv4_moe_plan dsv4_moe_plan;
int64_t dsv4_moe_workspace_bytes(int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                                 int64_t max_tokens);
int dsv4_moe_plan_create(dsv4_moe_plan** out, int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                         int64_t max_tokens, float swiglu_limit, uint8_t* slot_arena, int64_t n_slots,
                         void* workspace, int64_t workspace_bytes);
int dsv4_moe_plan_destroy(dsv4_moe_plan* plan);
int dsv4_moe_forward(dsv4_moe_plan* plan, int32_t profile, const void* x_bf16, int64_t n_tokens,
                     const float* route_weights, const int32_t* route_indices, const int32_t* slot_of_expert,
                     void* y_bf16, void* stream);
/* The router of the plan's layer (OffloadDeepseekV4MoE._route,
 * deepseek_v4.py:118-148; the same arguments and results as
 * dsv4_route_topk) for a decode batch of fewer than 256 tokens (and at most
 * the plan's max_tokens), with its scratch in the plan's workspace: partial
 * logits, a grid-wide barrier and the top-k in one launch when the grid fits
 * on the GPU at once, else dsv4_route_topk's two kernels.  The plan's status
 * (dsv4_moe_status) reports a barrier that timed out (DSV4_ETIMEOUT; the
 * affected picks are expert id n_experts, which the forward rejects).
 * Calls on one plan must not overlap on the GPU (they share its workspace,
 * as forwards do). */
int dsv4_moe_route(dsv4_moe_plan* plan, const void* x_bf16, const float* gate_w, const float* bias,
                   const int32_t* tid2eid, const int64_t* input_ids, int64_t vocab_size, int64_t n_tokens,
                   int32_t topk, int32_t score_func, int32_t renormalize, float route_scale, float* weights_out,
                   int32_t* indices_out, void* stream);
/* The same layer for a batch whose token count is known only on the device
 * (the rows that expert parallelism received): the first *n_tokens_dev
 * (<= max_tokens) rows of x and of the router outputs are used.  y_bf16 may
 * be NULL: the combine is then skipped and the per-assignment output rows
 * stay in the plan (dsv4_moe_output_rows), in sorted order: row inv[a] of
 * `rows` is assignment a = t * topk + j.  No counterpart in the reference. */
int dsv4_moe_forward_rows(dsv4_moe_plan* plan, int32_t profile, const void* x_bf16, int64_t max_tokens,
                          const int32_t* n_tokens_dev, const float* route_weights, const int32_t* route_indices,
                          const int32_t* slot_of_expert, void* y_bf16, void* stream);
/* dsv4_moe_forward_rows without y whose down GEMM writes the output row of
 * assignment a = t * topk + j to assign_dst[a] (any memory this GPU can
 * store to, another GPU's included; null: dropped) straight from its
 * epilogue, instead of the plan's output rows.  No counterpart in the
 * reference (the expert-parallel return fused into the GEMM). */
int dsv4_moe_forward_scatter(dsv4_moe_plan* plan, int32_t profile, const void* x_bf16, int64_t max_tokens,
                             const int32_t* n_tokens_dev, const float* route_weights, const int32_t* route_indices,
                             const int32_t* slot_of_expert, void* const* assign_dst, void* stream);
/* dsv4_moe_forward_scatter on rows quantised at their source
 * (dsv4_ep_dispatch_q; x_format DSV4_ROWS_FP8 with the bf16 profile,
 * DSV4_ROWS_MXFP4 with a4w4, rows of dsv4_ep_row_bytes bytes): the layer
 * only gathers them, with the results of the bf16 rows they came from.
 * Plans without a shared expert.  No counterpart in the reference. */
int dsv4_moe_forward_scatter_q(dsv4_moe_plan* plan, int32_t profile, const void* x_rows, int32_t x_format,
                               int64_t max_tokens, const int32_t* n_tokens_dev, const float* route_weights,
                               const int32_t* route_indices, const int32_t* slot_of_expert, void* const* assign_dst,
                               void* stream);
/* Device pointers of the last forward's per-assignment output rows (bf16
 * [rows, hidden], sorted by expert) and of inv (int32 [n_tokens * topk]). */
int dsv4_moe_output_rows(dsv4_moe_plan* plan, void** rows_bf16, int32_t** inv);
/* ------------------------------------------------------------------------ *
 * Shared expert fused into the routed launches (the reference runs it as a
 * separate dense MLP, deepseek_v4.py:87-100 and 264-265; its math is
 * model_npu.py Expert in "fp8" mode and MoE.forward's
 * `y = y + self.shared_experts(x)`, model_npu.py:532).  Weights: w1 / w3
 * [I, H] and w2 [H, I] E4M3 with one E8M0 scale per 128 x 128 block
 * (dequant_fp8_weight, npu_ops.py:161-167), packed once into an FP8 slot of
 * dsv4_shared_slot_bytes (same pairs, blocks and scale atoms as the routed
 * slot, one byte per element).  A plan made with with_shared = 1 treats the
 * shared expert as one more assignment of every token (expert id n_experts,
 * weight 1, last in the combine, so the fp32 sum adds it after the routed
 * rows before the one bf16 rounding, as model_npu does): in the bf16 profile
 * inside the same launches; in the a4w4 profile (packed E2M1 activations for
 * the routed GEMMs) as a first pass of its own whose output the routed
 * combine adds last.  route_weights / route_indices stay [T, k]. */
int64_t dsv4_shared_slot_bytes(int32_t hidden, int32_t inter);
int dsv4_pack_shared_host(const uint8_t* w1, const uint8_t* s1, const uint8_t* w2, const uint8_t* s2,
                          const uint8_t* w3, const uint8_t* s3, int32_t hidden, int32_t inter, uint8_t* slot_out);
int64_t dsv4_moe_workspace_bytes_ex(int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                                    int64_t max_tokens, int32_t with_shared);
int dsv4_moe_plan_create_ex(dsv4_moe_plan** out, int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                            int64_t max_tokens, float swiglu_limit, uint8_t* slot_arena, int64_t n_slots,
                            void* workspace, int64_t workspace_bytes, int32_t with_shared);
int dsv4_moe_forward_shared(dsv4_moe_plan* plan, int32_t profile, const void* x_bf16, int64_t n_tokens,
                            const float* route_weights, const int32_t* route_indices,
                            const int32_t* slot_of_expert, const uint8_t* shared_slot, void* y_bf16, void* stream);
/* Synchronises `stream`, returns the plan's device status word (0 or a
 * DSV4_E* code recorded by a kernel) and clears it. */
int dsv4_moe_status(dsv4_moe_plan* plan, void* stream);
/* Combine in a given order (deepseek_v4.py:195-197 index_add_, ascending
 * expert id per token): y[t] = bf16(sum_j rows[order[t*k + j]]) summed in
 * float32 from zero in j order; order < 0 skips.  Used by the expert-
 * parallel path, whose received rows are not grouped by expert. */
int dsv4_moe_combine_ordered(const void* rows_bf16, const int32_t* order, int64_t n_tokens, int32_t topk,
                             int32_t hidden, void* y_bf16, void* stream);

/* Per-stage device timing (no counterpart in the reference, which has no
 * timing hooks).  When enabled, dsv4_moe_forward records CUDA events on its
 * stream between its stages; dsv4_moe_stage_times waits for the last
 * forward's events and writes up to n elapsed times in ms: [0] align,
 * [1] activation quant + gather, [2] gate/up GEMM, [3] down GEMM,
 * [4] combine. */
int dsv4_moe_enable_timing(dsv4_moe_plan* plan, int32_t enable);
int dsv4_moe_stage_times(dsv4_moe_plan* plan, float* ms_out, int32_t n);
/* Tokens per GEMM tile (no counterpart in the reference): 64 or 112, or 0
 * for the library's choice (112 when the batch has at least 16 assignments
 * per expert with a4w4, 32 with bf16, else 64; the environment variable
 * DSV4_GEMM_BN overrides it).  The tile is also the padding of each expert's row group.
 * Takes effect from the next dsv4_moe_forward on the plan. */
int dsv4_moe_set_gemm_tile(dsv4_moe_plan* plan, int32_t tokens_per_tile);
/* Gate/up and down GEMMs in one launch (1), as two launches (0), or the
 * library's choice (-1, the default: one launch with the 64-token decode
 * tile, two with the 112-token prefill tile; the environment variable
 * DSV4_FUSED_FFN=0|1 replaces the default).
 * The fused launch stores the h rows of each expert chunk and starts that
 * chunk's down tiles as soon as all of its gate/up tiles are stored; results
 * are identical.  With stage timing on, the fused launch's time is reported
 * as the gate/up stage and the down stage is empty.
 * No counterpart in the reference (npu_grouped_matmul runs per projection). */
int dsv4_moe_set_ffn_fusion(dsv4_moe_plan* plan, int32_t enable);
/* Device pointers of the plan's align outputs (valid after a forward):
 * counts[E], offsets[E+1], sorted_flat[P], inv[P], active[E], n_active[1]. */
int dsv4_moe_debug_align(dsv4_moe_plan* plan, int32_t** counts, int32_t** offsets, int32_t** sorted_flat,
                         int32_t** inv, int32_t** active, int32_t** n_active);

/* ------------------------------------------------------------------------ *
 * Expert slot cache: the LRU bookkeeping of ExpertBank.get_packed
 * (offload.py:103-129; the engine's get_packed, engine.py:90-97), host only.
 * Maps (layer, expert) to a slot of the device arena.  A lookup serves a
 * whole batch of keys that must be resident together: a hit moves its key
 * to the most-recently-used end; a miss takes a free slot (0, 1, ... first)
 * or evicts the least recently used key that is not part of the batch, and
 * reports miss_out[i] = 1 so that the caller copies the expert's packed slot
 * into slot_out[i].  More distinct keys than slots: DSV4_ENOMEM and nothing
 * changes.  Not thread-safe (one cache per bank, as the reference's dict).
 * ------------------------------------------------------------------------ */
typedef struct dsv4_slotcache dsv4_slotcache;
int dsv4_slotcache_create(dsv4_slotcache** out, int64_t n_slots);
int dsv4_slotcache_destroy(dsv4_slotcache* cache);
int dsv4_slotcache_lookup(dsv4_slotcache* cache, const int64_t* layer, const int64_t* expert, int64_t n,
                          int32_t* slot_out, uint8_t* miss_out);
/* slot of a resident key, or -1; does not change the LRU order */
int32_t dsv4_slotcache_slot_of(const dsv4_slotcache* cache, int64_t layer, int64_t expert);
/* out4 = {hits, misses, evictions, resident keys} (offload.py:135-146 stats) */
int dsv4_slotcache_stats(const dsv4_slotcache* cache, int64_t* out4);
/* resident keys, least recently used first (up to cap of them); *n_out = resident count */
int dsv4_slotcache_snapshot(const dsv4_slotcache* cache, int64_t* layer_out, int64_t* expert_out,
                            int32_t* slot_out, int64_t cap, int64_t* n_out);
/* forget every key (ExpertBank.invalidate); the statistics are kept */
int dsv4_slotcache_clear(dsv4_slotcache* cache);

/* ------------------------------------------------------------------------ *
 * Device-resident slot directory: the same LRU as the dsv4_slotcache_*
 * calls (the packed-expert cache of ExpertBank.get_packed,
 * offload.py:103-129, one layer's batch at a time), kept in HBM so that an
 * offloaded layer never waits for the host.  dsv4_slotdir_acquire enqueues on `stream`:
 *   resolve: the layer's [T*k] expert ids (-1 = empty) are walked in
 *     ascending id order; hits move to the most-recently-used end, misses
 *     take a free slot (lowest first) or evict the least recently used key
 *     outside the batch; the (layer, expert) -> slot table is updated;
 *   fetch: each missed expert is copied by the GPU from its page-locked host
 *     slot (registered with dsv4_slotdir_set_sources; the host memory must be
 *     mapped for the device, as all cudaHostAlloc memory is under unified
 *     addressing) into its arena slot.
 * dsv4_slotdir_table gives the device table of a layer (int32 [n_experts],
 * slot or -1), the slot_of_expert argument of dsv4_moe_forward.
 * Mode DSV4_SLOTDIR_PREFETCH (predicted experts of a later layer, typically
 * on a side stream while the current layer computes) evicts only slots older
 * than the last DEMAND batch and skips what does not fit; the caller orders
 * each demand acquire after the previous prefetch (an event) and each
 * prefetch after the demand acquire it must not disturb.  Counters (int64 x 8):
 * demand hits, misses, evictions; prefetch hits, fetched, evictions,
 * skipped; acquire calls.  A demand batch with more distinct experts than
 * slots records DSV4_ENOMEM (dsv4_slotdir_status) and changes nothing.
 * ------------------------------------------------------------------------ */
#define DSV4_SLOTDIR_DEMAND 0
#define DSV4_SLOTDIR_PREFETCH 1
#define DSV4_SLOTDIR_MAX_SLOTS 32768
typedef struct dsv4_slotdir dsv4_slotdir;
int64_t dsv4_slotdir_workspace_bytes(int32_t n_layers, int32_t n_experts, int64_t n_slots);
int dsv4_slotdir_create(dsv4_slotdir** out, int32_t n_layers, int32_t n_experts, uint8_t* slot_arena,
                        int64_t n_slots, int64_t slot_bytes, void* workspace, int64_t workspace_bytes);
int dsv4_slotdir_destroy(dsv4_slotdir* dir);
/* host (page-locked) address of each (layer, expert) packed slot; host arrays */
int dsv4_slotdir_set_sources(dsv4_slotdir* dir, int64_t n, const int32_t* layers, const int32_t* experts,
                             const void* const* host_slots);
int dsv4_slotdir_acquire(dsv4_slotdir* dir, int32_t layer, const int32_t* indices, int64_t n_assign, int32_t mode,
                         void* stream);
int dsv4_slotdir_table(dsv4_slotdir* dir, int32_t layer, int32_t** slot_of_out);
/* synchronises `stream`, then reads the eight counters */
int dsv4_slotdir_stats(dsv4_slotdir* dir, int64_t* out8, void* stream);
/* synchronises `stream`; returns and clears the directory's status word */
int dsv4_slotdir_status(dsv4_slotdir* dir, void* stream);
/* synchronises `stream`; per slot the key (layer * n_experts + expert, or -1)
 * and the recency stamp (larger = more recent, 0 = free) */
int dsv4_slotdir_snapshot(dsv4_slotdir* dir, int32_t* slot_key_out, int64_t* stamp_out, void* stream);
/* forget every resident key (asynchronous on `stream`); counters are kept */
int dsv4_slotdir_clear(dsv4_slotdir* dir, void* stream);

/* ------------------------------------------------------------------------ *
 * Expert-parallel dispatch packing (no counterpart in the reference, whose
 * expert-parallel size is 1, deepseek_v4.py:82).  Expert e lives on rank
 * expert_owner[e] (device int32 [n_experts]; NULL: e / (n_experts / world),
 * which then must divide).  Every rank sends cap = n_tokens * topk rows to
 * every peer, so the all-to-all has a fixed shape (graph-capturable).  For
 * assignment a = t*topk + j with destination d the slot is d*cap + its rank
 * among the assignments to d (stable):
 *   send_x[slot] = x[t], send_meta[slot] = (expert, bits of the weight),
 *   slot_of_assignment[a] = slot;
 * padding slots get send_meta = (-1, 0), an empty assignment.
 * ordered_slots[t*topk + j] lists token t's slots in ascending expert order
 * (-1 after the last), the order in which the returned rows are added.
 * send_x: [world*cap, hidden] bf16; send_meta: [world*cap, 2] int32;
 * slot_of_assignment, ordered_slots: [n_tokens*topk] int32.  An expert id
 * of -1 is skipped; any other id outside [0, n_experts) (or an owner outside
 * [0, world)) sets DSV4_EINVAL in *status and is dropped.
 * ------------------------------------------------------------------------ */
int dsv4_ep_dispatch_pack(const void* x_bf16, const float* route_weights, const int32_t* route_indices,
                          int64_t n_tokens, int32_t topk, int32_t hidden, int32_t n_experts, int32_t world,
                          const int32_t* expert_owner, void* send_x_bf16, int32_t* send_meta,
                          int32_t* slot_of_assignment, int32_t* ordered_slots, int* status, void* stream);

/* ------------------------------------------------------------------------ *
 * Expert-parallel exchange over NVLink peer memory (no counterpart in the
 * reference).  Each rank owns one device block; peers map it through CUDA
 * IPC and write into it directly.  A token crosses once per destination
 * rank that holds one of its experts, not once per expert.  Per step:
 *   dsv4_ep_dispatch: each source first publishes to every peer how many of
 *     its tokens go there, then writes each such token's row, its k picks
 *     with the other ranks' experts set to -1 (weight 0), and its source
 *     into the owner's block, compact: owner d holds the tokens of source s
 *     at sum_{s'<s} n[s'->d] + r (r = stable rank of the token among those
 *     of s with an expert on d); waits (bounded, DSV4_ETIMEOUT in *status)
 *     until every source published; the number of tokens received is then in
 *     the device word *n_recv (dsv4_ep_buffers).  ordered_assignments[t*k+j]
 *     lists token t's assignments a = t*k + j' in ascending expert order
 *     (-1 after the last), the order in which the returned rows are added;
 *   (the routed-expert layer runs on recv_x / recv_indices / recv_weights,
 *     [tokens, k], with the device count: dsv4_moe_forward_rows)
 *   dsv4_ep_return: the output of each received assignment (token j, pick
 *     s, an expert of this rank) back into its source's `back` row t*k + s,
 *     read as row row_of_assignment[j*k + s] of `rows` (the layer's sorted
 *     output rows and its inv; NULL: row j*k + s), then waits for every owner;
 *   dsv4_moe_combine_ordered(back, ordered_assignments, ...) gives the output.
 * Every call is an asynchronous device operation with a fixed launch shape,
 * so a step can be captured in a CUDA graph.  All ranks must make the same
 * calls in the same order.  Buffers: recv_x [world*max_tokens, hidden] bf16,
 * recv_indices / recv_weights [world*max_tokens, topk], back
 * [max_tokens*topk, hidden] bf16.  After a DSV4_ETIMEOUT the step's data are
 * undefined and a late peer may still write into this rank's block: destroy
 * the handle and create a new one.  The IPC handle is
 * dsv4_ep_ipc_handle_bytes() bytes; dsv4_ep_connect takes all ranks'
 * handles, rank-major.
 * ------------------------------------------------------------------------ */
typedef struct dsv4_ep dsv4_ep;
int dsv4_ep_ipc_handle_bytes(void);
int dsv4_ep_create(dsv4_ep** out, int32_t device, int32_t rank, int32_t world, int64_t max_tokens, int32_t topk,
                   int32_t hidden, void* ipc_handle_out);
int dsv4_ep_connect(dsv4_ep* ep, const void* all_handles);
int dsv4_ep_buffers(dsv4_ep* ep, void** recv_x_bf16, int32_t** recv_indices, float** recv_weights, int32_t** n_recv,
                    void** back_bf16);
int dsv4_ep_dispatch(dsv4_ep* ep, const void* x_bf16, const float* route_weights, const int32_t* route_indices,
                     int64_t n_tokens, int32_t n_experts, const int32_t* expert_owner, int32_t* ordered_assignments,
                     int* status, void* stream);
/* dsv4_ep_dispatch with the rows sent in a quantised format (DSV4_ROWS_FP8
 * for the bf16 profile, DSV4_ROWS_MXFP4 for a4w4): each token is quantised
 * once at its source exactly as the owner's layer would quantise it, so the
 * owner's results are unchanged and a row crosses NVLink in 4128 (FP8) or
 * 2176 (MXFP4) bytes instead of 8192 at H = 4096.  recv_x then holds rows of
 * dsv4_ep_row_bytes(row_format, hidden) bytes, which
 * dsv4_moe_forward_scatter_q takes.  No counterpart in the reference. */
int64_t dsv4_ep_row_bytes(int32_t row_format, int32_t hidden);
int dsv4_ep_dispatch_q(dsv4_ep* ep, const void* x_bf16, const float* route_weights, const int32_t* route_indices,
                       int64_t n_tokens, int32_t n_experts, const int32_t* expert_owner, int32_t* ordered_assignments,
                       int32_t row_format, int* status, void* stream);
int dsv4_ep_return(dsv4_ep* ep, const void* rows_bf16, const int32_t* row_of_assignment, int* status, void* stream);
/* The return fused into the down GEMM: dsv4_ep_return_targets gives the
 * device table [world*max_tokens*topk] of each received assignment's
 * destination (row t*k + s of its source's `back`, in a peer's memory for
 * the other ranks; null for the other ranks' picks), filled by each
 * dsv4_ep_dispatch; dsv4_moe_forward_scatter(..., table) stores every output
 * row there from the GEMM's epilogue, so the rows cross NVLink while later
 * tiles compute; dsv4_ep_return_published then announces the returned rows
 * and waits for every owner's (bounded, DSV4_ETIMEOUT). */
int dsv4_ep_return_targets(dsv4_ep* ep, void*** assign_dst);
int dsv4_ep_return_published(dsv4_ep* ep, int* status, void* stream);
int dsv4_ep_destroy(dsv4_ep* ep);

#ifdef __cplusplus
}
#endif
#endif /* DSV4MOE_H */
