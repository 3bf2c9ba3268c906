/*
 * ds3_cuda.h — B200 (sm_100a) backend C-ABI for the qw3 engine's fused
 * per-layer path.
 *
 * The engine (src/ds3_engine.c of wzqhbustb/qw3) calls its GPU backend through
 * src/ds3_metal.h. This header offers the same entry points under a ds3_cuda_
 * prefix, with the same argument order, meaning and return convention, so the
 * engine can swap backends per op; each declaration cites the ds3_metal.h
 * line it replaces. Entries marked "new" have no Metal counterpart: they are
 * the fused kernels of this backend (one pass over HBM where the Metal path
 * makes two or three) and the stream/graph/timer plumbing a CUDA host needs.
 *
 * Conventions (as ds3_metal.m):
 *  - ops return 0 on success, -1 on error; allocators return NULL on failure;
 *    errors are printed to stderr;
 *  - rows are dense (row stride = n * element size);
 *  - in-place calls are legal where the Metal engine makes them
 *    (rms_norm(x, w, x), rope(src == dst), qk_norm_rope in place);
 *  - outside begin_batch/end_batch every op is synchronous: it launches,
 *    waits for the device and returns the status; inside a batch (or a graph
 *    capture) ops only enqueue, and end_batch waits and returns the status;
 *  - one device context per process (multi-GPU = one process per GPU; call
 *    ds3_cuda_set_device before ds3_cuda_init); state is not thread-safe;
 *  - inside a batch or graph, consecutive ops overlap (programmatic dependent
 *    launch): an op may read its weights (norm weights, the RoPE inputs'
 *    q_w / k_w, the embedding table, an fp32 router weight) before the op just before it has
 *    finished. So a weight must not be written by the op immediately before
 *    its use in the same batch or graph (make such a write, e.g. a
 *    dequantize_f32 that produces a norm weight, outside the batch, or put
 *    another op in between). Activations carry no such rule.
 *
 * Device-side errors (a token id outside the vocabulary, a bounded wait that
 * ran out) never trap: the kernel skips the bad row, writes zeros there and
 * sets a bit in a device error word, which the next synchronising call reads,
 * reports and clears (it then returns -1).
 */
#ifndef DS3_CUDA_H
#define DS3_CUDA_H

#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>

#if defined(__has_include)
#  if __has_include("ds3.h")
#    include "ds3.h"
#  endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; only these entry points are exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifndef DS3_H
/* GGUF tensor type ids; same values as ds3_type_t in the engine's src/ds3.h:201-216.
 * (When the engine's ds3.h is on the include path its enum is used instead.) */
typedef enum {
    DS3_TYPE_F32  = 0,
    DS3_TYPE_F16  = 1,
    DS3_TYPE_Q8_0 = 8,
    DS3_TYPE_Q4_K = 12,
    DS3_TYPE_Q6_K = 14
} ds3_type_t;
#endif

/* Opaque handle to a device buffer (ds3_metal.h:14). A view shares its
 * parent's allocation; freeing a view never frees the parent. */
typedef struct ds3_cuda_buffer ds3_cuda_buffer_t;

/* ------------------------------------------------------------------ */
/* Lifecycle                                                          */
/* ------------------------------------------------------------------ */

/* new: select the CUDA device this process drives; call before init. */
int  ds3_cuda_set_device(int device);
/* ds3_metal.h:19-20. Returns 0, or -1 if no usable sm_100 device is present. */
int  ds3_cuda_init(void);
void ds3_cuda_shutdown(void);

/* ------------------------------------------------------------------ */
/* Buffers                                                            */
/* ------------------------------------------------------------------ */

/* ds3_metal.h:25-26 */
ds3_cuda_buffer_t *ds3_cuda_buffer_alloc(size_t bytes);
void               ds3_cuda_buffer_free(ds3_cuda_buffer_t *buf);
/* ds3_metal.h:31. Metal aliases the mmap on unified memory; here the region is
 * copied once into device memory (a host-resident table would bound every
 * gather by the host link, not HBM). The result is read-only. `base` need not
 * be page-aligned. */
ds3_cuda_buffer_t *ds3_cuda_buffer_from_mmap(const void *base, size_t bytes);
/* ds3_metal.h:35-36 */
ds3_cuda_buffer_t *ds3_cuda_buffer_view(const ds3_cuda_buffer_t *base,
                                        size_t offset, size_t bytes);
/* new: wrap device memory owned by someone else (e.g. a framework tensor);
 * free() releases only the handle. */
ds3_cuda_buffer_t *ds3_cuda_buffer_wrap(void *device_ptr, size_t bytes);
/* new: device address and size of a buffer (views included). */
void  *ds3_cuda_buffer_device_ptr(const ds3_cuda_buffer_t *buf);
size_t ds3_cuda_buffer_size(const ds3_cuda_buffer_t *buf);
/* ds3_metal.h:39-42. Synchronous copies on the module stream. Writes to
 * read-only (from_mmap) buffers are refused. Inside a batch they are ordered
 * after the ops already enqueued. */
int ds3_cuda_buffer_write(ds3_cuda_buffer_t *buf, size_t offset,
                          const void *src, size_t bytes);
int ds3_cuda_buffer_read (ds3_cuda_buffer_t *buf, size_t offset,
                          void *dst, size_t bytes);

/* new: the same copies, enqueued on the module stream in order with the ops
 * and not waited for (graph-capturable). The host memory must stay valid and
 * unchanged until the stream is synchronised (ds3_cuda_synchronize or
 * end_batch); page-locked host memory lets the copies run at full link rate
 * without a staging copy. */
int ds3_cuda_buffer_write_async(ds3_cuda_buffer_t *buf, size_t offset,
                                const void *src, size_t bytes);
int ds3_cuda_buffer_read_async (ds3_cuda_buffer_t *buf, size_t offset,
                                void *dst, size_t bytes);

/* ------------------------------------------------------------------ */
/* Ops with a ds3_metal.h counterpart                                 */
/* ------------------------------------------------------------------ */

/* ds3_metal.h:53-57. out = x / sqrt(mean(x^2) + eps) * weight, per row. */
int ds3_cuda_rms_norm(const ds3_cuda_buffer_t *x,
                      const ds3_cuda_buffer_t *weight,
                      ds3_cuda_buffer_t       *out,
                      uint32_t n, uint32_t n_rows, float eps);

/* ds3_metal.h:64-69. NEOX RoPE over [n_rows, n_heads*head_dim]; positions int32 [n_rows]. */
int ds3_cuda_rope(const ds3_cuda_buffer_t *src,
                  ds3_cuda_buffer_t       *dst,
                  const ds3_cuda_buffer_t *positions,
                  uint32_t n_heads, uint32_t head_dim, uint32_t n_rows,
                  float theta_base);

/* ds3_metal.h:168-178 */
int ds3_cuda_buffer_copy_f32(const ds3_cuda_buffer_t *src, ds3_cuda_buffer_t *dst, size_t bytes);
int ds3_cuda_buffer_zero_f32(ds3_cuda_buffer_t *buf, size_t bytes);
int ds3_cuda_vec_add_inplace(ds3_cuda_buffer_t *acc, const ds3_cuda_buffer_t *addend, uint32_t n);
int ds3_cuda_vec_add(const ds3_cuda_buffer_t *a, const ds3_cuda_buffer_t *b,
                     ds3_cuda_buffer_t *c, uint32_t n);

/* ds3_metal.h:184-192. gather: dst[i] = src[ids[offset+i]];
 * scatter: dst[ids[offset+i]] += scores[offset+i] * src[i] (ids unique per call). */
int ds3_cuda_gather_rows_f32(const ds3_cuda_buffer_t *src, const ds3_cuda_buffer_t *ids,
                             ds3_cuda_buffer_t *dst,
                             uint32_t n_cols, uint32_t count, uint32_t offset);
int ds3_cuda_scatter_add_weighted_f32(const ds3_cuda_buffer_t *src,
                                      const ds3_cuda_buffer_t *scores,
                                      const ds3_cuda_buffer_t *ids,
                                      ds3_cuda_buffer_t *dst,
                                      uint32_t n_cols, uint32_t count, uint32_t offset);

/* ds3_metal.h:195-198. out = silu(gate) * up. */
int ds3_cuda_silu_mul_f32(const ds3_cuda_buffer_t *gate, const ds3_cuda_buffer_t *up,
                          ds3_cuda_buffer_t *out, uint32_t n);

/* ds3_metal.h:424-431. logits [n_layers][n_expert] -> indices/scores [n_layers][n_used]. */
int ds3_cuda_moe_router_topk_batch(const ds3_cuda_buffer_t *logits,
                                   ds3_cuda_buffer_t *indices, ds3_cuda_buffer_t *scores,
                                   uint32_t n_layers, uint32_t n_expert, uint32_t n_used,
                                   bool norm_topk_prob);
/* ds3_metal.h:437-445. logits [n_layers][n_tokens][n_expert] ->
 * [n_layers][n_tokens][n_used] (dense layer stride n_tokens*n_used). */
int ds3_cuda_moe_router_topk_batch_tokens(const ds3_cuda_buffer_t *logits,
                                          ds3_cuda_buffer_t *indices, ds3_cuda_buffer_t *scores,
                                          uint32_t n_layers, uint32_t n_tokens,
                                          uint32_t n_expert, uint32_t n_used,
                                          bool norm_topk_prob);

/* ds3_metal.h:280-290. k, v fp32 [n_tokens][n_kv_heads][head_dim] -> fp16 cache
 * rows seq_pos .. seq_pos+n_tokens-1 of [max_seq_len][n_kv_heads][head_dim]. */
int ds3_cuda_kv_cache_write_batch(const ds3_cuda_buffer_t *k, const ds3_cuda_buffer_t *v,
                                  ds3_cuda_buffer_t *k_cache, ds3_cuda_buffer_t *v_cache,
                                  uint32_t seq_pos, uint32_t n_tokens, uint32_t max_seq_len,
                                  uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim);

/* ds3_metal.h:457-462. begin_batch returns -1 if a batch is already open. */
int  ds3_cuda_begin_batch(void);
int  ds3_cuda_end_batch(void);
void ds3_cuda_synchronize(void);

/* ds3_metal.h:467-468. Enabled with DS3_CUDA_PROFILE=1 (or profile_enable). */
void ds3_cuda_profile_reset(void);
void ds3_cuda_profile_print(const char *label);

/* ------------------------------------------------------------------ */
/* Fused ops (new). They replace the sequences named beside each.     */
/* ------------------------------------------------------------------ */

/* Whole-tensor conversion to fp32 on the device (weights at load time).
 * Replaces ds3_ref_dequantize_tensor + buffer_write in the engine's
 * upload_dequantized_fp32 (src/ds3_engine.c:154-179), used for norm weights
 * stored in another type (:1609-1622). src: n_elements of `type` (F32, F16,
 * Q8_0, Q4_K, Q6_K; a whole number of blocks) as stored in the file; dst fp32
 * [n_elements]. Bit-exact with the reference dequant. */
int ds3_cuda_dequantize_f32(const ds3_cuda_buffer_t *src, ds3_type_t type, uint64_t n_elements,
                            ds3_cuda_buffer_t *dst);

/* Token-embedding gather + dequant on the device. Replaces the CPU loop
 * upload_token_embeddings (src/ds3_engine.c:273-290, ds3_ref_dequantize_row per
 * token) plus the host->device copy. table: [n_vocab] rows of `row_stride`
 * bytes of `type` (F32, F16, Q8_0, Q4_K, Q6_K); ids int32 [n_ids]; out fp32
 * [n_ids, n_cols]. Bit-exact with the reference dequant. */
int ds3_cuda_embed_rows(const ds3_cuda_buffer_t *table, const ds3_cuda_buffer_t *ids,
                        ds3_cuda_buffer_t *out,
                        uint32_t n_ids, uint32_t n_cols, uint32_t n_vocab,
                        ds3_type_t type, uint64_t row_stride);

/* Embedding gather + attn_norm RMSNorm in one pass: hidden_out gets the raw
 * rows (the residual the engine keeps, src/ds3_engine.c:734), norm_out the
 * normed rows (src/ds3_engine.c:744). hidden_out may be NULL. */
int ds3_cuda_embed_rms_norm(const ds3_cuda_buffer_t *table, const ds3_cuda_buffer_t *ids,
                            const ds3_cuda_buffer_t *weight,
                            ds3_cuda_buffer_t *hidden_out, ds3_cuda_buffer_t *norm_out,
                            uint32_t n_ids, uint32_t n_cols, uint32_t n_vocab,
                            ds3_type_t type, uint64_t row_stride, float eps);

/* Residual add + RMSNorm in one pass. Replaces vec_add_inplace + copy +
 * rms_norm (src/ds3_engine.c:857-866). sum_out = x + residual (may be NULL,
 * may alias x or residual); norm_out = rms_norm(sum) (may alias x). */
int ds3_cuda_add_rms_norm(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *residual,
                          const ds3_cuda_buffer_t *weight,
                          ds3_cuda_buffer_t *sum_out, ds3_cuda_buffer_t *norm_out,
                          uint32_t n, uint32_t n_rows, float eps);

/* Per-head Q/K RMSNorm + NEOX RoPE, in place. Replaces the two per-head
 * rms_norm calls (src/ds3_engine.c:789-792) and the per-token RoPE inside
 * attention (src/ds3_metal.m:1241-1266). q [n_rows, n_q_heads, head_dim],
 * k [n_rows, n_kv_heads, head_dim], stored as `storage` (DS3_TYPE_F32 or
 * DS3_TYPE_F16; math is fp32 either way); q_w/k_w fp32 [head_dim]; positions
 * int32 [n_rows]. k may be NULL when n_kv_heads == 0. */
int ds3_cuda_qk_norm_rope(ds3_cuda_buffer_t *q, ds3_cuda_buffer_t *k,
                          const ds3_cuda_buffer_t *q_w, const ds3_cuda_buffer_t *k_w,
                          const ds3_cuda_buffer_t *positions,
                          uint32_t n_rows, uint32_t n_q_heads, uint32_t n_kv_heads,
                          uint32_t head_dim, float theta_base, float eps,
                          ds3_type_t storage);

/* new: qk_norm_rope plus the KV-cache write of the same tokens, in one pass.
 * Replaces qk_norm_rope followed by kv_cache_write_batch (ds3_metal.h:280-290):
 * after q and k are normed and rotated in place, the rotated k rows and the v
 * rows (v [n_rows, n_kv_heads, 128], `storage` type, not modified) are
 * written, rounded to fp16, into k_cache / v_cache
 * [max_seq_len][n_kv_heads][128] at row positions[t]. head_dim must be 128;
 * a position outside [0, max_seq_len) skips that row's cache write and makes
 * the call return -1. */
int ds3_cuda_qk_norm_rope_kv(ds3_cuda_buffer_t *q, ds3_cuda_buffer_t *k, const ds3_cuda_buffer_t *v,
                             const ds3_cuda_buffer_t *q_w, const ds3_cuda_buffer_t *k_w,
                             const ds3_cuda_buffer_t *positions,
                             ds3_cuda_buffer_t *k_cache, ds3_cuda_buffer_t *v_cache,
                             uint32_t n_rows, uint32_t n_q_heads, uint32_t n_kv_heads,
                             uint32_t head_dim, uint32_t max_seq_len,
                             float theta_base, float eps, ds3_type_t storage);

/* Router softmax + top-k + renorm, one warp per token (the Metal kernel is
 * one thread per token, metal/moe.metal:566-624). logits [n_tokens, n_expert];
 * probs_out [n_tokens, n_expert] full softmax or NULL; idx int32 and scores
 * fp32 [n_tokens, n_used], ordered by descending probability. */
int ds3_cuda_router_softmax_topk(const ds3_cuda_buffer_t *logits,
                                 ds3_cuda_buffer_t *probs_out,
                                 ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores,
                                 uint32_t n_tokens, uint32_t n_expert, uint32_t n_used,
                                 bool norm_topk_prob);

/* new: per-expert token lists on the device. Replaces the host loop of
 * forward_chunk_post_gathered (src/ds3_engine.c:933-965) and the per-layer
 * readback of indices/scores it needs (:1256-1261). idx int32 / scores fp32
 * [n_tokens, n_used] (router output); counts int32 [n_expert]; ids int32 and
 * gscores fp32 [n_expert * cap]: the tokens that chose expert ex, ascending,
 * at ids[ex*cap + j] with their scores, exactly as the engine lays them out
 * (cap = n_tokens there). slot_of int32 [n_tokens * n_used] (or NULL) gets
 * ex*cap + j for each (token, slot): pass it as y_rows to
 * moe_combine_residual to read expert outputs in this layout. Slots past
 * counts[ex] are not written. counts[ex] is clamped to cap; a list that
 * would overflow, or an expert id outside [0, n_expert), makes the call
 * return -1 and leaves -1 in the affected slot_of entries. n_expert <= 256. */
int ds3_cuda_moe_expert_lists(const ds3_cuda_buffer_t *idx, const ds3_cuda_buffer_t *scores,
                              ds3_cuda_buffer_t *counts, ds3_cuda_buffer_t *ids,
                              ds3_cuda_buffer_t *gscores, ds3_cuda_buffer_t *slot_of,
                              uint32_t n_tokens, uint32_t n_expert, uint32_t n_used, uint32_t cap);

/* new: router projection + softmax + top-k + renorm in one call. Replaces
 * ds3_metal_moe_ffn_router (ds3_metal.h:380-387) followed by
 * moe_router_topk_batch_tokens. x fp32 [n_tokens, n_embd] (the ffn-normed
 * hidden state); w_router fp32 [n_expert][n_embd] (GGUF layout, dequantized);
 * logits_out fp32 [n_tokens, n_expert] or NULL (required unless n_expert is
 * 128 and n_embd a multiple of 64); idx / scores as router_softmax_topk.
 * Each logit is summed in the reference's order (from 0, ascending index,
 * multiply then add), so logits and top-k indices are bit-exact. */
int ds3_cuda_router_logits_topk(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *w_router,
                                ds3_cuda_buffer_t *logits_out,
                                ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores,
                                uint32_t n_tokens, uint32_t n_embd, uint32_t n_expert, uint32_t n_used,
                                bool norm_topk_prob);

/* new: the decode layer's FFN entry in one launch: residual add + ffn_norm
 * RMSNorm + router projection + softmax + top-k + renorm. Replaces
 * vec_add_inplace + buffer_copy_f32 + rms_norm + ds3_metal_moe_ffn_router +
 * moe_router_topk_batch_tokens (src/ds3_engine.c:508-535). sum_out = x +
 * residual (may alias residual or be NULL), norm_out = RMSNorm(sum) * weight
 * (may be NULL), both bit-identical to ds3_cuda_add_rms_norm; logits and
 * top-k as ds3_cuda_router_logits_topk over those normed rows (w_router fp32
 * [n_expert][n_embd]; logits_out may be NULL). Needs n_expert 128, n_used <= 32,
 * n_embd a multiple of 128 up to 2048 and 16-byte aligned rows; other shapes
 * return -1 (use add_rms_norm, then router_logits_topk). */
int ds3_cuda_add_rms_norm_router_topk(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *residual,
                                      const ds3_cuda_buffer_t *norm_weight, const ds3_cuda_buffer_t *w_router,
                                      ds3_cuda_buffer_t *sum_out, ds3_cuda_buffer_t *norm_out,
                                      ds3_cuda_buffer_t *logits_out, ds3_cuda_buffer_t *idx,
                                      ds3_cuda_buffer_t *scores, uint32_t n_tokens, uint32_t n_embd,
                                      uint32_t n_expert, uint32_t n_used, float eps, bool norm_topk_prob);

/* ds3_metal.h:380-387. Router logits of one token, the weight in its stored
 * type: gate_logits[e] = sum_i input[i] * W[e][i] (fp32, from 0, i
 * ascending, multiply then add, as ds3_ref_vec_matmul over the dequantised
 * weight), bit-exact. w_gate_inp: n_expert rows of n_embd elements of
 * router_type (F32, F16, Q8_0, Q4_K, Q6_K), router_row_stride bytes apart
 * (the GGUF nb[1]); input fp32 [n_embd]; gate_logits fp32 [n_expert]. A
 * weight other than dense F32 is converted to fp32 in a library-owned
 * device workspace first (n_expert * n_embd * 4 bytes, allocated on first
 * use and kept): make the first such call outside a graph capture. */
int ds3_cuda_moe_ffn_router(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                            ds3_cuda_buffer_t *gate_logits, uint32_t n_embd, uint32_t n_expert,
                            uint64_t router_row_stride, ds3_type_t router_type);

/* new: moe_ffn_router for n_tokens rows of input [n_tokens, n_embd] fused
 * with softmax + top-k + renorm (router_softmax_topk semantics): replaces
 * ds3_metal_moe_ffn_router per token followed by moe_router_topk_batch_tokens
 * (ds3_metal.h:437-445). gate_logits [n_tokens, n_expert] or NULL (required
 * unless n_expert is 128 and n_embd a multiple of 64); idx / scores
 * [n_tokens, n_used]. Same workspace rule as moe_ffn_router. */
int ds3_cuda_moe_ffn_router_topk(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                                 uint64_t router_row_stride, ds3_type_t router_type,
                                 ds3_cuda_buffer_t *gate_logits, ds3_cuda_buffer_t *idx,
                                 ds3_cuda_buffer_t *scores, uint32_t n_tokens, uint32_t n_embd,
                                 uint32_t n_expert, uint32_t n_used, bool norm_topk_prob);

/* new, with no counterpart in the reference: moe_ffn_router_topk for callers
 * that cannot let this library allocate device memory, for instance a host
 * whose GPU memory is all reserved up front by its own allocator, or one
 * that must not trigger an allocation (and its implicit device
 * synchronisation) in the middle of a step. Same arguments, results and
 * errors as moe_ffn_router_topk, but the fp32 copy of a router weight stored
 * in another type goes into a fixed scratch array inside the loaded library
 * (2 MiB per GPU that loads it, held until the process exits), so no call
 * ever allocates device memory. Limit: n_expert * n_embd <= 524288 (128
 * experts x 4096); larger shapes are refused with -1 and a message. The
 * first call on a device looks up the array's device address (no
 * allocation); make that first call before any stream capture. Every call
 * shares the one array and leaves its last contents there (each call
 * overwrites all it reads): calls that could run at the same time on the
 * GPU, e.g. graphs replayed on different streams, race on it. */
int ds3_cuda_moe_ffn_router_topk_noalloc(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                                         uint64_t router_row_stride, ds3_type_t router_type,
                                         ds3_cuda_buffer_t *gate_logits, ds3_cuda_buffer_t *idx,
                                         ds3_cuda_buffer_t *scores, uint32_t n_tokens, uint32_t n_embd,
                                         uint32_t n_expert, uint32_t n_used, bool norm_topk_prob);

/* SwiGLU with optional per-row routing weight:
 * out[r][c] = (silu(gate[r][c]) * up[r][c]) * row_weight[r]. row_weight may be
 * NULL (plain silu_mul, metal/moe.metal:95-108). */
int ds3_cuda_swiglu(const ds3_cuda_buffer_t *gate, const ds3_cuda_buffer_t *up,
                    const ds3_cuda_buffer_t *row_weight, ds3_cuda_buffer_t *out,
                    uint32_t n_rows, uint32_t n_cols);

/* Weighted expert combine + residual. Replaces zero + per-expert
 * scatter_add_weighted + vec_add (src/ds3_engine.c:1012-1019):
 * out[t] = residual[t] + sum_k w[t,k] * y[row(t,k)], accumulated from zero in
 * k order. row(t,k) = y_rows[t*n_used+k] (int32), or t*n_used+k when y_rows
 * is NULL. out may alias residual. A mapped row outside y (a -1 left by
 * moe_expert_lists, or an index past y's last row) counts as a zero row and
 * makes the call return -1; y is never read outside its buffer. */
int ds3_cuda_moe_combine_residual(const ds3_cuda_buffer_t *y, const ds3_cuda_buffer_t *y_rows,
                                  const ds3_cuda_buffer_t *w, const ds3_cuda_buffer_t *residual,
                                  ds3_cuda_buffer_t *out,
                                  uint32_t n_tokens, uint32_t n_used, uint32_t n_cols);

/* ------------------------------------------------------------------ */
/* Copy lanes (new): host transfers that overlap the ops              */
/* ------------------------------------------------------------------ */

/* Lane 0 is the module stream the ops run on; lanes 1 and 2 are two more
 * streams for host<->device copies, so that the next step's inputs can
 * arrive and the previous step's results leave while a step computes
 * (each direction has its own copy engine). lane_write / lane_read enqueue
 * a copy on a lane and do not wait (page-locked host memory, kept alive and
 * unchanged until the lanes are synchronised). Ordering between lanes is the
 * caller's: lane_record(lane, slot) records event slot `slot` (the timer
 * slots) at the current end of `lane`, and lane_wait(lane, slot) makes
 * everything enqueued on `lane` afterwards wait for it. ds3_cuda_synchronize
 * and end_batch wait for all three lanes. Not available while capturing a
 * graph. */
int ds3_cuda_lane_write(int lane, ds3_cuda_buffer_t *buf, size_t offset, const void *src, size_t bytes);
int ds3_cuda_lane_read(int lane, ds3_cuda_buffer_t *buf, size_t offset, void *dst, size_t bytes);
int ds3_cuda_lane_record(int lane, int slot);
int ds3_cuda_lane_wait(int lane, int slot);

/* ------------------------------------------------------------------ */
/* Streams, graphs, timers, errors (new)                              */
/* ------------------------------------------------------------------ */

/* The module stream (a cudaStream_t) all ops are enqueued on. */
void *ds3_cuda_stream(void);

/* Capture the ops enqueued between graph_begin and graph_end into a CUDA
 * graph (ops only enqueue while capturing). graph_launch enqueues one replay
 * without waiting; ds3_cuda_synchronize or end_batch waits. */
typedef struct ds3_cuda_graph ds3_cuda_graph_t;
int               ds3_cuda_graph_begin(void);
ds3_cuda_graph_t *ds3_cuda_graph_end(void);
int               ds3_cuda_graph_launch(ds3_cuda_graph_t *g);
void              ds3_cuda_graph_free(ds3_cuda_graph_t *g);

/* Event slots on the module stream (graph-capturable): mark(slot) records
 * slot; elapsed_ms(a, b) waits for b and returns the time between them, or a
 * negative value on error. Slots are 0 .. DS3_CUDA_TIMER_SLOTS-1. */
#define DS3_CUDA_TIMER_SLOTS 16384
int   ds3_cuda_timer_mark(int slot);
float ds3_cuda_timer_elapsed_ms(int slot_a, int slot_b);

/* Profiling switch (same effect as DS3_CUDA_PROFILE=1). */
void ds3_cuda_profile_enable(int on);

/* Last error message of this thread's calls ("" if none). */
const char *ds3_cuda_last_error(void);

/* new: self-test of the bounded-wait path. Launches one kernel that waits on
 * an mbarrier nothing will complete, giving up after `polls` polls, exactly
 * as the TMA-staged kernels do when a copy never lands. Returns 0 when the
 * wait ran out and was reported through the device error word (the word is
 * consumed), -1 otherwise. No fault, trap or hang is involved. */
int ds3_cuda_selftest_bounded_wait(uint32_t polls);

/* new: the compute capability the library's kernels were compiled for, as
 * the CUDA runtime reports it for a loaded kernel (major*10 + minor; 100 for
 * sm_100a code), or -1 without a usable device. Needs ds3_cuda_init. */
int ds3_cuda_kernel_binary_version(void);

/* Reads and clears the device error word (bit 0: bad token id; bit 1: a
 * bounded wait ran out). Synchronises the module stream. */
uint32_t ds3_cuda_device_errors(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* DS3_CUDA_H */
