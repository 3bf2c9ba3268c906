// Internal launchers: raw device pointers + a stream. The C-ABI layer in
// ds3_cuda.cu validates the public arguments, resolves buffers to pointers
// and calls these. Each returns the launch status (cudaGetLastError).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ds3 {

struct LaunchCtx {
    cudaStream_t stream;
    unsigned *err;  // device-visible error word (see common.cuh)
    int n_sm;
    bool pdl;       // launch with programmatic stream serialization
};

// One-time per-kernel set-up before its first launch (shared-memory carveout).
void prepare_kernel(const void *k);
// Exempt `k` from the common carveout (call before its first launch): for
// kernels whose occupancy needs most of the shared memory.
void keep_driver_carveout(const void *k);

// Launch `k` on c.stream, with the PDL attribute when c.pdl is set.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(const LaunchCtx &c, void (*k)(KArgs...), dim3 grid, dim3 block, Args... args)
{
    prepare_kernel(reinterpret_cast<const void *>(k));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Same, with `smem` bytes of dynamic shared memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_ks(const LaunchCtx &c, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args)
{
    prepare_kernel(reinterpret_cast<const void *>(k));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// x [rows, n] (+ r) -> sum_out (optional), norm_out. r == nullptr: plain RMSNorm.
cudaError_t launch_add_rms_norm(const LaunchCtx &c, const float *x, const float *r, const float *w,
                                float *sum_out, float *norm_out, int n, int64_t rows, float eps);

// Rows of a stored matrix (row_stride bytes apart, any supported type) ->
// dense fp32 [n_rows, n_cols], bit-exact with the reference dequant.
cudaError_t launch_dequantize_rows(const LaunchCtx &c, const uint8_t *src, int type, uint64_t row_stride,
                                   int64_t n_rows, int n_cols, float *out);
// Whole tensor of `type` (F32, F16, Q8_0, Q4_K, Q6_K) to fp32; n < 2^31.
cudaError_t launch_dequantize(const LaunchCtx &c, const uint8_t *src, int type, int64_t n, float *out);

// Embedding gather (+ RMSNorm when norm_out != nullptr).
cudaError_t launch_embed(const LaunchCtx &c, const uint8_t *table, int type, uint64_t row_stride,
                         int64_t n_vocab, const int32_t *ids, int64_t n_ids, int n_cols,
                         float *hidden_out, const float *w, float *norm_out, float eps);

// Per-head RMSNorm (when do_norm) + NEOX RoPE. storage: 0 = fp32, 1 = fp16.
// q: [rows, nq, hd] read from q_src, written to q_dst (may alias); same for k.
cudaError_t launch_qk_norm_rope(const LaunchCtx &c, const void *q_src, void *q_dst,
                                const void *k_src, void *k_dst, const float *q_w,
                                const float *k_w, const int32_t *pos, int64_t rows, int nq,
                                int nk, int hd, const float *freq, float eps, int do_norm,
                                int storage);

// qk_norm_rope in place plus fp16 KV-cache rows at positions[t] (head_dim 128).
cudaError_t launch_qk_norm_rope_kv(const LaunchCtx &c, void *q, void *k, const void *v, const float *q_w,
                                   const float *k_w, const int32_t *pos, int64_t rows, int nq, int nk,
                                   const float *freq, float eps, int storage, void *k_cache, void *v_cache,
                                   int max_seq);

// fp32 k/v [n_tokens][row_elems] -> fp16 cache rows seq_pos.. (row_elems = n_kv_heads * head_dim).
cudaError_t launch_kv_cache_write(const LaunchCtx &c, const float *k, const float *v, void *k_cache,
                                  void *v_cache, int64_t seq_pos, int64_t n_tokens, int64_t row_elems);

// Per-expert token lists from top-k (engine layout ids[ex*cap + j]), counts, slot map.
cudaError_t launch_moe_expert_lists(const LaunchCtx &c, const int32_t *idx, const float *scores, int32_t *counts,
                                    int32_t *ids, float *gscores, int32_t *slot_of, int64_t n_tokens, int n_used,
                                    int n_expert, int64_t cap);

cudaError_t launch_bounded_wait_selftest(const LaunchCtx &c, uint32_t polls);
// Compute capability (major*10 + minor) of the loaded kernel code, or -1.
int kernel_binary_version();

// Router projection (sequential fp32 dot products, reference order) + top-k.
bool router_gemv_fast(int64_t n_tokens, int n_embd, int n_expert, int n_used, const void *x, const void *W);
// Residual add + RMSNorm + router projection + top-k in one cluster kernel
// (128 experts, n_embd % 128 == 0 and <= 2048, 16-byte aligned rows).
bool add_norm_router_fast(int64_t n_tokens, int n_embd, int n_expert, int n_used, const void *x, const void *r,
                          const void *W);
cudaError_t launch_add_norm_router_topk(const LaunchCtx &c, const float *x, const float *r, const float *norm_w,
                                        const float *W, float *sum_out, float *norm_out, float *logits_out,
                                        int32_t *idx, float *scores, int64_t n_tokens, int n_embd, int n_expert,
                                        int n_used, int norm_topk, float eps);
// w_static: W is the caller's weight, which no op immediately before writes,
// so its copy may start before the programmatic-launch wait.
cudaError_t launch_router_gemv_topk(const LaunchCtx &c, const float *x, const float *W, float *logits_out,
                                    int32_t *idx, float *scores, int64_t n_tokens, int n_embd, int n_expert,
                                    int n_used, int norm_topk, bool w_static = false);

cudaError_t launch_router_topk(const LaunchCtx &c, const float *logits, float *probs_out,
                               int32_t *idx, float *scores, int64_t n_tokens, int n_expert,
                               int n_used, int norm_topk);

cudaError_t launch_swiglu(const LaunchCtx &c, const float *gate, const float *up,
                          const float *row_w, float *out, int64_t rows, int64_t cols);

cudaError_t launch_combine(const LaunchCtx &c, const float *y, const int32_t *y_rows,
                           const float *w, const float *residual, float *out, int64_t n_tokens,
                           int n_used, int64_t n_cols, int64_t n_y_rows);

cudaError_t launch_vec_add(const LaunchCtx &c, const float *a, const float *b, float *out,
                           int64_t n);

cudaError_t launch_gather_rows(const LaunchCtx &c, const float *src, const int32_t *ids,
                               float *dst, int64_t n_cols, int64_t count, int64_t n_src_rows);

cudaError_t launch_scatter_add_weighted(const LaunchCtx &c, const float *src, const float *scores,
                                        const int32_t *ids, float *dst, int64_t n_cols,
                                        int64_t count, int64_t n_dst_rows);

}  // namespace ds3
