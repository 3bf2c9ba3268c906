// MoE router: softmax over the experts, top-k selection and renormalisation
// (sm_100a).
//
// Reference: ds3_ref_softmax (src/ds3_reference.c:344-359), ds3_ref_topk
// (:466-490) and the renorm of ds3_ref_moe_ffn (:631-639); Metal
// moe_router_topk_batch(_tokens)_f32 (metal/moe.metal:499-624), which runs
// one thread per token with a 128-entry array.
//
// Here one warp owns one token: lane l holds experts l*V .. l*V+V-1 (one
// 128-bit load for 128 experts), max and sum are warp reductions, and each of
// the k selection rounds is a local scan over V values plus a 5-step warp
// arg-max. Selection runs on the logits with (value desc, index asc): the
// logits are identical on host and device and softmax is monotone, so the
// chosen indices and their order equal the reference's except where two
// distinct logits round to the same probability (an exact tie in the
// reference, where the lowest index wins). Scores are the probabilities of
// the chosen experts, renormalised by a sum taken in selection order.
#include <climits>

#include "common.cuh"
#include "launch.h"
#include "router_select.cuh"

namespace ds3 {
namespace {

__device__ __forceinline__ bool better(float v, int i, float bv, int bi)
{
    if (i == INT_MAX) return false;
    if (bi == INT_MAX) return true;
    return v > bv || (v == bv && i < bi);
}

template <int V>
__global__ void __launch_bounds__(128) router_warp(const float *logits, float *probs_out,
                                                   int32_t *idx, float *scores, int64_t n_tokens,
                                                   int n_used, int norm_topk)
{
    constexpr int E = 32 * V;
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (lane == 0 && t < n_tokens) prefetch_l2(logits + t * E, E * sizeof(float));
    pdl_wait();
    pdl_trigger();
    if (t >= n_tokens) return;
    const float *row = logits + t * E;

    float x[V];
    if constexpr (V % 4 == 0) {
#pragma unroll
        for (int j = 0; j < V; j += 4) {
            const float4 f = ld_stream(reinterpret_cast<const float4 *>(row + lane * V + j));
            x[j] = f.x; x[j + 1] = f.y; x[j + 2] = f.z; x[j + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; j++) x[j] = __ldcs(row + lane * V + j);
    }

    router_select<V>(x, lane, n_used, norm_topk, probs_out ? probs_out + t * E : nullptr, idx + t * n_used,
                     scores + t * n_used);
}

// Any n_expert / n_used (used when the warp layout does not fit): one thread
// per token, as the Metal kernel, re-reading the logits from global memory.
__global__ void router_thread(const float *logits, float *probs_out, int32_t *idx, float *scores,
                              int64_t n_tokens, int E, int n_used, int norm_topk)
{
    pdl_wait();
    pdl_trigger();
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_tokens) return;
    const float *row = logits + t * E;
    float mx = row[0];
    for (int e = 1; e < E; e++) mx = fmaxf(mx, row[e]);
    float total = 0.0f;
    for (int e = 0; e < E; e++) total = __fadd_rn(total, expf(__fsub_rn(row[e], mx)));
    const float inv = __fdiv_rn(1.0f, total);
    if (probs_out)
        for (int e = 0; e < E; e++) probs_out[t * E + e] = __fmul_rn(expf(__fsub_rn(row[e], mx)), inv);
    int32_t *ix = idx + t * n_used;
    float *sc = scores + t * n_used;
    float sum_sel = 0.0f;
    for (int k = 0; k < n_used; k++) {
        float bv = 0.0f;
        int bi = INT_MAX;
        for (int e = 0; e < E; e++) {
            bool taken = false;
            for (int q = 0; q < k; q++) taken |= (ix[q] == e);
            if (!taken && better(row[e], e, bv, bi)) {
                bv = row[e];
                bi = e;
            }
        }
        ix[k] = bi;
        sc[k] = __fmul_rn(expf(__fsub_rn(bv, mx)), inv);
        sum_sel = __fadd_rn(sum_sel, sc[k]);
    }
    if (norm_topk && sum_sel > 0.0f) {
        const float r = __fdiv_rn(1.0f, sum_sel);
        for (int k = 0; k < n_used; k++) sc[k] = __fmul_rn(sc[k], r);
    }
}

template <int V>
cudaError_t run_warp(const LaunchCtx &c, const float *logits, float *probs, int32_t *idx,
                     float *scores, int64_t n, int n_used, int norm)
{
    const int64_t blocks = (n + 3) / 4;
    launch_k(c, router_warp<V>, dim3((unsigned)blocks), dim3(128), logits, probs, idx, scores, n, n_used, norm);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router_topk(const LaunchCtx &c, const float *logits, float *probs_out,
                               int32_t *idx, float *scores, int64_t n_tokens, int n_expert,
                               int n_used, int norm_topk)
{
    if (n_tokens <= 0) return cudaSuccess;
    const bool al = ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(probs_out)) & 15u) == 0;
    if (n_used <= 32 && al) {
        switch (n_expert) {
        case 32: return run_warp<1>(c, logits, probs_out, idx, scores, n_tokens, n_used, norm_topk);
        case 64: return run_warp<2>(c, logits, probs_out, idx, scores, n_tokens, n_used, norm_topk);
        case 128: return run_warp<4>(c, logits, probs_out, idx, scores, n_tokens, n_used, norm_topk);
        case 256: return run_warp<8>(c, logits, probs_out, idx, scores, n_tokens, n_used, norm_topk);
        default: break;
        }
    }
    const int64_t blocks = (n_tokens + 127) / 128;
    launch_k(c, router_thread, dim3((unsigned)blocks), dim3(128), logits, probs_out, idx, scores, n_tokens,
                                                          n_expert, n_used, norm_topk);
    return cudaGetLastError();
}

}  // namespace ds3
