// Router projection fused with softmax / top-k / renorm (sm_100a).
//
// Reference: ds3_ref_moe_ffn computes the router logits with
// ds3_ref_vec_matmul (src/ds3_reference.c:424-434: for each expert, a float
// sum from 0 over i ascending of x[i] * W[e][i]) and then softmax, top-k and
// renorm (:627-639); the engine dispatches the projection as
// ds3_metal_moe_ffn_router (src/ds3_metal.h:380-387) and the selection as
// moe_router_topk_batch_tokens.
//
// The top-8 indices must match the reference exactly, which the logits do
// only if every dot product is accumulated in the reference's order. So the
// projection runs on the CUDA cores, one thread per (token, expert), each
// summing its 2048 products sequentially with separately rounded multiply
// and add (no FMA) - a tensor-core or tree-reduced dot product would round
// differently. A CTA owns 4 tokens x 128 experts, one expert per thread,
// with 4 independent sums per thread (one per token). W (GGUF layout
// [n_expert][n_embd]) is loaded 32 columns at a time with coalesced 128-bit
// loads (the next chunk prefetched into registers while the current one is
// consumed) and stored transposed in shared memory, so a warp's 32 experts
// read 32 consecutive words; each W word read serves 4 multiply-adds and the
// token columns come as 128-bit broadcast reads covering 4 columns. The logits then go through the same
// warp-level selection as router_softmax_topk (router_select.cuh).
#include "common.cuh"
#include "launch.h"
#include "router_select.cuh"

namespace ds3 {
namespace {

constexpr int kRgE = 128;                  // experts (fast path): 4 warps x 32 lanes
constexpr int kRgTok = 4;                  // tokens per CTA, one accumulator each per lane
constexpr int kRgKC = 32;                  // columns per chunk
constexpr int kRgThreads = kRgE;           // 128

__global__ void __launch_bounds__(kRgThreads) router_gemv_topk_k(const float *x, const float *W, float *logits_out,
                                                                 int32_t *idx, float *scores, int64_t n_tokens,
                                                                 int n_embd, int n_used, int norm_topk)
{
    __shared__ float ws[kRgKC][kRgE + 1];  // chunk of W, transposed; +1 keeps the transposing stores conflict-free
    __shared__ __align__(16) float xs[kRgTok][kRgKC];
    __shared__ __align__(16) float lg[kRgTok][kRgE];
    pdl_wait();
    pdl_trigger();
    const int e = threadIdx.x;  // expert owned by this thread
    const int64_t t0 = (int64_t)blockIdx.x * kRgTok;

    // Coalesced staging: float4 q = e + h*128 of the 128 x 32 chunk is row
    // q / 8, columns 4 * (q % 8) .. +3 (8 threads read 128 contiguous bytes).
    constexpr int kH = kRgE * kRgKC / 4 / kRgThreads;  // 8
    float4 w[kH];
    float xr = 0.0f;
    auto fetch = [&](int k0) {
#pragma unroll
        for (int h = 0; h < kH; h++) {
            const int q = e + h * kRgThreads;
            w[h] = __ldg(reinterpret_cast<const float4 *>(W + (int64_t)(q / 8) * n_embd + k0 + 4 * (q % 8)));
        }
        const int64_t tt = t0 + e / kRgKC;  // 128 threads stage 4 tokens x 32 columns
        xr = tt < n_tokens ? x[tt * n_embd + k0 + e % kRgKC] : 0.0f;
    };
    fetch(0);
    float acc[kRgTok];
#pragma unroll
    for (int j = 0; j < kRgTok; j++) acc[j] = 0.0f;
    for (int k0 = 0; k0 < n_embd; k0 += kRgKC) {
#pragma unroll
        for (int h = 0; h < kH; h++) {
            const int q = e + h * kRgThreads;
            const int r = q / 8, c = 4 * (q % 8);
            ws[c][r] = w[h].x;
            ws[c + 1][r] = w[h].y;
            ws[c + 2][r] = w[h].z;
            ws[c + 3][r] = w[h].w;
        }
        xs[e / kRgKC][e % kRgKC] = xr;
        __syncthreads();
        if (k0 + kRgKC < n_embd) fetch(k0 + kRgKC);  // next chunk in flight during the sums
#pragma unroll
        for (int i = 0; i < kRgKC / 4; i++) {
            float xv[kRgTok][4];
#pragma unroll
            for (int j = 0; j < kRgTok; j++) {
                const float4 v = *reinterpret_cast<const float4 *>(&xs[j][4 * i]);
                xv[j][0] = v.x; xv[j][1] = v.y; xv[j][2] = v.z; xv[j][3] = v.w;
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float wv = ws[4 * i + u][e];
#pragma unroll
                for (int j = 0; j < kRgTok; j++) acc[j] = __fadd_rn(acc[j], __fmul_rn(xv[j][u], wv));
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < kRgTok; j++) {
        lg[j][e] = acc[j];
        if (logits_out && t0 + j < n_tokens) logits_out[(t0 + j) * kRgE + e] = acc[j];
    }
    __syncthreads();

    const int warp = e >> 5, lane = e & 31;
    if (t0 + warp < n_tokens) {  // warp w selects for token t0 + w
        const float4 v = *reinterpret_cast<const float4 *>(&lg[warp][4 * lane]);
        const float xv[4] = {v.x, v.y, v.z, v.w};
        const int64_t tw = t0 + warp;
        router_select<4>(xv, lane, n_used, norm_topk, nullptr, idx + tw * n_used, scores + tw * n_used);
    }
}

// Any shape: one thread per (token, expert) straight from global memory, same
// sequential sum; the selection then runs as router_softmax_topk.
__global__ void router_logits_k(const float *x, const float *W, float *logits, int64_t n_tokens, int n_embd,
                                int n_expert)
{
    pdl_wait();
    pdl_trigger();
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= n_tokens * n_expert) return;
    const int64_t t = q / n_expert;
    const int e = (int)(q - t * n_expert);
    const float *xr = x + t * n_embd, *wr = W + (int64_t)e * n_embd;
    float acc = 0.0f;
    for (int i = 0; i < n_embd; i++) acc = __fadd_rn(acc, __fmul_rn(xr[i], wr[i]));
    logits[q] = acc;
}

}  // namespace

bool router_gemv_fast(int64_t n_tokens, int n_embd, int n_expert, int n_used, const void *x, const void *W)
{
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W);
    return n_expert == kRgE && n_embd % kRgKC == 0 && n_used <= 32 && (al & 15u) == 0 && n_tokens > 0;
}

cudaError_t launch_router_gemv_topk(const LaunchCtx &c, const float *x, const float *W, float *logits_out,
                                    int32_t *idx, float *scores, int64_t n_tokens, int n_embd, int n_expert,
                                    int n_used, int norm_topk)
{
    if (n_tokens <= 0) return cudaSuccess;
    if (router_gemv_fast(n_tokens, n_embd, n_expert, n_used, x, W)) {
        launch_k(c, router_gemv_topk_k, dim3((unsigned)((n_tokens + kRgTok - 1) / kRgTok)), dim3(kRgThreads), x, W,
                 logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk);
        return cudaGetLastError();
    }
    if (!logits_out) return cudaErrorInvalidValue;  // the general path needs the logits buffer
    const int64_t n = n_tokens * n_expert;
    launch_k(c, router_logits_k, dim3((unsigned)((n + 255) / 256)), dim3(256), x, W, logits_out, n_tokens, n_embd,
             n_expert);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_router_topk(c, logits_out, nullptr, idx, scores, n_tokens, n_expert, n_used, norm_topk);
}

}  // namespace ds3
