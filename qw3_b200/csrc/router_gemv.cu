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
// projection runs on the CUDA cores, one sum per (token, expert), each adding
// its 2048 products sequentially with separately rounded multiply and add (no
// FMA) - a tensor-core or tree-reduced dot product would round differently.
// Products are formed two at a time with the packed fp32 multiply of sm_100
// (mul.rn.f32x2, two independent IEEE products); the adds stay scalar and in
// order.
//
// Work split (fast path: 128 experts, n_embd % 64 == 0). A cluster of 4 CTAs
// shares up to 16 tokens and CTA r owns experts 32r .. 32r+31, so each CTA
// reads a quarter of W (GGUF layout [n_expert][n_embd]). Four compute warps
// hold lane = expert, 4 tokens each; four copy warps stream the CTA's 32 W
// rows and the cluster's token rows, 64 columns at a time, into a 6-stage
// ring in shared memory with 16-byte cp.async copies that complete on
// per-stage mbarriers (a copy warp arrives once its own copies have landed).
// Rows sit at a stride of 68 floats, so the 128-bit reads of 8 lanes (8
// different W rows) hit 32 distinct banks; token columns are broadcast reads.
// Each CTA asks for more than half an SM's shared memory, so the hardware
// places one CTA per SM, and the host sizes tokens per cluster from the number
// of clusters that can be resident at once, so one wave covers the tokens.
// When the sums are done, warp w stores its logits into the shared memory of
// CTA w (distributed shared memory), and after a cluster barrier CTA r runs
// the warp-level selection of router_softmax_topk (router_select.cuh) for
// tokens 4r .. 4r+3 of the cluster.
#include "common.cuh"
#include "launch.h"
#include "router_select.cuh"

namespace ds3 {
namespace {

constexpr int kRgE = 128;                    // experts on the fast path

constexpr int kClKC = 64;                    // columns per stage
constexpr int kClLd = kClKC + 4;             // padded row stride (floats), 16-byte multiple
constexpr int kClStages = 6;
constexpr int kClPW = 4;                     // copy warps
constexpr int kClSeg = kClKC / 4;            // 16-byte segments per row and stage
constexpr size_t kClMinSmem = 116 * 1024;    // > half an SM's shared memory: one CTA per SM

// CN CTAs per cluster, NW compute warps with TPW tokens each, PW copy warps.
// The launcher uses <4, 4, 4, 4>; at 512 tokens, 8x2 compute warps and 8 or
// 12 copy warps measured the same or slower, and 1 or 2 copy warps or 2-CTA
// clusters clearly slower.
// FUSE: the token rows are not streamed through the ring; each CTA first
// forms x + r and its RMSNorm for the cluster's tokens (add_rms_norm
// semantics, same reduction order) into a normed-row area of up to
// kFuseMaxEmbd floats per token, which the sums then read.
constexpr int kFuseMaxEmbd = 2048;
constexpr int64_t kSmallT = 128;  // token counts served with one token per compute warp

template <int CN, int NW, int TPW, int PW = kClPW, bool FUSE = false>
struct ClLayout {
    static constexpr int kEpC = kRgE / CN;                            // experts per CTA
    static constexpr int kEpL = kEpC / 32;                            // experts per lane
    static constexpr int kThreads = 32 * (NW + PW);
    static constexpr int kTok = NW * TPW;                             // max tokens per cluster
    static constexpr int kSel = kTok / CN;                            // tokens each CTA selects for
    static constexpr int kStageFloats = (kEpC + (FUSE ? 0 : kTok)) * kClLd;
    static constexpr size_t kNormFloats = FUSE ? (size_t)kTok * kFuseMaxEmbd : 0;
    static constexpr size_t kSmemUsed =
        (size_t)kClStages * kStageFloats * 4 + (size_t)kSel * kRgE * 4 + kNormFloats * 4;
    static constexpr size_t kSmem = kSmemUsed > kClMinSmem ? kSmemUsed : kClMinSmem;
    static_assert(kTok <= 32 && kTok % CN == 0 && kSel <= NW + PW && kEpC % 32 == 0, "layout");
};

// Arguments of the fused add + RMSNorm prologue (FUSE only).
struct AddNorm {
    const float *r;   // residual [n_tokens, n_embd]
    const float *w;   // ffn_norm weight [n_embd]
    float *sum_out;   // x + r, or nullptr
    float *norm_out;  // normed rows, or nullptr
    float eps;
    int w_early;      // W is a weight no preceding op writes: its copy may start before the PDL wait
};

__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// Store one float into the shared memory of CTA `rank` of this cluster, at the
// offset `local` has in this CTA.
__device__ __forceinline__ void st_cluster_f32(const float *local, uint32_t rank, float v)
{
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// Arrive on `bar` once this thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// tpc = tokens per cluster (<= NW * TPW), chosen by the host so that the
// clusters fill the GPU in one wave.
template <int CN, int NW, int TPW, int PW, bool FUSE>
__global__ void __launch_bounds__(ClLayout<CN, NW, TPW, PW, FUSE>::kThreads, 1)
    router_gemv_cluster_k(const float *x, const float *W, float *logits_out, int32_t *idx, float *scores,
                          int64_t n_tokens, int n_embd, int n_used, int norm_topk, int tpc, unsigned *err,
                          const AddNorm an)
{
    using L = ClLayout<CN, NW, TPW, PW, FUSE>;
    extern __shared__ __align__(16) float sm[];
    float *lgx = sm + kClStages * L::kStageFloats;  // [kSel][128] logits of the tokens this CTA selects for
    float *xn = lgx + L::kSel * kRgE;               // FUSE: [kTok][n_embd] normed rows of the cluster's tokens
    __shared__ __align__(8) uint64_t full[kClStages], empty[kClStages];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int64_t t0 = (int64_t)(blockIdx.x / CN) * tpc;
    const int nt = n_tokens - t0 < tpc ? (int)(n_tokens - t0) : tpc;
    const int e0 = (int)rank * L::kEpC;
    const int n_chunks = n_embd / kClKC;  // n_embd % kClKC == 0 on this path
    if (threadIdx.x == 0) {
        for (int s = 0; s < kClStages; s++) {
            mbar_init(&full[s], 32 * PW);
            mbar_init(&empty[s], NW);
        }
        mbar_init_fence();
    }
    __syncthreads();
    cluster_arrive_relaxed();  // every CTA of the cluster has started (waited on before the logit exchange)
    pdl_wait();
    pdl_trigger();

    if constexpr (FUSE) {
        // x + r and its RMSNorm for the cluster's tokens, one warp per token,
        // with add_rms_norm's reduction (lane l sums the squares of float4
        // l, l+32, ... in order, then a butterfly), so the normed rows equal
        // that kernel's bit for bit. Every CTA of the cluster forms them in
        // its own shared memory for its own sums; rank 0 writes sum_out /
        // norm_out at the very end, after a cluster barrier, so outputs that
        // alias x or r (the engine keeps the sum in the residual buffer) are
        // never overwritten while another CTA still reads them.
        // Only the compute warps do this (they meet on named barrier 1), so
        // the copy warps start streaming W at once. Loads are issued in
        // batches of 8 float4 per lane before any is used (one round trip per
        // batch instead of one per float4).
        if (warp < NW) {
            const int vpl = n_embd / 128;
            for (int tl = warp; tl < nt; tl += NW) {
                const int64_t t = t0 + tl;
                const float4 *xr = reinterpret_cast<const float4 *>(x + t * n_embd);
                const float4 *rr = reinterpret_cast<const float4 *>(an.r + t * n_embd);
                float4 *xs = reinterpret_cast<float4 *>(xn + (size_t)tl * n_embd);
                float ss = 0.0f;
                for (int i0 = 0; i0 < vpl; i0 += 8) {
                    float4 a[8], b[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) {
                            a[u] = __ldcg(xr + (i0 + u) * 32 + lane);
                            b[u] = __ldcg(rr + (i0 + u) * 32 + lane);
                        }
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) {
                            const float4 v = f4_add(a[u], b[u]);
                            xs[(i0 + u) * 32 + lane] = v;
                            ss = f4_sumsq(v, ss);
                        }
                }
                ss = warp_sum(ss);
                const float inv = rms_inv(ss, n_embd, an.eps);
                const float4 *w4 = reinterpret_cast<const float4 *>(an.w);
                for (int i0 = 0; i0 < vpl; i0 += 8) {
                    float4 wv[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) wv[u] = __ldg(w4 + (i0 + u) * 32 + lane);
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) {
                            const int e = (i0 + u) * 32 + lane;
                            xs[e] = f4_norm(xs[e], inv, wv[u]);
                        }
                }
            }
            // The normed rows are complete before any compute warp reads them.
            asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
        }
    }

    bool ok = true;
    float acc[L::kEpL][TPW];
#pragma unroll
    for (int m = 0; m < L::kEpL; m++)
#pragma unroll
        for (int j = 0; j < TPW; j++) acc[m][j] = 0.0f;
    if (warp >= NW) {
        // Copy warps: 16-byte async copies of the kEpC W rows and nt token
        // rows of each stage; every copy thread arrives on full[s] once its
        // own copies have landed.
        const int pt = threadIdx.x - 32 * NW;
        for (int c = 0; c < n_chunks; c++) {
            const int s = c % kClStages;
            if (c >= kClStages && !mbar_wait(&empty[s], ((c / kClStages) - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            const int k0 = c * kClKC;
            float *st = sm + s * L::kStageFloats;
            for (int q = pt; q < (L::kEpC + (FUSE ? 0 : L::kTok)) * kClSeg; q += 32 * PW) {
                const int row = q / kClSeg, seg = q % kClSeg;
                if (row < L::kEpC)
                    cp_async16(st + row * kClLd + 4 * seg, W + (int64_t)(e0 + row) * n_embd + k0 + 4 * seg);
                else if (row - L::kEpC < nt)
                    cp_async16(st + row * kClLd + 4 * seg, x + (t0 + row - L::kEpC) * n_embd + k0 + 4 * seg);
            }
            cp_async_arrive(&full[s]);
        }
        // Do not leave with copies in flight.
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        for (int c = 0; c < n_chunks; c++) {
            const int s = c % kClStages;
            if (!mbar_wait(&full[s], (c / kClStages) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            const float *st = sm + s * L::kStageFloats;
            // Token j of this warp: column k0 + 4i of its row (stage rows at
            // stride kClLd, or the normed rows at stride n_embd).
            const float *xr = FUSE ? xn + (size_t)(warp * TPW) * n_embd + c * kClKC : st + (L::kEpC + warp * TPW) * kClLd;
            const int xld = FUSE ? n_embd : kClLd;
#pragma unroll
            for (int i = 0; i < kClKC / 4; i++) {
                float wv[L::kEpL][4];
#pragma unroll
                for (int m = 0; m < L::kEpL; m++) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(st + (lane + 32 * m) * kClLd + 4 * i);
                    wv[m][0] = w4.x; wv[m][1] = w4.y; wv[m][2] = w4.z; wv[m][3] = w4.w;
                }
                // Products of columns (k, k+1) and (k+2, k+3) two at a time for
                // every sum, then the four sequential adds, round-robin over the
                // independent sums so consecutive adds do not wait on each other.
                float pr[L::kEpL][TPW][4];
#pragma unroll
                for (int j = 0; j < TPW; j++) {
                    const float4 v = *reinterpret_cast<const float4 *>(xr + j * xld + 4 * i);
#pragma unroll
                    for (int m = 0; m < L::kEpL; m++) {
                        const float2 p01 = mul2_rn(make_float2(v.x, v.y), make_float2(wv[m][0], wv[m][1]));
                        const float2 p23 = mul2_rn(make_float2(v.z, v.w), make_float2(wv[m][2], wv[m][3]));
                        pr[m][j][0] = p01.x; pr[m][j][1] = p01.y; pr[m][j][2] = p23.x; pr[m][j][3] = p23.y;
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++)
#pragma unroll
                    for (int j = 0; j < TPW; j++)
#pragma unroll
                        for (int m = 0; m < L::kEpL; m++) acc[m][j] = __fadd_rn(acc[m][j], pr[m][j][u]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    if (!ok) flag_error(err, kErrWaitTimeout);

    cluster_wait_acquire();  // all CTAs resident before the remote stores
    if (warp < NW) {
#pragma unroll
        for (int j = 0; j < TPW; j++) {
            const int tl = warp * TPW + j;
            if (tl < nt) {
#pragma unroll
                for (int m = 0; m < L::kEpL; m++) {
                    const int e = e0 + lane + 32 * m;
                    if (logits_out) logits_out[(t0 + tl) * kRgE + e] = acc[m][j];
                    st_cluster_f32(lgx + (tl % L::kSel) * kRgE + e, (uint32_t)(tl / L::kSel), acc[m][j]);
                }
            }
        }
    }
    cluster_arrive_release();
    cluster_wait_acquire();
    if constexpr (FUSE) {
        // Every CTA of the cluster has read x and r by now: rank 0 stores the
        // sum (recomputed, the same single rounding) and the normed rows.
        if (rank == 0 && (an.sum_out || an.norm_out)) {
            const int vpl = n_embd / 128;
            for (int tl = warp; tl < nt; tl += NW + PW) {
                const int64_t t = t0 + tl;
                const float4 *xr = reinterpret_cast<const float4 *>(x + t * n_embd);
                const float4 *rr = reinterpret_cast<const float4 *>(an.r + t * n_embd);
                const float4 *xs = reinterpret_cast<const float4 *>(xn + (size_t)tl * n_embd);
                for (int i0 = 0; i0 < vpl; i0 += 8) {
                    float4 a[8], b[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) {
                            a[u] = __ldcg(xr + (i0 + u) * 32 + lane);
                            b[u] = __ldcg(rr + (i0 + u) * 32 + lane);
                        }
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (i0 + u < vpl) {
                            const int e = (i0 + u) * 32 + lane;
                            if (an.sum_out) reinterpret_cast<float4 *>(an.sum_out + t * n_embd)[e] = f4_add(a[u], b[u]);
                            if (an.norm_out) reinterpret_cast<float4 *>(an.norm_out + t * n_embd)[e] = xs[e];
                        }
                }
            }
        }
    }
    if (idx && warp < L::kSel) {  // idx == nullptr: logits only
        const int tl = (int)rank * L::kSel + warp;  // this CTA selects for tokens kSel*rank ..
        if (tl < nt) {
            const float4 v = *reinterpret_cast<const float4 *>(lgx + warp * kRgE + 4 * lane);
            const float xv[4] = {v.x, v.y, v.z, v.w};
            const int64_t tw = t0 + tl;
            router_select<4>(xv, lane, n_used, norm_topk, nullptr, idx + tw * n_used, scores + tw * n_used);
        }
    }
}

template <int CN, int NW, int TPW, int PW = kClPW, bool FUSE = false>
cudaError_t launch_cluster(const LaunchCtx &c, const float *x, const float *W, float *logits_out, int32_t *idx,
                           float *scores, int64_t n_tokens, int n_embd, int n_used, int norm_topk,
                           const AddNorm &an = AddNorm{})
{
    using L = ClLayout<CN, NW, TPW, PW, FUSE>;
    auto kern = router_gemv_cluster_k<CN, NW, TPW, PW, FUSE>;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(L::kThreads);
    cfg.dynamicSmemBytes = L::kSmem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CN;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static int max_clusters = 0;  // clusters resident at once, queried once per process
    if (max_clusters == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmem);
        if (e != cudaSuccess) return e;
        cfg.gridDim = dim3(CN);
        cfg.numAttrs = 1;
        e = cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg);
        if (e != cudaSuccess) return e;
        if (max_clusters < 1) max_clusters = 1;
    }
    // Fewest tokens per cluster that still lets one wave of clusters cover n_tokens.
    int64_t tpc = (n_tokens + max_clusters - 1) / max_clusters;
    if (tpc > L::kTok) tpc = L::kTok;
    if (tpc < 1) tpc = 1;
    cfg.gridDim = dim3((unsigned)(((n_tokens + tpc - 1) / tpc) * CN));
    cfg.numAttrs = c.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk,
                              (int)tpc, c.err, an);
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

// ------------------------------------------------------------------------
// Decode-size token counts (up to 8 tokens per cluster): the weight stays
// resident. A cluster of 8 CTAs covers the 128 experts, CTA r holding rows
// 16r .. 16r+15 of W whole in shared memory (one 1-D bulk copy per row, at a
// padded stride), and the cluster's TOK token rows (or, fused, their
// add + RMSNorm computed in place). Lane l of a compute warp sums expert
// 16r + (l & 15) for token 2*warp + (l >> 4), i ascending, multiply then add
// as the reference does: the only serial chain is the n_embd adds, with no
// ring of stages to synchronise on. Logits go to the CTA whose rank is the
// token (distributed shared memory), which then runs the selection.
constexpr int kResE = 16;   // experts per CTA
constexpr int kResCN = 8;   // CTAs per cluster
constexpr int kResMaxEmbd = 2048;

// Threads per CTA: TOK / 2 summing warps, at least 4 warps (the fused
// prologue gives each warp a token).
__host__ __device__ constexpr int res_threads(int tok) { return tok * 16 > 128 ? tok * 16 : 128; }

__host__ __device__ constexpr size_t res_smem(int tok, int n_embd)
{
    return ((size_t)kResE * (n_embd + 4) + (size_t)tok * n_embd + kRgE) * sizeof(float);
}

template <int TOK, bool FUSE>
__global__ void __launch_bounds__(res_threads(TOK), 1)
    router_gemv_resident_k(const float *x, const float *W, float *logits_out, int32_t *idx, float *scores,
                           int64_t n_tokens, int n_embd, int n_used, int norm_topk, unsigned *err, const AddNorm an)
{
    extern __shared__ __align__(16) float sm[];
    const int ldw = n_embd + 4;
    float *ws = sm;                          // [16][ldw]
    float *xs = ws + (size_t)kResE * ldw;    // [TOK][n_embd]
    float *lg = xs + (size_t)TOK * n_embd;   // [128] logits of the token this CTA selects for
    __shared__ __align__(8) uint64_t bar;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int64_t t0 = (int64_t)(blockIdx.x / kResCN) * TOK;
    const int nt = n_tokens - t0 < TOK ? (int)(n_tokens - t0) : TOK;
    const int e0 = (int)rank * kResE;
    const uint32_t row_bytes = (uint32_t)n_embd * 4u;
    const uint32_t tx = kResE * row_bytes + (FUSE ? 0u : (uint32_t)nt * row_bytes);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
        if (an.w_early) {
            // The weight (the caller's, never written by the op just before
            // it) is copied while the previous kernel runs; the barrier
            // expects the token rows too, copied after the wait.
            mbar_expect_tx(&bar, tx);
            for (int j = 0; j < kResE; j++)
                bulk_g2s(ws + (size_t)j * ldw, W + (size_t)(e0 + j) * n_embd, row_bytes, &bar);
        } else {
            prefetch_l2(W + (size_t)e0 * n_embd, (uint64_t)kResE * row_bytes);
        }
        // The cluster's token rows: hints only (they may be the previous
        // kernel's output; they are read after the wait).
        prefetch_l2(x + t0 * n_embd, (uint64_t)nt * row_bytes);
        if (FUSE) prefetch_l2(an.r + t0 * n_embd, (uint64_t)nt * row_bytes);
    }
    __syncthreads();
    cluster_arrive_relaxed();
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        if (!an.w_early) {
            mbar_expect_tx(&bar, tx);
            for (int j = 0; j < kResE; j++)
                bulk_g2s(ws + (size_t)j * ldw, W + (size_t)(e0 + j) * n_embd, row_bytes, &bar);
        }
        if constexpr (!FUSE)
            for (int k = 0; k < nt; k++) bulk_g2s(xs + (size_t)k * n_embd, x + (t0 + k) * n_embd, row_bytes, &bar);
    }
    if constexpr (FUSE) {
        // x + r and its RMSNorm (add_rms_norm's reduction order, so the normed
        // rows equal that kernel's bit for bit), one warp per token; every CTA
        // forms them for its own sums. The lane's share of the norm weight
        // (static) is loaded once, the x / r rows of a token all at once.
        const int vpl = n_embd / 128;  // <= 16
        float4 wv[16];
#pragma unroll
        for (int u = 0; u < 16; u++)
            if (u < vpl) wv[u] = __ldg(reinterpret_cast<const float4 *>(an.w) + u * 32 + lane);
        for (int tl = warp; tl < nt; tl += res_threads(TOK) / 32) {
            const int64_t t = t0 + tl;
            const float4 *xr = reinterpret_cast<const float4 *>(x + t * n_embd);
            const float4 *rr = reinterpret_cast<const float4 *>(an.r + t * n_embd);
            float4 *xo = reinterpret_cast<float4 *>(xs + (size_t)tl * n_embd);
            float4 a[16], b[16];
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (u < vpl) {
                    a[u] = __ldcg(xr + u * 32 + lane);
                    b[u] = __ldcg(rr + u * 32 + lane);
                }
            float ss = 0.0f;
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (u < vpl) {
                    a[u] = f4_add(a[u], b[u]);
                    ss = f4_sumsq(a[u], ss);
                }
            ss = warp_sum(ss);
            const float inv = rms_inv(ss, n_embd, an.eps);
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (u < vpl) xo[u * 32 + lane] = f4_norm(a[u], inv, wv[u]);
        }
    }
    bool ok = mbar_wait(&bar, 0, kWaitLimit);
    __syncthreads();  // fused normed rows, and every thread past its wait
    ok = __syncthreads_and(ok);
    if (!ok && threadIdx.x == 0) flag_error(err, kErrWaitTimeout);

    const int e = lane & 15, tk = 2 * warp + (lane >> 4);
    float acc = 0.0f;
    if (ok && tk < nt) {
        // Software-pipelined over groups of 16 columns: the products of the
        // next group (two IEEE products per mul.rn.f32x2) and the shared-memory
        // reads of the group after it are issued before the 16 adds of the
        // current group, so the chain of dependent adds is the only wait.
        const float *wr = ws + (size_t)e * ldw;
        const float *xr = xs + (size_t)tk * n_embd;
        float pc[16], pn[16];
        float4 wb[4], xb[4];
        auto load = [&](int at) {
#pragma unroll
            for (int g = 0; g < 4; g++) {
                wb[g] = *reinterpret_cast<const float4 *>(wr + at + 4 * g);
                xb[g] = *reinterpret_cast<const float4 *>(xr + at + 4 * g);
            }
        };
        auto products = [&](float *pr) {
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const float2 p01 = mul2_rn(make_float2(xb[g].x, xb[g].y), make_float2(wb[g].x, wb[g].y));
                const float2 p23 = mul2_rn(make_float2(xb[g].z, xb[g].w), make_float2(wb[g].z, wb[g].w));
                pr[4 * g] = p01.x;
                pr[4 * g + 1] = p01.y;
                pr[4 * g + 2] = p23.x;
                pr[4 * g + 3] = p23.y;
            }
        };
        load(0);
        products(pc);
        load(16 < n_embd ? 16 : 0);
        for (int i = 0; i < n_embd; i += 16) {
            products(pn);                                       // columns i+16 .. i+31
            load(i + 32 < n_embd ? i + 32 : 0);                 // columns i+32 .. (unused past the end)
#pragma unroll
            for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, pc[u]);  // columns i .. i+15, in order
#pragma unroll
            for (int u = 0; u < 16; u++) pc[u] = pn[u];
        }
    }
    cluster_wait_acquire();  // every CTA resident before the remote stores
    if (tk < nt) {
        if (logits_out) logits_out[(t0 + tk) * kRgE + e0 + e] = acc;
        st_cluster_f32(lg + e0 + e, (uint32_t)tk, acc);
    }
    cluster_arrive_release();
    cluster_wait_acquire();
    if constexpr (FUSE) {
        // Every CTA has read x and r: each stores an eighth of the columns of
        // every token's sum (recomputed, the same single rounding) and normed
        // row, so outputs that alias x or r are only written now.
        if (an.sum_out || an.norm_out) {
            const int per = n_embd / 4 / kResCN;  // float4 columns per CTA
            for (int q = threadIdx.x; q < nt * per; q += blockDim.x) {
                const int tl = q / per, k = (int)rank * per + q % per;
                const int64_t t = t0 + tl;
                const float4 xv = __ldcg(reinterpret_cast<const float4 *>(x + t * n_embd) + k);
                const float4 rv = __ldcg(reinterpret_cast<const float4 *>(an.r + t * n_embd) + k);
                if (an.sum_out) reinterpret_cast<float4 *>(an.sum_out + t * n_embd)[k] = f4_add(xv, rv);
                if (an.norm_out)
                    reinterpret_cast<float4 *>(an.norm_out + t * n_embd)[k] =
                        reinterpret_cast<const float4 *>(xs + (size_t)tl * n_embd)[k];
            }
        }
    }
    if (idx && warp == 0 && (int)rank < nt) {
        const float4 v = *reinterpret_cast<const float4 *>(lg + 4 * lane);
        const float xv[4] = {v.x, v.y, v.z, v.w};
        const int64_t tw = t0 + rank;
        router_select<4>(xv, lane, n_used, norm_topk, nullptr, idx + tw * n_used, scores + tw * n_used);
    }
}

template <int TOK, bool FUSE>
cudaError_t launch_resident(const LaunchCtx &c, const float *x, const float *W, float *logits_out, int32_t *idx,
                            float *scores, int64_t n_tokens, int n_embd, int n_used, int norm_topk,
                            const AddNorm &an)
{
    auto kern = router_gemv_resident_k<TOK, FUSE>;
    static bool configured = false;
    if (!configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)res_smem(TOK, kResMaxEmbd));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((n_tokens + TOK - 1) / TOK) * kResCN));
    cfg.blockDim = dim3(res_threads(TOK));
    cfg.dynamicSmemBytes = res_smem(TOK, n_embd);
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kResCN;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk, c.err,
                              an);
}

// Clusters of 8 resident at once for the resident-weight kernel with TOK
// tokens per cluster (queried once per TOK).
template <int TOK>
int resident_clusters()
{
    static int n = -1;
    if (n < 0) {
        auto kern = router_gemv_resident_k<TOK, false>;
        n = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)res_smem(TOK, kResMaxEmbd)) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(kResCN);
            cfg.blockDim = dim3(res_threads(TOK));
            cfg.dynamicSmemBytes = res_smem(TOK, kResMaxEmbd);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kResCN;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
        }
        cudaGetLastError();
    }
    return n;
}

// Runs the resident-weight kernel when the shape allows it and one wave of
// clusters covers the tokens; returns cudaErrorNotSupported otherwise.
template <bool FUSE>
cudaError_t try_resident(const LaunchCtx &c, const float *x, const float *W, float *logits_out, int32_t *idx,
                         float *scores, int64_t n_tokens, int n_embd, int n_used, int norm_topk, const AddNorm &an)
{
    if (n_embd > kResMaxEmbd || n_embd % 128 != 0) return cudaErrorNotSupported;
    if (n_tokens <= 2LL * resident_clusters<2>())
        return launch_resident<2, FUSE>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk, an);
    if (n_tokens <= 4LL * resident_clusters<4>())
        return launch_resident<4, FUSE>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk, an);
    if (n_tokens <= 8LL * resident_clusters<8>())
        return launch_resident<8, FUSE>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk, an);
    return cudaErrorNotSupported;
}

}  // namespace

bool router_gemv_fast(int64_t n_tokens, int n_embd, int n_expert, int n_used, const void *x, const void *W)
{
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W);
    return n_expert == kRgE && n_embd % kClKC == 0 && n_used <= 32 && (al & 15u) == 0 && n_tokens > 0;
}

cudaError_t launch_router_gemv_topk(const LaunchCtx &c, const float *x, const float *W, float *logits_out,
                                    int32_t *idx, float *scores, int64_t n_tokens, int n_embd, int n_expert,
                                    int n_used, int norm_topk, bool w_static)
{
    if (n_tokens <= 0) return cudaSuccess;
    if (!idx && !logits_out) return cudaErrorInvalidValue;
    if (router_gemv_fast(n_tokens, n_embd, n_expert, n_used, x, W)) {
        // Each sum is a chain of n_embd dependent adds, so a warp's time is set
        // by how many tokens it holds; up to kSmallT tokens (decode batches)
        // one token per compute warp keeps that chain 4x shorter.
        const cudaError_t er =
            try_resident<false>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk,
                                AddNorm{nullptr, nullptr, nullptr, nullptr, 0.0f, w_static ? 1 : 0});
        if (er != cudaErrorNotSupported) return er;
        if (n_tokens <= kSmallT)
            return launch_cluster<4, 4, 1, 4>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk);
        return launch_cluster<4, 4, 4, 4>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk);
    }
    if (!logits_out) return cudaErrorInvalidValue;  // the general path needs the logits buffer
    const int64_t n = n_tokens * n_expert;
    launch_k(c, router_logits_k, dim3((unsigned)((n + 255) / 256)), dim3(256), x, W, logits_out, n_tokens, n_embd,
             n_expert);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !idx) return e;
    return launch_router_topk(c, logits_out, nullptr, idx, scores, n_tokens, n_expert, n_used, norm_topk);
}

bool add_norm_router_fast(int64_t n_tokens, int n_embd, int n_expert, int n_used, const void *x, const void *r,
                          const void *W)
{
    const uintptr_t al = reinterpret_cast<uintptr_t>(r);
    return router_gemv_fast(n_tokens, n_embd, n_expert, n_used, x, W) && n_embd % 128 == 0 &&
           n_embd <= kFuseMaxEmbd && (al & 15u) == 0;
}

cudaError_t launch_add_norm_router_topk(const LaunchCtx &c, const float *x, const float *r, const float *norm_w,
                                        const float *W, float *sum_out, float *norm_out, float *logits_out,
                                        int32_t *idx, float *scores, int64_t n_tokens, int n_embd, int n_expert,
                                        int n_used, int norm_topk, float eps)
{
    if (n_tokens <= 0) return cudaSuccess;
    if (!add_norm_router_fast(n_tokens, n_embd, n_expert, n_used, x, r, W)) return cudaErrorInvalidValue;
    const AddNorm an{r, norm_w, sum_out, norm_out, eps, 1};
    const cudaError_t er = try_resident<true>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk, an);
    if (er != cudaErrorNotSupported) return er;
    if (n_tokens <= kSmallT)
        return launch_cluster<4, 4, 1, 4, true>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used,
                                                norm_topk, an);
    return launch_cluster<4, 4, 4, 4, true>(c, x, W, logits_out, idx, scores, n_tokens, n_embd, n_used, norm_topk,
                                            an);
}

}  // namespace ds3
