// Device-side MoE token permutation (sm_100a): per-expert token lists built
// from the router's top-k on the GPU.
//
// Reference: the host loop of forward_chunk_post_gathered
// (src/ds3_engine.c:933-965), which reads idx/scores back to the host every
// layer (:1256-1261) and writes, for expert ex, the tokens that chose it to
// ids[ex * M + j] (j = running count, so tokens in ascending order, each
// token's k slots in order) and their scores alongside; counts[ex] = j.
//
// One CTA per expert, all experts in parallel. CTA ex walks the T*K
// (token, slot) entries in entry order, 4096 at a time, 4 consecutive entries
// per thread: each thread counts its hits, one CTA-wide exclusive scan (two
// warp scans) gives every hit its rank, and a running base carries over
// between passes. Every hit lands at ids[ex*cap + j] in the
// engine's order, with no atomics and no memory beyond the outputs.
// slot_of[t*K+k] = ex*cap + j is written by the CTA of the entry's expert; it
// is the row map moe_combine_residual takes to read expert outputs laid out
// per expert. CTA 0 also flags entries whose expert id is out of range.
#include "common.cuh"
#include "launch.h"

namespace ds3 {
namespace {

constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kPerThread = 4;                              // consecutive entries per thread
constexpr int kRouteChunk = kRouteThreads * kPerThread;    // 4096 = 512 tokens x top-8 in one pass

__global__ void __launch_bounds__(kRouteThreads) moe_expert_lists_k(
    const int32_t *idx, const float *scores, int32_t *counts, int32_t *ids, float *gscores, int32_t *slot_of,
    int64_t n_entries, int n_used, int n_expert, int64_t cap, unsigned *err)
{
    __shared__ int32_t wpre[kRouteWarps];
    __shared__ int32_t total;
    pdl_wait();
    pdl_trigger();
    const int ex = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int64_t base = 0;
    for (int64_t s0 = 0; s0 < n_entries; s0 += kRouteChunk) {
        // Entries s0 + 4*tid .. +3: ids and scores are loaded together, before
        // either is used, so the pass costs one memory round trip.
        const int64_t i0 = s0 + (int64_t)kPerThread * tid;
        int ev[kPerThread];
        float sv[kPerThread];
#pragma unroll
        for (int c = 0; c < kPerThread; c++) {
            const bool in = i0 + c < n_entries;
            ev[c] = in ? idx[i0 + c] : -1;
            sv[c] = in ? scores[i0 + c] : 0.0f;
        }
        int mine = 0;
#pragma unroll
        for (int c = 0; c < kPerThread; c++) {
            mine += ev[c] == ex;
            if (ex == 0 && i0 + c < n_entries && (ev[c] < 0 || ev[c] >= n_expert)) {
                flag_error(err, kErrBadId);
                if (slot_of) slot_of[i0 + c] = -1;
            }
        }
        // Exclusive scan of the hit counts over the CTA, in entry order.
        int inc = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) wpre[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            const int v = wpre[lane];
            int w = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(kFull, w, o);
                if (lane >= o) w += y;
            }
            wpre[lane] = w - v;
            if (lane == 31) total = w;
        }
        __syncthreads();
        int64_t j = base + wpre[warp] + (inc - mine);
#pragma unroll
        for (int c = 0; c < kPerThread; c++) {
            if (ev[c] != ex) continue;
            const int64_t i = i0 + c;
            if (j < cap) {
                const int64_t slot = (int64_t)ex * cap + j;
                ids[slot] = (int32_t)(i / n_used);
                gscores[slot] = sv[c];
                if (slot_of) slot_of[i] = (int32_t)slot;
            } else {
                flag_error(err, kErrBadId);
                if (slot_of) slot_of[i] = -1;
            }
            j++;
        }
        base += total;
        __syncthreads();  // wpre / total are rewritten by the next pass
    }
    // Clamped to the list capacity: a consumer looping j < counts[ex] stays
    // inside this expert's list (an overflow is already flagged above).
    if (tid == 0) counts[ex] = (int32_t)(base < cap ? base : cap);
}

// Self-test of the bounded mbarrier wait: the barrier expects one arrival
// that never comes; the wait must give up after `polls` polls and record the
// timeout in the error word.
__global__ void bounded_wait_selftest_k(uint32_t polls, unsigned *err)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
    }
    __syncwarp();
    if (!mbar_wait(&bar, 0, polls) && threadIdx.x == 0) flag_error(err, kErrWaitTimeout);
}

}  // namespace

int kernel_binary_version()
{
    cudaFuncAttributes a;
    if (cudaFuncGetAttributes(&a, bounded_wait_selftest_k) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return a.binaryVersion;
}

cudaError_t launch_bounded_wait_selftest(const LaunchCtx &c, uint32_t polls)
{
    bounded_wait_selftest_k<<<1, 32, 0, c.stream>>>(polls, c.err);
    return cudaGetLastError();
}

cudaError_t launch_moe_expert_lists(const LaunchCtx &c, const int32_t *idx, const float *scores, int32_t *counts,
                                    int32_t *ids, float *gscores, int32_t *slot_of, int64_t n_tokens, int n_used,
                                    int n_expert, int64_t cap)
{
    if (n_expert <= 0 || n_expert > 65535) return cudaErrorInvalidValue;
    launch_k(c, moe_expert_lists_k, dim3((unsigned)n_expert), dim3(kRouteThreads), idx, scores, counts, ids, gscores, slot_of,
             n_tokens * n_used, n_used, n_expert, cap, c.err);
    return cudaGetLastError();
}

}  // namespace ds3
