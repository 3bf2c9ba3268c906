// Warp-level router selection shared by the router kernels: softmax over
// the 32*V logits a warp holds (lane l: experts l*V .. l*V+V-1), top n_used
// by (logit desc, index asc), optional renorm; see router.cu for the
// reference semantics.
#pragma once

#include <climits>

#include "common.cuh"

namespace ds3 {

// Monotone map of a (non-NaN) float onto unsigned integers.
__device__ __forceinline__ unsigned order_key(float x)
{
    const unsigned u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// probs_row (may be null): [32*V] full softmax; idx_row / sc_row: [n_used].
template <int V>
__device__ __forceinline__ void router_select(const float *x, int lane, int n_used, int norm_topk, float *probs_row,
                                              int32_t *idx_row, float *sc_row)
{
    float mx = x[0];
#pragma unroll
    for (int j = 1; j < V; j++) mx = fmaxf(mx, x[j]);
    mx = warp_max(mx);
    float p[V];
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < V; j++) {
        p[j] = expf(__fsub_rn(x[j], mx));
        part = __fadd_rn(part, p[j]);
    }
    const float total = warp_sum(part);
    const float inv = __fdiv_rn(1.0f, total);
#pragma unroll
    for (int j = 0; j < V; j++) p[j] = __fmul_rn(p[j], inv);

    if (probs_row) {
        float *po = probs_row + lane * V;
        if constexpr (V % 4 == 0) {
#pragma unroll
            for (int j = 0; j < V; j += 4)
                *reinterpret_cast<float4 *>(po + j) = make_float4(p[j], p[j + 1], p[j + 2], p[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < V; j++) po[j] = p[j];
        }
    }

    // Selection keys: the float order of the logits as unsigned integers, so a
    // round is a local scan plus one redux.sync max and one ballot (lowest
    // lane = lowest expert index among equal logits; -0 is folded into +0).
    unsigned key[V];
#pragma unroll
    for (int j = 0; j < V; j++) key[j] = order_key(__fadd_rn(x[j], 0.0f));
    unsigned used = 0;
    int my_idx = -1;
    float my_sc = 0.0f;
    float sum_sel = 0.0f;
    for (int k = 0; k < n_used; k++) {
        unsigned best = 0;
        int bj = -1;
#pragma unroll
        for (int j = 0; j < V; j++)
            if (!((used >> j) & 1u) && key[j] > best) {
                best = key[j];
                bj = j;
            }
        const unsigned m = __reduce_max_sync(kFull, best);
        const unsigned ball = __ballot_sync(kFull, bj >= 0 && best == m);
        if (ball == 0) break;  // fewer experts than n_used (host rejects this)
        const int owner = __ffs(ball) - 1;
        const int sel = __shfl_sync(kFull, bj, owner);
        float pj = p[0];
#pragma unroll
        for (int j = 1; j < V; j++)
            if (j == sel) pj = p[j];
        if (lane == owner) used |= 1u << sel;
        const float sc = __shfl_sync(kFull, pj, owner);
        sum_sel = __fadd_rn(sum_sel, sc);
        if (lane == k) {
            my_idx = owner * V + sel;
            my_sc = sc;
        }
    }
    if (norm_topk && sum_sel > 0.0f) my_sc = __fmul_rn(my_sc, __fdiv_rn(1.0f, sum_sel));
    if (lane < n_used) {
        idx_row[lane] = my_idx;
        sc_row[lane] = my_sc;
    }
}

}  // namespace ds3
