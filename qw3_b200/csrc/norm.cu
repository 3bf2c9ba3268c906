// RMSNorm and fused residual-add + RMSNorm (sm_100a).
//
// Reference semantics: ds3_ref_rms_norm (src/ds3_reference.c:329-342),
// ds3_ref_add (:455-460); Metal kernel metal/rms_norm.metal:16-69.
//
// Fast path: one warp per row, the whole row held in registers (VPL float4
// per lane, n = 128 * VPL), so x and the residual are read from HBM exactly
// once and sum/normed are written exactly once: 16 B/elem for add+norm with
// the sum stored, 8 B/elem for a plain norm. Loads are 128-bit, coalesced
// (lane l reads float4 l, l+32, ...), all issued before the first use.
// Generic path (any n): one CTA per row, two passes (the second hits L1/L2).
#include "common.cuh"
#include "launch.h"

namespace ds3 {
namespace {

template <int VPL>
__global__ void __launch_bounds__(128) add_rms_norm_warp(const float *x, const float *r,
                                                         const float *w, float *sum_out,
                                                         float *norm_out, int64_t rows, float eps)
{
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    constexpr int n = VPL * 128;
    const float4 *xr = reinterpret_cast<const float4 *>(x + row * n);

    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = ld_stream(xr + i * 32 + lane);
    if (r) {
        const float4 *rr = reinterpret_cast<const float4 *>(r + row * n);
        float4 b[VPL];
#pragma unroll
        for (int i = 0; i < VPL; i++) b[i] = ld_stream(rr + i * 32 + lane);
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] = f4_add(v[i], b[i]);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; i++) ss = f4_sumsq(v[i], ss);
    ss = warp_sum(ss);
    const float inv = rms_inv_n<n>(ss, eps);

    if (sum_out) {
        float4 *so = reinterpret_cast<float4 *>(sum_out + row * n);
#pragma unroll
        for (int i = 0; i < VPL; i++) so[i * 32 + lane] = v[i];
    }
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    float4 *no = reinterpret_cast<float4 *>(norm_out + row * n);
#pragma unroll
    for (int i = 0; i < VPL; i++) no[i * 32 + lane] = f4_norm(v[i], inv, ld_param(w4 + i * 32 + lane));
}

// Any n. Pass 1: s = x (+ r), written to sum_out when given, sum of squares.
// Pass 2: every thread revisits exactly the elements it produced (same index
// mapping), reading s back from sum_out (or recomputing x + r), so aliasing
// of sum_out / norm_out with x or r is safe.
__global__ void __launch_bounds__(256) add_rms_norm_block(const float *x, const float *r,
                                                          const float *w, float *sum_out,
                                                          float *norm_out, int n, float eps)
{
    pdl_wait();
    pdl_trigger();
    __shared__ float part[32];
    const int64_t row = blockIdx.x;
    const float *xr = x + row * n;
    const float *rr = r ? r + row * n : nullptr;
    float *sr = sum_out ? sum_out + row * n : nullptr;
    float *nr = norm_out + row * n;

    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float s = xr[i];
        if (rr) s = __fadd_rn(s, rr[i]);
        if (sr) sr[i] = s;
        ss = sq_acc(ss, s);
    }
    ss = warp_sum(ss);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) part[wid] = ss;
    __syncthreads();
    if (wid == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) part[0] = t;
    }
    __syncthreads();
    const float inv = rms_inv(part[0], n, eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float s;
        if (sr) s = sr[i];
        else s = rr ? __fadd_rn(xr[i], rr[i]) : xr[i];
        nr[i] = norm_mul(s, inv, w[i]);
    }
}

template <int VPL>
cudaError_t run_warp(const LaunchCtx &c, const float *x, const float *r, const float *w,
                     float *sum_out, float *norm_out, int64_t rows, float eps)
{
    const int warps = 4;
    const int64_t blocks = (rows + warps - 1) / warps;
    launch_k(c, add_rms_norm_warp<VPL>, dim3((unsigned)blocks), dim3(warps * 32), x, r, w, sum_out, norm_out,
                                                                          rows, eps);
    return cudaGetLastError();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t launch_add_rms_norm(const LaunchCtx &c, const float *x, const float *r, const float *w,
                                float *sum_out, float *norm_out, int n, int64_t rows, float eps)
{
    if (rows <= 0 || n <= 0) return cudaSuccess;
    const bool vec = (n % 128) == 0 && aligned16(x) && aligned16(w) && aligned16(norm_out) &&
                     (!r || aligned16(r)) && (!sum_out || aligned16(sum_out));
    if (vec) {
        switch (n / 128) {
        case 1: return run_warp<1>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 2: return run_warp<2>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 4: return run_warp<4>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 6: return run_warp<6>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 8: return run_warp<8>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 12: return run_warp<12>(c, x, r, w, sum_out, norm_out, rows, eps);
        case 16: return run_warp<16>(c, x, r, w, sum_out, norm_out, rows, eps);
        default: break;
        }
    }
    if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    launch_k(c, add_rms_norm_block, dim3((unsigned)rows), dim3(256), x, r, w, sum_out, norm_out, n, eps);
    return cudaGetLastError();
}

}  // namespace ds3
