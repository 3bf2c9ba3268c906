// Routed-expert elementwise kernels and the small FP32 helpers (sm_100a):
// SwiGLU (optionally weighted), weighted combine + residual, vec_add,
// gather/scatter of rows.
//
// References: ds3_ref_silu / ds3_ref_mul (src/ds3_reference.c:436-448),
// moe_expert_silu_mul_f32 (metal/moe.metal:95-108); the weighted expert
// accumulation and residual add of ds3_ref_moe_ffn / ds3_ref_layer_forward
// (src/ds3_reference.c:642, :674-678, :777); vec_add / gather_rows /
// scatter_add_weighted (metal/elementwise.metal:146-211).
//
// All are streaming kernels: 128-bit loads/stores, several independent
// 16-byte loads in flight per thread, grids sized to fill the 148 SMs.
#include "common.cuh"
#include "launch.h"

namespace ds3 {
namespace {

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float silu_mul(float g, float u)
{
    // (g / (1 + expf(-g))) * u, each step rounded as the reference's C.
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(s, u);
}

// ------------------------------------------------------------------ SwiGLU
// Each thread owns kSwigluUnits float4 units (stride = total threads) and
// issues all 2 x kSwigluUnits 128-bit loads before computing, so at the
// 4096 x 768 shape one resident wave holds the whole input in flight.
constexpr int kSwigluUnits = 4;

template <typename Index>
__global__ void __launch_bounds__(256, 4) swiglu_vec(const float4 *gate, const float4 *up,
                                                     const float *row_w, float4 *out, Index units,
                                                     Index cols4)
{
    pdl_wait();
    pdl_trigger();
    const Index stride = (Index)gridDim.x * blockDim.x;
    for (Index u0 = (Index)blockIdx.x * blockDim.x + threadIdx.x; u0 < units; u0 += stride * kSwigluUnits) {
        float4 g[kSwigluUnits], v[kSwigluUnits];
#pragma unroll
        for (int k = 0; k < kSwigluUnits; k++) {
            const Index u = u0 + k * stride;
            if (u < units) {
                g[k] = ld_stream(gate + u);
                v[k] = ld_stream(up + u);
            }
        }
#pragma unroll
        for (int k = 0; k < kSwigluUnits; k++) {
            const Index u = u0 + k * stride;
            if (u >= units) break;
            float4 o = make_float4(silu_mul(g[k].x, v[k].x), silu_mul(g[k].y, v[k].y),
                                   silu_mul(g[k].z, v[k].z), silu_mul(g[k].w, v[k].w));
            if (row_w) {
                const float w = __ldg(row_w + u / cols4);
                o = make_float4(__fmul_rn(o.x, w), __fmul_rn(o.y, w), __fmul_rn(o.z, w), __fmul_rn(o.w, w));
            }
            out[u] = o;
        }
    }
}

// Non-persistent variant: CTA b owns units [b*256*U, (b+1)*256*U); thread t
// handles units base + t + k*256 (k < U, coalesced per k), all 2*U loads
// issued before any result is used.
template <int U>
__global__ void __launch_bounds__(256) swiglu_blk(const float4 *gate, const float4 *up, const float *row_w,
                                                  float4 *out, uint32_t units, uint32_t cols4)
{
    if (threadIdx.x < 2) {  // this CTA's gate / up ranges, into L2 while the previous kernel runs
        const uint32_t u0 = blockIdx.x * (256u * U);
        const uint32_t n = units - u0 < 256u * U ? units - u0 : 256u * U;
        prefetch_l2((threadIdx.x ? up : gate) + u0, (uint64_t)n * sizeof(float4));
    }
    pdl_wait();
    pdl_trigger();
    const uint32_t base = blockIdx.x * (256u * U) + threadIdx.x;
    float4 g[U], v[U];
    float rw[U];
    // All loads, the routing weight included, are issued before any is used,
    // so the launch costs one memory round trip.
#pragma unroll
    for (int k = 0; k < U; k++) {
        const uint32_t u = base + 256u * k;
        rw[k] = 1.0f;
        if (u < units) {
            g[k] = ld_stream_inflight(gate + u);
            v[k] = ld_stream_inflight(up + u);
            if (row_w) rw[k] = ld_param_f(row_w + u / cols4);
        }
    }
#pragma unroll
    for (int k = 0; k < U; k++) {
        const uint32_t u = base + 256u * k;
        if (u >= units) break;
        float4 o = make_float4(silu_mul(g[k].x, v[k].x), silu_mul(g[k].y, v[k].y), silu_mul(g[k].z, v[k].z),
                               silu_mul(g[k].w, v[k].w));
        if (row_w) {
            const float w = rw[k];
            o = make_float4(__fmul_rn(o.x, w), __fmul_rn(o.y, w), __fmul_rn(o.z, w), __fmul_rn(o.w, w));
        }
        out[u] = o;
    }
}

__global__ void swiglu_scalar(const float *gate, const float *up, const float *row_w, float *out,
                              int64_t n, int64_t cols)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float o = silu_mul(gate[i], up[i]);
        if (row_w) o = __fmul_rn(o, row_w[i / cols]);
        out[i] = o;
    }
}

// --------------------------------------------------------- combine + residual
// One thread per (token, float4 column): all n_used expert rows of that
// column are loaded before the sum, which runs from zero in k order.
// A mapped row outside [0, n_y_rows) (a -1 from moe_expert_lists for a bad
// expert id or a full list) reads as a zero row and sets the bad-id bit of
// the error word; y is never read out of bounds.
__device__ __forceinline__ bool row_ok(int64_t r, int64_t n_y_rows, unsigned *err, bool report)
{
    if (r >= 0 && r < n_y_rows) return true;
    if (report) flag_error(err, kErrBadId);
    return false;
}

template <int K>
__global__ void __launch_bounds__(128) combine_vec(const float4 *y, const int32_t *y_rows,
                                                   const float *w, const float4 *residual,
                                                   float4 *out, int64_t n_tokens, int n_used,
                                                   int64_t cols4, int64_t n_y_rows, unsigned *err)
{
    pdl_wait();
    pdl_trigger();
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n_tokens * cols4) return;
    const int64_t t = e / cols4;
    const int64_t c = e - t * cols4;
    const int nk = K > 0 ? K : n_used;
    const float4 res = ld_stream(residual + e);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (K > 0) {
        float4 yv[K];
        float wk[K];
#pragma unroll
        for (int k = 0; k < K; k++) {
            const int64_t r = y_rows ? (int64_t)y_rows[t * K + k] : t * K + k;
            yv[k] = row_ok(r, n_y_rows, err, c == 0) ? ld_stream(y + r * cols4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            wk[k] = __ldg(w + t * K + k);
        }
#pragma unroll
        for (int k = 0; k < K; k++) {
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk[k], yv[k].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk[k], yv[k].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk[k], yv[k].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk[k], yv[k].w));
        }
    } else {
        for (int k = 0; k < nk; k++) {
            const int64_t r = y_rows ? (int64_t)y_rows[t * nk + k] : t * nk + k;
            const float4 yv =
                row_ok(r, n_y_rows, err, c == 0) ? ld_stream(y + r * cols4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float wk = __ldg(w + t * nk + k);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk, yv.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk, yv.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk, yv.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk, yv.w));
        }
    }
    out[e] = f4_add(res, acc);
}

// Token-major expert outputs, 8 experts, 32-bit indices: the nine 128-bit
// loads are volatile asm statements, so all are issued before the first is
// consumed (the generic kernel lets the compiler interleave them with the
// sum; measured at T=512: 7.3 vs 7.6-8.2 us).
template <int U>
__global__ void __launch_bounds__(128) combine8_tokmajor(const float4 *y, const float *w, const float4 *residual,
                                                         float4 *out, uint32_t n_tokens, uint32_t cols4)
{
    const uint32_t total = n_tokens * cols4;
    const uint32_t base = blockIdx.x * (128u * U) + threadIdx.x;
    {
        // Lane k < 8 of each warp prefetches the warp's columns of expert row
        // k into L2, lane 8 those of the residual (split where the warp's 32
        // units straddle two tokens), while the previous kernel runs.
        const uint32_t lane = threadIdx.x & 31;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t e0 = base - lane + 128u * u;
            if (lane < 9 && e0 < total) {
                const uint32_t e1 = (e0 + 32 < total ? e0 + 32 : total);  // one past the warp's last unit
                for (uint32_t a = e0; a < e1;) {
                    const uint32_t t = a / cols4, c = a - t * cols4;
                    const uint32_t n = (cols4 - c < e1 - a) ? cols4 - c : e1 - a;
                    prefetch_l2(lane < 8 ? y + (t * 8 + lane) * cols4 + c : residual + a, (uint64_t)n * sizeof(float4));
                    a += n;
                }
            }
        }
    }
    pdl_wait();
    pdl_trigger();
    float4 yv[U][8], res[U];
    float wk[U][8];
#pragma unroll
    for (int u = 0; u < U; u++) {
        const uint32_t e = base + 128u * u;
        if (e >= total) continue;
        const uint32_t t = e / cols4, c = e - t * cols4;
#pragma unroll
        for (int k = 0; k < 8; k++) yv[u][k] = ld_stream_inflight(y + (t * 8 + k) * cols4 + c);
        res[u] = ld_stream_inflight(residual + e);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        const uint32_t e = base + 128u * u;
        if (e >= total) continue;
        const uint32_t t = e / cols4;
#pragma unroll
        for (int k = 0; k < 8; k++) wk[u][k] = __ldg(w + t * 8 + k);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        const uint32_t e = base + 128u * u;
        if (e >= total) continue;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk[u][k], yv[u][k].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk[u][k], yv[u][k].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk[u][k], yv[u][k].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk[u][k], yv[u][k].w));
        }
        out[e] = f4_add(res[u], acc);
    }
}

__global__ void combine_scalar(const float *y, const int32_t *y_rows, const float *w,
                               const float *residual, float *out, int64_t n_tokens, int n_used,
                               int64_t cols, int64_t n_y_rows, unsigned *err)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_tokens * cols;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / cols, c = e - t * cols;
        float acc = 0.0f;
        for (int k = 0; k < n_used; k++) {
            const int64_t r = y_rows ? (int64_t)y_rows[t * n_used + k] : t * n_used + k;
            const float yv = row_ok(r, n_y_rows, err, c == 0) ? y[r * cols + c] : 0.0f;
            acc = __fadd_rn(acc, __fmul_rn(w[t * n_used + k], yv));
        }
        out[e] = __fadd_rn(residual[e], acc);
    }
}

// ----------------------------------------------------------------- vec_add
// Up to 2^31 float4 units: one unit per thread, both loads issued before the
// add, a non-persistent grid (the same shape as swiglu_blk).
__global__ void __launch_bounds__(256) vec_add_blk(const float4 *a, const float4 *b, float4 *c, uint32_t n4)
{
    pdl_wait();
    pdl_trigger();
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i >= n4) return;
    const float4 x = ld_stream_inflight(a + i), y = ld_stream_inflight(b + i);
    c[i] = f4_add(x, y);
}

__global__ void vec_add_vec(const float4 *a, const float4 *b, float4 *c, int64_t n4)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x)
        c[i] = f4_add(ld_stream(a + i), ld_stream(b + i));
}

__global__ void vec_add_scalar(const float *a, const float *b, float *c, int64_t n)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        c[i] = __fadd_rn(a[i], b[i]);
}

// ------------------------------------------------------- gather / scatter
__global__ void gather_rows_k(const float *src, const int32_t *ids, float *dst, int64_t n_cols,
                              int64_t count, int64_t n_src_rows, unsigned *err)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count * n_cols;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / n_cols, j = e - i * n_cols;
        const int64_t r = ids[i];
        if (r < 0 || r >= n_src_rows) {
            if (j == 0) flag_error(err, kErrBadId);
            dst[e] = 0.0f;
            continue;
        }
        dst[e] = src[r * n_cols + j];
    }
}

__global__ void scatter_add_k(const float *src, const float *scores, const int32_t *ids, float *dst,
                              int64_t n_cols, int64_t count, int64_t n_dst_rows, unsigned *err)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count * n_cols;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / n_cols, j = e - i * n_cols;
        const int64_t r = ids[i];
        if (r < 0 || r >= n_dst_rows) {
            if (j == 0) flag_error(err, kErrBadId);
            continue;
        }
        float *d = dst + r * n_cols + j;
        *d = __fadd_rn(*d, __fmul_rn(scores[i], src[e]));
    }
}

unsigned grid_for(const LaunchCtx &c, int64_t work, int threads, int per_sm)
{
    int64_t b = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)c.n_sm * per_sm;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (unsigned)b;
}

}  // namespace

cudaError_t launch_swiglu(const LaunchCtx &c, const float *gate, const float *up,
                          const float *row_w, float *out, int64_t rows, int64_t cols)
{
    const int64_t n = rows * cols;
    if (n <= 0) return cudaSuccess;
    if (cols % 4 == 0 && al16(gate) && al16(up) && al16(out)) {
        const int64_t units = n / 4;
        // Non-persistent blocks (measured, 4096 x 768: 7.9 us vs 9.7 us for the
        // persistent grid-stride kernel; 32768 x 768: 46 us vs 56 us).
        if (units < ((int64_t)1 << 31)) {
            auto *g4 = reinterpret_cast<const float4 *>(gate);
            auto *u4 = reinterpret_cast<const float4 *>(up);
            auto *o4 = reinterpret_cast<float4 *>(out);
            const uint32_t uu = (uint32_t)units, c4 = (uint32_t)(cols / 4);
            // Two units per thread at every size: at the 4096 x 768 chunk shape the
            // grid then nearly fits one resident wave, so the next kernel's CTAs
            // become resident (and start their L2 prefetch) sooner; measured in
            // the T=512 step 29.0 vs 29.7 us with one unit (3 or 4 units: 30.3).
            launch_k(c, swiglu_blk<2>, dim3((uu + 511) / 512), dim3(256), g4, u4, row_w, o4, uu, c4);
            return cudaGetLastError();
        }
        // Beyond 2^31 units: the persistent grid-stride kernel with 64-bit indices.
        static int occ = 0;
        if (!occ && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, swiglu_vec<int64_t>, 256, 0) != cudaSuccess)
            occ = 4;
        const unsigned blocks = grid_for(c, (units + kSwigluUnits - 1) / kSwigluUnits, 256, occ > 0 ? occ : 4);
        launch_k(c, swiglu_vec<int64_t>, dim3(blocks), dim3(256), reinterpret_cast<const float4 *>(gate),
                 reinterpret_cast<const float4 *>(up), row_w, reinterpret_cast<float4 *>(out), units, cols / 4);
    } else {
        launch_k(c, swiglu_scalar, dim3(grid_for(c, n, 256, 16)), dim3(256), gate, up, row_w, out, n, cols);
    }
    return cudaGetLastError();
}

cudaError_t launch_combine(const LaunchCtx &c, const float *y, const int32_t *y_rows,
                           const float *w, const float *residual, float *out, int64_t n_tokens,
                           int n_used, int64_t n_cols, int64_t n_y_rows)
{
    if (n_tokens <= 0 || n_cols <= 0) return cudaSuccess;
    if (n_cols % 4 == 0 && al16(y) && al16(residual) && al16(out)) {
        const int64_t cols4 = n_cols / 4;
        const int64_t total = n_tokens * cols4;
        const unsigned blocks = (unsigned)((total + 127) / 128);
        auto *y4 = reinterpret_cast<const float4 *>(y);
        auto *r4 = reinterpret_cast<const float4 *>(residual);
        auto *o4 = reinterpret_cast<float4 *>(out);
        if (n_used == 8 && !y_rows && total * 8 < ((int64_t)1 << 31)) {
            const uint32_t tt = (uint32_t)n_tokens, c4 = (uint32_t)cols4, tot = (uint32_t)total;
            // Two units per thread: half the threads, so the next kernel's CTAs
            // find room to become resident early (T=512 step 29.3 -> 28.8 us).
            launch_k(c, combine8_tokmajor<2>, dim3((tot + 255) / 256), dim3(128), y4, w, r4, o4, tt, c4);
            return cudaGetLastError();
        }
        if (n_used == 8)
            launch_k(c, combine_vec<8>, dim3(blocks), dim3(128), y4, y_rows, w, r4, o4, n_tokens, n_used, cols4,
                     n_y_rows, c.err);
        else
            launch_k(c, combine_vec<0>, dim3(blocks), dim3(128), y4, y_rows, w, r4, o4, n_tokens, n_used, cols4,
                     n_y_rows, c.err);
    } else {
        launch_k(c, combine_scalar, dim3(grid_for(c, n_tokens * n_cols, 256, 16)), dim3(256), 
            y, y_rows, w, residual, out, n_tokens, n_used, n_cols, n_y_rows, c.err);
    }
    return cudaGetLastError();
}

cudaError_t launch_vec_add(const LaunchCtx &c, const float *a, const float *b, float *out, int64_t n)
{
    if (n <= 0) return cudaSuccess;
    if (n % 4 == 0 && al16(a) && al16(b) && al16(out) && n / 4 < ((int64_t)1 << 31))
        launch_k(c, vec_add_blk, dim3((unsigned)((n / 4 + 255) / 256)), dim3(256), reinterpret_cast<const float4 *>(a),
                 reinterpret_cast<const float4 *>(b), reinterpret_cast<float4 *>(out), (uint32_t)(n / 4));
    else if (n % 4 == 0 && al16(a) && al16(b) && al16(out))
        launch_k(c, vec_add_vec, dim3(grid_for(c, n / 4, 256, 16)), dim3(256), 
            reinterpret_cast<const float4 *>(a), reinterpret_cast<const float4 *>(b),
            reinterpret_cast<float4 *>(out), n / 4);
    else
        launch_k(c, vec_add_scalar, dim3(grid_for(c, n, 256, 16)), dim3(256), a, b, out, n);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const LaunchCtx &c, const float *src, const int32_t *ids,
                               float *dst, int64_t n_cols, int64_t count, int64_t n_src_rows)
{
    if (count <= 0 || n_cols <= 0) return cudaSuccess;
    launch_k(c, gather_rows_k, dim3(grid_for(c, count * n_cols, 256, 16)), dim3(256), src, ids, dst, n_cols, count,
                                                                             n_src_rows, c.err);
    return cudaGetLastError();
}

cudaError_t launch_scatter_add_weighted(const LaunchCtx &c, const float *src, const float *scores,
                                        const int32_t *ids, float *dst, int64_t n_cols,
                                        int64_t count, int64_t n_dst_rows)
{
    if (count <= 0 || n_cols <= 0) return cudaSuccess;
    launch_k(c, scatter_add_k, dim3(grid_for(c, count * n_cols, 256, 16)), dim3(256), 
        src, scores, ids, dst, n_cols, count, n_dst_rows, c.err);
    return cudaGetLastError();
}

}  // namespace ds3
