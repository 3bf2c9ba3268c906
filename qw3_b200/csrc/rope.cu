// Per-head Q/K RMSNorm fused with NEOX RoPE (sm_100a).
//
// Reference: per-head ds3_ref_rms_norm (src/ds3_reference.c:526-533, engine
// src/ds3_engine.c:789-792) followed by ds3_ref_rope (:361-402); Metal
// metal/rope.metal:88-123 with the host frequency table of
// src/ds3_metal.m:478-489.
//
// Fast path (head_dim = 128): one warp owns a group of up to 8 heads of one
// token; lane l holds elements 4l..4l+3 of each head (one 128-bit load per
// head, coalesced). RoPE pairs (i, i+64) live in lanes l and l^16, exchanged
// with one shuffle. The angle of pair i depends only on (position, i), so a
// warp computes the 64 cos/sin values of its token once (2 sincosf per lane,
// shared through a shuffle) and reuses them for all its heads. Each element
// is read once and written once: 2 x 4 B (fp32) or 2 x 2 B (fp16 storage).
//
// Numerics: freq[i] = powf(theta, (float)i * (-2/hd)) is built on the host
// with the C library (same as the reference), the angle is the fp32 product
// (float)pos * freq[i] rounded once, cos/sin are CUDA's accurate sincosf, and
// the rotation is x0*c - x1*s / x0*s + x1*c with each product and sum rounded
// separately.
#include "common.cuh"
#include "launch.h"

namespace ds3 {
namespace {

struct FreqTable {
    float f[256];  // head_dim / 2 entries used (head_dim <= 512)
};

constexpr int kHeadsPerWarp = 8;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
    __device__ static float4 load(const float *p) { return ld_stream(reinterpret_cast<const float4 *>(p)); }
    __device__ static void store(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
};
template <>
struct Vec4<__half> {
    __device__ static float4 load(const __half *p)
    {
        const uint2 u = __ldcs(reinterpret_cast<const uint2 *>(p));
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    __device__ static void store(__half *p, float4 v)
    {
        __half2 a = __floats2half2_rn(v.x, v.y);
        __half2 b = __floats2half2_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<unsigned *>(&a);
        u.y = *reinterpret_cast<unsigned *>(&b);
        *reinterpret_cast<uint2 *>(p) = u;
    }
};

__device__ __forceinline__ float rot_lo(float own, float other, float c, float s)
{
    return __fsub_rn(__fmul_rn(own, c), __fmul_rn(other, s));  // x0*c - x1*s
}
__device__ __forceinline__ float rot_hi(float own, float other, float c, float s)
{
    return __fadd_rn(__fmul_rn(other, s), __fmul_rn(own, c));  // x0*s + x1*c
}

template <typename T>
__global__ void __launch_bounds__(128) qk_norm_rope_hd128(
    const T *q_src, T *q_dst, const T *k_src, T *k_dst, const float *q_w, const float *k_w,
    const int32_t *pos, int64_t rows, int nq, int nk, int chunks_q, int chunks_k,
    const __grid_constant__ FreqTable ft, float eps, int do_norm)
{
    const int lane = threadIdx.x & 31;
    const int chunks = chunks_q + chunks_k;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t t = gw / chunks;
    if (t >= rows) return;
    const int ch = (int)(gw - t * chunks);

    const T *src;
    T *dst;
    const float *w;
    int h0, nh;
    if (ch < chunks_q) {
        h0 = ch * kHeadsPerWarp;
        nh = min(kHeadsPerWarp, nq - h0);
        src = q_src + (t * nq + h0) * 128;
        dst = q_dst + (t * nq + h0) * 128;
        w = q_w;
    } else {
        h0 = (ch - chunks_q) * kHeadsPerWarp;
        nh = min(kHeadsPerWarp, nk - h0);
        src = k_src + (t * nk + h0) * 128;
        dst = k_dst + (t * nk + h0) * 128;
        w = k_w;
    }

    float4 v[kHeadsPerWarp];
#pragma unroll
    for (int h = 0; h < kHeadsPerWarp; h++)
        if (h < nh) v[h] = Vec4<T>::load(src + h * 128 + 4 * lane);

    // cos/sin of pairs i = 4*(lane&15) + j: lanes < 16 compute j = 0,1, lanes
    // >= 16 compute j = 2,3, then swap halves with lane^16.
    const float p = (float)pos[t];
    const int ib = 4 * (lane & 15) + ((lane < 16) ? 0 : 2);
    float s0, c0, s1, c1;
    sincosf(__fmul_rn(p, ft.f[ib]), &s0, &c0);
    sincosf(__fmul_rn(p, ft.f[ib + 1]), &s1, &c1);
    const float os0 = __shfl_xor_sync(kFull, s0, 16), oc0 = __shfl_xor_sync(kFull, c0, 16);
    const float os1 = __shfl_xor_sync(kFull, s1, 16), oc1 = __shfl_xor_sync(kFull, c1, 16);
    const bool lo = lane < 16;
    const float cs[4] = {lo ? c0 : oc0, lo ? c1 : oc1, lo ? oc0 : c0, lo ? oc1 : c1};
    const float sn[4] = {lo ? s0 : os0, lo ? s1 : os1, lo ? os0 : s0, lo ? os1 : s1};

    float4 wv = make_float4(1.f, 1.f, 1.f, 1.f);
    if (do_norm) wv = ld_param(reinterpret_cast<const float4 *>(w) + lane);

#pragma unroll
    for (int h = 0; h < kHeadsPerWarp; h++) {
        if (h >= nh) break;
        float4 x = v[h];
        if (do_norm) {
            const float ss = warp_sum(f4_sumsq(x, 0.0f));
            x = f4_norm(x, rms_inv(ss, 128, eps), wv);
        }
        float4 o;
        o.x = __shfl_xor_sync(kFull, x.x, 16);
        o.y = __shfl_xor_sync(kFull, x.y, 16);
        o.z = __shfl_xor_sync(kFull, x.z, 16);
        o.w = __shfl_xor_sync(kFull, x.w, 16);
        float4 y;
        if (lo) {
            y = make_float4(rot_lo(x.x, o.x, cs[0], sn[0]), rot_lo(x.y, o.y, cs[1], sn[1]),
                            rot_lo(x.z, o.z, cs[2], sn[2]), rot_lo(x.w, o.w, cs[3], sn[3]));
        } else {
            y = make_float4(rot_hi(x.x, o.x, cs[0], sn[0]), rot_hi(x.y, o.y, cs[1], sn[1]),
                            rot_hi(x.z, o.z, cs[2], sn[2]), rot_hi(x.w, o.w, cs[3], sn[3]));
        }
        Vec4<T>::store(dst + h * 128 + 4 * lane, y);
    }
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Any even head_dim <= 512: one CTA of hd/2 threads per (token, head);
// thread i owns the pair (i, i + hd/2).
template <typename T>
__global__ void qk_norm_rope_generic(const T *q_src, T *q_dst, const T *k_src, T *k_dst,
                                     const float *q_w, const float *k_w, const int32_t *pos,
                                     int nq, int nk, int hd, const __grid_constant__ FreqTable ft,
                                     float eps, int do_norm)
{
    __shared__ float part[32];
    const int64_t t = blockIdx.x;
    const int head = blockIdx.y;
    const int half = hd / 2;
    const int i = threadIdx.x;
    const T *src;
    T *dst;
    const float *w;
    if (head < nq) {
        src = q_src + (t * nq + head) * hd;
        dst = q_dst + (t * nq + head) * hd;
        w = q_w;
    } else {
        src = k_src + (t * nk + (head - nq)) * hd;
        dst = k_dst + (t * nk + (head - nq)) * hd;
        w = k_w;
    }
    const bool act = i < half;  // blockDim is rounded up to whole warps
    float a = act ? to_f(src[i]) : 0.0f;
    float b = act ? to_f(src[i + half]) : 0.0f;
    if (do_norm) {
        float ss = sq_acc(sq_acc(0.0f, a), b);
        ss = warp_sum(ss);
        if ((i & 31) == 0) part[i >> 5] = ss;
        __syncthreads();
        if (i < 32) {
            float s = i < (int)(blockDim.x >> 5) ? part[i] : 0.0f;
            s = warp_sum(s);
            if (i == 0) part[0] = s;
        }
        __syncthreads();
        const float inv = rms_inv(part[0], hd, eps);
        if (act) {
            a = norm_mul(a, inv, w[i]);
            b = norm_mul(b, inv, w[i + half]);
        }
    }
    if (!act) return;
    float s, c;
    sincosf(__fmul_rn((float)pos[t], ft.f[i]), &s, &c);
    dst[i] = from_f<T>(rot_lo(a, b, c, s));
    dst[i + half] = from_f<T>(rot_hi(b, a, c, s));
}

template <typename T>
cudaError_t run(const LaunchCtx &c, const void *qs, void *qd, const void *ks, void *kd,
                const float *q_w, const float *k_w, const int32_t *pos, int64_t rows, int nq,
                int nk, int hd, int use_hd128, const FreqTable &ft, float eps, int do_norm)
{
    if (use_hd128) {
        const int cq = (nq + kHeadsPerWarp - 1) / kHeadsPerWarp;
        const int ck = (nk + kHeadsPerWarp - 1) / kHeadsPerWarp;
        const int64_t warps = rows * (cq + ck);
        const int64_t blocks = (warps + 3) / 4;
        qk_norm_rope_hd128<T><<<(unsigned)blocks, 128, 0, c.stream>>>(
            (const T *)qs, (T *)qd, (const T *)ks, (T *)kd, q_w, k_w, pos, rows, nq, nk, cq, ck, ft,
            eps, do_norm);
    } else {
        dim3 grid((unsigned)rows, (unsigned)(nq + nk));
        const int threads = ((hd / 2 + 31) / 32) * 32;
        qk_norm_rope_generic<T><<<grid, threads, 0, c.stream>>>((const T *)qs, (T *)qd, (const T *)ks,
                                                                (T *)kd, q_w, k_w, pos, nq, nk, hd, ft,
                                                                eps, do_norm);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qk_norm_rope(const LaunchCtx &c, const void *q_src, void *q_dst,
                                const void *k_src, void *k_dst, const float *q_w,
                                const float *k_w, const int32_t *pos, int64_t rows, int nq,
                                int nk, int hd, const float *freq, float eps, int do_norm,
                                int storage)
{
    if (rows <= 0 || nq + nk <= 0) return cudaSuccess;
    if (hd <= 0 || hd % 2 || hd > 512 || rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    FreqTable ft;
    for (int i = 0; i < hd / 2; i++) ft.f[i] = freq[i];
    // The 128-wide kernel moves 4 elements per lane: 16 B (fp32) or 8 B (fp16)
    // per access, and reads the norm weights as float4.
    const uintptr_t m = storage ? 7u : 15u;
    const uintptr_t data = reinterpret_cast<uintptr_t>(q_src) | reinterpret_cast<uintptr_t>(q_dst) |
                           reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(k_dst);
    const uintptr_t wts = reinterpret_cast<uintptr_t>(q_w) | reinterpret_cast<uintptr_t>(k_w);
    const int use_hd = (hd == 128 && (data & m) == 0 && (!do_norm || (wts & 15u) == 0)) ? 128 : 0;
    if (storage)
        return run<__half>(c, q_src, q_dst, k_src, k_dst, q_w, k_w, pos, rows, nq, nk, hd, use_hd, ft, eps,
                           do_norm);
    return run<float>(c, q_src, q_dst, k_src, k_dst, q_w, k_w, pos, rows, nq, nk, hd, use_hd, ft, eps,
                      do_norm);
}

}  // namespace ds3
