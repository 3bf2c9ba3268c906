// Device helpers shared by the ds3_cuda kernels (sm_100a).
//
// Rounding discipline: where a kernel must reproduce the reference CPU
// kernels bit for bit (dequant, residual add, combine) or within a few ulp
// (norms, RoPE, softmax, SwiGLU), every multiply/add that the reference writes
// as separate C operations is issued with an explicit round-to-nearest
// intrinsic (__fmul_rn, __fadd_rn, __fsub_rn, __fdiv_rn, __fsqrt_rn). nvcc
// never contracts those into an FMA, so the device performs the same roundings
// in the same order as the reference's C code.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace ds3 {

constexpr unsigned kFull = 0xffffffffu;

// Device error word, mapped from pinned host memory: kernels store 1 into a
// slot (plain stores, no read-modify-write) and the host reads it after a
// synchronisation. Slot meanings:
enum : int { kErrBadId = 0, kErrWaitTimeout = 1, kErrSlots = 4 };

__device__ __forceinline__ void flag_error(unsigned *err, int slot)
{
    if (err) *(volatile unsigned *)(err + slot) = 1u;
}

__device__ __forceinline__ float warp_sum(float v)
{
    // Butterfly: lane i and lane i^o add the same two values, so every lane
    // ends with the bit-identical total.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// 1 / sqrt(ss / n + eps), each step correctly rounded as in the reference
// (ds3_reference.c: ss /= n; ss += eps; rms = 1.0f / sqrtf(ss)).
__device__ __forceinline__ float rms_inv(float ss, int n, float eps)
{
    float m = __fdiv_rn(ss, (float)n);
    m = __fadd_rn(m, eps);
    return __fdiv_rn(1.0f, __fsqrt_rn(m));
}

// Same for a compile-time power-of-two n: ss / n and ss * (1/n) are the same
// correctly rounded value (scaling by a power of two), so the divide becomes
// one multiply.
template <int N>
__device__ __forceinline__ float rms_inv_pow2(float ss, float eps)
{
    static_assert((N & (N - 1)) == 0, "power of two");
    float m = __fmul_rn(ss, 1.0f / (float)N);
    m = __fadd_rn(m, eps);
    return __fdiv_rn(1.0f, __fsqrt_rn(m));
}

template <int N>
__device__ __forceinline__ float rms_inv_n(float ss, float eps)
{
    if constexpr ((N & (N - 1)) == 0) return rms_inv_pow2<N>(ss, eps);
    else return rms_inv(ss, N, eps);
}

// (x * inv) * w, left to right as the reference writes it.
__device__ __forceinline__ float norm_mul(float x, float inv, float w)
{
    return __fmul_rn(__fmul_rn(x, inv), w);
}

__device__ __forceinline__ float sq_acc(float acc, float x) { return fmaf(x, x, acc); }

// Packed fp32 pairs (the f32x2 instructions of sm_100): each half is one IEEE
// round-to-nearest operation, bit-identical to __fmul_rn / __fadd_rn /
// __fsub_rn / fmaf applied to that half alone. Operands already in adjacent
// registers need no moves. Caution, measured on sm_100a with CUDA 12.9: a
// mul2_rn whose result feeds an add2_rn / sub2_rn is contracted into one
// packed FMA (a single rounding), despite the .rn qualifiers and with
// --fmad=false too. Where the reference rounds the product, keep the sum
// scalar (__fadd_rn after a packed product is not contracted).
__device__ __forceinline__ unsigned long long f2_bits(float2 a)
{
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
__device__ __forceinline__ float2 f2_val(unsigned long long r)
{
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b)
{
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(d);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b)
{
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(d);
}
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b)
{
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(d);
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c)
{
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_val(d);
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b)
{
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y),
                       __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

__device__ __forceinline__ float f4_sumsq(float4 v, float acc)
{
    acc = sq_acc(acc, v.x);
    acc = sq_acc(acc, v.y);
    acc = sq_acc(acc, v.z);
    return sq_acc(acc, v.w);
}

__device__ __forceinline__ float4 f4_norm(float4 v, float inv, float4 w)
{
    return make_float4(norm_mul(v.x, inv, w.x), norm_mul(v.y, inv, w.y),
                       norm_mul(v.z, inv, w.z), norm_mul(v.w, inv, w.w));
}

// Streaming (evict-first) 128-bit load for activations read exactly once.
// These are coherent loads (ld.global.cs), so they stay correct for the
// in-place calls where the same warp later writes the row it read.
__device__ __forceinline__ float4 ld_stream(const float4 *p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_param(const float4 *p) { return __ldg(p); }

// Same load as ld_stream, as a volatile asm statement: the compiler keeps
// such loads in program order, so a kernel that issues a batch of them before
// using any result really has the whole batch in flight (the scheduler may
// otherwise interleave loads with their uses to save registers, turning one
// DRAM round trip into several).
__device__ __forceinline__ float4 ld_stream_inflight(const float4 *p)
{
    float4 v;
    asm volatile("ld.global.cs.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// A read-only scalar load kept in program order with the volatile loads around
// it (so it is issued with them, not after their results are used).
__device__ __forceinline__ float ld_param_f(const float *p)
{
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// ------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, 1-D) helpers.
// ------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_init_fence()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Plain arrival (release semantics: this thread's earlier shared-memory
// writes are visible to threads that complete their wait on the phase).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One bulk copy global -> shared (no multicast); completion is signalled on
// `bar` as transaction bytes. dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Bounded wait on an mbarrier phase. Returns false if the phase did not
// complete within `limit` polls; the caller records the timeout and stops.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit)
{
    const uint32_t a = smem_addr(bar);
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

constexpr uint32_t kWaitLimit = 1u << 22;

// ------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel of this library calls
// pdl_wait() — unconditionally, in every CTA, before any early return and
// before it touches activations — and then pdl_trigger(). pdl_wait returns
// once the preceding grid in the stream has completed and its writes are
// visible, so a chain of PDL launches keeps full stream order for the data;
// the trigger lets the next kernel be launched and its CTAs made resident
// while this one works, hiding launch latency. Triggering only after the wait
// keeps at most one dependent grid waiting behind a running one. Only static
// parameters (norm weights, embedding table, frequency table) may be read
// before pdl_wait. Without the PDL launch attribute both are no-ops.
// ------------------------------------------------------------------------
// ------------------------------------------------------------------------
// L2 prefetch ahead of pdl_wait. A kernel whose CTAs are already resident
// while the previous grid runs (PDL) asks the L2 for the activation bytes it
// is about to read (cp.async.bulk.prefetch.L2: a hint, no data returned), so
// the DRAM round trip overlaps the previous kernel instead of following it.
// This is safe for any input, including one the previous grid writes: every
// global store lands in the L2, the device's point of coherence, so a load
// issued after pdl_wait sees the final data whatever was prefetched before.
// (Loads made before the wait to steer a prefetch must bypass L1 — ld.cg —
// since L1 is not coherent with the other SMs' stores.) Only the part of
// [p, p + bytes) that lies on whole 16-byte units is prefetched, so nothing
// outside the range is touched.
// ------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_l2(const void *p, uint64_t bytes)
{
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t end = (a + bytes) & ~(uintptr_t)15;
    a = (a + 15) & ~(uintptr_t)15;
    while (a < end) {
        const uint32_t n = (uint32_t)((end - a) < 65536u ? (end - a) : 65536u);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
        a += n;
    }
}

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }


}  // namespace ds3
