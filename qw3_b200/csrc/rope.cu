// Per-head Q/K RMSNorm fused with NEOX RoPE (sm_100a).
//
// Reference: per-head ds3_ref_rms_norm (src/ds3_reference.c:526-533, engine
// src/ds3_engine.c:789-792) followed by ds3_ref_rope (:361-402); Metal
// metal/rope.metal:88-123 with the host frequency table of
// src/ds3_metal.m:478-489.
//
// Fast path (head_dim = 128, qk_norm_rope_tile): a CTA owns 2 tokens. The
// angle of pair i depends only on (position, i), so the CTA computes the 64
// cos/sin values of each token once into shared memory. Warps take groups of
// 4 heads with 8 lanes per head; each lane holds 8 elements of the first half
// of the head and their 8 RoPE partners (i + 64), loaded with 128-bit
// accesses that cover 128 contiguous bytes per 8 lanes; the RMS sum needs 3
// shuffles and the rotation none. Each element is read once and written
// once: 2 x 4 B (fp32) or 2 x 2 B (fp16).
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

__device__ __forceinline__ float rot_lo(float own, float other, float c, float s)
{
    return __fsub_rn(__fmul_rn(own, c), __fmul_rn(other, s));  // x0*c - x1*s
}
__device__ __forceinline__ float rot_hi(float own, float other, float c, float s)
{
    return __fadd_rn(__fmul_rn(other, s), __fmul_rn(own, c));  // x0*s + x1*c
}

// One lane's share of a 128-wide head when 8 lanes hold the head (j = lane
// within the 8): `lo` = 8 elements from the first half of the head and `hi`
// = their RoPE partners (index + 64), so the rotation is lane-local. Each
// load/store instruction of the 8 lanes covers 128 contiguous bytes.
//   fp32: lo = {4j..4j+3, 32+4j..32+4j+3}, pair index of lo[e] = pidx(j, e)
//   fp16: lo = {8j..8j+7}
// Lane-major tables of per-pair values (cos, sin, norm weight): the value
// lane j needs for its element e sits at tab_pos(j, e), so a lane reads its 8
// values with two 128-bit loads, and 8 lanes together read 128 contiguous
// bytes (no bank conflicts).
__host__ __device__ constexpr int tab_pos(int j, int e) { return ((e >> 2) * 8 + j) * 4 + (e & 3); }

template <typename T>
struct HeadSlice;
template <>
struct HeadSlice<float> {
    __device__ static int pidx(int j, int e) { return (e < 4) ? 4 * j + e : 32 + 4 * j + (e - 4); }
    // Position of pair index p in a lane-major table (see tab_pos).
    __device__ static int tab(int p) { return p < 32 ? tab_pos(p >> 2, p & 3) : tab_pos((p - 32) >> 2, 4 + (p & 3)); }
    __device__ static void load(const float *head, int j, float *lo, float *hi)
    {
        const float4 *q = reinterpret_cast<const float4 *>(head);
        const float4 a = ld_stream(q + j), b = ld_stream(q + 8 + j);
        const float4 c = ld_stream(q + 16 + j), d = ld_stream(q + 24 + j);
        lo[0] = a.x; lo[1] = a.y; lo[2] = a.z; lo[3] = a.w;
        lo[4] = b.x; lo[5] = b.y; lo[6] = b.z; lo[7] = b.w;
        hi[0] = c.x; hi[1] = c.y; hi[2] = c.z; hi[3] = c.w;
        hi[4] = d.x; hi[5] = d.y; hi[6] = d.z; hi[7] = d.w;
    }
    __device__ static void store(float *head, int j, const float *lo, const float *hi)
    {
        float4 *q = reinterpret_cast<float4 *>(head);
        q[j] = make_float4(lo[0], lo[1], lo[2], lo[3]);
        q[8 + j] = make_float4(lo[4], lo[5], lo[6], lo[7]);
        q[16 + j] = make_float4(hi[0], hi[1], hi[2], hi[3]);
        q[24 + j] = make_float4(hi[4], hi[5], hi[6], hi[7]);
    }
};
template <>
struct HeadSlice<__half> {
    __device__ static int pidx(int j, int e) { return 8 * j + e; }
    __device__ static int tab(int p) { return tab_pos(p >> 3, p & 7); }
    __device__ static void unpack(uint4 u, float *v)
    {
        const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
        }
    }
    __device__ static uint4 pack(const float *v)
    {
        unsigned w[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
            w[k] = *reinterpret_cast<unsigned *>(&h);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    __device__ static void load(const __half *head, int j, float *lo, float *hi)
    {
        const uint4 *q = reinterpret_cast<const uint4 *>(head);
        unpack(__ldcs(q + j), lo);
        unpack(__ldcs(q + 8 + j), hi);
    }
    __device__ static void store(__half *head, int j, const float *lo, const float *hi)
    {
        uint4 *q = reinterpret_cast<uint4 *>(head);
        q[j] = pack(lo);
        q[8 + j] = pack(hi);
    }
};

// head_dim = 128. A CTA of kTileWarps warps owns kTileTok tokens. While the
// head rows are being loaded, the CTA computes the cos/sin of the 64 rotation
// pairs of each of its tokens once into shared memory (one sincosf per pair).
// Each warp handles groups of 4 heads, 8 lanes per head (HeadSlice layout):
// the RMS sum is 3 shuffles and the rotation needs no data exchange.
constexpr int kTileTok = 2;
constexpr int kTileWarps = 9;
constexpr int kTok1Warps = 5;  // one-token tiles: up to 10 groups of 4 heads

// fp16 copy of a lane's 16 values into a 128-wide cache row, at the element
// positions HeadSlice<T> uses for that lane.
__device__ __forceinline__ void cache_store(__half *row, int j, const float *lo, const float *hi, float)
{
    uint2 *r = reinterpret_cast<uint2 *>(row);
    auto pk = [](float a, float b, float c, float d) {
        __half2 x = __floats2half2_rn(a, b), y = __floats2half2_rn(c, d);
        return make_uint2(*reinterpret_cast<unsigned *>(&x), *reinterpret_cast<unsigned *>(&y));
    };
    r[j] = pk(lo[0], lo[1], lo[2], lo[3]);            // elements 4j..4j+3
    r[8 + j] = pk(lo[4], lo[5], lo[6], lo[7]);        // 32+4j..
    r[16 + j] = pk(hi[0], hi[1], hi[2], hi[3]);       // 64+4j..
    r[24 + j] = pk(hi[4], hi[5], hi[6], hi[7]);       // 96+4j..
}
__device__ __forceinline__ void cache_store(__half *row, int j, const float *lo, const float *hi, __half)
{
    HeadSlice<__half>::store(row, j, lo, hi);
}

// KV = true additionally handles the V heads of each token (no norm, no
// rotation) and writes the rotated K rows and the V rows, rounded to fp16,
// into the KV cache at row positions[t] ([max_seq][n_kv_heads][128]).
// Warps per CTA: 9 (18 groups of 4 heads for 2 tokens x 36 heads, 2 per
// warp); with V, 2 x 40 heads = 20 groups over 10 warps, still 2 per warp.
template <bool KV>
__host__ __device__ constexpr int tile_warps() { return KV ? 10 : 9; }

template <typename T, bool KV, int W>
__host__ __device__ constexpr int tile_min_blocks() { return W <= 5 ? 5 : ((sizeof(T) == 2 && !KV) ? 4 : 3); }

template <typename T, bool KV, int TT = kTileTok, int W = tile_warps<KV>()>
__global__ void __launch_bounds__(W * 32, tile_min_blocks<T, KV, W>()) qk_norm_rope_tile(
    const T *q_src, T *q_dst, const T *k_src, T *k_dst, const float *q_w, const float *k_w,
    const int32_t *pos, int64_t rows, int nq, int nk, const __grid_constant__ FreqTable ft, float eps,
    int do_norm, const T *v_src, __half *k_cache, __half *v_cache, int max_seq, unsigned *err)
{
    constexpr int kMaxG = 2;
    constexpr int kW = W;
    __shared__ __align__(16) float cs[TT][64];
    __shared__ __align__(16) float sn[TT][64];
    __shared__ __align__(16) float wq[128];
    __shared__ __align__(16) float wk[128];

    const int tid = threadIdx.x;
    if (do_norm) {  // static parameters: safe to read before the wait
        for (int i = tid; i < 256; i += W * 32) {
            if (i < 128) wq[i] = q_w[i];
            else if (nk > 0) wk[i - 128] = k_w[i - 128];
        }
    }
    {
        // The tile's q / k (/ v) rows are contiguous: one L2 prefetch each,
        // issued while the previous kernel runs.
        const int64_t tb = (int64_t)blockIdx.x * TT;
        const int64_t nt = rows - tb < TT ? rows - tb : TT;
        if ((tid & 31) == 0 && nt > 0) {
            const int which = tid >> 5;
            if (which == 0) prefetch_l2(q_src + tb * nq * 128, (uint64_t)nt * nq * 128 * sizeof(T));
            else if (which == 1 && nk > 0) prefetch_l2(k_src + tb * nk * 128, (uint64_t)nt * nk * 128 * sizeof(T));
            else if (KV && which == 2 && nk > 0) prefetch_l2(v_src + tb * nk * 128, (uint64_t)nt * nk * 128 * sizeof(T));
        }
    }
    pdl_wait();
    pdl_trigger();

    const int64_t t0 = (int64_t)blockIdx.x * TT;
    const int lane = tid & 31, warp = tid >> 5;
    const int sub = lane >> 3;  // head within the group of 4
    const int j = lane & 7;     // slice of the head
    const int nh = nq + nk + (KV ? nk : 0);
    const int n_heads = TT * nh;
    const int n_groups = (n_heads + 3) >> 2;

    float lo[kMaxG][8], hi[kMaxG][8];
    T *headp[kMaxG];
    __half *cachep[kMaxG];
    int meta[kMaxG];  // bit 0: active, bit 1: K head, bit 2: V head, bits 3+: local token
#pragma unroll
    for (int gi = 0; gi < kMaxG; gi++) {
        const int g = warp + gi * kW;
        const int h = 4 * g + sub;
        meta[gi] = 0;
        headp[gi] = nullptr;
        cachep[gi] = nullptr;
        if (g < n_groups && h < n_heads) {
            const int tl = h / nh, hh = h - tl * nh;
            const int64_t t = t0 + tl;
            if (t < rows) {
                const bool is_v = KV && hh >= nq + nk;
                const bool is_k = !is_v && hh >= nq;
                const int kvh = is_v ? hh - nq - nk : hh - nq;
                const int64_t off = (is_k || is_v) ? (t * nk + kvh) * 128 : (t * nq + hh) * 128;
                headp[gi] = is_v ? nullptr : (is_k ? k_dst : q_dst) + off;
                meta[gi] = 1 | (is_k ? 2 : 0) | (is_v ? 4 : 0) | (tl << 3);
                HeadSlice<T>::load((is_v ? v_src : is_k ? k_src : q_src) + off, j, lo[gi], hi[gi]);
                if (KV && (is_k || is_v)) {
                    const int p = pos[t];
                    if (p >= 0 && p < max_seq) {
                        cachep[gi] = (is_v ? v_cache : k_cache) + ((int64_t)p * nk + kvh) * 128;
                    } else if (j == 0) {
                        flag_error(err, kErrBadId);
                    }
                }
            }
        }
        if (!(meta[gi] & 1)) {
#pragma unroll
            for (int e = 0; e < 8; e++) lo[gi][e] = hi[gi][e] = 0.0f;
        }
    }

    // cos/sin of this tile's tokens, computed while the loads above are in flight
    if (tid < TT * 64) {
        const int tl = tid >> 6, i = tid & 63;
        const int64_t t = t0 + tl;
        float s = 0.0f, c = 1.0f;
        if (t < rows) sincosf(__fmul_rn((float)pos[t], ft.f[i]), &s, &c);
        cs[tl][i] = c;
        sn[tl][i] = s;
    }
    __syncthreads();

#pragma unroll
    for (int gi = 0; gi < kMaxG; gi++) {
        if (warp + gi * kW >= n_groups) break;  // warp-uniform
        float *xl = lo[gi], *xh = hi[gi];
        const bool is_v = meta[gi] & 4;
        if (do_norm) {
            float ss = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) ss = sq_acc(sq_acc(ss, xl[e]), xh[e]);
            ss += __shfl_xor_sync(kFull, ss, 1);
            ss += __shfl_xor_sync(kFull, ss, 2);
            ss += __shfl_xor_sync(kFull, ss, 4);
            const float inv = rms_inv_pow2<128>(ss, eps);
            const float *w = (meta[gi] & 2) ? wk : wq;
            if (!is_v) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int pi = HeadSlice<T>::pidx(j, e);
                    xl[e] = norm_mul(xl[e], inv, w[pi]);
                    xh[e] = norm_mul(xh[e], inv, w[pi + 64]);
                }
            }
        }
        const int tl = meta[gi] >> 3;
        float yl[8], yh[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int pi = HeadSlice<T>::pidx(j, e);
            const float c = cs[tl][pi], s = sn[tl][pi];
            yl[e] = is_v ? xl[e] : rot_lo(xl[e], xh[e], c, s);  // x0*c - x1*s
            yh[e] = is_v ? xh[e] : rot_hi(xh[e], xl[e], c, s);  // x0*s + x1*c
        }
        if (headp[gi]) HeadSlice<T>::store(headp[gi], j, yl, yh);
        if (KV && cachep[gi]) cache_store(cachep[gi], j, yl, yh, T());
    }
}

// Shared-memory counterpart of HeadSlice<__half>::load (same element layout);
// the staged kernel below is used for fp16 storage only.
__device__ __forceinline__ void head_from_smem(const __half *head, int j, float *lo, float *hi)
{
    const uint4 *q = reinterpret_cast<const uint4 *>(head);
    HeadSlice<__half>::unpack(q[j], lo);
    HeadSlice<__half>::unpack(q[8 + j], hi);
}

// Norm (optional) and rotation of one lane's 8 + 8 elements from lane-major
// tables: w = [lo 64 | hi 64] weights, c / sn = 64 cos / sin. The products
// and sums are those of norm_mul / rot_lo / rot_hi, the products two elements
// per packed f32x2 instruction, so every element is rounded as by the scalar
// code; only the sum of squares is accumulated in four partial sums.
__device__ __forceinline__ void norm_rotate_packed(float *xl, float *xh, int j, const float *w, const float *c,
                                                   const float *sn, bool do_norm, float eps)
{
    if (do_norm) {
        float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const float2 l = make_float2(xl[e], xl[e + 1]), h = make_float2(xh[e], xh[e + 1]);
            al = fma2_rn(l, l, al);
            ah = fma2_rn(h, h, ah);
        }
        float ss = (al.x + al.y) + (ah.x + ah.y);
        ss += __shfl_xor_sync(kFull, ss, 1);
        ss += __shfl_xor_sync(kFull, ss, 2);
        ss += __shfl_xor_sync(kFull, ss, 4);
        const float inv = rms_inv_pow2<128>(ss, eps);
        const float2 i2 = make_float2(inv, inv);
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const float4 wl = *reinterpret_cast<const float4 *>(w + tab_pos(j, 4 * q));
            const float4 wh = *reinterpret_cast<const float4 *>(w + 64 + tab_pos(j, 4 * q));
            float2 a = mul2_rn(mul2_rn(make_float2(xl[4 * q], xl[4 * q + 1]), i2), make_float2(wl.x, wl.y));
            float2 b = mul2_rn(mul2_rn(make_float2(xl[4 * q + 2], xl[4 * q + 3]), i2), make_float2(wl.z, wl.w));
            xl[4 * q] = a.x; xl[4 * q + 1] = a.y; xl[4 * q + 2] = b.x; xl[4 * q + 3] = b.y;
            a = mul2_rn(mul2_rn(make_float2(xh[4 * q], xh[4 * q + 1]), i2), make_float2(wh.x, wh.y));
            b = mul2_rn(mul2_rn(make_float2(xh[4 * q + 2], xh[4 * q + 3]), i2), make_float2(wh.z, wh.w));
            xh[4 * q] = a.x; xh[4 * q + 1] = a.y; xh[4 * q + 2] = b.x; xh[4 * q + 3] = b.y;
        }
    }
#pragma unroll
    for (int q = 0; q < 2; q++) {
        const float4 c4 = *reinterpret_cast<const float4 *>(c + tab_pos(j, 4 * q));
        const float4 s4 = *reinterpret_cast<const float4 *>(sn + tab_pos(j, 4 * q));
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int e = 4 * q + 2 * h;
            const float2 cc = h ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
            const float2 ss = h ? make_float2(s4.z, s4.w) : make_float2(s4.x, s4.y);
            const float2 lo = make_float2(xl[e], xl[e + 1]), hi = make_float2(xh[e], xh[e + 1]);
            // Products two at a time; the sums stay scalar (a packed product
            // feeding a packed sum is fused into one FMA by the compiler).
            const float2 lc = mul2_rn(lo, cc), hs = mul2_rn(hi, ss), ls = mul2_rn(lo, ss), hc = mul2_rn(hi, cc);
            xl[e] = __fsub_rn(lc.x, hs.x);  // x0*c - x1*s
            xl[e + 1] = __fsub_rn(lc.y, hs.y);
            xh[e] = __fadd_rn(ls.x, hc.x);  // x0*s + x1*c
            xh[e + 1] = __fadd_rn(ls.y, hc.y);
        }
    }
}

// fp16 storage, head_dim 128, large token counts: a persistent CTA streams
// tiles of TT consecutive tokens through an NS-stage ring in shared memory. A
// tile's q rows (and its k rows) are contiguous in memory, so each is one 1-D
// bulk async copy (TMA, no multicast). The kernel is warp-specialised: warp W
// (the producer) issues each tile's copies and computes the tile's cos/sin
// into the stage's own table, up to NS tiles ahead; the W compute warps wait
// on the stage's "full" mbarrier (the copies' bytes plus the producer's 32
// arrivals after its table writes), process groups of 4 heads from shared
// memory (HeadSlice layout, lane-major tables) straight to global memory, and
// release the stage on its "empty" mbarrier. No CTA barrier separates the
// tiles. All waits are bounded.
template <int TT, int NS, int W>
__global__ void __launch_bounds__((W + 1) * 32) qk_norm_rope_ws(
    const __half *q_src, __half *q_dst, const __half *k_src, __half *k_dst, const float *q_w, const float *k_w,
    const int32_t *pos, int64_t rows, int nq, int nk, const __grid_constant__ FreqTable ft, float eps, int do_norm,
    unsigned *err)
{
    using T = __half;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(16) float cs[NS][TT][64];
    __shared__ __align__(16) float sn[NS][TT][64];
    __shared__ __align__(16) float wq[128];
    __shared__ __align__(16) float wk[128];
    __shared__ __align__(8) uint64_t full[NS], empty[NS];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nh = nq + nk;
    const size_t stage_elems = (size_t)TT * nh * 128;
    if (do_norm) {  // static parameters: safe to read before the wait
        for (int i = tid; i < 256; i += (W + 1) * 32) {
            const int m = i & 127, at = (m & 64) + HeadSlice<T>::tab(m & 63);
            if (i < 128) wq[at] = q_w[m];
            else if (nk > 0) wk[at] = k_w[m];
        }
    }
    if (tid == 0) {
        for (int st = 0; st < NS; st++) {
            mbar_init(&full[st], 33);  // producer lane 0's expect_tx + 32 lanes after the cos/sin writes
            mbar_init(&empty[st], W);
        }
        mbar_init_fence();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();

    const int64_t n_tiles = (rows + TT - 1) / TT;
    const int64_t G = gridDim.x;
    T *stage_base = reinterpret_cast<T *>(ring);
    bool ok = true;
    if (warp == W) {
        int issued = 0;
        for (int64_t tile = blockIdx.x; tile < n_tiles; tile += G, issued++) {
            const int st = issued % NS;
            if (issued >= NS && !mbar_wait(&empty[st], ((issued / NS) - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            const int64_t t0 = tile * TT;
            const int tok = (int)((rows - t0 < TT) ? rows - t0 : TT);
            if (lane == 0) {
                const uint32_t qb = (uint32_t)(tok * nq * 128 * sizeof(T));
                const uint32_t kb = (uint32_t)(tok * nk * 128 * sizeof(T));
                T *dst = stage_base + st * stage_elems;
                mbar_expect_tx(&full[st], qb + kb);
                bulk_g2s(dst, q_src + t0 * nq * 128, qb, &full[st]);
                if (kb) bulk_g2s(dst + (size_t)TT * nq * 128, k_src + t0 * nk * 128, kb, &full[st]);
            }
#pragma unroll
            for (int tl = 0; tl < TT; tl++) {
                const float pf = tl < tok ? (float)pos[t0 + tl] : 0.0f;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int pr = lane + 32 * h;
                    float sv = 0.0f, cv = 1.0f;
                    if (tl < tok) sincosf(__fmul_rn(pf, ft.f[pr]), &sv, &cv);
                    cs[st][tl][HeadSlice<T>::tab(pr)] = cv;
                    sn[st][tl][HeadSlice<T>::tab(pr)] = sv;
                }
            }
            mbar_arrive(&full[st]);  // release: the table writes are visible to the waiting warps
        }
        // Do not leave with copies in flight: the last stages issued must land.
        for (int k = issued - 1; k >= 0 && k >= issued - NS; k--)
            if (!mbar_wait(&full[k % NS], (k / NS) & 1, kWaitLimit)) ok = false;
    } else {
        const int sub = lane >> 3, j = lane & 7;
        int it = 0;
        for (int64_t tile = blockIdx.x; tile < n_tiles; tile += G, it++) {
            const int st = it % NS;
            if (!mbar_wait(&full[st], (it / NS) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            const int64_t t0 = tile * TT;
            const int tok = (int)((rows - t0 < TT) ? rows - t0 : TT);
            const T *sq = stage_base + st * stage_elems;
            const T *sk = sq + (size_t)TT * nq * 128;
            const int n_heads = tok * nh;
            const int n_groups = (n_heads + 3) >> 2;
            for (int g = warp; g < n_groups; g += W) {
                const int h = 4 * g + sub;
                const bool act = h < n_heads;
                const int hc = act ? h : 0;
                const int tl = TT == 1 ? 0 : TT == 2 ? (hc >= nh ? 1 : 0) : hc / nh, hh = hc - tl * nh;
                const bool is_k = hh >= nq;
                const T *src = is_k ? sk + (size_t)(tl * nk + (hh - nq)) * 128 : sq + (size_t)(tl * nq + hh) * 128;
                float xl[8], xh[8];
                head_from_smem(src, j, xl, xh);
                norm_rotate_packed(xl, xh, j, is_k ? wk : wq, cs[st][tl], sn[st][tl], do_norm, eps);
                if (act) {
                    const int64_t t = t0 + tl;
                    T *dst = is_k ? k_dst + (t * nk + (hh - nq)) * 128 : q_dst + (t * nq + hh) * 128;
                    HeadSlice<T>::store(dst, j, xl, xh);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
    if (!ok && lane == 0) flag_error(err, kErrWaitTimeout);
}

template <int TT, int NS, int W>
cudaError_t run_ws(const LaunchCtx &c, const void *qs, void *qd, const void *ks, void *kd, const float *q_w,
                   const float *k_w, const int32_t *pos, int64_t rows, int nq, int nk, const FreqTable &ft, float eps,
                   int do_norm)
{
    auto kern = qk_norm_rope_ws<TT, NS, W>;
    const size_t smem = (size_t)NS * TT * (nq + nk) * 128 * sizeof(__half);
    static size_t configured = 0;
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
        keep_driver_carveout(reinterpret_cast<const void *>(kern));
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (W + 1) * 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t tiles = (rows + TT - 1) / TT;
    const int64_t cap = (int64_t)c.n_sm * per_sm;
    launch_ks(c, kern, dim3((unsigned)(tiles < cap ? tiles : cap)), dim3((W + 1) * 32), smem, (const __half *)qs,
              (__half *)qd, (const __half *)ks, (__half *)kd, q_w, k_w, pos, rows, nq, nk, ft, eps, do_norm, c.err);
    return cudaGetLastError();
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
    pdl_wait();
    pdl_trigger();
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
        // One token per CTA (5 warps, 2 groups of 4 heads each) whenever the
        // token's heads fit: 512 small CTAs keep more loads in flight per SM
        // than 256 two-token CTAs (T=512: 5.35 vs 5.88 us; T=32768 alike).
        if ((nq + nk + 3) / 4 <= 2 * kTok1Warps) {
            launch_k(c, qk_norm_rope_tile<T, false, 1, kTok1Warps>, dim3((unsigned)rows), dim3(kTok1Warps * 32),
                     (const T *)qs, (T *)qd, (const T *)ks, (T *)kd, q_w, k_w, pos, rows, nq, nk, ft, eps, do_norm,
                     (const T *)nullptr, (__half *)nullptr, (__half *)nullptr, 0, c.err);
            return cudaGetLastError();
        }
        const int64_t blocks = (rows + kTileTok - 1) / kTileTok;
        launch_k(c, qk_norm_rope_tile<T, false>, dim3((unsigned)blocks), dim3(kTileWarps * 32), (const T *)qs,
                 (T *)qd, (const T *)ks, (T *)kd, q_w, k_w, pos, rows, nq, nk, ft, eps, do_norm, (const T *)nullptr,
                 (__half *)nullptr, (__half *)nullptr, 0, c.err);
    } else {
        dim3 grid((unsigned)rows, (unsigned)(nq + nk));
        const int threads = ((hd / 2 + 31) / 32) * 32;
        launch_k(c, qk_norm_rope_generic<T>, dim3(grid), dim3(threads), (const T *)qs, (T *)qd, (const T *)ks,
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
    // The 128-wide kernel moves 16 contiguous elements per lane with 16-byte
    // accesses, so head rows must be 16-byte aligned.
    const uintptr_t m = 15u;
    const uintptr_t data = reinterpret_cast<uintptr_t>(q_src) | reinterpret_cast<uintptr_t>(q_dst) |
                           reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(k_dst);
    const uintptr_t wts = reinterpret_cast<uintptr_t>(q_w) | reinterpret_cast<uintptr_t>(k_w);
    const int groups = (kTileTok * (nq + nk) + 3) / 4;
    const int use_hd = (hd == 128 && (data & m) == 0 && groups <= kTileWarps * 2) ? 128 : 0;
    (void)wts;
    // fp16 storage at large token counts: the warp-specialised staged kernel
    // (T=32768: 98.5 us, against 109 us for a staged kernel with two CTA
    // barriers per tile and 180 us for the register-tile kernel; fp32 is
    // faster with the register-tile kernel). 2-token tiles, 3 stages, 9
    // compute warps measured best against 2 or 4 stages, 6 or 12 warps, and
    // 1- or 4-token tiles.
    if (use_hd && storage && rows >= 2048) {
        const uintptr_t al = reinterpret_cast<uintptr_t>(q_src) | reinterpret_cast<uintptr_t>(k_src);
        if ((al & 15u) == 0) {
            return run_ws<2, 3, 9>(c, q_src, q_dst, k_src, k_dst, q_w, k_w, pos, rows, nq, nk, ft, eps, do_norm);
        }
    }
    if (storage)
        return run<__half>(c, q_src, q_dst, k_src, k_dst, q_w, k_w, pos, rows, nq, nk, hd, use_hd, ft, eps,
                           do_norm);
    return run<float>(c, q_src, q_dst, k_src, k_dst, q_w, k_w, pos, rows, nq, nk, hd, use_hd, ft, eps,
                      do_norm);
}

cudaError_t launch_qk_norm_rope_kv(const LaunchCtx &c, void *q, void *k, const void *v, const float *q_w,
                                   const float *k_w, const int32_t *pos, int64_t rows, int nq, int nk,
                                   const float *freq, float eps, int storage, void *k_cache, void *v_cache,
                                   int max_seq)
{
    if (rows <= 0) return cudaSuccess;
    const int groups = (kTileTok * (nq + 2 * nk) + 3) / 4;
    constexpr int kW = tile_warps<true>();
    const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_cache) |
                         reinterpret_cast<uintptr_t>(v_cache);
    if ((al & 15u) || groups > kW * 2 || rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    FreqTable ft;
    for (int i = 0; i < 64; i++) ft.f[i] = freq[i];
    if ((nq + 2 * nk + 3) / 4 <= 2 * kTok1Warps) {
        const dim3 grid((unsigned)rows), block(kTok1Warps * 32);
        if (storage)
            launch_k(c, qk_norm_rope_tile<__half, true, 1, kTok1Warps>, grid, block, (const __half *)q, (__half *)q,
                     (const __half *)k, (__half *)k, q_w, k_w, pos, rows, nq, nk, ft, eps, 1, (const __half *)v,
                     (__half *)k_cache, (__half *)v_cache, max_seq, c.err);
        else
            launch_k(c, qk_norm_rope_tile<float, true, 1, kTok1Warps>, grid, block, (const float *)q, (float *)q,
                     (const float *)k, (float *)k, q_w, k_w, pos, rows, nq, nk, ft, eps, 1, (const float *)v,
                     (__half *)k_cache, (__half *)v_cache, max_seq, c.err);
        return cudaGetLastError();
    }
    const int64_t blocks = (rows + kTileTok - 1) / kTileTok;
    if (storage)
        launch_k(c, qk_norm_rope_tile<__half, true>, dim3((unsigned)blocks), dim3(kW * 32),
                 (const __half *)q, (__half *)q, (const __half *)k, (__half *)k, q_w, k_w, pos, rows, nq, nk, ft, eps,
                 1, (const __half *)v, (__half *)k_cache, (__half *)v_cache, max_seq, c.err);
    else
        launch_k(c, qk_norm_rope_tile<float, true>, dim3((unsigned)blocks), dim3(kW * 32),
                 (const float *)q, (float *)q, (const float *)k, (float *)k, q_w, k_w, pos, rows, nq, nk, ft, eps, 1,
                 (const float *)v, (__half *)k_cache, (__half *)v_cache, max_seq, c.err);
    return cudaGetLastError();
}

namespace {
// KV-cache write of a chunk, metal/attention.metal:66-87: row seq_pos + t of
// the fp16 cache [max_seq][n_kv_heads][head_dim] gets half(k[t]), half(v[t]).
__global__ void kv_cache_write_k(const float *k, const float *v, __half *kc, __half *vc, int64_t seq_pos,
                                 int64_t n_elems, int64_t row_elems)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_elems;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t dst = seq_pos * row_elems + e;
        kc[dst] = __float2half_rn(k[e]);
        vc[dst] = __float2half_rn(v[e]);
    }
}
}  // namespace

cudaError_t launch_kv_cache_write(const LaunchCtx &c, const float *k, const float *v, void *k_cache,
                                  void *v_cache, int64_t seq_pos, int64_t n_tokens, int64_t row_elems)
{
    const int64_t n = n_tokens * row_elems;
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)c.n_sm * 16) blocks = (int64_t)c.n_sm * 16;
    launch_k(c, kv_cache_write_k, dim3((unsigned)blocks), dim3(256), k, v, (__half *)k_cache, (__half *)v_cache,
             seq_pos, n, row_elems);
    return cudaGetLastError();
}

}  // namespace ds3
