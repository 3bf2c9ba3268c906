// Token-embedding gather + dequant (+ fused RMSNorm) on the device (sm_100a).
//
// Reference: ds3_ref_dequantize_row (src/ds3_reference.c:194-241) with the
// Q4_K / Q6_K / Q8_0 block decoders (:87-113, :130-158, :173-184), called per
// token on the CPU by upload_token_embeddings (src/ds3_engine.c:273-290).
// Here the table stays resident in HBM and one warp produces one token row.
//
// Fast path (Q4_K / Q6_K, n_cols = 256 * NB, NB in {1,2,4,8}):
//  - the quantised row (NB * 144 or NB * 210 bytes) is staged in shared
//    memory by a 1-D bulk async copy (TMA, cp.async.bulk) completing on a
//    per-warp mbarrier; two slots per warp, so the copy of the warp's next row
//    is in flight while the current one is unpacked;
//  - rows that are not 16-byte aligned/sized fall back to a byte copy by the
//    warp into the same slot;
//  - unpack: lane l produces float4 number k*32+l of the row (k < 2*NB), so
//    each store instruction writes 512 contiguous bytes; 6-bit scale/min pairs
//    and fp16 d/dmin are decoded in registers;
//  - every value is (d*sc)*q - dmin*m (Q4_K) or (d*sc)*(q-32) (Q6_K) with
//    explicit round-to-nearest ops in the reference's order: bit-exact.
//  - with a norm weight, the row stays in registers and the warp also writes
//    rms_norm(row): one pass, 17,540 B per 2048-wide Q4_K token.
// Generic path (other types/widths): one thread per output element.
//
// An id outside [0, n_vocab) is not read: its row is written as zeros and the
// bad-id slot of the device error word is set (the CPU reference returns -1).
#include "common.cuh"
#include "launch.h"

namespace ds3 {
namespace {

constexpr int kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeQ4K = 12, kTypeQ6K = 14;
constexpr int kWarps = 4;

template <int TYPE>
struct BlockBytes;
template <>
struct BlockBytes<kTypeQ4K> {
    static constexpr int v = 144;
};
template <>
struct BlockBytes<kTypeQ6K> {
    static constexpr int v = 210;
};

__device__ __forceinline__ float h2f(const uint8_t *p)
{
    const unsigned short u = *reinterpret_cast<const unsigned short *>(p);
    return __half2float(__ushort_as_half(u));
}

// Q4_K row in shared memory -> this lane's 2*NB float4 (ds3_reference.c:76-113).
// STORE: write each float4 to dst[k*32 + lane] as soon as it is decoded
// (nothing held in registers); otherwise return the row in out[].
template <int NB, bool STORE>
__device__ __forceinline__ void unpack_q4k(const uint8_t *rowp, int lane, float4 *out, float4 *dst)
{
    const int hi = (lane >> 3) & 1;  // 0: low nibbles, 1: high nibbles
    const int sh = hi * 4;
#pragma unroll
    for (int k = 0; k < 2 * NB; k++) {
        const uint8_t *blk = rowp + (k >> 1) * 144;
        const int grp = 2 * (k & 1) + (lane >> 4);  // 64-weight group 0..3
        const int j = 2 * grp + hi;                 // scale/min pair 0..7
        const float d = h2f(blk);
        const float dmin = h2f(blk + 2);
        const uint8_t *s = blk + 4;
        unsigned sc, mn;
        if (j < 4) {
            sc = s[j] & 63u;
            mn = s[j + 4] & 63u;
        } else {
            sc = (s[j + 4] & 15u) | ((unsigned)(s[j - 4] >> 6) << 4);
            mn = (unsigned)(s[j + 4] >> 4) | ((unsigned)(s[j] >> 6) << 4);
        }
        const float d1 = __fmul_rn(d, (float)sc);
        const float m1 = __fmul_rn(dmin, (float)mn);
        const uint32_t q = *reinterpret_cast<const uint32_t *>(blk + 16 + 32 * grp + 4 * (lane & 7));
        const float4 r = make_float4(__fsub_rn(__fmul_rn(d1, (float)((q >> (0 + sh)) & 15u)), m1),
                                     __fsub_rn(__fmul_rn(d1, (float)((q >> (8 + sh)) & 15u)), m1),
                                     __fsub_rn(__fmul_rn(d1, (float)((q >> (16 + sh)) & 15u)), m1),
                                     __fsub_rn(__fmul_rn(d1, (float)((q >> (24 + sh)) & 15u)), m1));
        if constexpr (STORE) dst[k * 32 + lane] = r;
        else out[k] = r;
    }
}

__device__ __forceinline__ uint32_t ld_u32_from_u16(const uint8_t *p)
{
    const unsigned short *h = reinterpret_cast<const unsigned short *>(p);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}

// Q6_K row in shared memory -> this lane's 2*NB float4 (ds3_reference.c:130-158).
template <int NB, bool STORE>
__device__ __forceinline__ void unpack_q6k(const uint8_t *rowp, int lane, float4 *out, float4 *dst)
{
    const int quad = lane >> 3;           // which of q1..q4 (32-weight quarter)
    const int l = 4 * (lane & 7);         // first of 4 positions in the quarter
    const int is = (lane & 7) >> 2;       // l / 16
    const int nsh = (quad >= 2) ? 4 : 0;  // q3/q4 use the high nibble
    const int hsh = 2 * quad;             // 2-bit field of qh
#pragma unroll
    for (int k = 0; k < 2 * NB; k++) {
        const uint8_t *blk = rowp + (k >> 1) * 210;
        const int half = k & 1;
        const uint32_t lq = ld_u32_from_u16(blk + 64 * half + 32 * (quad & 1) + l);
        const uint32_t hq = ld_u32_from_u16(blk + 128 + 32 * half + l);
        const int sc = (int)reinterpret_cast<const int8_t *>(blk)[192 + 8 * half + is + 2 * quad];
        const float dsc = __fmul_rn(h2f(blk + 208), (float)sc);
        float v[4];
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int q = (int)(((lq >> (8 * b + nsh)) & 15u) | (((hq >> (8 * b + hsh)) & 3u) << 4)) - 32;
            v[b] = __fmul_rn(dsc, (float)q);
        }
        if constexpr (STORE) dst[k * 32 + lane] = make_float4(v[0], v[1], v[2], v[3]);
        else out[k] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

template <int TYPE, int NB, bool STORE>
__device__ __forceinline__ void unpack_row(const uint8_t *rowp, int lane, float4 *out, float4 *dst)
{
    if constexpr (TYPE == kTypeQ4K) unpack_q4k<NB, STORE>(rowp, lane, out, dst);
    else unpack_q6k<NB, STORE>(rowp, lane, out, dst);
}

template <int NB>
__device__ __forceinline__ void emit_row(float4 *v, int lane, int64_t row, float *hidden,
                                         const float *w, float *norm, float eps)
{
    constexpr int n = NB * 256;
    if (hidden) {
        float4 *h = reinterpret_cast<float4 *>(hidden + row * n);
#pragma unroll
        for (int k = 0; k < 2 * NB; k++) h[k * 32 + lane] = v[k];
    }
    if (norm) {
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < 2 * NB; k++) ss = f4_sumsq(v[k], ss);
        ss = warp_sum(ss);
        const float inv = rms_inv_n<n>(ss, eps);
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        float4 *o = reinterpret_cast<float4 *>(norm + row * n);
#pragma unroll
        for (int k = 0; k < 2 * NB; k++) o[k * 32 + lane] = f4_norm(v[k], inv, ld_param(w4 + k * 32 + lane));
    }
}

// Decode one staged row: with a norm, keep it in registers and emit hidden +
// norm; without, stream each decoded float4 straight to the output row.
template <int TYPE, int NB, bool NORM>
__device__ __forceinline__ void decode_row(const uint8_t *rowp, int lane, int64_t row, float *hidden,
                                           const float *w, float *norm, float eps)
{
    if constexpr (NORM) {
        float4 v[2 * NB];
        unpack_row<TYPE, NB, false>(rowp, lane, v, nullptr);
        emit_row<NB>(v, lane, row, hidden, w, norm, eps);
    } else {
        unpack_row<TYPE, NB, true>(rowp, lane, nullptr, reinterpret_cast<float4 *>(hidden + row * NB * 256));
    }
}

template <int NB>
__device__ __forceinline__ void zero_row(int lane, int64_t row, float *hidden, float *norm)
{
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 2 * NB; k++) {
        if (hidden) reinterpret_cast<float4 *>(hidden + row * NB * 256)[k * 32 + lane] = z;
        if (norm) reinterpret_cast<float4 *>(norm + row * NB * 256)[k * 32 + lane] = z;
    }
}

struct EmbedArgs {
    const uint8_t *table;
    const int32_t *ids;
    float *hidden;
    const float *w;
    float *norm;
    int64_t n_ids;
    int64_t n_vocab;
    uint64_t row_stride;
    float eps;
    unsigned *err;
    int use_bulk;
};

template <int TYPE, int NB, bool NORM>
__global__ void __launch_bounds__(kWarps * 32) embed_warp(const EmbedArgs a)
{
    constexpr int kRowBytes = NB * BlockBytes<TYPE>::v;
    constexpr int kSlot = (kRowBytes + 15) & ~15;
    __shared__ __align__(128) uint8_t slots[kWarps][2][kSlot];
    __shared__ __align__(8) uint64_t bars[kWarps][2];

    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;  // <= kWarps
    const int64_t stride = (int64_t)gridDim.x * warps;
    int64_t cur = (int64_t)blockIdx.x * warps + wid;
    // While the previous kernel runs: read this warp's first id past L1 and
    // prefetch that table row into L2 (a hint only: the id is read again
    // after the wait, and a stale or bad id just prefetches nothing useful).
    const int32_t hint = cur < a.n_ids ? __ldcg(a.ids + cur) : -1;
    const bool hint_ok = hint >= 0 && hint < a.n_vocab;
    if (lane == 0 && hint_ok) prefetch_l2(a.table + (uint64_t)hint * a.row_stride, kRowBytes);
    pdl_wait();
    pdl_trigger();
    if (cur >= a.n_ids) return;  // whole warp leaves together; no CTA barrier below

    if (!a.use_bulk) {
        // Byte-copy staging: the warp copies the row into its slot, then unpacks.
        for (; cur < a.n_ids; cur += stride) {
            const int32_t id = a.ids[cur];
            if (id < 0 || id >= a.n_vocab) {
                if (lane == 0) flag_error(a.err, kErrBadId);
                zero_row<NB>(lane, cur, a.hidden, a.norm);
            } else {
                const uint8_t *src = a.table + (uint64_t)id * a.row_stride;
                for (int i = lane; i < kRowBytes; i += 32) slots[wid][0][i] = src[i];
                __syncwarp();
                decode_row<TYPE, NB, NORM>(slots[wid][0], lane, cur, a.hidden, a.w, a.norm, a.eps);
                __syncwarp();
            }
        }
        return;
    }

    if (lane == 0) {
        mbar_init(&bars[wid][0], 1);
        mbar_init(&bars[wid][1], 1);
        mbar_init_fence();
    }
    __syncwarp();

    auto issue = [&](int s, int32_t id) {
        if (lane == 0) {
            mbar_expect_tx(&bars[wid][s], kRowBytes);
            bulk_g2s(slots[wid][s], a.table + (uint64_t)id * a.row_stride, kRowBytes, &bars[wid][s]);
        }
    };

    uint32_t parity = 0;  // bit s: phase parity to wait for on slot s
    int slot = 0;
    // The first row's copy starts from the hinted id (now read after the
    // wait, so the table row is current) while the id itself is read again;
    // if the id changed meanwhile, that copy is let land and the right row is
    // fetched. This saves the id's round trip on the common path.
    if (hint_ok) issue(slot, hint);
    int32_t cur_id = a.ids[cur];
    bool cur_ok = cur_id >= 0 && cur_id < a.n_vocab;
    if (cur_id != hint) {
        if (hint_ok) {
            if (!__all_sync(kFull, mbar_wait(&bars[wid][slot], 0, kWaitLimit))) {
                if (lane == 0) flag_error(a.err, kErrWaitTimeout);
                return;
            }
            parity ^= 1u;
            __syncwarp();
        }
        if (cur_ok) issue(slot, cur_id);
    }

    while (cur < a.n_ids) {
        const int64_t nxt = cur + stride;
        int32_t nxt_id = -1;
        bool nxt_ok = false;
        if (nxt < a.n_ids) {
            nxt_id = a.ids[nxt];
            nxt_ok = nxt_id >= 0 && nxt_id < a.n_vocab;
            if (nxt_ok) issue(slot ^ 1, nxt_id);
        }
        if (cur_ok) {
            const bool done = __all_sync(kFull, mbar_wait(&bars[wid][slot], (parity >> slot) & 1u, kWaitLimit));
            parity ^= 1u << slot;
            if (!done) {
                // Record the timeout, let this warp's copies land (bounded), stop.
                if (lane == 0) flag_error(a.err, kErrWaitTimeout);
                mbar_wait(&bars[wid][slot], ((parity >> slot) & 1u) ^ 1u, kWaitLimit);
                if (nxt_ok) mbar_wait(&bars[wid][slot ^ 1], (parity >> (slot ^ 1)) & 1u, kWaitLimit);
                return;
            }
            decode_row<TYPE, NB, NORM>(slots[wid][slot], lane, cur, a.hidden, a.w, a.norm, a.eps);
            __syncwarp();  // slot free before it is refilled two rows later
        } else {
            if (lane == 0) flag_error(a.err, kErrBadId);
            zero_row<NB>(lane, cur, a.hidden, a.norm);
        }
        cur = nxt;
        cur_id = nxt_id;
        cur_ok = nxt_ok;
        slot ^= 1;
    }
}

// ------------------------------------------------------------------------
// Generic path: any supported type / width, one thread per output element.
// ------------------------------------------------------------------------
__device__ float dequant_one(int type, const uint8_t *row, int c)
{
    switch (type) {
    case kTypeF32: return reinterpret_cast<const float *>(row)[c];
    case kTypeF16: {
        const unsigned short u = reinterpret_cast<const unsigned short *>(row)[c];
        return __half2float(__ushort_as_half(u));
    }
    case kTypeQ8_0: {
        const uint8_t *blk = row + (c >> 5) * 34;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        return __fmul_rn((float)(int8_t)blk[2 + (c & 31)], d);
    }
    case kTypeQ4K: {
        const uint8_t *blk = row + (c >> 8) * 144;
        const int w = c & 255, grp = w >> 6, hi = (w >> 5) & 1, l = w & 31, j = 2 * grp + hi;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
        const uint8_t *s = blk + 4;
        unsigned sc, mn;
        if (j < 4) {
            sc = s[j] & 63u;
            mn = s[j + 4] & 63u;
        } else {
            sc = (s[j + 4] & 15u) | ((unsigned)(s[j - 4] >> 6) << 4);
            mn = (unsigned)(s[j + 4] >> 4) | ((unsigned)(s[j] >> 6) << 4);
        }
        const uint8_t qb = blk[16 + 32 * grp + l];
        const unsigned q = hi ? (qb >> 4) : (qb & 15u);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
    }
    case kTypeQ6K: {
        const uint8_t *blk = row + (c >> 8) * 210;
        const int w = c & 255, half = w >> 7, t = w & 127, quad = t >> 5, l = t & 31, is = l >> 4;
        const uint8_t lb = blk[64 * half + 32 * (quad & 1) + l];
        const uint8_t hb = blk[128 + 32 * half + l];
        const unsigned nib = (quad >= 2) ? (lb >> 4) : (lb & 15u);
        const int q = (int)(nib | (((hb >> (2 * quad)) & 3u) << 4)) - 32;
        const int sc = (int)(int8_t)blk[192 + 8 * half + is + 2 * quad];
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[208] | (blk[209] << 8))));
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    default: return 0.0f;
    }
}

__global__ void embed_generic(const uint8_t *table, int type, uint64_t row_stride, int64_t n_vocab,
                              const int32_t *ids, int64_t n_ids, int n_cols, float *out,
                              unsigned *err)
{
    pdl_wait();
    pdl_trigger();
    const int64_t total = n_ids * n_cols;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / n_cols;
        const int c = (int)(e - i * n_cols);
        const int32_t id = ids[i];
        if (id < 0 || id >= n_vocab) {
            if (c == 0) flag_error(err, kErrBadId);
            out[e] = 0.0f;
            continue;
        }
        out[e] = dequant_one(type, table + (uint64_t)id * row_stride, c);
    }
}

// Whole-tensor conversion to fp32 (weights at load time): element e of a
// tensor stored as consecutive blocks is element e of one long row.
__global__ void dequant_tensor_k(const uint8_t *src, int type, int64_t n, float *out)
{
    pdl_wait();
    pdl_trigger();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        out[e] = dequant_one(type, src, (int)e);
}

// Rows of a stored matrix with any row stride (bytes) -> dense fp32 rows.
__global__ void dequant_rows_k(const uint8_t *src, int type, uint64_t row_stride, int64_t n_rows, int n_cols,
                               float *out)
{
    pdl_wait();
    pdl_trigger();
    const int64_t n = n_rows * n_cols;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / n_cols;
        out[e] = dequant_one(type, src + (uint64_t)r * row_stride, (int)(e - r * n_cols));
    }
}

template <int TYPE, int NB>
cudaError_t run_fast(const LaunchCtx &c, const EmbedArgs &a)
{
    // Few rows: one warp per CTA so the rows spread over every SM.
    const int warps = a.n_ids < 8 * (int64_t)c.n_sm ? 1 : kWarps;
    const int64_t need = (a.n_ids + warps - 1) / warps;
    // One row per warp, no persistent grid: the scattered 8 KB output rows
    // drain best when warps retire and new ones start (measured at T=32768:
    // Q6_K 52 us vs 56-71 us for one or two resident waves of persistent
    // warps; Q4_K + norm 89 us vs 99 us). The kernel's two-slot TMA pipeline
    // still serves any warp that is given more than one row.
    auto kern = a.norm ? embed_warp<TYPE, NB, true> : embed_warp<TYPE, NB, false>;
    const int64_t blocks = need;
    launch_k(c, kern, dim3((unsigned)blocks), dim3(warps * 32), a);
    return cudaGetLastError();
}

template <int TYPE>
cudaError_t run_fast_nb(const LaunchCtx &c, const EmbedArgs &a, int nb)
{
    switch (nb) {
    case 1: return run_fast<TYPE, 1>(c, a);
    case 2: return run_fast<TYPE, 2>(c, a);
    case 4: return run_fast<TYPE, 4>(c, a);
    case 8: return run_fast<TYPE, 8>(c, a);
    default: return cudaErrorInvalidValue;
    }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t launch_embed(const LaunchCtx &c, const uint8_t *table, int type, uint64_t row_stride,
                         int64_t n_vocab, const int32_t *ids, int64_t n_ids, int n_cols,
                         float *hidden_out, const float *w, float *norm_out, float eps)
{
    if (n_ids <= 0) return cudaSuccess;
    const int nb = n_cols / 256;
    const bool fast_shape = (type == kTypeQ4K || type == kTypeQ6K) && n_cols % 256 == 0 &&
                            (nb == 1 || nb == 2 || nb == 4 || nb == 8);
    const bool fast_align = (!hidden_out || al16(hidden_out)) && (!norm_out || (al16(norm_out) && al16(w)));
    if (fast_shape && fast_align) {
        EmbedArgs a;
        a.table = table;
        a.ids = ids;
        a.hidden = hidden_out;
        a.w = w;
        a.norm = norm_out;
        a.n_ids = n_ids;
        a.n_vocab = n_vocab;
        a.row_stride = row_stride;
        a.eps = eps;
        a.err = c.err;
        const uint64_t row_bytes = (uint64_t)nb * (type == kTypeQ4K ? 144 : 210);
        a.use_bulk = al16(table) && row_stride % 16 == 0 && row_bytes % 16 == 0;
        return type == kTypeQ4K ? run_fast_nb<kTypeQ4K>(c, a, nb) : run_fast_nb<kTypeQ6K>(c, a, nb);
    }
    // Generic: dequant into hidden (or into norm_out as scratch), then norm in place.
    float *dst = hidden_out ? hidden_out : norm_out;
    const int64_t total = n_ids * (int64_t)n_cols;
    int64_t blocks = (total + 255) / 256;
    if (blocks > (int64_t)c.n_sm * 32) blocks = (int64_t)c.n_sm * 32;
    launch_k(c, embed_generic, dim3((unsigned)blocks), dim3(256), table, type, row_stride, n_vocab, ids, n_ids,
                                                          n_cols, dst, c.err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !norm_out) return e;
    return launch_add_rms_norm(c, dst, nullptr, w, nullptr, norm_out, n_cols, n_ids, eps);
}

cudaError_t launch_dequantize(const LaunchCtx &c, const uint8_t *src, int type, int64_t n, float *out)
{
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 32LL * c.n_sm) blocks = 32LL * c.n_sm;
    launch_k(c, dequant_tensor_k, dim3((unsigned)blocks), dim3(256), src, type, n, out);
    return cudaGetLastError();
}

cudaError_t launch_dequantize_rows(const LaunchCtx &c, const uint8_t *src, int type, uint64_t row_stride,
                                   int64_t n_rows, int n_cols, float *out)
{
    const int64_t n = n_rows * n_cols;
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 32LL * c.n_sm) blocks = 32LL * c.n_sm;
    launch_k(c, dequant_rows_k, dim3((unsigned)blocks), dim3(256), src, type, row_stride, n_rows, n_cols, out);
    return cudaGetLastError();
}

}  // namespace ds3
