/*
 * ds3_oracle.c — CPU restatement of the reference's per-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see ds3_oracle.h): the checker for the CUDA path,
 * never linked into or called by the product.
 *
 * Build with -O2 -ffp-contract=off (oracle/Makefile) so that no multiply-add
 * is fused: every expression below then rounds exactly as the reference's
 * ds3_reference.c does on the same machine, and the tests confirm that the two
 * agree bit for bit.
 *
 * Reference line numbers are for wzqhbustb/qw3 src/ds3_reference.c unless
 * another file is named.
 */
#include "ds3_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int ds3o_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int clamp_threads(int nthreads)
{
    if (nthreads < 1) return 1;
    return nthreads;
}

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32. Follows ds3_reference.c:21-27 (native _Float16 conversion,
 * which is exact for every half value).                                     */
/* ------------------------------------------------------------------------ */
float ds3o_fp16_to_fp32(uint16_t h)
{
    _Float16 v;
    memcpy(&v, &h, sizeof v);
    return (float)v;
}

uint16_t ds3o_fp32_to_fp16(float f)
{
    _Float16 v = (_Float16)f; /* round to nearest even */
    uint16_t h;
    memcpy(&h, &v, sizeof h);
    return h;
}

/* ------------------------------------------------------------------------ */
/* Block layouts: ds3_reference.c:65-70 (Q4_K, 144 B), :119-124 (Q6_K, 210 B),
 * :164-167 (Q8_0, 34 B). Offsets are spelled out so the restatement does not
 * depend on struct packing.                                                 */
/* ------------------------------------------------------------------------ */
#define Q4K_BYTES 144
#define Q6K_BYTES 210
#define Q80_BYTES 34
#define QK_K      256

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 6-bit (scale, min) pair j of the 12 packed bytes: ds3_reference.c:76-85. */
static void q4k_scale_min(int j, const uint8_t *s, unsigned *sc, unsigned *mn)
{
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (s[j + 4] & 15u) | ((unsigned)(s[j - 4] >> 6) << 4);
        *mn = (unsigned)(s[j + 4] >> 4) | ((unsigned)(s[j] >> 6) << 4);
    }
}

/* Q4_K super-block: ds3_reference.c:87-113.  y = (d*sc)*q - dmin*m per 32. */
static void q4k_block(const uint8_t *blk, float *y)
{
    const float d  = ds3o_fp16_to_fp32(rd16(blk));
    const float dm = ds3o_fp16_to_fp32(rd16(blk + 2));
    const uint8_t *scales = blk + 4;
    const uint8_t *qs = blk + 16;
    for (int g = 0; g < 4; g++) {          /* 64 weights per step */
        unsigned sc, mn;
        q4k_scale_min(2 * g, scales, &sc, &mn);
        const float d_lo = d * (float)sc;
        const float m_lo = dm * (float)mn;
        q4k_scale_min(2 * g + 1, scales, &sc, &mn);
        const float d_hi = d * (float)sc;
        const float m_hi = dm * (float)mn;
        const uint8_t *q = qs + 32 * g;
        for (int l = 0; l < 32; l++) y[64 * g + l]      = d_lo * (float)(q[l] & 15) - m_lo;
        for (int l = 0; l < 32; l++) y[64 * g + 32 + l] = d_hi * (float)(q[l] >> 4) - m_hi;
    }
}

/* Q6_K super-block: ds3_reference.c:130-158.  y = (d*sc)*(q-32). */
static void q6k_block(const uint8_t *blk, float *y)
{
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t  *sc = (const int8_t *)(blk + 192);
    const float d = ds3o_fp16_to_fp32(rd16(blk + 208));
    for (int half = 0; half < 2; half++) {
        const uint8_t *L = ql + 64 * half;
        const uint8_t *H = qh + 32 * half;
        const int8_t  *S = sc + 8 * half;
        float *o = y + 128 * half;
        for (int l = 0; l < 32; l++) {
            const int is = l / 16;
            const int v0 = (int)((L[l]      & 15) | (((H[l] >> 0) & 3) << 4)) - 32;
            const int v1 = (int)((L[l + 32] & 15) | (((H[l] >> 2) & 3) << 4)) - 32;
            const int v2 = (int)((L[l]      >> 4) | (((H[l] >> 4) & 3) << 4)) - 32;
            const int v3 = (int)((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32;
            o[l]      = d * (float)S[is + 0] * (float)v0;
            o[l + 32] = d * (float)S[is + 2] * (float)v1;
            o[l + 64] = d * (float)S[is + 4] * (float)v2;
            o[l + 96] = d * (float)S[is + 6] * (float)v3;
        }
    }
}

/* Q8_0 block: ds3_reference.c:173-184.  y = q * d. */
static void q80_block(const uint8_t *blk, float *y)
{
    const float d = ds3o_fp16_to_fp32(rd16(blk));
    const int8_t *q = (const int8_t *)(blk + 2);
    for (int j = 0; j < 32; j++) y[j] = (float)q[j] * d;
}

/* Type switch of ds3_ref_dequantize_row, ds3_reference.c:209-240. */
int ds3o_dequant_row(int type, const void *row, int64_t n_cols, float *out)
{
    const uint8_t *p = (const uint8_t *)row;
    switch (type) {
    case DS3O_TYPE_F32:
        memcpy(out, p, (size_t)n_cols * sizeof(float));
        return 0;
    case DS3O_TYPE_F16:
        for (int64_t i = 0; i < n_cols; i++) out[i] = ds3o_fp16_to_fp32(rd16(p + 2 * i));
        return 0;
    case DS3O_TYPE_Q4_K:
        if (n_cols % QK_K) return -1;
        for (int64_t b = 0; b < n_cols / QK_K; b++) q4k_block(p + b * Q4K_BYTES, out + b * QK_K);
        return 0;
    case DS3O_TYPE_Q6_K:
        if (n_cols % QK_K) return -1;
        for (int64_t b = 0; b < n_cols / QK_K; b++) q6k_block(p + b * Q6K_BYTES, out + b * QK_K);
        return 0;
    case DS3O_TYPE_Q8_0:
        if (n_cols % 32) return -1;
        for (int64_t b = 0; b < n_cols / 32; b++) q80_block(p + b * Q80_BYTES, out + b * 32);
        return 0;
    default:
        return -1;
    }
}

/* Embedding gather: the per-token loop of upload_token_embeddings,
 * src/ds3_engine.c:273-290, with the row bounds check of ds3_reference.c:201-205. */
int ds3o_embed_rows(const void *table, int type, uint64_t row_stride, int64_t n_vocab,
                    const int32_t *ids, int64_t n_ids, int64_t n_cols,
                    float *out, int nthreads)
{
    int rc = 0;
    const uint8_t *base = (const uint8_t *)table;
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static) reduction(|:rc)
    for (int64_t i = 0; i < n_ids; i++) {
        float *o = out + i * n_cols;
        const int32_t id = ids[i];
        if (id < 0 || id >= n_vocab) {
            memset(o, 0, (size_t)n_cols * sizeof(float));
            rc |= 1;
            continue;
        }
        if (ds3o_dequant_row(type, base + (uint64_t)id * row_stride, n_cols, o) != 0) rc |= 1;
    }
    return rc ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* RMSNorm: ds3_reference.c:329-342. Sequential float sum of squares,
 * mean = ss/n, + eps, rms = 1/sqrtf, out = (x*rms)*w.                       */
/* ------------------------------------------------------------------------ */
void ds3o_rms_norm(const float *x, const float *w, float eps, int n, float *out)
{
    float acc = 0.0f;
    for (int i = 0; i < n; i++) acc += x[i] * x[i];
    acc /= (float)n;
    acc += eps;
    const float inv = 1.0f / sqrtf(acc);
    for (int i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

void ds3o_rms_norm_rows(const float *x, const float *w, float eps, int n,
                        int64_t n_rows, float *out, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) ds3o_rms_norm(x + r * n, w, eps, n, out + r * n);
}

/* Residual add then norm, the engine sequence vec_add_inplace -> copy ->
 * rms_norm of src/ds3_engine.c:857-866; the add is ds3_ref_add,
 * ds3_reference.c:455-460. */
void ds3o_add_rms_norm(const float *x, const float *r, const float *w, float eps,
                       int n, int64_t n_rows, float *sum_out, float *norm_out,
                       int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t row = 0; row < n_rows; row++) {
        float *tmp = (float *)malloc((size_t)n * sizeof(float));
        const float *a = x + row * n, *b = r + row * n;
        for (int i = 0; i < n; i++) tmp[i] = a[i] + b[i];
        if (sum_out) memcpy(sum_out + row * n, tmp, (size_t)n * sizeof(float));
        ds3o_rms_norm(tmp, w, eps, n, norm_out + row * n);
        free(tmp);
    }
}

int ds3o_embed_rms_norm(const void *table, int type, uint64_t row_stride, int64_t n_vocab,
                        const int32_t *ids, int64_t n_ids, int64_t n_cols,
                        const float *w, float eps, float *hidden_out, float *norm_out,
                        int nthreads)
{
    int rc = ds3o_embed_rows(table, type, row_stride, n_vocab, ids, n_ids, n_cols,
                             hidden_out, nthreads);
    ds3o_rms_norm_rows(hidden_out, w, eps, (int)n_cols, n_ids, norm_out, nthreads);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* NEOX RoPE: ds3_reference.c:361-402. Pairs (i, i+hd/2),
 * freq = powf(theta, (float)i * (-2/hd)), angle = pos*freq in float.        */
/* ------------------------------------------------------------------------ */
static void rope_head(float *x, int pos, int head_dim, float theta)
{
    const float step = -2.0f / head_dim;
    const int half = head_dim / 2;
    for (int i = 0; i < half; i++) {
        const float freq = powf(theta, (float)i * step);
        const float ang = pos * freq;
        const float c = cosf(ang);
        const float s = sinf(ang);
        const float a = x[i];
        const float b = x[i + half];
        x[i]        = a * c - b * s;
        x[i + half] = a * s + b * c;
    }
}

void ds3o_rope_token(float *q, float *k, int pos, int n_q_head, int n_kv_head,
                     int head_dim, float theta)
{
    for (int h = 0; h < n_q_head; h++) rope_head(q + h * head_dim, pos, head_dim, theta);
    for (int h = 0; h < n_kv_head; h++) rope_head(k + h * head_dim, pos, head_dim, theta);
}

void ds3o_rope_rows(const float *src, float *dst, const int32_t *positions,
                    int n_heads, int head_dim, int64_t n_rows, float theta, int nthreads)
{
    const int64_t row_elems = (int64_t)n_heads * head_dim;
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) {
        if (dst != src) memcpy(dst + r * row_elems, src + r * row_elems,
                               (size_t)row_elems * sizeof(float));
        for (int h = 0; h < n_heads; h++)
            rope_head(dst + r * row_elems + (int64_t)h * head_dim, positions[r], head_dim, theta);
    }
}

/* Per-head QK RMSNorm (ds3_reference.c:526-533, engine src/ds3_engine.c:789-792)
 * followed by RoPE of the same token (ds3_reference.c:536). */
void ds3o_qk_norm_rope(float *q, float *k, const float *q_w, const float *k_w,
                       const int32_t *positions, int64_t n_rows, int n_q_head,
                       int n_kv_head, int head_dim, float theta, float eps, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_rows; t++) {
        float *qt = q + t * (int64_t)n_q_head * head_dim;
        float *kt = k + t * (int64_t)n_kv_head * head_dim;
        for (int h = 0; h < n_q_head; h++)
            ds3o_rms_norm(qt + h * head_dim, q_w, eps, head_dim, qt + h * head_dim);
        for (int h = 0; h < n_kv_head; h++)
            ds3o_rms_norm(kt + h * head_dim, k_w, eps, head_dim, kt + h * head_dim);
        ds3o_rope_token(qt, kt, positions[t], n_q_head, n_kv_head, head_dim, theta);
    }
}

/* ------------------------------------------------------------------------ */
/* Softmax: ds3_reference.c:344-359.                                         */
/* ------------------------------------------------------------------------ */
void ds3o_softmax(float *x, int n)
{
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float total = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        total += x[i];
    }
    const float inv = 1.0f / total;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* Selection top-k: ds3_reference.c:466-490. Strict '>' over ascending index,
 * so among equal values the lowest index is taken first. */
void ds3o_topk(const float *scores, int n, int k, int32_t *idx_out, float *val_out)
{
    unsigned char *taken = (unsigned char *)calloc((size_t)n, 1);
    for (int r = 0; r < k; r++) {
        float best = -1e30f;
        int at = -1;
        for (int j = 0; j < n; j++) {
            if (!taken[j] && scores[j] > best) { best = scores[j]; at = j; }
        }
        if (at < 0) { idx_out[r] = -1; val_out[r] = best; continue; }
        taken[at] = 1;
        idx_out[r] = at;
        val_out[r] = best;
    }
    free(taken);
}

/* Router: softmax + top-k (ds3_reference.c:627-629) and the renormalisation
 * of ds3_reference.c:632-639 (sequential sum in k order, scale by 1/sum). */
void ds3o_router_softmax_topk(const float *logits, int64_t n_tokens, int n_expert, int n_used,
                              int norm_topk_prob, float *probs_out, int32_t *idx_out,
                              float *scores_out, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++) {
        float *p = (float *)malloc((size_t)n_expert * sizeof(float));
        memcpy(p, logits + t * n_expert, (size_t)n_expert * sizeof(float));
        ds3o_softmax(p, n_expert);
        if (probs_out) memcpy(probs_out + t * n_expert, p, (size_t)n_expert * sizeof(float));
        int32_t *ix = idx_out + t * n_used;
        float *sc = scores_out + t * n_used;
        ds3o_topk(p, n_expert, n_used, ix, sc);
        if (norm_topk_prob) {
            float s = 0.0f;
            for (int i = 0; i < n_used; i++) s += sc[i];
            if (s > 0.0f) {
                const float inv = 1.0f / s;
                for (int i = 0; i < n_used; i++) sc[i] *= inv;
            }
        }
        free(p);
    }
}

/* ------------------------------------------------------------------------ */
/* SwiGLU: silu (ds3_reference.c:436-441) then mul (:443-448), i.e.
 * (g / (1 + expf(-g))) * u, then times the routing weight of the row.       */
/* ------------------------------------------------------------------------ */
void ds3o_swiglu(const float *gate, const float *up, const float *row_weight, float *out,
                 int64_t n_rows, int64_t n_cols, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) {
        const float *g = gate + r * n_cols, *u = up + r * n_cols;
        float *o = out + r * n_cols;
        for (int64_t c = 0; c < n_cols; c++) {
            const float s = g[c] / (1.0f + expf(-g[c]));
            float v = s * u[c];
            if (row_weight) v = v * row_weight[r];
            o[c] = v;
        }
    }
}

/* Weighted expert accumulation from zero in k order (ds3_reference.c:642 and
 * :674-678) followed by the residual add (ds3_reference.c:777, ds3_ref_add). */
void ds3o_moe_combine_residual(const float *y, const int32_t *y_rows, const float *w,
                               const float *residual, float *out, int64_t n_tokens,
                               int n_used, int64_t n_cols, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++) {
        for (int64_t c = 0; c < n_cols; c++) {
            float acc = 0.0f;
            for (int k = 0; k < n_used; k++) {
                const int64_t row = y_rows ? (int64_t)y_rows[t * n_used + k] : t * n_used + k;
                acc += w[t * n_used + k] * y[row * n_cols + c];
            }
            out[t * n_cols + c] = residual[t * n_cols + c] + acc;
        }
    }
}

/* scatter_add_weighted_f32, metal/elementwise.metal:198-211. */
void ds3o_scatter_add_weighted(const float *src, const float *scores, const int32_t *ids,
                               float *dst, int64_t n_cols, int64_t count, int64_t offset)
{
    for (int64_t i = 0; i < count; i++) {
        const int64_t row = ids[offset + i];
        const float wt = scores[offset + i];
        for (int64_t j = 0; j < n_cols; j++) dst[row * n_cols + j] += wt * src[i * n_cols + j];
    }
}

/* gather_rows_f32, metal/elementwise.metal:175-186. */
void ds3o_gather_rows(const float *src, const int32_t *ids, float *dst, int64_t n_cols,
                      int64_t count, int64_t offset)
{
    for (int64_t i = 0; i < count; i++)
        memcpy(dst + i * n_cols, src + (int64_t)ids[offset + i] * n_cols,
               (size_t)n_cols * sizeof(float));
}

/* kv_cache_write_batch, metal/attention.metal:66-87 (and ds3_metal.m:1588-1660):
 * k_cache[(seq_pos + t) * row + e] = half(k[t * row + e]), same for v. The
 * engine's cache is fp16 (src/ds3.h:179-182); conversion rounds to nearest. */
void ds3o_kv_cache_write(const float *k, const float *v, const int32_t *row_of, int64_t seq_pos,
                         int64_t n_tokens, int64_t row_elems, uint16_t *k_cache, uint16_t *v_cache)
{
    for (int64_t t = 0; t < n_tokens; t++) {
        const int64_t dst = (row_of ? (int64_t)row_of[t] : seq_pos + t) * row_elems;
        for (int64_t e = 0; e < row_elems; e++) {
            k_cache[dst + e] = ds3o_fp32_to_fp16(k[t * row_elems + e]);
            v_cache[dst + e] = ds3o_fp32_to_fp16(v[t * row_elems + e]);
        }
    }
}

/* Per-expert token lists: forward_chunk_post_gathered, src/ds3_engine.c:933-954
 * (counts zeroed, then for t ascending, k ascending: slot ex*M + counts[ex]++). */
int ds3o_moe_expert_lists(const int32_t *idx, const float *scores, int64_t n_tokens, int n_used,
                          int n_expert, int64_t cap, int32_t *counts, int32_t *ids, float *gscores,
                          int32_t *slot_of)
{
    int rc = 0;
    memset(counts, 0, (size_t)n_expert * sizeof(int32_t));
    for (int64_t t = 0; t < n_tokens; t++) {
        for (int k = 0; k < n_used; k++) {
            const int64_t i = t * n_used + k;
            const int32_t ex = idx[i];
            if (ex < 0 || ex >= n_expert || counts[ex] >= cap) {
                rc = -1;
                if (slot_of) slot_of[i] = -1;
                continue;
            }
            const int64_t slot = (int64_t)ex * cap + counts[ex];
            ids[slot] = (int32_t)t;
            gscores[slot] = scores[i];
            if (slot_of) slot_of[i] = (int32_t)slot;
            counts[ex]++;
        }
    }
    return rc;
}

/* Vector x matrix as ds3_ref_vec_matmul, src/ds3_reference.c:424-434. */
void ds3o_router_logits(const float *x, const float *W, int64_t n_tokens, int n_embd, int n_expert,
                        float *logits, int nthreads)
{
#pragma omp parallel for num_threads(clamp_threads(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++) {
        const float *xr = x + t * n_embd;
        for (int e = 0; e < n_expert; e++) {
            const float *wr = W + (int64_t)e * n_embd;
            float acc = 0.0f;
            for (int i = 0; i < n_embd; i++) acc += xr[i] * wr[i];
            logits[t * n_expert + e] = acc;
        }
    }
}
