/*
 * ref_harness.c — drives the UNMODIFIED reference CPU kernels
 * (wzqhbustb/qw3 src/ds3_reference.c, compiled from the reference tree by
 * oracle/Makefile into oracle/_ref/libds3ref.so).
 *
 * TEST INFRASTRUCTURE ONLY: used to pin the restatement in ds3_oracle.c, to
 * generate the golden fixtures in tests/golden/, and as the timed CPU
 * baseline of bench.py. The product never loads it.
 *
 * Each ds3r_* entry has the signature of the matching ds3o_* entry in
 * ds3_oracle.h, so a test can run either library on the same inputs. The
 * loops over rows/tokens are the only code here; every value is computed by
 * a ds3_ref_* call. The few pieces of arithmetic the reference performs
 * inline rather than in a function are restated and marked "glue".
 */
#include "ds3_reference.h"

#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ds3.h declares this logging switch; the engine's ds3_log.c defines it. */
int ds3_log_quiet = 1;

static int nt(int n) { return n < 1 ? 1 : n; }

int ds3r_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

int ds3r_embed_rows(const void *table, int type, uint64_t row_stride, int64_t n_vocab,
                    const int32_t *ids, int64_t n_ids, int64_t n_cols,
                    float *out, int nthreads)
{
    ds3_tensor_t t;
    memset(&t, 0, sizeof t);
    t.type = (ds3_type_t)type;
    t.n_dims = 2;
    t.ne[0] = (uint64_t)n_cols;
    t.ne[1] = (uint64_t)n_vocab;
    t.nb[1] = row_stride;
    t.data = (void *)table;
    t.size = (size_t)(row_stride * (uint64_t)n_vocab);
    int rc = 0;
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static) reduction(|:rc)
    for (int64_t i = 0; i < n_ids; i++) {
        if (ds3_ref_dequantize_row(&t, ids[i], out + i * n_cols) != 0) {
            memset(out + i * n_cols, 0, (size_t)n_cols * sizeof(float));
            rc |= 1;
        }
    }
    return rc ? -1 : 0;
}

void ds3r_rms_norm_rows(const float *x, const float *w, float eps, int n,
                        int64_t n_rows, float *out, int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) ds3_ref_rms_norm(x + r * n, w, eps, n, out + r * n);
}

void ds3r_add_rms_norm(const float *x, const float *r, const float *w, float eps,
                       int n, int64_t n_rows, float *sum_out, float *norm_out,
                       int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t row = 0; row < n_rows; row++) {
        float *tmp = (float *)malloc((size_t)n * sizeof(float));
        ds3_ref_add(x + row * n, r + row * n, tmp, n);
        if (sum_out) memcpy(sum_out + row * n, tmp, (size_t)n * sizeof(float));
        ds3_ref_rms_norm(tmp, w, eps, n, norm_out + row * n);
        free(tmp);
    }
}

int ds3r_embed_rms_norm(const void *table, int type, uint64_t row_stride, int64_t n_vocab,
                        const int32_t *ids, int64_t n_ids, int64_t n_cols,
                        const float *w, float eps, float *hidden_out, float *norm_out,
                        int nthreads)
{
    int rc = ds3r_embed_rows(table, type, row_stride, n_vocab, ids, n_ids, n_cols,
                             hidden_out, nthreads);
    ds3r_rms_norm_rows(hidden_out, w, eps, (int)n_cols, n_ids, norm_out, nthreads);
    return rc;
}

/* The reference's RoPE hard-codes theta = DS3_ROPE_THETA (1e6); `theta` is
 * accepted for signature parity with the restatement and must be 1e6. */
void ds3r_qk_norm_rope(float *q, float *k, const float *q_w, const float *k_w,
                       const int32_t *positions, int64_t n_rows, int n_q_head,
                       int n_kv_head, int head_dim, float theta, float eps, int nthreads)
{
    (void)theta;
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_rows; t++) {
        float *qt = q + t * (int64_t)n_q_head * head_dim;
        float *kt = k + t * (int64_t)n_kv_head * head_dim;
        for (int h = 0; h < n_q_head; h++)
            ds3_ref_rms_norm(qt + h * head_dim, q_w, eps, head_dim, qt + h * head_dim);
        for (int h = 0; h < n_kv_head; h++)
            ds3_ref_rms_norm(kt + h * head_dim, k_w, eps, head_dim, kt + h * head_dim);
        ds3_ref_rope(qt, kt, positions[t], n_q_head, n_kv_head, head_dim);
    }
}

void ds3r_rope_rows(const float *src, float *dst, const int32_t *positions,
                    int n_heads, int head_dim, int64_t n_rows, float theta, int nthreads)
{
    (void)theta;
    const int64_t row_elems = (int64_t)n_heads * head_dim;
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) {
        if (dst != src) memcpy(dst + r * row_elems, src + r * row_elems,
                               (size_t)row_elems * sizeof(float));
        /* ds3_ref_rope rotates q heads then k heads; pass all heads as q. */
        ds3_ref_rope(dst + r * row_elems, NULL, positions[r], n_heads, 0, head_dim);
    }
}

void ds3r_router_softmax_topk(const float *logits, int64_t n_tokens, int n_expert, int n_used,
                              int norm_topk_prob, float *probs_out, int32_t *idx_out,
                              float *scores_out, int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++) {
        float *p = (float *)malloc((size_t)n_expert * sizeof(float));
        int *ix = (int *)malloc((size_t)n_used * sizeof(int));
        memcpy(p, logits + t * n_expert, (size_t)n_expert * sizeof(float));
        ds3_ref_softmax(p, n_expert);
        if (probs_out) memcpy(probs_out + t * n_expert, p, (size_t)n_expert * sizeof(float));
        float *sc = scores_out + t * n_used;
        ds3_ref_topk(p, n_expert, n_used, ix, sc);
        for (int i = 0; i < n_used; i++) idx_out[t * n_used + i] = ix[i];
        if (norm_topk_prob) { /* glue: ds3_reference.c:632-639 */
            float s = 0.0f;
            for (int i = 0; i < n_used; i++) s += sc[i];
            if (s > 0.0f) {
                const float inv = 1.0f / s;
                for (int i = 0; i < n_used; i++) sc[i] *= inv;
            }
        }
        free(ix);
        free(p);
    }
}

void ds3r_swiglu(const float *gate, const float *up, const float *row_weight, float *out,
                 int64_t n_rows, int64_t n_cols, int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t r = 0; r < n_rows; r++) {
        float *o = out + r * n_cols;
        ds3_ref_silu(gate + r * n_cols, o, (int)n_cols);
        ds3_ref_mul(o, up + r * n_cols, o, (int)n_cols);
        if (row_weight) { /* glue: routing weight of the row */
            const float wt = row_weight[r];
            for (int64_t c = 0; c < n_cols; c++) o[c] = o[c] * wt;
        }
    }
}

void ds3r_moe_combine_residual(const float *y, const int32_t *y_rows, const float *w,
                               const float *residual, float *out, int64_t n_tokens,
                               int n_used, int64_t n_cols, int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++) {
        float *acc = (float *)calloc((size_t)n_cols, sizeof(float));
        for (int k = 0; k < n_used; k++) { /* glue: ds3_reference.c:674-678 */
            const int64_t row = y_rows ? (int64_t)y_rows[t * n_used + k] : t * n_used + k;
            const float wt = w[t * n_used + k];
            const float *yr = y + row * n_cols;
            for (int64_t c = 0; c < n_cols; c++) acc[c] += wt * yr[c];
        }
        ds3_ref_add(residual + t * n_cols, acc, out + t * n_cols, (int)n_cols);
        free(acc);
    }
}

void ds3r_router_logits(const float *x, const float *W, int64_t n_tokens, int n_embd, int n_expert,
                        float *logits, int nthreads)
{
#pragma omp parallel for num_threads(nt(nthreads)) schedule(static)
    for (int64_t t = 0; t < n_tokens; t++)
        ds3_ref_vec_matmul(x + t * n_embd, W, logits + t * n_expert, n_embd, n_expert);
}
