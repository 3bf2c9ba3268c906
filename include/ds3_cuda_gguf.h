/*
 * ds3_cuda_gguf.h - GGUF v3 reader and binding of the tensors the fused
 * per-layer path reads, for the B200 backend (libds3cuda.so).
 *
 * Counterparts in the qw3 engine:
 *   - src/ds3_gguf.h:141-176   ds3_gguf_open / _close / _find_tensor /
 *                              _find_metadata / _get_metadata_{string,u32,f32}
 *   - src/ds3_weights.c:48-99  make_tensor (shape, type, byte strides)
 *   - src/ds3_weights.c:106-215 ds3_weights_load (tensor names per layer)
 *   - src/ds3_engine.c:1609-1622 upload_norm_weight (any norm type -> FP32 on
 *                              the device) and :273-290 (token_embd upload)
 *
 * The file is mmap'd read-only; descriptors point into the mapping, as in the
 * engine. Parsing follows the same order and rules as ds3_gguf_open (magic
 * "GGUF", version >= 3, metadata key/value pairs, tensor infos, data region
 * at the next multiple of general.alignment, default 32). It additionally
 * rejects a file whose tensor data would run past the end of the file, and
 * tensor types it cannot size (the engine logs those and keeps size 0).
 */
#ifndef DS3_CUDA_GGUF_H
#define DS3_CUDA_GGUF_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "ds3_cuda.h"

#pragma GCC visibility push(default)

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ds3_cuda_gguf ds3_cuda_gguf_t;

/* One tensor descriptor (mirrors ds3_gguf_tensor_info_t, src/ds3_gguf.h:111-122,
 * plus the byte strides make_tensor derives, src/ds3_weights.c:63-95).
 * name is NOT NUL-terminated; name_len gives its length. */
typedef struct {
    const char *name;
    uint64_t name_len;
    uint32_t n_dims;       /* 1..4 */
    uint64_t ne[4];        /* unused dimensions are 1 */
    uint64_t nb[4];        /* byte strides: nb[0] block bytes, nb[1] row bytes, ... */
    uint32_t type;         /* ggml type id (ds3_type_t values) */
    uint64_t offset;       /* from the start of the tensor data region */
    uint64_t size;         /* bytes in the file */
    const void *data;      /* into the mapping */
} ds3_cuda_gguf_tensor_t;

/* Open and parse; NULL on failure (ds3_cuda_last_error() says why). Needs no
 * GPU. Replaces ds3_gguf_open. */
ds3_cuda_gguf_t *ds3_cuda_gguf_open(const char *path);
/* Unmap and free. Replaces ds3_gguf_close. */
void ds3_cuda_gguf_close(ds3_cuda_gguf_t *g);

uint32_t ds3_cuda_gguf_version(const ds3_cuda_gguf_t *g);
uint32_t ds3_cuda_gguf_alignment(const ds3_cuda_gguf_t *g);
uint64_t ds3_cuda_gguf_data_offset(const ds3_cuda_gguf_t *g);   /* file offset of the tensor data */
uint64_t ds3_cuda_gguf_n_tensors(const ds3_cuda_gguf_t *g);
uint64_t ds3_cuda_gguf_n_metadata(const ds3_cuda_gguf_t *g);

/* Descriptor i (0-based, file order); 0 on success, -1 if out of range. */
int ds3_cuda_gguf_tensor(const ds3_cuda_gguf_t *g, uint64_t i, ds3_cuda_gguf_tensor_t *out);
/* Descriptor by exact name; 0 on success, -1 if absent. Replaces
 * ds3_gguf_find_tensor (first match in file order). */
int ds3_cuda_gguf_find_tensor(const ds3_cuda_gguf_t *g, const char *name, ds3_cuda_gguf_tensor_t *out);

/* Typed metadata reads; false when the key is absent or has another type.
 * Replace ds3_gguf_get_metadata_{string,u32,f32}. The string is not
 * NUL-terminated. */
bool ds3_cuda_gguf_get_string(const ds3_cuda_gguf_t *g, const char *key, const char **out, size_t *len);
bool ds3_cuda_gguf_get_u32(const ds3_cuda_gguf_t *g, const char *key, uint32_t *out);
bool ds3_cuda_gguf_get_f32(const ds3_cuda_gguf_t *g, const char *key, float *out);

/* Device-resident tensors of the fused per-layer path for n_layer layers,
 * bound by the engine's names (src/ds3_weights.c:122-138):
 *   token_embd.weight                 kept in its file type (Q4_K, Q6_K, Q8_0,
 *                                     F16 or F32), copied as is
 *   output_norm.weight                \
 *   blk.N.attn_norm.weight             |
 *   blk.N.attn_q_norm.weight           |  converted to FP32 on the device
 *   blk.N.attn_k_norm.weight           |  (any of F32, F16, Q8_0, Q4_K, Q6_K)
 *   blk.N.ffn_norm.weight              |
 *   blk.N.ffn_gate_inp.weight         /   (router, [n_expert][n_embd])
 * Missing tensors fail the load, as in ds3_weights_load; q/k norms are
 * required when require_qk_norm is true (the engine's DS3_HAS_QK_NORM). */
typedef struct {
    uint32_t n_layer;
    uint32_t n_embd;            /* token_embd ne[0] */
    uint32_t n_vocab;           /* token_embd ne[1] */
    uint32_t head_dim;          /* attn_q_norm ne[0] (0 without q/k norms) */
    uint32_t n_expert;          /* ffn_gate_inp ne[1] */
    uint32_t token_embd_type;
    uint64_t token_embd_row_stride;   /* bytes per vocabulary row */
    ds3_cuda_buffer_t *token_embd;
    ds3_cuda_buffer_t *output_norm;   /* fp32 [n_embd] */
    ds3_cuda_buffer_t **attn_norm;    /* [n_layer] fp32 [n_embd] */
    ds3_cuda_buffer_t **attn_q_norm;  /* [n_layer] fp32 [head_dim] or NULL entries */
    ds3_cuda_buffer_t **attn_k_norm;
    ds3_cuda_buffer_t **ffn_norm;     /* [n_layer] fp32 [n_embd] */
    ds3_cuda_buffer_t **ffn_gate_inp; /* [n_layer] fp32 [n_expert][n_embd] */
} ds3_cuda_path_weights_t;

/* Needs ds3_cuda_init(). NULL on failure (ds3_cuda_last_error() says why). */
ds3_cuda_path_weights_t *ds3_cuda_path_weights_load(const ds3_cuda_gguf_t *g, uint32_t n_layer,
                                                    bool require_qk_norm);
void ds3_cuda_path_weights_free(ds3_cuda_path_weights_t *w);

#ifdef __cplusplus
}
#endif

#pragma GCC visibility pop

#endif /* DS3_CUDA_GGUF_H */
