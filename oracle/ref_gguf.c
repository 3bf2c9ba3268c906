/* Harness over the UNMODIFIED GGUF reader of the reference engine
 * (src/ds3_gguf.c of wzqhbustb/qw3), compiled where it lies into
 * oracle/_ref/libds3gguf.so by oracle/Makefile. Test infrastructure only:
 * flattens the parsed header and tensor table into plain arrays for ctypes.
 */
#include <stdint.h>
#include <string.h>

#include "ds3_gguf.h"

void *ds3rg_open(const char *path) { return ds3_gguf_open(path); }
void ds3rg_close(void *g) { ds3_gguf_close((ds3_gguf_t *)g); }

/* out[0..4] = version, alignment, n_tensors, n_metadata, tensor data offset */
void ds3rg_header(const void *h, uint64_t out[5])
{
    const ds3_gguf_t *g = (const ds3_gguf_t *)h;
    out[0] = g->version;
    out[1] = g->alignment;
    out[2] = g->n_tensors;
    out[3] = g->n_metadata;
    out[4] = g->tensor_data_offset;
}

/* Tensor i: name into name[cap] (NUL-terminated, truncated), and
 * out[0..9] = n_dims, ne[0..3], type, offset, size, data - mapping base,
 * name length. Returns -1 if i is out of range. */
int ds3rg_tensor(const void *h, uint64_t i, char *name, size_t cap, uint64_t out[10])
{
    const ds3_gguf_t *g = (const ds3_gguf_t *)h;
    if (i >= g->n_tensors) return -1;
    const ds3_gguf_tensor_info_t *t = &g->tensors[i];
    size_t n = t->name.len < cap - 1 ? (size_t)t->name.len : cap - 1;
    memcpy(name, t->name.data, n);
    name[n] = 0;
    out[0] = t->n_dims;
    for (int d = 0; d < 4; d++) out[1 + d] = t->ne[d];
    out[5] = t->type;
    out[6] = t->offset;
    out[7] = t->size;
    out[8] = (uint64_t)((const uint8_t *)t->data - (const uint8_t *)g->mmap_base);
    out[9] = t->name.len;
    return 0;
}

int ds3rg_get_u32(const void *h, const char *key, uint32_t *v)
{
    return ds3_gguf_get_metadata_u32((const ds3_gguf_t *)h, key, v);
}
int ds3rg_get_f32(const void *h, const char *key, float *v)
{
    return ds3_gguf_get_metadata_f32((const ds3_gguf_t *)h, key, v);
}
int ds3rg_get_string(const void *h, const char *key, const char **s, size_t *len)
{
    return ds3_gguf_get_metadata_string((const ds3_gguf_t *)h, key, s, len);
}
