// GGUF v3 reader and the device binding of the fused path's tensors.
//
// Parsing follows the engine's ds3_gguf_open (src/ds3_gguf.c:179-356): header
// (magic, version >= 3, tensor count, metadata count), the metadata key/value
// pairs (general.alignment, when stored as uint32, overrides the default of
// 32), the tensor infos (name, n_dims <= 4, ne[], type, offset), and the data
// region at the first multiple of the alignment after the infos. Tensor sizes
// use the same block sizes and bytes per block, a trailing partial block
// counting as a whole one (:311-344). Byte strides follow make_tensor
// (src/ds3_weights.c:63-95), including nb[1] = 0 for 1-D tensors.
//
// Deliberate differences, all of them on files the engine would misread:
//   - an unknown metadata value type, a zero alignment, a tensor type without
//     a known block size and tensor data running past the end of the file
//     reject the file (the engine logs the first and third and parses on,
//     divides by zero on the second, and checks the fourth only in its test
//     program, tests/test_gguf.c:75-88);
//   - arrays of arrays are skipped element by element as the GGUF
//     specification defines them (the engine does not skip them).
#include "ds3_cuda_gguf.h"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace ds3 {
void report_error(const char *msg);  // ds3_cuda.cu
}

namespace {

void fail(const char *fmt, ...)
{
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    ds3::report_error(msg);
}

enum : uint32_t {
    kMetaU8 = 0, kMetaI8, kMetaU16, kMetaI16, kMetaU32, kMetaI32, kMetaF32, kMetaBool, kMetaString, kMetaArray,
    kMetaU64, kMetaI64, kMetaF64
};

// Little-endian reads from an unaligned byte pointer.
uint64_t le(const uint8_t *p, int bytes)
{
    uint64_t v = 0;
    for (int i = bytes - 1; i >= 0; i--) v = (v << 8) | p[i];
    return v;
}

// Bounds-checked cursor over the mapping; any overrun clears ok.
struct Cursor {
    const uint8_t *p, *end;
    bool ok = true;
    bool take(uint64_t n)
    {
        if (!ok || (uint64_t)(end - p) < n) return ok = false;
        p += n;
        return true;
    }
    uint64_t num(int bytes)
    {
        const uint8_t *at = p;
        return take((uint64_t)bytes) ? le(at, bytes) : 0;
    }
    // GGUF string: u64 length + bytes.
    const char *str(uint64_t *len)
    {
        *len = num(8);
        const uint8_t *at = p;
        return take(*len) ? reinterpret_cast<const char *>(at) : nullptr;
    }
};

int scalar_bytes(uint32_t type)
{
    switch (type) {
    case kMetaU8: case kMetaI8: case kMetaBool: return 1;
    case kMetaU16: case kMetaI16: return 2;
    case kMetaU32: case kMetaI32: case kMetaF32: return 4;
    case kMetaU64: case kMetaI64: case kMetaF64: return 8;
    default: return 0;
    }
}

// Skip one value of `type`; false on an unknown type or an overrun.
bool skip_value(Cursor &c, uint32_t type, int depth)
{
    if (const int b = scalar_bytes(type)) return c.take((uint64_t)b);
    if (type == kMetaString) {
        uint64_t n;
        c.str(&n);
        return c.ok;
    }
    if (type == kMetaArray && depth < 8) {
        const uint32_t et = (uint32_t)c.num(4);
        const uint64_t n = c.num(8);
        if (!c.ok) return false;
        if (const int b = scalar_bytes(et)) {
            if (n > UINT64_MAX / (uint64_t)b) return c.ok = false;
            return c.take(n * (uint64_t)b);
        }
        for (uint64_t i = 0; i < n; i++)
            if (!skip_value(c, et, depth + 1)) return false;
        return true;
    }
    return c.ok = false;
}

// Bytes per block and elements per block of a tensor type (0 if unknown);
// the table of src/ds3_gguf.c:314-330.
bool type_geometry(uint32_t type, uint64_t *block_bytes, uint64_t *block_elems)
{
    struct G { uint32_t t; uint64_t bytes, elems; };
    static const G table[] = {{0, 4, 1},     {1, 2, 1},     {2, 18, 32},   {6, 22, 32},   {8, 34, 32},
                              {10, 84, 256}, {11, 110, 256}, {12, 144, 256}, {13, 176, 256}, {14, 210, 256},
                              {15, 290, 256}, {16, 66, 256}, {17, 74, 256},  {18, 98, 256}};
    for (const G &g : table)
        if (g.t == type) {
            *block_bytes = g.bytes;
            *block_elems = g.elems;
            return true;
        }
    return false;
}

struct Meta {
    const char *key;
    uint64_t key_len;
    uint32_t type;
    const uint8_t *value;  // first byte of the value in the mapping
};

bool name_is(const char *s, uint64_t len, const char *want)
{
    return strlen(want) == len && memcmp(s, want, len) == 0;
}

}  // namespace

struct ds3_cuda_gguf {
    int fd = -1;
    void *base = MAP_FAILED;
    size_t bytes = 0;
    uint32_t version = 0;
    uint32_t alignment = 32;
    uint64_t data_offset = 0;
    std::vector<Meta> meta;
    std::vector<ds3_cuda_gguf_tensor_t> tensors;
};

extern "C" {

void ds3_cuda_gguf_close(ds3_cuda_gguf_t *g)
{
    if (!g) return;
    if (g->base != MAP_FAILED) munmap(g->base, g->bytes);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

ds3_cuda_gguf_t *ds3_cuda_gguf_open(const char *path)
{
    if (!path) {
        fail("gguf_open: path is NULL");
        return nullptr;
    }
    ds3_cuda_gguf_t *g = new ds3_cuda_gguf_t();
    g->fd = open(path, O_RDONLY);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        fail("gguf_open: cannot open %s", path);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }
    g->bytes = (size_t)st.st_size;
    if (g->bytes > 0) g->base = mmap(nullptr, g->bytes, PROT_READ, MAP_SHARED, g->fd, 0);
    if (g->base == MAP_FAILED) {
        fail("gguf_open: cannot map %s (%zu bytes)", path, g->bytes);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }
    const uint8_t *b = static_cast<const uint8_t *>(g->base);
    Cursor c{b, b + g->bytes};

    const uint32_t magic = (uint32_t)c.num(4);
    if (!c.ok || magic != 0x46554747u) {
        fail("gguf_open: %s: bad magic", path);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }
    g->version = (uint32_t)c.num(4);
    if (!c.ok || g->version < 3) {
        fail("gguf_open: %s: version %u, need 3", path, g->version);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }
    const uint64_t n_tensors = c.num(8), n_meta = c.num(8);
    // Every metadata pair and tensor info takes at least 12 bytes, which
    // bounds the counts before anything is reserved.
    if (!c.ok || n_tensors > g->bytes / 12 || n_meta > g->bytes / 12) {
        fail("gguf_open: %s: truncated header or impossible counts", path);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }

    g->meta.reserve(n_meta);
    for (uint64_t i = 0; i < n_meta; i++) {
        Meta m;
        m.key = c.str(&m.key_len);
        m.type = (uint32_t)c.num(4);
        m.value = c.p;
        if (!c.ok || !skip_value(c, m.type, 0)) {
            fail("gguf_open: %s: metadata pair %llu unreadable (value type %u)", path, (unsigned long long)i,
                 m.type);
            ds3_cuda_gguf_close(g);
            return nullptr;
        }
        if (m.type == kMetaU32 && name_is(m.key, m.key_len, "general.alignment"))
            g->alignment = (uint32_t)le(m.value, 4);
        g->meta.push_back(m);
    }
    if (g->alignment == 0) {
        fail("gguf_open: %s: general.alignment is 0", path);
        ds3_cuda_gguf_close(g);
        return nullptr;
    }

    g->tensors.reserve(n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        ds3_cuda_gguf_tensor_t t;
        memset(&t, 0, sizeof t);
        t.name = c.str(&t.name_len);
        t.n_dims = (uint32_t)c.num(4);
        if (c.ok && t.n_dims > 4) {
            fail("gguf_open: %s: tensor %.*s has %u dimensions (at most 4)", path, (int)t.name_len, t.name,
                 t.n_dims);
            ds3_cuda_gguf_close(g);
            return nullptr;
        }
        for (uint32_t d = 0; d < 4; d++) t.ne[d] = d < t.n_dims ? c.num(8) : 1;
        t.type = (uint32_t)c.num(4);
        t.offset = c.num(8);
        if (!c.ok) {
            fail("gguf_open: %s: tensor info %llu truncated", path, (unsigned long long)i);
            ds3_cuda_gguf_close(g);
            return nullptr;
        }
        g->tensors.push_back(t);
    }

    const uint64_t info_end = (uint64_t)(c.p - b);
    g->data_offset = info_end + (g->alignment - info_end % g->alignment) % g->alignment;
    for (ds3_cuda_gguf_tensor_t &t : g->tensors) {
        uint64_t bb, be;
        if (!type_geometry(t.type, &bb, &be)) {
            fail("gguf_open: %s: tensor %.*s has unknown type %u", path, (int)t.name_len, t.name, t.type);
            ds3_cuda_gguf_close(g);
            return nullptr;
        }
        uint64_t n = 1;
        for (uint32_t d = 0; d < t.n_dims; d++) n *= t.ne[d];
        t.size = (n / be) * bb + (n % be ? bb : 0);
        t.nb[0] = t.n_dims ? bb : 0;
        t.nb[1] = t.n_dims >= 2 ? bb * (t.ne[0] / be) : 0;
        for (int d = 2; d < 4; d++) t.nb[d] = t.nb[d - 1] * t.ne[d - 1];
        if (g->data_offset > g->bytes || t.offset > g->bytes - g->data_offset ||
            t.size > g->bytes - g->data_offset - t.offset) {
            fail("gguf_open: %s: tensor %.*s (offset %llu, %llu bytes) runs past the end of the file", path,
                 (int)t.name_len, t.name, (unsigned long long)t.offset, (unsigned long long)t.size);
            ds3_cuda_gguf_close(g);
            return nullptr;
        }
        t.data = b + g->data_offset + t.offset;
    }
    return g;
}

uint32_t ds3_cuda_gguf_version(const ds3_cuda_gguf_t *g) { return g ? g->version : 0; }
uint32_t ds3_cuda_gguf_alignment(const ds3_cuda_gguf_t *g) { return g ? g->alignment : 0; }
uint64_t ds3_cuda_gguf_data_offset(const ds3_cuda_gguf_t *g) { return g ? g->data_offset : 0; }
uint64_t ds3_cuda_gguf_n_tensors(const ds3_cuda_gguf_t *g) { return g ? g->tensors.size() : 0; }
uint64_t ds3_cuda_gguf_n_metadata(const ds3_cuda_gguf_t *g) { return g ? g->meta.size() : 0; }

int ds3_cuda_gguf_tensor(const ds3_cuda_gguf_t *g, uint64_t i, ds3_cuda_gguf_tensor_t *out)
{
    if (!g || !out || i >= g->tensors.size()) return -1;
    *out = g->tensors[i];
    return 0;
}

int ds3_cuda_gguf_find_tensor(const ds3_cuda_gguf_t *g, const char *name, ds3_cuda_gguf_tensor_t *out)
{
    if (!g || !name) return -1;
    for (const ds3_cuda_gguf_tensor_t &t : g->tensors)
        if (name_is(t.name, t.name_len, name)) {
            if (out) *out = t;
            return 0;
        }
    return -1;
}

static const Meta *find_meta(const ds3_cuda_gguf_t *g, const char *key, uint32_t type)
{
    if (!g || !key) return nullptr;
    for (const Meta &m : g->meta)
        if (m.type == type && name_is(m.key, m.key_len, key)) return &m;
    return nullptr;
}

bool ds3_cuda_gguf_get_string(const ds3_cuda_gguf_t *g, const char *key, const char **out, size_t *len)
{
    const Meta *m = find_meta(g, key, kMetaString);
    if (!m || !out || !len) return false;
    *len = (size_t)le(m->value, 8);
    *out = reinterpret_cast<const char *>(m->value + 8);
    return true;
}

bool ds3_cuda_gguf_get_u32(const ds3_cuda_gguf_t *g, const char *key, uint32_t *out)
{
    const Meta *m = find_meta(g, key, kMetaU32);
    if (!m || !out) return false;
    *out = (uint32_t)le(m->value, 4);
    return true;
}

bool ds3_cuda_gguf_get_f32(const ds3_cuda_gguf_t *g, const char *key, float *out)
{
    const Meta *m = find_meta(g, key, kMetaF32);
    if (!m || !out) return false;
    const uint32_t u = (uint32_t)le(m->value, 4);
    memcpy(out, &u, 4);
    return true;
}

// ---------------------------------------------------------------------------
// Device binding of the path's tensors.
// ---------------------------------------------------------------------------

static uint64_t n_elements(const ds3_cuda_gguf_tensor_t &t)
{
    uint64_t n = 1;
    for (uint32_t d = 0; d < t.n_dims; d++) n *= t.ne[d];
    return n;
}

// A weight the kernels read as fp32: copied as is when the file holds F32,
// else copied raw and converted on the device (the engine converts on the
// host, src/ds3_engine.c:154-179 and :1609-1622; the values are the same).
static ds3_cuda_buffer_t *upload_f32(const ds3_cuda_gguf_tensor_t &t)
{
    const uint64_t n = n_elements(t);
    if (t.type == DS3_TYPE_F32) return ds3_cuda_buffer_from_mmap(t.data, (size_t)t.size);
    ds3_cuda_buffer_t *raw = ds3_cuda_buffer_from_mmap(t.data, (size_t)t.size);
    ds3_cuda_buffer_t *out = raw ? ds3_cuda_buffer_alloc((size_t)n * 4) : nullptr;
    if (!out || ds3_cuda_dequantize_f32(raw, (ds3_type_t)t.type, n, out) != 0) {
        ds3_cuda_buffer_free(out);
        out = nullptr;
    } else {
        ds3_cuda_synchronize();  // the raw copy is freed next
    }
    ds3_cuda_buffer_free(raw);
    return out;
}

void ds3_cuda_path_weights_free(ds3_cuda_path_weights_t *w)
{
    if (!w) return;
    ds3_cuda_buffer_free(w->token_embd);
    ds3_cuda_buffer_free(w->output_norm);
    ds3_cuda_buffer_t **lists[] = {w->attn_norm, w->attn_q_norm, w->attn_k_norm, w->ffn_norm, w->ffn_gate_inp};
    for (ds3_cuda_buffer_t **l : lists) {
        if (!l) continue;
        for (uint32_t i = 0; i < w->n_layer; i++) ds3_cuda_buffer_free(l[i]);
        free(l);
    }
    free(w);
}

ds3_cuda_path_weights_t *ds3_cuda_path_weights_load(const ds3_cuda_gguf_t *g, uint32_t n_layer, bool require_qk_norm)
{
    if (!g || n_layer == 0) {
        fail("path_weights_load: need an open file and n_layer > 0");
        return nullptr;
    }
    ds3_cuda_path_weights_t *w = (ds3_cuda_path_weights_t *)calloc(1, sizeof(ds3_cuda_path_weights_t));
    if (!w) return nullptr;
    w->n_layer = n_layer;
    ds3_cuda_buffer_t ***lists[] = {&w->attn_norm, &w->attn_q_norm, &w->attn_k_norm, &w->ffn_norm,
                                    &w->ffn_gate_inp};
    for (ds3_cuda_buffer_t ***l : lists)
        if (!(*l = (ds3_cuda_buffer_t **)calloc(n_layer, sizeof(ds3_cuda_buffer_t *)))) {
            ds3_cuda_path_weights_free(w);
            return nullptr;
        }

    ds3_cuda_gguf_tensor_t t;
    if (ds3_cuda_gguf_find_tensor(g, "token_embd.weight", &t) != 0 || t.n_dims != 2) {
        fail("path_weights_load: token_embd.weight missing or not 2-D");
        ds3_cuda_path_weights_free(w);
        return nullptr;
    }
    w->n_embd = (uint32_t)t.ne[0];
    w->n_vocab = (uint32_t)t.ne[1];
    w->token_embd_type = t.type;
    w->token_embd_row_stride = t.nb[1];
    if (!(w->token_embd = ds3_cuda_buffer_from_mmap(t.data, (size_t)t.size))) {
        ds3_cuda_path_weights_free(w);
        return nullptr;
    }

    // One fp32 weight: name, expected element count (0 = any), destination.
    auto bind = [&](const char *name, uint64_t want, bool required, ds3_cuda_buffer_t **dst) -> bool {
        ds3_cuda_gguf_tensor_t x;
        if (ds3_cuda_gguf_find_tensor(g, name, &x) != 0) {
            if (required) fail("path_weights_load: missing %s", name);
            return !required;
        }
        if (want && n_elements(x) != want) {
            fail("path_weights_load: %s has %llu elements, expected %llu", name, (unsigned long long)n_elements(x),
                 (unsigned long long)want);
            return false;
        }
        return (*dst = upload_f32(x)) != nullptr;
    };
    bool ok = bind("output_norm.weight", w->n_embd, true, &w->output_norm);
    char name[128];
    for (uint32_t l = 0; ok && l < n_layer; l++) {
        snprintf(name, sizeof name, "blk.%u.attn_norm.weight", l);
        ok = ok && bind(name, w->n_embd, true, &w->attn_norm[l]);
        snprintf(name, sizeof name, "blk.%u.attn_q_norm.weight", l);
        ok = ok && bind(name, 0, require_qk_norm, &w->attn_q_norm[l]);
        snprintf(name, sizeof name, "blk.%u.attn_k_norm.weight", l);
        ok = ok && bind(name, 0, require_qk_norm, &w->attn_k_norm[l]);
        snprintf(name, sizeof name, "blk.%u.ffn_norm.weight", l);
        ok = ok && bind(name, w->n_embd, true, &w->ffn_norm[l]);
        snprintf(name, sizeof name, "blk.%u.ffn_gate_inp.weight", l);
        ds3_cuda_gguf_tensor_t r;
        if (ok && ds3_cuda_gguf_find_tensor(g, name, &r) == 0) {
            if (r.n_dims != 2 || r.ne[0] != w->n_embd || (w->n_expert && r.ne[1] != w->n_expert)) {
                fail("path_weights_load: %s is not [n_expert][%u]", name, w->n_embd);
                ok = false;
            }
            w->n_expert = (uint32_t)r.ne[1];
        }
        ok = ok && bind(name, 0, true, &w->ffn_gate_inp[l]);
        if (ok && l == 0 && w->attn_q_norm[0]) {
            ds3_cuda_gguf_tensor_t q;
            snprintf(name, sizeof name, "blk.0.attn_q_norm.weight");
            ds3_cuda_gguf_find_tensor(g, name, &q);
            w->head_dim = (uint32_t)n_elements(q);
        }
    }
    if (!ok) {
        ds3_cuda_path_weights_free(w);
        return nullptr;
    }
    return w;
}

}  // extern "C"
