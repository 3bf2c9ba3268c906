// ds3_cuda.cu — the C-ABI of include/ds3_cuda.h: device/stream lifecycle,
// buffers, synchronous vs batched dispatch, graphs, timers, profiling, and
// host-side argument validation in front of every kernel launcher.
//
// Mirrors the behaviour of the Metal backend (src/ds3_metal.m of
// wzqhbustb/qw3): 0/-1 returns with a message on stderr, NULL from failed
// allocators, synchronous ops outside a batch (ds3_metal.m:534-541), enqueue
// only inside begin_batch/end_batch (:2847-2889), nested begin refused
// (:2849-2852), read-only buffers refuse writes (:439), views share the
// parent allocation (:416-435).
#include "ds3_cuda.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "launch.h"

struct ds3_cuda_buffer {
    char *base;      // start of the underlying allocation (or wrapped region)
    size_t bytes;    // size of this buffer / view
    size_t offset;   // byte offset of this view inside `base`
    bool read_only;  // from_mmap copies
    bool owns;       // true only for ds3_cuda_buffer_alloc / from_mmap results
};

struct ds3_cuda_graph {
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

namespace {

struct ProfileRec {
    const char *op;
    cudaEvent_t a, b;
};

struct State {
    bool inited = false;
    int device = 0;
    int n_sm = 148;
    cudaStream_t stream = nullptr;
    cudaStream_t lanes[2] = {nullptr, nullptr};  // copy lanes 1 and 2 (lane 0 is `stream`)
    unsigned *err_host = nullptr;  // pinned + mapped; kErrSlots words
    unsigned *err_dev = nullptr;
    bool batch = false;
    bool capturing = false;
    bool profile = false;
    bool pdl = true;  // DS3_CUDA_PDL=0 disables programmatic dependent launch
    // Library-owned device workspace: the fp32 copy of a router matrix stored
    // in another type (moe_ffn_router*). Earlier, smaller allocations stay
    // alive until shutdown: graphs captured before a growth still use them.
    float *ws = nullptr;
    size_t ws_bytes = 0;
    std::vector<void *> ws_old;
    std::vector<cudaEvent_t> timers;
    std::vector<cudaEvent_t> event_pool;
    std::vector<ProfileRec> prof;
};

State G;
thread_local std::string g_last_error;

void set_error(const char *fmt, ...)
{
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    g_last_error = msg;
    fprintf(stderr, "ds3_cuda: %s\n", msg);
}

bool deferred() { return G.batch || G.capturing; }

ds3::LaunchCtx ctx() { return ds3::LaunchCtx{G.stream, G.err_dev, G.n_sm, G.pdl}; }

void *dptr(const ds3_cuda_buffer_t *b) { return b ? (void *)(b->base + b->offset) : nullptr; }

bool need(const char *op, const char *name, const ds3_cuda_buffer_t *b, size_t bytes)
{
    if (!b) {
        set_error("%s: %s is NULL", op, name);
        return false;
    }
    if (b->bytes < bytes) {
        set_error("%s: %s holds %zu bytes, needs %zu", op, name, b->bytes, bytes);
        return false;
    }
    return true;
}

bool writable(const char *op, const char *name, const ds3_cuda_buffer_t *b)
{
    if (b && b->read_only) {
        set_error("%s: %s is read-only", op, name);
        return false;
    }
    return true;
}

bool ready(const char *op)
{
    if (!G.inited) {
        set_error("%s: backend not initialised (call ds3_cuda_init)", op);
        return false;
    }
    return true;
}

uint32_t take_device_errors()
{
    uint32_t bits = 0;
    for (int i = 0; i < ds3::kErrSlots; i++) {
        if (((volatile unsigned *)G.err_host)[i]) bits |= 1u << i;
        ((volatile unsigned *)G.err_host)[i] = 0;
    }
    return bits;
}

// Waits for the stream, then reports launch/async errors and device error bits.
int sync_and_check(const char *op)
{
    cudaError_t e = cudaStreamSynchronize(G.stream);
    for (cudaStream_t l : G.lanes)
        if (e == cudaSuccess && l) e = cudaStreamSynchronize(l);
    if (e != cudaSuccess) {
        set_error("%s: %s", op, cudaGetErrorString(e));
        return -1;
    }
    const uint32_t bits = take_device_errors();
    if (bits) {
        set_error("%s: device reported%s%s", op, (bits & 1u) ? " token/row id out of range" : "",
                  (bits & 2u) ? " bounded wait timed out" : "");
        return -1;
    }
    return 0;
}

cudaEvent_t pool_event()
{
    if (!G.event_pool.empty()) {
        cudaEvent_t e = G.event_pool.back();
        G.event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Profiling bracket around one launch (not while capturing a graph).
struct ProfScope {
    const char *op;
    cudaEvent_t a = nullptr;
    explicit ProfScope(const char *o) : op(o)
    {
        if (G.profile && !G.capturing) {
            a = pool_event();
            cudaEventRecord(a, G.stream);
        }
    }
    void close()
    {
        if (!a) return;
        cudaEvent_t b = pool_event();
        cudaEventRecord(b, G.stream);
        G.prof.push_back({op, a, b});
        a = nullptr;
    }
};

// Common tail of every op: launch status, then (outside a batch) wait + checks.
int finish(const char *op, cudaError_t launch, ProfScope &ps)
{
    ps.close();
    if (launch != cudaSuccess) {
        set_error("%s: launch failed: %s", op, cudaGetErrorString(launch));
        return -1;
    }
    if (deferred()) return 0;
    return sync_and_check(op);
}

// At least `bytes` of library workspace, or nullptr (error set). It only
// grows outside a graph capture (an allocation cannot be captured).
float *workspace(const char *op, size_t bytes)
{
    if (G.ws_bytes >= bytes) return G.ws;
    if (G.capturing) {
        set_error("%s: the library workspace needs %zu bytes; make this call once outside a graph capture first",
                  op, bytes);
        return nullptr;
    }
    void *p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        set_error("%s: workspace of %zu bytes: %s", op, bytes, cudaGetErrorString(e));
        return nullptr;
    }
    if (G.ws) G.ws_old.push_back(G.ws);
    G.ws = (float *)p;
    G.ws_bytes = bytes;
    return G.ws;
}

int rope_freqs(uint32_t head_dim, float theta, float *freq)
{
    // ds3_reference.c:369-377: freq_i = powf(theta, (float)i * (-2.0f / head_dim)).
    const float step = -2.0f / (float)head_dim;
    for (uint32_t i = 0; i < head_dim / 2; i++) freq[i] = powf(theta, (float)i * step);
    return 0;
}

}  // namespace

namespace ds3 {
constexpr int kMaxPrepared = 256;
const void *g_prepared[kMaxPrepared];  // kernels already set up
int g_n_prepared = 0;

// Every kernel launched through launch_k asks for the same L1/shared split.
// Consecutive kernels with different splits cannot share an SM (it must
// drain to switch), which defeats programmatic dependent launch; one split
// for all lets the next kernel's CTAs become resident while the previous
// kernel finishes. 50 % measured best on the T=512 step (34.1 us vs 35.4 us
// with the driver's per-kernel choice; 45-55 % alike, 60 % slows the RoPE
// kernel, 40 % and below starve the TMA-staged norm). DS3_CUDA_CARVEOUT
// overrides it (-1 leaves the driver's choice).
void prepare_kernel(const void *k)
{
    static const int carve = [] {
        const char *v = getenv("DS3_CUDA_CARVEOUT");
        return v ? atoi(v) : 50;
    }();
    if (carve < 0) return;
    for (int i = 0; i < g_n_prepared; i++)
        if (g_prepared[i] == k) return;
    cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, carve);
    if (g_n_prepared < kMaxPrepared) g_prepared[g_n_prepared++] = k;
}

void keep_driver_carveout(const void *k)
{
    for (int i = 0; i < g_n_prepared; i++)
        if (g_prepared[i] == k) return;
    if (g_n_prepared < kMaxPrepared) g_prepared[g_n_prepared++] = k;
}

// Shared with the other host modules of the library (gguf.cpp).
void report_error(const char *msg)
{
    g_last_error = msg;
    fprintf(stderr, "ds3_cuda: %s\n", msg);
}
}  // namespace ds3

extern "C" {

// ------------------------------------------------------------------ lifecycle
int ds3_cuda_set_device(int device)
{
    if (G.inited) {
        set_error("set_device: call before ds3_cuda_init");
        return -1;
    }
    G.device = device;
    return 0;
}

int ds3_cuda_init(void)
{
    if (G.inited) return 0;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        set_error("init: no CUDA device (%s)", e != cudaSuccess ? cudaGetErrorString(e) : "count 0");
        cudaGetLastError();
        return -1;
    }
    if (G.device < 0 || G.device >= n) {
        set_error("init: device %d out of range [0,%d)", G.device, n);
        return -1;
    }
    if ((e = cudaSetDevice(G.device)) != cudaSuccess) {
        set_error("init: cudaSetDevice: %s", cudaGetErrorString(e));
        return -1;
    }
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, G.device);
    if (prop.major != 10) {
        set_error("init: device %d is sm_%d%d; this build targets sm_100a (B200)", G.device, prop.major,
                  prop.minor);
        return -1;
    }
    G.n_sm = prop.multiProcessorCount;
    if ((e = cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking)) != cudaSuccess) {
        set_error("init: stream: %s", cudaGetErrorString(e));
        return -1;
    }
    for (cudaStream_t &l : G.lanes)
        if ((e = cudaStreamCreateWithFlags(&l, cudaStreamNonBlocking)) != cudaSuccess) {
            set_error("init: copy lane: %s", cudaGetErrorString(e));
            return -1;
        }
    if ((e = cudaHostAlloc((void **)&G.err_host, ds3::kErrSlots * sizeof(unsigned), cudaHostAllocMapped)) !=
        cudaSuccess) {
        set_error("init: error word: %s", cudaGetErrorString(e));
        return -1;
    }
    memset(G.err_host, 0, ds3::kErrSlots * sizeof(unsigned));
    cudaHostGetDevicePointer((void **)&G.err_dev, G.err_host, 0);
    G.timers.assign(DS3_CUDA_TIMER_SLOTS, nullptr);
    const char *p = getenv("DS3_CUDA_PROFILE");
    G.profile = p && p[0] == '1';
    const char *q = getenv("DS3_CUDA_PDL");
    G.pdl = !(q && q[0] == '0');
    G.inited = true;
    return 0;
}

void ds3_cuda_shutdown(void)
{
    if (!G.inited) return;
    cudaStreamSynchronize(G.stream);
    for (auto &r : G.prof) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    G.prof.clear();
    for (auto e : G.event_pool) cudaEventDestroy(e);
    G.event_pool.clear();
    for (auto e : G.timers)
        if (e) cudaEventDestroy(e);
    G.timers.clear();
    if (G.ws) cudaFree(G.ws);
    for (void *p : G.ws_old) cudaFree(p);
    for (cudaStream_t l : G.lanes)
        if (l) {
            cudaStreamSynchronize(l);
            cudaStreamDestroy(l);
        }
    cudaFreeHost(G.err_host);
    cudaStreamDestroy(G.stream);
    G = State();
}

// -------------------------------------------------------------------- buffers
ds3_cuda_buffer_t *ds3_cuda_buffer_alloc(size_t bytes)
{
    if (!ready("buffer_alloc") || bytes == 0) return nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        set_error("buffer_alloc(%zu): %s", bytes, cudaGetErrorString(e));
        return nullptr;
    }
    auto *b = (ds3_cuda_buffer_t *)calloc(1, sizeof(ds3_cuda_buffer_t));
    if (!b) {
        cudaFree(p);
        return nullptr;
    }
    b->base = (char *)p;
    b->bytes = bytes;
    b->owns = true;
    return b;
}

ds3_cuda_buffer_t *ds3_cuda_buffer_from_mmap(const void *base, size_t bytes)
{
    if (!base || bytes == 0) return nullptr;
    ds3_cuda_buffer_t *b = ds3_cuda_buffer_alloc(bytes);
    if (!b) return nullptr;
    cudaError_t e = cudaMemcpy(b->base, base, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        set_error("buffer_from_mmap: %s", cudaGetErrorString(e));
        ds3_cuda_buffer_free(b);
        return nullptr;
    }
    b->read_only = true;
    return b;
}

ds3_cuda_buffer_t *ds3_cuda_buffer_view(const ds3_cuda_buffer_t *base, size_t offset, size_t bytes)
{
    if (!base || offset > base->bytes || bytes == 0 || offset + bytes > base->bytes) return nullptr;
    auto *v = (ds3_cuda_buffer_t *)calloc(1, sizeof(ds3_cuda_buffer_t));
    if (!v) return nullptr;
    v->base = base->base;
    v->offset = base->offset + offset;
    v->bytes = bytes;
    v->read_only = base->read_only;
    v->owns = false;
    return v;
}

ds3_cuda_buffer_t *ds3_cuda_buffer_wrap(void *device_ptr, size_t bytes)
{
    if (!device_ptr || bytes == 0) return nullptr;
    auto *v = (ds3_cuda_buffer_t *)calloc(1, sizeof(ds3_cuda_buffer_t));
    if (!v) return nullptr;
    v->base = (char *)device_ptr;
    v->bytes = bytes;
    return v;
}

void ds3_cuda_buffer_free(ds3_cuda_buffer_t *buf)
{
    if (!buf) return;
    if (buf->owns && G.inited) cudaFree(buf->base);
    free(buf);
}

void *ds3_cuda_buffer_device_ptr(const ds3_cuda_buffer_t *buf) { return dptr(buf); }
size_t ds3_cuda_buffer_size(const ds3_cuda_buffer_t *buf) { return buf ? buf->bytes : 0; }

int ds3_cuda_buffer_write(ds3_cuda_buffer_t *buf, size_t offset, const void *src, size_t bytes)
{
    if (!ready("buffer_write")) return -1;
    if (!buf || !src || offset + bytes > buf->bytes || buf->read_only) {
        set_error("buffer_write: bad arguments (offset %zu + %zu, size %zu%s)", offset, bytes,
                  buf ? buf->bytes : 0, buf && buf->read_only ? ", read-only" : "");
        return -1;
    }
    if (G.capturing) {
        set_error("buffer_write: not allowed during graph capture");
        return -1;
    }
    cudaError_t e = cudaMemcpyAsync((char *)dptr(buf) + offset, src, bytes, cudaMemcpyHostToDevice, G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_write: %s", cudaGetErrorString(e));
        return -1;
    }
    e = cudaStreamSynchronize(G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_write: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int ds3_cuda_buffer_read(ds3_cuda_buffer_t *buf, size_t offset, void *dst, size_t bytes)
{
    if (!ready("buffer_read")) return -1;
    if (!buf || !dst || offset + bytes > buf->bytes) {
        set_error("buffer_read: bad arguments");
        return -1;
    }
    if (G.capturing) {
        set_error("buffer_read: not allowed during graph capture");
        return -1;
    }
    cudaError_t e = cudaMemcpyAsync(dst, (char *)dptr(buf) + offset, bytes, cudaMemcpyDeviceToHost, G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_read: %s", cudaGetErrorString(e));
        return -1;
    }
    e = cudaStreamSynchronize(G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_read: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int ds3_cuda_buffer_write_async(ds3_cuda_buffer_t *buf, size_t offset, const void *src, size_t bytes)
{
    if (!ready("buffer_write_async")) return -1;
    if (!buf || !src || offset + bytes > buf->bytes || buf->read_only) {
        set_error("buffer_write_async: bad arguments");
        return -1;
    }
    cudaError_t e = cudaMemcpyAsync((char *)dptr(buf) + offset, src, bytes, cudaMemcpyHostToDevice, G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_write_async: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int ds3_cuda_buffer_read_async(ds3_cuda_buffer_t *buf, size_t offset, void *dst, size_t bytes)
{
    if (!ready("buffer_read_async")) return -1;
    if (!buf || !dst || offset + bytes > buf->bytes) {
        set_error("buffer_read_async: bad arguments");
        return -1;
    }
    cudaError_t e = cudaMemcpyAsync(dst, (char *)dptr(buf) + offset, bytes, cudaMemcpyDeviceToHost, G.stream);
    if (e != cudaSuccess) {
        set_error("buffer_read_async: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// ------------------------------------------------------- ops (Metal mirror)
int ds3_cuda_rms_norm(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *weight, ds3_cuda_buffer_t *out,
                      uint32_t n, uint32_t n_rows, float eps)
{
    const char *op = "rms_norm";
    if (!ready(op)) return -1;
    const size_t rb = (size_t)n * n_rows * sizeof(float);
    if (n == 0 || !need(op, "x", x, rb) || !need(op, "weight", weight, n * sizeof(float)) ||
        !need(op, "out", out, rb) || !writable(op, "out", out))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_add_rms_norm(ctx(), (const float *)dptr(x), nullptr, (const float *)dptr(weight),
                                           nullptr, (float *)dptr(out), (int)n, n_rows, eps),
                  ps);
}

int ds3_cuda_rope(const ds3_cuda_buffer_t *src, ds3_cuda_buffer_t *dst, const ds3_cuda_buffer_t *positions,
                  uint32_t n_heads, uint32_t head_dim, uint32_t n_rows, float theta_base)
{
    const char *op = "rope";
    if (!ready(op)) return -1;
    if (head_dim == 0 || head_dim % 2 || head_dim > 512) {
        set_error("%s: head_dim %u must be even and <= 512", op, head_dim);
        return -1;
    }
    const size_t rb = (size_t)n_rows * n_heads * head_dim * sizeof(float);
    if (!need(op, "src", src, rb) || !need(op, "dst", dst, rb) || !writable(op, "dst", dst) ||
        !need(op, "positions", positions, (size_t)n_rows * 4))
        return -1;
    float freq[256];
    rope_freqs(head_dim, theta_base, freq);
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_qk_norm_rope(ctx(), dptr(src), dptr(dst), nullptr, nullptr, nullptr, nullptr,
                                           (const int32_t *)dptr(positions), n_rows, (int)n_heads, 0,
                                           (int)head_dim, freq, 0.0f, 0, 0),
                  ps);
}

int ds3_cuda_buffer_copy_f32(const ds3_cuda_buffer_t *src, ds3_cuda_buffer_t *dst, size_t bytes)
{
    const char *op = "buffer_copy_f32";
    if (!ready(op)) return -1;
    if (bytes % 4 || !need(op, "src", src, bytes) || !need(op, "dst", dst, bytes) || !writable(op, "dst", dst))
        return -1;
    ProfScope ps(op);
    return finish(op, cudaMemcpyAsync(dptr(dst), dptr(src), bytes, cudaMemcpyDeviceToDevice, G.stream), ps);
}

int ds3_cuda_buffer_zero_f32(ds3_cuda_buffer_t *buf, size_t bytes)
{
    const char *op = "buffer_zero_f32";
    if (!ready(op)) return -1;
    if (bytes % 4 || !need(op, "buf", buf, bytes) || !writable(op, "buf", buf)) return -1;
    ProfScope ps(op);
    return finish(op, cudaMemsetAsync(dptr(buf), 0, bytes, G.stream), ps);
}

int ds3_cuda_vec_add_inplace(ds3_cuda_buffer_t *acc, const ds3_cuda_buffer_t *addend, uint32_t n)
{
    const char *op = "vec_add_inplace";
    if (!ready(op)) return -1;
    const size_t b = (size_t)n * 4;
    if (!need(op, "acc", acc, b) || !need(op, "addend", addend, b) || !writable(op, "acc", acc)) return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_vec_add(ctx(), (const float *)dptr(acc), (const float *)dptr(addend),
                                      (float *)dptr(acc), n),
                  ps);
}

int ds3_cuda_vec_add(const ds3_cuda_buffer_t *a, const ds3_cuda_buffer_t *b, ds3_cuda_buffer_t *c, uint32_t n)
{
    const char *op = "vec_add";
    if (!ready(op)) return -1;
    const size_t nb = (size_t)n * 4;
    if (!need(op, "a", a, nb) || !need(op, "b", b, nb) || !need(op, "c", c, nb) || !writable(op, "c", c))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_vec_add(ctx(), (const float *)dptr(a), (const float *)dptr(b), (float *)dptr(c), n),
                  ps);
}

int ds3_cuda_gather_rows_f32(const ds3_cuda_buffer_t *src, const ds3_cuda_buffer_t *ids, ds3_cuda_buffer_t *dst,
                             uint32_t n_cols, uint32_t count, uint32_t offset)
{
    const char *op = "gather_rows_f32";
    if (!ready(op)) return -1;
    const size_t row = (size_t)n_cols * 4;
    if (n_cols == 0 || !need(op, "src", src, row) || !need(op, "ids", ids, ((size_t)offset + count) * 4) ||
        !need(op, "dst", dst, row * count) || !writable(op, "dst", dst))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_gather_rows(ctx(), (const float *)dptr(src), (const int32_t *)dptr(ids) + offset,
                                          (float *)dptr(dst), n_cols, count, (int64_t)(src->bytes / row)),
                  ps);
}

int ds3_cuda_scatter_add_weighted_f32(const ds3_cuda_buffer_t *src, const ds3_cuda_buffer_t *scores,
                                      const ds3_cuda_buffer_t *ids, ds3_cuda_buffer_t *dst, uint32_t n_cols,
                                      uint32_t count, uint32_t offset)
{
    const char *op = "scatter_add_weighted_f32";
    if (!ready(op)) return -1;
    const size_t row = (size_t)n_cols * 4;
    const size_t tbl = ((size_t)offset + count) * 4;
    if (n_cols == 0 || !need(op, "src", src, row * count) || !need(op, "scores", scores, tbl) ||
        !need(op, "ids", ids, tbl) || !need(op, "dst", dst, row) || !writable(op, "dst", dst))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_scatter_add_weighted(ctx(), (const float *)dptr(src), (const float *)dptr(scores) + offset,
                                                   (const int32_t *)dptr(ids) + offset, (float *)dptr(dst), n_cols,
                                                   count, (int64_t)(dst->bytes / row)),
                  ps);
}

int ds3_cuda_silu_mul_f32(const ds3_cuda_buffer_t *gate, const ds3_cuda_buffer_t *up, ds3_cuda_buffer_t *out,
                          uint32_t n)
{
    const char *op = "silu_mul_f32";
    if (!ready(op)) return -1;
    const size_t b = (size_t)n * 4;
    if (!need(op, "gate", gate, b) || !need(op, "up", up, b) || !need(op, "out", out, b) ||
        !writable(op, "out", out))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_swiglu(ctx(), (const float *)dptr(gate), (const float *)dptr(up), nullptr,
                                     (float *)dptr(out), 1, n),
                  ps);
}

static int router_common(const char *op, const ds3_cuda_buffer_t *logits, ds3_cuda_buffer_t *probs,
                         ds3_cuda_buffer_t *indices, ds3_cuda_buffer_t *scores, uint64_t rows, uint32_t n_expert,
                         uint32_t n_used, bool norm)
{
    if (!ready(op)) return -1;
    if (n_expert == 0 || n_used == 0 || n_used > n_expert || n_used > 64) {
        set_error("%s: need 0 < n_used (%u) <= min(n_expert (%u), 64)", op, n_used, n_expert);
        return -1;
    }
    const size_t lb = rows * n_expert * 4, ob = rows * n_used * 4;
    if (!need(op, "logits", logits, lb) || !need(op, "indices", indices, ob) || !need(op, "scores", scores, ob) ||
        !writable(op, "indices", indices) || !writable(op, "scores", scores) ||
        (probs && (!need(op, "probs", probs, lb) || !writable(op, "probs", probs))))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_router_topk(ctx(), (const float *)dptr(logits), (float *)dptr(probs),
                                          (int32_t *)dptr(indices), (float *)dptr(scores), (int64_t)rows,
                                          (int)n_expert, (int)n_used, norm ? 1 : 0),
                  ps);
}

int ds3_cuda_moe_router_topk_batch(const ds3_cuda_buffer_t *logits, ds3_cuda_buffer_t *indices,
                                   ds3_cuda_buffer_t *scores, uint32_t n_layers, uint32_t n_expert, uint32_t n_used,
                                   bool norm_topk_prob)
{
    return router_common("moe_router_topk_batch", logits, nullptr, indices, scores, n_layers, n_expert, n_used,
                         norm_topk_prob);
}

int ds3_cuda_moe_router_topk_batch_tokens(const ds3_cuda_buffer_t *logits, ds3_cuda_buffer_t *indices,
                                          ds3_cuda_buffer_t *scores, uint32_t n_layers, uint32_t n_tokens,
                                          uint32_t n_expert, uint32_t n_used, bool norm_topk_prob)
{
    return router_common("moe_router_topk_batch_tokens", logits, nullptr, indices, scores,
                         (uint64_t)n_layers * n_tokens, n_expert, n_used, norm_topk_prob);
}

// ------------------------------------------------------------ batch / profile
int ds3_cuda_begin_batch(void)
{
    if (!ready("begin_batch")) return -1;
    if (G.batch) {
        set_error("begin_batch: a batch is already open");
        return -1;
    }
    G.batch = true;
    return 0;
}

int ds3_cuda_end_batch(void)
{
    if (!G.inited) return -1;
    G.batch = false;
    if (G.capturing) return 0;
    return sync_and_check("end_batch");
}

void ds3_cuda_synchronize(void)
{
    if (G.inited && !G.capturing) sync_and_check("synchronize");
}

void ds3_cuda_profile_enable(int on) { G.profile = on != 0; }

void ds3_cuda_profile_reset(void)
{
    if (!G.inited) return;
    cudaStreamSynchronize(G.stream);
    for (auto &r : G.prof) {
        G.event_pool.push_back(r.a);
        G.event_pool.push_back(r.b);
    }
    G.prof.clear();
}

void ds3_cuda_profile_print(const char *label)
{
    if (!G.inited || !G.profile) return;
    cudaStreamSynchronize(G.stream);
    std::map<std::string, std::pair<int, double>> acc;
    double total = 0.0;
    for (auto &r : G.prof) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
            auto &s = acc[r.op];
            s.first++;
            s.second += ms;
            total += ms;
        }
    }
    fprintf(stderr, "[ds3_cuda profile] %s: launches=%zu gpu_ms=%.3f\n", label ? label : "", G.prof.size(), total);
    for (auto &kv : acc)
        fprintf(stderr, "  %-28s n=%-6d gpu_ms=%.3f\n", kv.first.c_str(), kv.second.first, kv.second.second);
}

// ----------------------------------------------------------------- fused ops
int ds3_cuda_embed_rows(const ds3_cuda_buffer_t *table, const ds3_cuda_buffer_t *ids, ds3_cuda_buffer_t *out,
                        uint32_t n_ids, uint32_t n_cols, uint32_t n_vocab, ds3_type_t type, uint64_t row_stride)
{
    return ds3_cuda_embed_rms_norm(table, ids, nullptr, out, nullptr, n_ids, n_cols, n_vocab, type, row_stride,
                                   0.0f);
}

static bool type_row_bytes(ds3_type_t type, uint32_t n_cols, uint64_t *bytes)
{
    switch ((int)type) {
    case 0: *bytes = (uint64_t)n_cols * 4; return true;
    case 1: *bytes = (uint64_t)n_cols * 2; return true;
    case 8: if (n_cols % 32) return false; *bytes = (uint64_t)n_cols / 32 * 34; return true;
    case 12: if (n_cols % 256) return false; *bytes = (uint64_t)n_cols / 256 * 144; return true;
    case 14: if (n_cols % 256) return false; *bytes = (uint64_t)n_cols / 256 * 210; return true;
    default: return false;
    }
}

int ds3_cuda_dequantize_f32(const ds3_cuda_buffer_t *src, ds3_type_t type, uint64_t n_elements, ds3_cuda_buffer_t *dst)
{
    const char *op = "dequantize_f32";
    if (!ready(op)) return -1;
    uint64_t rb = 0;
    const uint32_t n = (uint32_t)n_elements;
    if (n_elements == 0 || n_elements >= (1ull << 31) || !type_row_bytes(type, n, &rb)) {
        set_error("%s: unsupported type %d or element count %llu", op, (int)type, (unsigned long long)n_elements);
        return -1;
    }
    if (!need(op, "src", src, (size_t)rb) || !need(op, "dst", dst, (size_t)n_elements * 4) ||
        !writable(op, "dst", dst))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_dequantize(ctx(), (const uint8_t *)dptr(src), (int)type, (int64_t)n_elements,
                                         (float *)dptr(dst)),
                  ps);
}

int ds3_cuda_embed_rms_norm(const ds3_cuda_buffer_t *table, const ds3_cuda_buffer_t *ids,
                            const ds3_cuda_buffer_t *weight, ds3_cuda_buffer_t *hidden_out,
                            ds3_cuda_buffer_t *norm_out, uint32_t n_ids, uint32_t n_cols, uint32_t n_vocab,
                            ds3_type_t type, uint64_t row_stride, float eps)
{
    const char *op = norm_out ? "embed_rms_norm" : "embed_rows";
    if (!ready(op)) return -1;
    uint64_t rb = 0;
    if (n_cols == 0 || !type_row_bytes(type, n_cols, &rb)) {
        set_error("%s: unsupported type %d or n_cols %u", op, (int)type, n_cols);
        return -1;
    }
    if (row_stride < rb) {
        set_error("%s: row_stride %llu < row bytes %llu", op, (unsigned long long)row_stride,
                  (unsigned long long)rb);
        return -1;
    }
    if (n_vocab == 0 || !need(op, "table", table, (size_t)(row_stride * (n_vocab - 1) + rb))) return -1;
    const size_t ob = (size_t)n_ids * n_cols * 4;
    if (!need(op, "ids", ids, (size_t)n_ids * 4)) return -1;
    if (!hidden_out && !norm_out) {
        set_error("%s: no output buffer", op);
        return -1;
    }
    if (hidden_out && (!need(op, "hidden_out", hidden_out, ob) || !writable(op, "hidden_out", hidden_out)))
        return -1;
    if (norm_out && (!need(op, "norm_out", norm_out, ob) || !writable(op, "norm_out", norm_out) ||
                     !need(op, "weight", weight, (size_t)n_cols * 4)))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_embed(ctx(), (const uint8_t *)dptr(table), (int)type, row_stride, n_vocab,
                                    (const int32_t *)dptr(ids), n_ids, (int)n_cols, (float *)dptr(hidden_out),
                                    (const float *)dptr(weight), (float *)dptr(norm_out), eps),
                  ps);
}

int ds3_cuda_add_rms_norm(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *residual,
                          const ds3_cuda_buffer_t *weight, ds3_cuda_buffer_t *sum_out, ds3_cuda_buffer_t *norm_out,
                          uint32_t n, uint32_t n_rows, float eps)
{
    const char *op = "add_rms_norm";
    if (!ready(op)) return -1;
    const size_t rb = (size_t)n * n_rows * 4;
    if (n == 0 || !need(op, "x", x, rb) || !need(op, "residual", residual, rb) ||
        !need(op, "weight", weight, (size_t)n * 4) || !need(op, "norm_out", norm_out, rb) ||
        !writable(op, "norm_out", norm_out) ||
        (sum_out && (!need(op, "sum_out", sum_out, rb) || !writable(op, "sum_out", sum_out))))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_add_rms_norm(ctx(), (const float *)dptr(x), (const float *)dptr(residual),
                                           (const float *)dptr(weight), (float *)dptr(sum_out),
                                           (float *)dptr(norm_out), (int)n, n_rows, eps),
                  ps);
}

int ds3_cuda_qk_norm_rope(ds3_cuda_buffer_t *q, ds3_cuda_buffer_t *k, const ds3_cuda_buffer_t *q_w,
                          const ds3_cuda_buffer_t *k_w, const ds3_cuda_buffer_t *positions, uint32_t n_rows,
                          uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim, float theta_base, float eps,
                          ds3_type_t storage)
{
    const char *op = "qk_norm_rope";
    if (!ready(op)) return -1;
    if ((int)storage != 0 && (int)storage != 1) {
        set_error("%s: storage must be DS3_TYPE_F32 or DS3_TYPE_F16", op);
        return -1;
    }
    if (head_dim == 0 || head_dim % 2 || head_dim > 512) {
        set_error("%s: head_dim %u must be even and <= 512", op, head_dim);
        return -1;
    }
    const size_t es = (int)storage == 1 ? 2 : 4;
    const size_t qb = (size_t)n_rows * n_q_heads * head_dim * es;
    const size_t kb = (size_t)n_rows * n_kv_heads * head_dim * es;
    if (!need(op, "q", q, qb) || !writable(op, "q", q) || !need(op, "q_w", q_w, (size_t)head_dim * 4) ||
        !need(op, "positions", positions, (size_t)n_rows * 4))
        return -1;
    if (n_kv_heads && (!need(op, "k", k, kb) || !writable(op, "k", k) || !need(op, "k_w", k_w, (size_t)head_dim * 4)))
        return -1;
    float freq[256];
    rope_freqs(head_dim, theta_base, freq);
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_qk_norm_rope(ctx(), dptr(q), dptr(q), dptr(k), dptr(k), (const float *)dptr(q_w),
                                           (const float *)dptr(k_w), (const int32_t *)dptr(positions), n_rows,
                                           (int)n_q_heads, (int)n_kv_heads, (int)head_dim, freq, eps, 1,
                                           (int)storage),
                  ps);
}

int ds3_cuda_qk_norm_rope_kv(ds3_cuda_buffer_t *q, ds3_cuda_buffer_t *k, const ds3_cuda_buffer_t *v,
                             const ds3_cuda_buffer_t *q_w, const ds3_cuda_buffer_t *k_w,
                             const ds3_cuda_buffer_t *positions, ds3_cuda_buffer_t *k_cache,
                             ds3_cuda_buffer_t *v_cache, uint32_t n_rows, uint32_t n_q_heads, uint32_t n_kv_heads,
                             uint32_t head_dim, uint32_t max_seq_len, float theta_base, float eps, ds3_type_t storage)
{
    const char *op = "qk_norm_rope_kv";
    if (!ready(op)) return -1;
    if ((int)storage != 0 && (int)storage != 1) {
        set_error("%s: storage must be DS3_TYPE_F32 or DS3_TYPE_F16", op);
        return -1;
    }
    if (head_dim != 128 || n_kv_heads == 0 || max_seq_len == 0) {
        set_error("%s: needs head_dim 128 (got %u), n_kv_heads > 0, max_seq_len > 0", op, head_dim);
        return -1;
    }
    const size_t es = (int)storage == 1 ? 2 : 4;
    const size_t qb = (size_t)n_rows * n_q_heads * 128 * es, kb = (size_t)n_rows * n_kv_heads * 128 * es;
    const size_t cb = (size_t)max_seq_len * n_kv_heads * 128 * 2;
    if (!need(op, "q", q, qb) || !writable(op, "q", q) || !need(op, "k", k, kb) || !writable(op, "k", k) ||
        !need(op, "v", v, kb) || !need(op, "q_w", q_w, 512) || !need(op, "k_w", k_w, 512) ||
        !need(op, "positions", positions, (size_t)n_rows * 4) || !need(op, "k_cache", k_cache, cb) ||
        !writable(op, "k_cache", k_cache) || !need(op, "v_cache", v_cache, cb) || !writable(op, "v_cache", v_cache))
        return -1;
    float freq[256];
    rope_freqs(head_dim, theta_base, freq);
    ProfScope ps(op);
    const cudaError_t e = ds3::launch_qk_norm_rope_kv(
        ctx(), dptr(q), dptr(k), dptr(v), (const float *)dptr(q_w), (const float *)dptr(k_w),
        (const int32_t *)dptr(positions), n_rows, (int)n_q_heads, (int)n_kv_heads, freq, eps, (int)storage,
        dptr(k_cache), dptr(v_cache), (int)max_seq_len);
    if (e == cudaErrorInvalidValue) {
        set_error("%s: buffers must be 16-byte aligned and n_q_heads + 2*n_kv_heads <= 40", op);
        ps.close();
        return -1;
    }
    return finish(op, e, ps);
}

int ds3_cuda_kv_cache_write_batch(const ds3_cuda_buffer_t *k, const ds3_cuda_buffer_t *v, ds3_cuda_buffer_t *k_cache,
                                  ds3_cuda_buffer_t *v_cache, uint32_t seq_pos, uint32_t n_tokens,
                                  uint32_t max_seq_len, uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim)
{
    const char *op = "kv_cache_write_batch";
    (void)n_q_heads;
    if (!ready(op)) return -1;
    if (n_tokens == 0) return 0;
    if ((uint64_t)seq_pos + n_tokens > max_seq_len) {
        set_error("%s: seq_pos=%u n_tokens=%u exceeds max_seq_len=%u", op, seq_pos, n_tokens, max_seq_len);
        return -1;
    }
    const size_t row = (size_t)n_kv_heads * head_dim;
    const size_t cb = (size_t)max_seq_len * row * 2;
    if (row == 0 || !need(op, "k", k, n_tokens * row * 4) || !need(op, "v", v, n_tokens * row * 4) ||
        !need(op, "k_cache", k_cache, cb) || !writable(op, "k_cache", k_cache) || !need(op, "v_cache", v_cache, cb) ||
        !writable(op, "v_cache", v_cache))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_kv_cache_write(ctx(), (const float *)dptr(k), (const float *)dptr(v), dptr(k_cache),
                                             dptr(v_cache), seq_pos, n_tokens, (int64_t)row),
                  ps);
}

int ds3_cuda_router_softmax_topk(const ds3_cuda_buffer_t *logits, ds3_cuda_buffer_t *probs_out,
                                 ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores, uint32_t n_tokens,
                                 uint32_t n_expert, uint32_t n_used, bool norm_topk_prob)
{
    return router_common("router_softmax_topk", logits, probs_out, idx, scores, n_tokens, n_expert, n_used,
                         norm_topk_prob);
}

int ds3_cuda_router_logits_topk(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *w_router,
                                ds3_cuda_buffer_t *logits_out, ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores,
                                uint32_t n_tokens, uint32_t n_embd, uint32_t n_expert, uint32_t n_used,
                                bool norm_topk_prob)
{
    const char *op = "router_logits_topk";
    if (!ready(op)) return -1;
    if (n_embd == 0 || n_expert == 0 || n_used == 0 || n_used > n_expert || n_used > 64) {
        set_error("%s: need n_embd > 0 and 0 < n_used <= min(n_expert, 64)", op);
        return -1;
    }
    const size_t ob = (size_t)n_tokens * n_used * 4;
    if (!need(op, "x", x, (size_t)n_tokens * n_embd * 4) || !need(op, "w_router", w_router, (size_t)n_expert * n_embd * 4) ||
        !need(op, "idx", idx, ob) || !writable(op, "idx", idx) || !need(op, "scores", scores, ob) ||
        !writable(op, "scores", scores) ||
        (logits_out && (!need(op, "logits_out", logits_out, (size_t)n_tokens * n_expert * 4) ||
                        !writable(op, "logits_out", logits_out))))
        return -1;
    if (!logits_out && !ds3::router_gemv_fast(n_tokens, (int)n_embd, (int)n_expert, (int)n_used, dptr(x), dptr(w_router))) {
        set_error("%s: logits_out is required for this shape (fast path: n_expert 128, n_embd %% 64 == 0)", op);
        return -1;
    }
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_router_gemv_topk(ctx(), (const float *)dptr(x), (const float *)dptr(w_router),
                                               (float *)dptr(logits_out), (int32_t *)dptr(idx), (float *)dptr(scores),
                                               n_tokens, (int)n_embd, (int)n_expert, (int)n_used,
                                               norm_topk_prob ? 1 : 0, true),
                  ps);
}

int ds3_cuda_add_rms_norm_router_topk(const ds3_cuda_buffer_t *x, const ds3_cuda_buffer_t *residual,
                                      const ds3_cuda_buffer_t *norm_weight, const ds3_cuda_buffer_t *w_router,
                                      ds3_cuda_buffer_t *sum_out, ds3_cuda_buffer_t *norm_out,
                                      ds3_cuda_buffer_t *logits_out, ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores,
                                      uint32_t n_tokens, uint32_t n_embd, uint32_t n_expert, uint32_t n_used,
                                      float eps, bool norm_topk_prob)
{
    const char *op = "add_rms_norm_router_topk";
    if (!ready(op)) return -1;
    if (n_used == 0 || n_used > n_expert) {
        set_error("%s: need 0 < n_used (%u) <= n_expert (%u)", op, n_used, n_expert);
        return -1;
    }
    const size_t rb = (size_t)n_tokens * n_embd * 4, ob = (size_t)n_tokens * n_used * 4;
    if (!need(op, "x", x, rb) || !need(op, "residual", residual, rb) ||
        !need(op, "norm_weight", norm_weight, (size_t)n_embd * 4) ||
        !need(op, "w_router", w_router, (size_t)n_expert * n_embd * 4) || !need(op, "idx", idx, ob) ||
        !writable(op, "idx", idx) || !need(op, "scores", scores, ob) || !writable(op, "scores", scores) ||
        (sum_out && (!need(op, "sum_out", sum_out, rb) || !writable(op, "sum_out", sum_out))) ||
        (norm_out && (!need(op, "norm_out", norm_out, rb) || !writable(op, "norm_out", norm_out))) ||
        (logits_out && (!need(op, "logits_out", logits_out, (size_t)n_tokens * n_expert * 4) ||
                        !writable(op, "logits_out", logits_out))))
        return -1;
    if (n_tokens == 0) return 0;
    if (!ds3::add_norm_router_fast(n_tokens, (int)n_embd, (int)n_expert, (int)n_used, dptr(x), dptr(residual),
                                   dptr(w_router))) {
        set_error("%s: needs n_expert 128, n_used <= 32, n_embd a multiple of 128 up to 2048 and 16-byte aligned "
                  "rows (otherwise call add_rms_norm, then router_logits_topk)", op);
        return -1;
    }
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_add_norm_router_topk(ctx(), (const float *)dptr(x), (const float *)dptr(residual),
                                                   (const float *)dptr(norm_weight), (const float *)dptr(w_router),
                                                   (float *)dptr(sum_out), (float *)dptr(norm_out),
                                                   (float *)dptr(logits_out), (int32_t *)dptr(idx),
                                                   (float *)dptr(scores), n_tokens, (int)n_embd, (int)n_expert,
                                                   (int)n_used, norm_topk_prob ? 1 : 0, eps),
                  ps);
}

// Router projection with the weight in its stored type (F32, F16, Q8_0,
// Q4_K or Q6_K rows, `row_stride` bytes apart, as the GGUF holds them). A
// dense F32 matrix is used in place; any other is first converted to fp32 in
// the library workspace by the bit-exact row dequant, so the logits equal
// ds3_ref_vec_matmul over the reference's dequantised weights.
static int moe_router_typed(const char *op, const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w,
                            uint64_t row_stride, ds3_type_t type, ds3_cuda_buffer_t *logits, ds3_cuda_buffer_t *idx,
                            ds3_cuda_buffer_t *scores, uint32_t n_tokens, uint32_t n_embd, uint32_t n_expert,
                            uint32_t n_used, bool norm)
{
    if (!ready(op)) return -1;
    uint64_t rb = 0;
    if (n_embd == 0 || n_expert == 0 || !type_row_bytes(type, n_embd, &rb)) {
        set_error("%s: unsupported router type %d or n_embd %u", op, (int)type, n_embd);
        return -1;
    }
    if (row_stride < rb) {
        set_error("%s: router_row_stride %llu < row bytes %llu", op, (unsigned long long)row_stride,
                  (unsigned long long)rb);
        return -1;
    }
    if (idx && (n_used == 0 || n_used > n_expert || n_used > 64)) {
        set_error("%s: need 0 < n_used (%u) <= min(n_expert (%u), 64)", op, n_used, n_expert);
        return -1;
    }
    const size_t ob = (size_t)n_tokens * n_used * 4;
    if (!need(op, "input", input, (size_t)n_tokens * n_embd * 4) ||
        !need(op, "w_gate_inp", w, (size_t)(row_stride * (n_expert - 1) + rb)) ||
        (logits && (!need(op, "gate_logits", logits, (size_t)n_tokens * n_expert * 4) ||
                    !writable(op, "gate_logits", logits))) ||
        (idx && (!need(op, "idx", idx, ob) || !writable(op, "idx", idx) || !need(op, "scores", scores, ob) ||
                 !writable(op, "scores", scores))))
        return -1;
    if (!logits && !idx) {
        set_error("%s: no output buffer", op);
        return -1;
    }
    if (n_tokens == 0) return 0;
    const float *wf = (const float *)dptr(w);
    ProfScope ps(op);
    if ((int)type != 0 || row_stride != rb) {
        float *buf = workspace(op, (size_t)n_expert * n_embd * 4);
        if (!buf) {
            ps.close();
            return -1;
        }
        const cudaError_t e = ds3::launch_dequantize_rows(ctx(), (const uint8_t *)dptr(w), (int)type, row_stride,
                                                          n_expert, (int)n_embd, buf);
        if (e != cudaSuccess) return finish(op, e, ps);
        wf = buf;
    }
    if (!logits && !ds3::router_gemv_fast(n_tokens, (int)n_embd, (int)n_expert, (int)n_used, dptr(input), wf)) {
        set_error("%s: gate_logits is required for this shape (fast path: n_expert 128, n_embd %% 64 == 0)", op);
        ps.close();
        return -1;
    }
    return finish(op,
                  ds3::launch_router_gemv_topk(ctx(), (const float *)dptr(input), wf, (float *)dptr(logits),
                                               (int32_t *)dptr(idx), (float *)dptr(scores), n_tokens, (int)n_embd,
                                               (int)n_expert, (int)(idx ? n_used : 0), norm ? 1 : 0),
                  ps);
}

int ds3_cuda_moe_ffn_router(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                            ds3_cuda_buffer_t *gate_logits, uint32_t n_embd, uint32_t n_expert,
                            uint64_t router_row_stride, ds3_type_t router_type)
{
    return moe_router_typed("moe_ffn_router", input, w_gate_inp, router_row_stride, router_type, gate_logits,
                            nullptr, nullptr, 1, n_embd, n_expert, 0, false);
}

int ds3_cuda_moe_ffn_router_topk(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                                 uint64_t router_row_stride, ds3_type_t router_type, ds3_cuda_buffer_t *gate_logits,
                                 ds3_cuda_buffer_t *idx, ds3_cuda_buffer_t *scores, uint32_t n_tokens,
                                 uint32_t n_embd, uint32_t n_expert, uint32_t n_used, bool norm_topk_prob)
{
    const char *op = "moe_ffn_router_topk";
    if (!idx || !scores) {
        set_error("%s: idx and scores are required", op);
        return -1;
    }
    return moe_router_typed(op, input, w_gate_inp, router_row_stride, router_type, gate_logits, idx, scores,
                            n_tokens, n_embd, n_expert, n_used, norm_topk_prob);
}

// ---------------------------------------------- allocation-free router entry
// A router call for callers that cannot let this library allocate device
// memory: the fp32 copy of a stored router weight goes into a fixed scratch
// array that is part of the loaded library (a file-scope __device__ array),
// not into the workspace moe_ffn_router_topk allocates on first use. Every
// GPU that loads the library holds the array until the process exits.
static constexpr size_t kNoAllocRouterMaxElems = 524288;  // n_expert * n_embd; 2 MiB of fp32
static __device__ __align__(256) float g_noalloc_router_scratch[kNoAllocRouterMaxElems];

// Device address of the scratch array for the current device. The array's
// name in host code is only a host-side stand-in, never a device address, so
// the address is looked up once per device (with that device current) and
// cached; the lookup allocates nothing.
static float *noalloc_router_scratch(const char *op)
{
    constexpr int kMaxDevices = 64;
    static float *addr[kMaxDevices] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error("%s: no current device (%s)", op, e != cudaSuccess ? cudaGetErrorString(e) : "index out of range");
        return nullptr;
    }
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_router_scratch);
        if (e != cudaSuccess || !p) {
            set_error("%s: cudaGetSymbolAddress of the scratch array: %s", op, cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<float *>(p);
    }
    return addr[dev];
}

int ds3_cuda_moe_ffn_router_topk_noalloc(const ds3_cuda_buffer_t *input, const ds3_cuda_buffer_t *w_gate_inp,
                                         uint64_t router_row_stride, ds3_type_t router_type,
                                         ds3_cuda_buffer_t *gate_logits, ds3_cuda_buffer_t *idx,
                                         ds3_cuda_buffer_t *scores, uint32_t n_tokens, uint32_t n_embd,
                                         uint32_t n_expert, uint32_t n_used, bool norm_topk_prob)
{
    const char *op = "moe_ffn_router_topk_noalloc";
    if (!ready(op)) return -1;
    uint64_t rb = 0;
    if (n_embd == 0 || n_expert == 0 || !type_row_bytes(router_type, n_embd, &rb)) {
        set_error("%s: unsupported router type %d or n_embd %u", op, (int)router_type, n_embd);
        return -1;
    }
    if ((uint64_t)n_expert * n_embd > kNoAllocRouterMaxElems) {
        set_error("%s: n_expert * n_embd = %llu exceeds the fixed scratch of %zu elements; use "
                  "ds3_cuda_moe_ffn_router_topk",
                  op, (unsigned long long)n_expert * n_embd, kNoAllocRouterMaxElems);
        return -1;
    }
    if (router_row_stride < rb) {
        set_error("%s: router_row_stride %llu < row bytes %llu", op, (unsigned long long)router_row_stride,
                  (unsigned long long)rb);
        return -1;
    }
    if (!idx || !scores || n_used == 0 || n_used > n_expert || n_used > 64) {
        set_error("%s: need idx, scores and 0 < n_used (%u) <= min(n_expert (%u), 64)", op, n_used, n_expert);
        return -1;
    }
    const size_t ob = (size_t)n_tokens * n_used * 4;
    if (!need(op, "input", input, (size_t)n_tokens * n_embd * 4) ||
        !need(op, "w_gate_inp", w_gate_inp, (size_t)(router_row_stride * (n_expert - 1) + rb)) ||
        (gate_logits && (!need(op, "gate_logits", gate_logits, (size_t)n_tokens * n_expert * 4) ||
                         !writable(op, "gate_logits", gate_logits))) ||
        !need(op, "idx", idx, ob) || !writable(op, "idx", idx) || !need(op, "scores", scores, ob) ||
        !writable(op, "scores", scores))
        return -1;
    float *scratch = noalloc_router_scratch(op);
    if (!scratch) return -1;
    if (n_tokens == 0) return 0;
    const float *wf = (const float *)dptr(w_gate_inp);
    if ((int)router_type != 0 || router_row_stride != rb) {
        // Every element the projection reads is written here first, so the
        // previous call's contents never need clearing.
        const cudaError_t e = ds3::launch_dequantize_rows(ctx(), (const uint8_t *)dptr(w_gate_inp), (int)router_type,
                                                          router_row_stride, n_expert, (int)n_embd, scratch);
        if (e != cudaSuccess) {
            set_error("%s: launch failed: %s", op, cudaGetErrorString(e));
            return -1;
        }
        wf = scratch;
    }
    if (!gate_logits && !ds3::router_gemv_fast(n_tokens, (int)n_embd, (int)n_expert, (int)n_used, dptr(input), wf)) {
        set_error("%s: gate_logits is required for this shape (fast path: n_expert 128, n_embd %% 64 == 0)", op);
        return -1;
    }
    const cudaError_t e =
        ds3::launch_router_gemv_topk(ctx(), (const float *)dptr(input), wf, (float *)dptr(gate_logits),
                                     (int32_t *)dptr(idx), (float *)dptr(scores), n_tokens, (int)n_embd,
                                     (int)n_expert, (int)n_used, norm_topk_prob ? 1 : 0);
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", op, cudaGetErrorString(e));
        return -1;
    }
    if (deferred()) return 0;
    return sync_and_check(op);
}

int ds3_cuda_moe_expert_lists(const ds3_cuda_buffer_t *idx, const ds3_cuda_buffer_t *scores, ds3_cuda_buffer_t *counts,
                              ds3_cuda_buffer_t *ids, ds3_cuda_buffer_t *gscores, ds3_cuda_buffer_t *slot_of,
                              uint32_t n_tokens, uint32_t n_expert, uint32_t n_used, uint32_t cap)
{
    const char *op = "moe_expert_lists";
    if (!ready(op)) return -1;
    if (n_expert == 0 || n_expert > 256 || n_used == 0 || cap == 0) {
        set_error("%s: need 0 < n_expert <= 256, n_used > 0, cap > 0", op);
        return -1;
    }
    const size_t ent = (size_t)n_tokens * n_used * 4, lists = (size_t)n_expert * cap * 4;
    if (!need(op, "idx", idx, ent) || !need(op, "scores", scores, ent) || !need(op, "counts", counts, n_expert * 4) ||
        !writable(op, "counts", counts) || !need(op, "ids", ids, lists) || !writable(op, "ids", ids) ||
        !need(op, "gscores", gscores, lists) || !writable(op, "gscores", gscores) ||
        (slot_of && (!need(op, "slot_of", slot_of, ent) || !writable(op, "slot_of", slot_of))))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_moe_expert_lists(ctx(), (const int32_t *)dptr(idx), (const float *)dptr(scores),
                                               (int32_t *)dptr(counts), (int32_t *)dptr(ids), (float *)dptr(gscores),
                                               (int32_t *)dptr(slot_of), n_tokens, (int)n_used, (int)n_expert, cap),
                  ps);
}

int ds3_cuda_swiglu(const ds3_cuda_buffer_t *gate, const ds3_cuda_buffer_t *up, const ds3_cuda_buffer_t *row_weight,
                    ds3_cuda_buffer_t *out, uint32_t n_rows, uint32_t n_cols)
{
    const char *op = "swiglu";
    if (!ready(op)) return -1;
    const size_t b = (size_t)n_rows * n_cols * 4;
    if (!need(op, "gate", gate, b) || !need(op, "up", up, b) || !need(op, "out", out, b) ||
        !writable(op, "out", out) || (row_weight && !need(op, "row_weight", row_weight, (size_t)n_rows * 4)))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_swiglu(ctx(), (const float *)dptr(gate), (const float *)dptr(up),
                                     (const float *)dptr(row_weight), (float *)dptr(out), n_rows, n_cols),
                  ps);
}

int ds3_cuda_moe_combine_residual(const ds3_cuda_buffer_t *y, const ds3_cuda_buffer_t *y_rows,
                                  const ds3_cuda_buffer_t *w, const ds3_cuda_buffer_t *residual, ds3_cuda_buffer_t *out,
                                  uint32_t n_tokens, uint32_t n_used, uint32_t n_cols)
{
    const char *op = "moe_combine_residual";
    if (!ready(op)) return -1;
    const size_t rb = (size_t)n_tokens * n_cols * 4;
    const size_t tk = (size_t)n_tokens * n_used;
    if (n_used == 0 || n_cols == 0) {
        set_error("%s: n_used and n_cols must be > 0", op);
        return -1;
    }
    // Without a row map y holds n_tokens*n_used rows; with one, any row it names.
    if (!need(op, "y", y, y_rows ? (size_t)n_cols * 4 : tk * n_cols * 4) || !need(op, "w", w, tk * 4) ||
        !need(op, "residual", residual, rb) || !need(op, "out", out, rb) || !writable(op, "out", out) ||
        (y_rows && !need(op, "y_rows", y_rows, tk * 4)))
        return -1;
    ProfScope ps(op);
    return finish(op,
                  ds3::launch_combine(ctx(), (const float *)dptr(y), (const int32_t *)dptr(y_rows),
                                      (const float *)dptr(w), (const float *)dptr(residual), (float *)dptr(out),
                                      n_tokens, (int)n_used, n_cols, (int64_t)(y->bytes / ((size_t)n_cols * 4))),
                  ps);
}

// ------------------------------------------------------------- copy lanes
static cudaStream_t lane_stream(const char *op, int lane)
{
    if (!ready(op)) return nullptr;
    if (G.capturing) {
        set_error("%s: copy lanes are not available during graph capture", op);
        return nullptr;
    }
    if (lane < 0 || lane > 2) {
        set_error("%s: lane %d out of range 0..2", op, lane);
        return nullptr;
    }
    return lane == 0 ? G.stream : G.lanes[lane - 1];
}

int ds3_cuda_lane_write(int lane, ds3_cuda_buffer_t *buf, size_t offset, const void *src, size_t bytes)
{
    const char *op = "lane_write";
    cudaStream_t s = lane_stream(op, lane);
    if (!s) return -1;
    if (!buf || !src || offset + bytes > buf->bytes || buf->read_only) {
        set_error("%s: bad arguments", op);
        return -1;
    }
    const cudaError_t e = cudaMemcpyAsync((char *)dptr(buf) + offset, src, bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        set_error("%s: %s", op, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int ds3_cuda_lane_read(int lane, ds3_cuda_buffer_t *buf, size_t offset, void *dst, size_t bytes)
{
    const char *op = "lane_read";
    cudaStream_t s = lane_stream(op, lane);
    if (!s) return -1;
    if (!buf || !dst || offset + bytes > buf->bytes) {
        set_error("%s: bad arguments", op);
        return -1;
    }
    const cudaError_t e = cudaMemcpyAsync(dst, (char *)dptr(buf) + offset, bytes, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) {
        set_error("%s: %s", op, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

static cudaEvent_t slot_event(const char *op, int slot)
{
    if (slot < 0 || slot >= DS3_CUDA_TIMER_SLOTS) {
        set_error("%s: slot %d out of range", op, slot);
        return nullptr;
    }
    if (!G.timers[slot] && cudaEventCreate(&G.timers[slot]) != cudaSuccess) {
        set_error("%s: cudaEventCreate failed", op);
        return nullptr;
    }
    return G.timers[slot];
}

int ds3_cuda_lane_record(int lane, int slot)
{
    const char *op = "lane_record";
    cudaStream_t s = lane_stream(op, lane);
    if (!s) return -1;
    cudaEvent_t ev = slot_event(op, slot);
    if (!ev) return -1;
    const cudaError_t e = cudaEventRecord(ev, s);
    if (e != cudaSuccess) {
        set_error("%s: %s", op, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int ds3_cuda_lane_wait(int lane, int slot)
{
    const char *op = "lane_wait";
    cudaStream_t s = lane_stream(op, lane);
    if (!s) return -1;
    cudaEvent_t ev = slot_event(op, slot);
    if (!ev) return -1;
    const cudaError_t e = cudaStreamWaitEvent(s, ev, 0);
    if (e != cudaSuccess) {
        set_error("%s: %s", op, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// --------------------------------------------------- stream / graph / timers
void *ds3_cuda_stream(void) { return G.inited ? (void *)G.stream : nullptr; }

int ds3_cuda_graph_begin(void)
{
    if (!ready("graph_begin")) return -1;
    if (G.capturing || G.batch) {
        set_error("graph_begin: a batch or capture is already open");
        return -1;
    }
    cudaError_t e = cudaStreamBeginCapture(G.stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        set_error("graph_begin: %s", cudaGetErrorString(e));
        return -1;
    }
    G.capturing = true;
    return 0;
}

ds3_cuda_graph_t *ds3_cuda_graph_end(void)
{
    if (!G.inited || !G.capturing) {
        set_error("graph_end: no capture open");
        return nullptr;
    }
    G.capturing = false;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(G.stream, &g);
    if (e != cudaSuccess || !g) {
        set_error("graph_end: %s", cudaGetErrorString(e));
        return nullptr;
    }
    cudaGraphExec_t x = nullptr;
    e = cudaGraphInstantiate(&x, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        set_error("graph_end: instantiate: %s", cudaGetErrorString(e));
        return nullptr;
    }
    auto *h = new ds3_cuda_graph{g, x};
    return h;
}

int ds3_cuda_graph_launch(ds3_cuda_graph_t *g)
{
    if (!ready("graph_launch") || !g) return -1;
    cudaError_t e = cudaGraphLaunch(g->exec, G.stream);
    if (e != cudaSuccess) {
        set_error("graph_launch: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

void ds3_cuda_graph_free(ds3_cuda_graph_t *g)
{
    if (!g) return;
    if (G.inited) {
        cudaGraphExecDestroy(g->exec);
        cudaGraphDestroy(g->graph);
    }
    delete g;
}

int ds3_cuda_timer_mark(int slot)
{
    if (!ready("timer_mark")) return -1;
    if (slot < 0 || slot >= DS3_CUDA_TIMER_SLOTS) {
        set_error("timer_mark: slot %d out of range", slot);
        return -1;
    }
    if (!G.timers[slot] && cudaEventCreate(&G.timers[slot]) != cudaSuccess) {
        set_error("timer_mark: cudaEventCreate failed");
        return -1;
    }
    cudaError_t e = cudaEventRecordWithFlags(G.timers[slot], G.stream, G.capturing ? cudaEventRecordExternal : 0);
    if (e != cudaSuccess) {
        set_error("timer_mark: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

float ds3_cuda_timer_elapsed_ms(int a, int b)
{
    if (!G.inited || a < 0 || b < 0 || a >= DS3_CUDA_TIMER_SLOTS || b >= DS3_CUDA_TIMER_SLOTS || !G.timers[a] ||
        !G.timers[b])
        return -1.0f;
    if (cudaEventSynchronize(G.timers[b]) != cudaSuccess) return -1.0f;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, G.timers[a], G.timers[b]) != cudaSuccess) return -1.0f;
    return ms;
}

int ds3_cuda_selftest_bounded_wait(uint32_t polls)
{
    if (!ready("selftest_bounded_wait") || G.capturing) return -1;
    if (polls == 0 || polls > (1u << 20)) {
        set_error("selftest_bounded_wait: polls must be in 1..2^20");
        return -1;
    }
    cudaStreamSynchronize(G.stream);
    take_device_errors();  // start from a clean word
    if (ds3::launch_bounded_wait_selftest(ctx(), polls) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(G.stream) != cudaSuccess) return -1;
    const uint32_t bits = take_device_errors();
    return (bits & (1u << ds3::kErrWaitTimeout)) ? 0 : -1;
}

const char *ds3_cuda_last_error(void) { return g_last_error.c_str(); }

int ds3_cuda_kernel_binary_version(void)
{
    if (!ready("kernel_binary_version")) return -1;
    return ds3::kernel_binary_version();
}


uint32_t ds3_cuda_device_errors(void)
{
    if (!G.inited) return 0;
    if (!G.capturing) cudaStreamSynchronize(G.stream);
    return take_device_errors();
}

}  // extern "C"
