// k3_ctx.cu -- the device context behind both headers: device selection, the library
// stream, sticky status, device error flag, allocation, host-argument staging and the
// HBM weight cache, events, graphs and launch accounting.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "k3_common.cuh"

__device__ int k3_dev_err[2];
__device__ int k3_dev_diag[4];
__device__ long long k3_wait_cycles = 4000000000LL;

namespace k3 {

namespace {

struct WeightCopy { void *dev; size_t bytes; };

struct Ctx {
    bool ready = false;
    int device = -1;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    bool graph_prio = true;        // k3d_graph_end keeps the nodes' stream priorities
    int sms = 0;
    int status = 0;
    char msg[512] = {0};
    int abort_on_error = 0;
    int cache_weights = 0;
    long launches = 0;
    std::unordered_map<const void *, WeightCopy> wcache;
    size_t wcache_bytes = 0;
    void *scratch[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t scratch_bytes[6] = {0, 0, 0, 0, 0, 0};
    void *arena = nullptr;
    size_t arena_bytes = 0;
    size_t arena_top = 0;
    cudaGraph_t capturing = nullptr;
    bool prof = false;
    struct Sec { std::vector<std::pair<cudaEvent_t, cudaEvent_t>> done; cudaEvent_t open = nullptr;
                 double ms = 0.0; long count = 0; };
    std::map<std::string, Sec> secs;
    std::vector<cudaEvent_t> pool;
    cudaStream_t side = nullptr;          // second stream for independent work in a layer
    cudaEvent_t side_ev[4] = {nullptr, nullptr, nullptr, nullptr};
};

Ctx g;

void record(int code, const char *text)
{
    if (code && !g.status) {
        g.status = code;
        snprintf(g.msg, sizeof g.msg, "%s", text);
    }
    if (code) {
        fprintf(stderr, "k3cuda: error %d (%s): %s\n", code, k3d_strerror(code), text);
        if (g.abort_on_error) abort();
    }
}

bool capturing_now()
{
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(g.stream, &cs);
    return cs != cudaStreamCaptureStatusNone;
}

cudaEvent_t pool_event()
{
    if (!g.pool.empty()) { cudaEvent_t e = g.pool.back(); g.pool.pop_back(); return e; }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}

// fold finished event pairs of one section into its total
void prof_collect(Ctx::Sec &sec)
{
    for (auto &pr : sec.done) {
        float ms = 0.f;
        cudaEventSynchronize(pr.second);
        if (cudaEventElapsedTime(&ms, pr.first, pr.second) == cudaSuccess) {
            sec.ms += ms;
            sec.count++;
        } else {
            cudaGetLastError();
        }
        g.pool.push_back(pr.first);
        g.pool.push_back(pr.second);
    }
    sec.done.clear();
}

}  // namespace

std::recursive_mutex g_mu;

void allow_dyn_smem(const void *func)
{
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, g.device < 0 ? 0 : g.device);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, func) != cudaSuccess) { cudaGetLastError(); return; }
    const int want = optin - (int)fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, want) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ECUDA, "cannot raise dynamic shared memory to %d bytes", want);
    }
}

void prof_begin(const char *section)
{
    if (!g.prof || capturing_now()) return;
    auto &sec = g.secs[section];
    if (sec.open) return;
    sec.open = pool_event();
    cudaEventRecord(sec.open, g.stream);
}

void prof_end(const char *section)
{
    if (!g.prof) return;
    auto it = g.secs.find(section);
    if (it == g.secs.end() || !it->second.open) return;
    cudaEvent_t e = pool_event();
    cudaEventRecord(e, g.stream);
    it->second.done.push_back({it->second.open, e});
    it->second.open = nullptr;
    if (it->second.done.size() > 256) prof_collect(it->second);
}

int fail(int code, const char *fmt, ...)
{
    char buf[480];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    record(code, buf);
    return code;
}

int ensure_ctx()
{
    if (g.ready) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != g.device) cudaSetDevice(g.device);
        return K3D_OK;
    }
    return k3d_init(0);
}

cudaStream_t stream() { return g.stream; }

// The side stream and its fork/join events, created on first use. Work forked onto it is
// always joined back into the main stream before the call returns, so synchronising the
// main stream (or capturing it into a graph) covers it.
cudaStream_t side_stream()
{
    if (!g.side) {
        if (cudaStreamCreateWithFlags(&g.side, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            g.side = nullptr;
        }
        for (int i = 0; i < 4 && g.side; i++)
            if (cudaEventCreateWithFlags(&g.side_ev[i], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                g.side = nullptr;
            }
    }
    return g.side;
}

cudaEvent_t side_event(int i) { return g.side_ev[i & 3]; }

bool profiling() { return g.prof; }

bool pdl_enabled()
{
    static const bool on = [] {
        const char *v = getenv("K3_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}
int sm_count() { return g.sms; }
void note_launch(int n) { g.launches += n; }

int check_launch(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(K3D_ECUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return K3D_OK;
}

bool is_device_ptr(const void *p)
{
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

void *scratch(size_t bytes, int slot)
{
    if (slot < 0 || slot > 5) return nullptr;
    if (bytes == 0) bytes = 256;
    if (g.scratch_bytes[slot] >= bytes) return g.scratch[slot];
    if (g.scratch[slot]) {
        cudaStreamSynchronize(g.stream);
        if (g.side) cudaStreamSynchronize(g.side);
        cudaFree(g.scratch[slot]);
    }
    g.scratch[slot] = nullptr; g.scratch_bytes[slot] = 0;
    size_t want = bytes + bytes / 4;
    if (cudaMalloc(&g.scratch[slot], want) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ENOMEM, "scratch of %zu bytes", want);
        return nullptr;
    }
    g.scratch_bytes[slot] = want;
    return g.scratch[slot];
}

// ------------------------------------------------------------------- staging ----
Stage::Stage() { base = g.arena_top; }
Stage::~Stage() { g.arena_top = base; }

void *Stage::arena(size_t bytes)
{
    size_t off = (g.arena_top + 255) & ~(size_t)255;
    size_t need = off + bytes;
    if (need > g.arena_bytes) {
        // Grow only when nothing staged is live; earlier pointers must stay valid.
        if (g.arena_top != 0) {
            err = fail(K3D_ENOMEM, "staging arena exhausted mid-call (%zu bytes)", need);
            return nullptr;
        }
        if (g.arena) { cudaStreamSynchronize(g.stream); cudaFree(g.arena); }
        g.arena = nullptr; g.arena_bytes = 0;
        size_t want = need < ((size_t)64 << 20) ? ((size_t)64 << 20) : need * 2;
        if (cudaMalloc(&g.arena, want) != cudaSuccess) {
            cudaGetLastError();
            err = fail(K3D_ENOMEM, "staging arena of %zu bytes", want);
            return nullptr;
        }
        g.arena_bytes = want;
    }
    g.arena_top = need;
    return (char *)g.arena + off;
}

const void *Stage::weight(const void *p, size_t bytes)
{
    if (err) return nullptr;
    if (!p) { err = fail(K3D_EINVAL, "null weight pointer"); return nullptr; }
    if (is_device_ptr(p)) return p;
    if (!g.cache_weights) return in(p, bytes);
    auto it = g.wcache.find(p);
    if (it != g.wcache.end() && it->second.bytes >= bytes) return it->second.dev;
    if (it != g.wcache.end()) {
        cudaStreamSynchronize(g.stream);
        cudaFree(it->second.dev);
        g.wcache_bytes -= it->second.bytes;
        g.wcache.erase(it);
    }
    void *d = nullptr;
    if (cudaMalloc(&d, bytes ? bytes : 16) != cudaSuccess) {
        cudaGetLastError();
        err = fail(K3D_ENOMEM, "HBM copy of a %zu-byte host weight", bytes);
        return nullptr;
    }
    if (cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d);
        err = fail(K3D_ECUDA, "upload of a host weight");
        return nullptr;
    }
    g.wcache[p] = WeightCopy{d, bytes};
    g.wcache_bytes += bytes;
    any_host = true;
    return d;
}

const void *Stage::in(const void *p, size_t bytes)
{
    if (err) return nullptr;
    if (!p) { err = fail(K3D_EINVAL, "null input pointer"); return nullptr; }
    if (is_device_ptr(p)) return p;
    void *d = arena(bytes);
    if (!d) return nullptr;
    if (cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) {
        cudaGetLastError();
        err = fail(K3D_ECUDA, "staging a host input");
        return nullptr;
    }
    any_host = true;
    return d;
}

void *Stage::out(void *p, size_t bytes)
{
    if (err) return nullptr;
    if (!p) { err = fail(K3D_EINVAL, "null output pointer"); return nullptr; }
    if (is_device_ptr(p)) return p;
    if (n_out >= 16) { err = fail(K3D_EINVAL, "too many staged outputs"); return nullptr; }
    void *d = arena(bytes);
    if (!d) return nullptr;
    outs[n_out++] = Out{p, d, bytes};
    any_host = true;
    return d;
}

void *Stage::inout(void *p, size_t bytes)
{
    if (err) return nullptr;
    if (!p) { err = fail(K3D_EINVAL, "null state pointer"); return nullptr; }
    if (is_device_ptr(p)) return p;
    void *d = const_cast<void *>(in(p, bytes));
    if (!d) return nullptr;
    if (n_out >= 16) { err = fail(K3D_EINVAL, "too many staged outputs"); return nullptr; }
    outs[n_out++] = Out{p, d, bytes};
    return d;
}

int Stage::finish()
{
    if (err) return err;
    for (int i = 0; i < n_out; i++) {
        if (cudaMemcpyAsync(outs[i].host, outs[i].dev, outs[i].bytes,
                            cudaMemcpyDeviceToHost, g.stream) != cudaSuccess) {
            cudaGetLastError();
            return fail(K3D_ECUDA, "copying a staged output back");
        }
    }
    if (any_host) {
        cudaError_t e = cudaStreamSynchronize(g.stream);
        if (e != cudaSuccess) return fail(K3D_ECUDA, "stream sync: %s", cudaGetErrorString(e));
        return device_flag_status();
    }
    return K3D_OK;
}

// The device error flag (after a synchronisation), as a status with the kernel's location
// details when it gave any.
int device_flag_status()
{
    int flag[2] = {0, 0};
    cudaMemcpyFromSymbol(flag, k3_dev_err, sizeof flag);
    if (!flag[0]) return K3D_OK;
    int diag[4] = {0, 0, 0, 0};
    cudaMemcpyFromSymbol(diag, k3_dev_diag, sizeof diag);
    if (diag[3])
        return fail(K3D_EDEVICE, "device error %d at site %d (%d, %d, %d)", flag[0], flag[1], diag[0],
                    diag[1], diag[2]);
    return fail(K3D_EDEVICE, "device error %d at site %d", flag[0], flag[1]);
}

}  // namespace k3

using namespace k3;

// ------------------------------------------------------------------- C ABI ----
extern "C" {

int k3d_init(int device)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (g.ready && g.device == device) { cudaSetDevice(device); return K3D_OK; }
    // One device per process: the workspaces, the side stream and each kernel's one-time
    // shared-memory opt-in belong to the device the context was made on.
    if (g.ready)
        return fail(K3D_EINVAL, "k3d_init(%d): this process's context is on device %d; one "
                    "device per process", device, g.device);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return fail(K3D_ENODEV, "no CUDA device is available; libk3cuda has no CPU path");
    }
    if (device < 0 || device >= n) return fail(K3D_ENODEV, "device %d of %d", device, n);
    if (cudaSetDevice(device) != cudaSuccess) return fail(K3D_ENODEV, "cudaSetDevice(%d)", device);
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, device);
    if (p.major < 10) {
        return fail(K3D_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a",
                    device, p.major, p.minor);
    }
    // the library's stream at the device's highest priority, the side stream (shared
    // expert, x split) at the default, lowest one: where both have CTAs waiting, the block
    // scheduler starts the router and routed experts first (graphs keep the priorities:
    // k3d_graph_end instantiates with node priorities). Stack 534.2 -> 541.8 tok/s.
    cudaStream_t s;
    int prio_lo = 0, prio_hi = 0;
    if (cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi) != cudaSuccess) {
        cudaGetLastError();
        prio_hi = 0;
    }
    if (cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, prio_hi) != cudaSuccess)
        return fail(K3D_ECUDA, "stream creation");
    g.device = device;
    g.stream = s;
    g.own_stream = true;
    g.sms = p.multiProcessorCount;
    int zero[4] = {0, 0, 0, 0};
    cudaMemcpyToSymbol(k3_dev_err, zero, 2 * sizeof(int));
    cudaMemcpyToSymbol(k3_dev_diag, zero, sizeof zero);
    g.ready = true;
    return K3D_OK;
}

int k3d_device(void) { return g.device; }

int k3d_status(void) { return g.status; }

void k3d_clear_status(void)
{
    g.status = 0;
    g.msg[0] = 0;
    if (g.ready) {
        int zero[4] = {0, 0, 0, 0};
        cudaMemcpyToSymbol(k3_dev_err, zero, 2 * sizeof(int));
        cudaMemcpyToSymbol(k3_dev_diag, zero, sizeof zero);
    }
}

const char *k3d_strerror(int code)
{
    switch (code) {
    case K3D_OK: return "ok";
    case K3D_ENODEV: return "no usable CUDA device";
    case K3D_EINVAL: return "invalid argument";
    case K3D_ENOMEM: return "device allocation failed";
    case K3D_ECUDA: return "CUDA runtime error";
    case K3D_EDEVICE: return "device-side error flag raised";
    case K3D_EUNSUPPORTED: return "unsupported by this library";
    case K3D_ENCCL: return "NCCL error";
    case K3D_EBOUND: return "capacity bound exceeded";
    case K3D_ETIMEOUT: return "bounded device wait gave up";
    default: return "unknown";
    }
}

const char *k3d_last_message(void) { return g.msg; }

int k3d_set_wait_limit(long long cycles)
{
    K3_TRY(ensure_ctx());
    const long long v = cycles > 0 ? cycles : 4000000000LL;
    if (cudaMemcpyToSymbol(k3_wait_cycles, &v, sizeof v) != cudaSuccess)
        return fail(K3D_ECUDA, "k3d_set_wait_limit");
    return K3D_OK;
}
void k3d_set_abort_on_error(int on) { g.abort_on_error = on; }

int k3d_device_error(int *code, int *site)
{
    int flag[2] = {0, 0};
    if (ensure_ctx()) return g.status;
    cudaMemcpyFromSymbol(flag, k3_dev_err, sizeof flag);
    if (code) *code = flag[0];
    if (site) *site = flag[1];
    return K3D_OK;
}

void *k3d_alloc(size_t bytes)
{
    if (ensure_ctx()) return nullptr;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ENOMEM, "k3d_alloc(%zu)", bytes);
        return nullptr;
    }
    return p;
}

void k3d_free(void *p)
{
    if (!p || !g.ready) return;
    cudaStreamSynchronize(g.stream);
    cudaFree(p);
}

int k3d_upload(void *dst, const void *src, size_t bytes)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src) return fail(K3D_EINVAL, "k3d_upload null pointer");
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g.stream) != cudaSuccess ||
        cudaStreamSynchronize(g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "k3d_upload of %zu bytes", bytes);
    }
    return K3D_OK;
}

int k3d_download(void *dst, const void *src, size_t bytes)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src) return fail(K3D_EINVAL, "k3d_download null pointer");
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess ||
        cudaStreamSynchronize(g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "k3d_download of %zu bytes", bytes);
    }
    return K3D_OK;
}

int k3d_memset(void *dst, int value, size_t bytes)
{
    K3_TRY(ensure_ctx());
    if (cudaMemsetAsync(dst, value, bytes, g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "k3d_memset");
    }
    return K3D_OK;
}

int k3d_copy(void *dst, const void *src, size_t bytes)
{
    K3_TRY(ensure_ctx());
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "k3d_copy");
    }
    return K3D_OK;
}

int k3d_copy2d(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows)
{
    K3_TRY(ensure_ctx());
    if (cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDeviceToDevice, g.stream) !=
        cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "k3d_copy2d");
    }
    return K3D_OK;
}

void k3d_set_weight_cache(int on) { g.cache_weights = on != 0; if (!on) k3d_forget_all(); }

void k3d_forget(const void *host_ptr)
{
    auto it = g.wcache.find(host_ptr);
    if (it == g.wcache.end()) return;
    cudaStreamSynchronize(g.stream);
    cudaFree(it->second.dev);
    g.wcache_bytes -= it->second.bytes;
    g.wcache.erase(it);
}

void k3d_forget_all(void)
{
    if (g.ready) cudaStreamSynchronize(g.stream);
    for (auto &kv : g.wcache) cudaFree(kv.second.dev);
    g.wcache.clear();
    g.wcache_bytes = 0;
}

size_t k3d_weight_cache_bytes(void) { return g.wcache_bytes; }

int k3d_sync(void)
{
    K3_TRY(ensure_ctx());
    cudaError_t e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) return fail(K3D_ECUDA, "k3d_sync: %s", cudaGetErrorString(e));
    return device_flag_status();
}

void *k3d_stream(void) { ensure_ctx(); return (void *)g.stream; }

int k3d_set_stream(void *s)
{
    K3_TRY(ensure_ctx());
    g.stream = (cudaStream_t)s;
    return K3D_OK;
}

void *k3d_event_create(void)
{
    if (ensure_ctx()) return nullptr;
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    return (void *)e;
}

int k3d_event_record(void *ev)
{
    K3_TRY(ensure_ctx());
    if (cudaEventRecord((cudaEvent_t)ev, g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "event record");
    }
    return K3D_OK;
}

float k3d_event_elapsed_ms(void *a, void *b)
{
    float ms = -1.0f;
    cudaEventSynchronize((cudaEvent_t)b);
    if (cudaEventElapsedTime(&ms, (cudaEvent_t)a, (cudaEvent_t)b) != cudaSuccess) {
        cudaGetLastError();
        return -1.0f;
    }
    return ms;
}

void k3d_event_destroy(void *ev) { if (ev) cudaEventDestroy((cudaEvent_t)ev); }

int k3d_set_graph_priorities(int on)
{
    g.graph_prio = on != 0;
    return K3D_OK;
}

int k3d_graph_begin(void)
{
    K3_TRY(ensure_ctx());
    if (cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "graph capture begin");
    }
    return K3D_OK;
}

void *k3d_graph_end(void)
{
    if (ensure_ctx()) return nullptr;
    cudaGraph_t graph = nullptr;
    if (cudaStreamEndCapture(g.stream, &graph) != cudaSuccess || !graph) {
        cudaGetLastError();
        fail(K3D_ECUDA, "graph capture end");
        return nullptr;
    }
    cudaGraphExec_t ex = nullptr;
    // node priorities: each captured kernel keeps its stream's priority (see k3d_init);
    // without them every node runs at the priority of the stream the graph is launched on
    const unsigned long long flags = g.graph_prio ? cudaGraphInstantiateFlagUseNodePriority : 0;
    if (cudaGraphInstantiate(&ex, graph, flags) != cudaSuccess) {
        cudaGetLastError();
        cudaGraphDestroy(graph);
        fail(K3D_ECUDA, "graph instantiate");
        return nullptr;
    }
    cudaGraphDestroy(graph);
    return (void *)ex;
}

int k3d_graph_launch(void *ex)
{
    K3_TRY(ensure_ctx());
    if (cudaGraphLaunch((cudaGraphExec_t)ex, g.stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ECUDA, "graph launch");
    }
    return K3D_OK;
}

void k3d_graph_destroy(void *ex) { if (ex) cudaGraphExecDestroy((cudaGraphExec_t)ex); }

void *k3d_host_alloc(size_t bytes)
{
    if (ensure_ctx()) return nullptr;
    void *p = nullptr;
    if (cudaMallocHost(&p, bytes ? bytes : 16) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ENOMEM, "k3d_host_alloc(%zu)", bytes);
        return nullptr;
    }
    return p;
}

void k3d_host_free(void *p) { if (p) cudaFreeHost(p); }

void k3d_prof_enable(int on) { ensure_ctx(); g.prof = on != 0; }

void k3d_prof_reset(void)
{
    for (auto &kv : g.secs) {
        prof_collect(kv.second);
        kv.second.ms = 0.0;
        kv.second.count = 0;
    }
}

double k3d_prof_ms(const char *section, long *count)
{
    auto it = g.secs.find(section);
    if (it == g.secs.end()) { if (count) *count = 0; return 0.0; }
    prof_collect(it->second);
    if (count) *count = it->second.count;
    return it->second.ms;
}

long k3d_launch_count(void) { return g.launches; }
void k3d_launch_count_reset(void) { g.launches = 0; }
int  k3d_sm_count(void) { ensure_ctx(); return g.sms; }

}  // extern "C"
