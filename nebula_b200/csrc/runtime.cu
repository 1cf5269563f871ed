// Runtime entry points of the qwen/gpu.h ABI: device memory, copies, the
// per-thread capture stream and CUDA graphs, tensor sizes and the pinned
// expert uploader. Semantics follow the reference (qwen/gpu.cu:10-85); the
// code is this library's own.
#include <cstdlib>
#include <cstring>
#include <new>
#include "common.cuh"

namespace nb {
thread_local cudaStream_t launch_stream = 0;
}
using nb::launch_stream;

namespace {
struct Graph {
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool capturing = false;
};
}  // namespace

extern "C" void qg_graph_destroy(void *ptr) {
    Graph *g = static_cast<Graph *>(ptr);
    if (!g) return;
    if (g->capturing) {
        cudaGraph_t partial = nullptr;
        cudaStreamEndCapture(g->stream, &partial);
        if (partial) cudaGraphDestroy(partial);
        launch_stream = 0;
    }
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    if (g->stream) cudaStreamDestroy(g->stream);
    delete g;
}

// Starts a thread-local capture: every later launch from this thread goes to
// the capture stream until qg_graph_end (reference qwen/gpu.cu:21-28).
extern "C" int qg_graph_begin(void **out) {
    if (!out || *out || launch_stream) return cudaErrorInvalidValue;
    Graph *g = new (std::nothrow) Graph;
    if (!g) return cudaErrorMemoryAllocation;
    int rc = cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking);
    if (!rc) rc = cudaStreamBeginCapture(g->stream, cudaStreamCaptureModeThreadLocal);
    if (rc) {
        qg_graph_destroy(g);
        return rc;
    }
    g->capturing = true;
    launch_stream = g->stream;
    *out = g;
    return 0;
}

extern "C" int qg_graph_end(void *ptr) {
    Graph *g = static_cast<Graph *>(ptr);
    if (!g || !g->capturing) return cudaErrorInvalidValue;
    int rc = cudaStreamEndCapture(g->stream, &g->graph);
    g->capturing = false;
    launch_stream = 0;
    if (!rc) rc = cudaGraphInstantiate(&g->exec, g->graph, 0);
    return rc;
}

// Replays on the legacy default stream, ordered with qg_write/qg_read.
extern "C" int qg_graph_launch(void *ptr) {
    Graph *g = static_cast<Graph *>(ptr);
    return g && g->exec ? cudaGraphLaunch(g->exec, 0) : cudaErrorInvalidValue;
}

extern "C" void *qg_alloc(size_t n) {
    void *p = nullptr;
    return cudaMalloc(&p, n) == cudaSuccess ? p : nullptr;
}
extern "C" void qg_free(void *p) {
    if (p) cudaFree(p);
}
extern "C" int qg_write(void *d, const void *s, size_t n) { return cudaMemcpy(d, s, n, cudaMemcpyHostToDevice); }
extern "C" int qg_read(void *d, const void *s, size_t n) { return cudaMemcpy(d, s, n, cudaMemcpyDeviceToHost); }
extern "C" int qg_copy(void *d, const void *s, size_t n) {
    return cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToDevice, launch_stream);
}
extern "C" int qg_zero(void *d, size_t n) { return cudaMemsetAsync(d, 0, n, launch_stream); }
extern "C" int qg_sync(void) { return cudaDeviceSynchronize(); }
extern "C" int qg_memory(size_t *f, size_t *t) { return cudaMemGetInfo(f, t); }
extern "C" const char *qg_error(int e) { return cudaGetErrorString(static_cast<cudaError_t>(e)); }

// Bytes of a 4-D GGML tensor whose first dimension is the row length
// (reference qwen/gpu.cu:114-120): rejects ragged blocks and overflow.
extern "C" int qg_tensor_bytes(int type, const uint64_t dims[4], uint64_t *bytes) {
    if (!dims || !bytes || dims[0] < 1 || dims[0] > 2147483647ULL) return cudaErrorInvalidValue;
    uint64_t n = nb::row_bytes(type, static_cast<int>(dims[0]));
    if (!n) return cudaErrorInvalidValue;
    for (int i = 1; i < 4; i++) {
        if (!dims[i] || dims[i] > UINT64_MAX / n) return cudaErrorInvalidValue;
        n *= dims[i];
    }
    *bytes = n;
    return 0;
}

// ---- expert uploader -----------------------------------------------------
// Two pinned slabs so the host can pack expert e+1 while expert e's copy is
// in flight; event pairs time each copy (reference qwen/gpu.cu:48-85).
namespace {
struct Uploader {
    unsigned char *stage[2] = {nullptr, nullptr};
    cudaEvent_t begin[2] = {nullptr, nullptr}, end[2] = {nullptr, nullptr};
    int next = 0;
    bool pending[2] = {false, false};
    size_t capacity = 0;
    double seconds = 0;
};

int upload_finish(Uploader *u, int i, bool wait) {
    if (!u->pending[i]) return cudaSuccess;
    cudaError_t rc = wait ? cudaEventSynchronize(u->end[i]) : cudaEventQuery(u->end[i]);
    if (rc == cudaErrorNotReady) return cudaSuccess;
    if (rc != cudaSuccess) return rc;
    float ms = 0;
    rc = cudaEventElapsedTime(&ms, u->begin[i], u->end[i]);
    if (rc != cudaSuccess) return rc;
    u->seconds += ms / 1000.0;
    u->pending[i] = false;
    return cudaSuccess;
}
}  // namespace

extern "C" void qg_upload_destroy(void *ptr) {
    Uploader *u = static_cast<Uploader *>(ptr);
    if (!u) return;
    for (int i = 0; i < 2; i++)
        if (u->pending[i]) cudaEventSynchronize(u->end[i]);
    for (int i = 0; i < 2; i++) {
        if (u->stage[i]) cudaFreeHost(u->stage[i]);
        if (u->begin[i]) cudaEventDestroy(u->begin[i]);
        if (u->end[i]) cudaEventDestroy(u->end[i]);
    }
    delete u;
}

extern "C" void *qg_upload_create(size_t bytes) {
    Uploader *u = new (std::nothrow) Uploader;
    if (!u) return nullptr;
    u->capacity = bytes;
    for (int i = 0; i < 2; i++) {
        if (cudaHostAlloc(reinterpret_cast<void **>(&u->stage[i]), bytes, 0) != cudaSuccess ||
            cudaEventCreate(&u->begin[i]) != cudaSuccess || cudaEventCreate(&u->end[i]) != cudaSuccess) {
            qg_upload_destroy(u);
            return nullptr;
        }
    }
    return u;
}

extern "C" int qg_upload_expert(void *ptr, void *dst, const void *g, size_t ng, const void *up, size_t nu,
                                const void *down, size_t nd) {
    Uploader *u = static_cast<Uploader *>(ptr);
    if (!u || !dst || ng > u->capacity || nu > u->capacity - ng || nd > u->capacity - ng - nu)
        return cudaErrorInvalidValue;
    int i = u->next;
    int rc = upload_finish(u, i, true);
    if (rc) return rc;
    std::memcpy(u->stage[i], g, ng);
    std::memcpy(u->stage[i] + ng, up, nu);
    std::memcpy(u->stage[i] + ng + nu, down, nd);
    if ((rc = cudaEventRecord(u->begin[i], 0))) return rc;
    if ((rc = cudaMemcpyAsync(dst, u->stage[i], ng + nu + nd, cudaMemcpyHostToDevice, 0))) return rc;
    if ((rc = cudaEventRecord(u->end[i], 0))) return rc;
    u->pending[i] = true;
    u->next = 1 - i;
    return cudaSuccess;
}

extern "C" double qg_upload_seconds(void *ptr) {
    Uploader *u = static_cast<Uploader *>(ptr);
    if (!u) return 0;
    for (int i = 0; i < 2; i++)
        if (upload_finish(u, i, false)) return -1;
    return u->seconds;
}
