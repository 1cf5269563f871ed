// Runtime entry points of the qwen/gpu.h ABI: device memory and copies, the
// per-thread launch stream and CUDA graph capture. (Tensor sizes and the
// expert uploads live in loader.cu.)
//
// Capture model (the ABI's contract, qwen/gpu.h:4-5,18-21): qg_graph_begin
// makes a fresh non-blocking stream the calling thread's launch stream and
// starts a thread-local capture on it, so every entry point this thread calls
// afterwards records into the graph instead of running; qg_graph_end
// instantiates it and returns the thread to the legacy default stream, where
// qg_graph_launch replays it (ordered with qg_write / qg_read).
#include <new>
#include "common.cuh"

namespace nb {
thread_local cudaStream_t launch_stream asm("nebula_launch_stream") = 0;
}
using nb::launch_stream;

namespace {

class CaptureGraph {
  public:
    ~CaptureGraph() {
        if (recording_) abandon();
        if (exec_) cudaGraphExecDestroy(exec_);
        if (graph_) cudaGraphDestroy(graph_);
        if (stream_) cudaStreamDestroy(stream_);
    }

    int start() {
        int rc = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
        if (rc) return rc;
        if ((rc = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal))) return rc;
        recording_ = true;
        launch_stream = stream_;
        return cudaSuccess;
    }

    int finish() {
        if (!recording_) return cudaErrorInvalidValue;
        recording_ = false;
        launch_stream = 0;
        int rc = cudaStreamEndCapture(stream_, &graph_);
        return rc ? rc : cudaGraphInstantiate(&exec_, graph_, 0);
    }

    int replay() const { return exec_ ? cudaGraphLaunch(exec_, 0) : cudaErrorInvalidValue; }

  private:
    // A capture destroyed before qg_graph_end: end it and drop the partial graph.
    void abandon() {
        cudaGraph_t partial = nullptr;
        cudaStreamEndCapture(stream_, &partial);
        if (partial) cudaGraphDestroy(partial);
        recording_ = false;
        launch_stream = 0;
    }

    cudaStream_t stream_ = nullptr;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t exec_ = nullptr;
    bool recording_ = false;
};

}  // namespace

extern "C" int qg_graph_begin(void **graph) {
    // one capture per thread at a time, into an empty handle
    if (!graph || *graph || launch_stream) return cudaErrorInvalidValue;
    auto *g = new (std::nothrow) CaptureGraph;
    if (!g) return cudaErrorMemoryAllocation;
    if (int rc = g->start()) {
        delete g;
        return rc;
    }
    *graph = g;
    return cudaSuccess;
}

extern "C" int qg_graph_end(void *graph) {
    return graph ? static_cast<CaptureGraph *>(graph)->finish() : cudaErrorInvalidValue;
}

extern "C" int qg_graph_launch(void *graph) {
    return graph ? static_cast<const CaptureGraph *>(graph)->replay() : cudaErrorInvalidValue;
}

extern "C" void qg_graph_destroy(void *graph) { delete static_cast<CaptureGraph *>(graph); }

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
