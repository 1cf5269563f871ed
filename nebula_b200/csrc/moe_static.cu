// qg_moe_routed_static: the routed-expert entry point with a library-owned
// scratch in place of the caller's workspace.
//
// It serves callers that cannot allocate device memory where they call the
// MoE step: a runtime whose device memory is reserved in full up front by
// another allocator (a cudaMalloc there fails or steals from that pool), or a
// serving loop that must not take the device-wide synchronisation a
// cudaMalloc/cudaFree can imply. Such callers get a fixed per-device scratch:
// one static __device__ array, found with cudaGetSymbolAddress the first time
// each device is used (with that device current) and zeroed then, because the
// workspace's status words and counters must start at zero (every call leaves
// them at zero again). Nothing here allocates.
//
// The first call on a device does that set-up (a symbol lookup, a memset and a
// synchronisation), so it belongs before any stream capture. All calls on a
// device share the one scratch: calls that overlap (from other host threads or
// on other streams) race on it.
//
// Errors: a caller of this entry point has no workspace pointer, so it can
// neither read qg_moe_status nor zero the scratch after a bounded wait ran out
// (the only device-side error; the counters of such a call stay where they
// stopped). Each call therefore starts with a one-CTA kernel that clears the
// scratch's status words and counters when the previous call left the error
// word set; the failed call's own output rows are not repaired. Invalid routes
// are reported as NaN rows, as on every MoE entry point. The per-device address
// is looked up once per process: cudaDeviceReset on a device that has used this
// entry point is not supported.
#include <mutex>
#include "moe_decode.cuh"

namespace {

// Largest workspace this entry point serves (qg_moe_workspace_bytes): batches
// of up to 28 tokens at hidden 2048 / FFN 512 and up to 23 at 2560 / 640;
// verify batches (T <= 17, 4.7 MiB at 2048 / 512) fit both.
constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_moe_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void *g_scratch[kMaxDevices];

// This device's scratch, looked up and zeroed on first use.
int device_scratch(void **out) {
    int dev = 0;
    int rc = cudaGetDevice(&dev);
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch[dev]) {
        void *p = nullptr;
        if ((rc = cudaGetSymbolAddress(&p, g_moe_scratch))) return rc;
        if ((rc = cudaMemset(p, 0, kStaticScratchBytes))) return rc;
        if ((rc = cudaDeviceSynchronize())) return rc;
        g_scratch[dev] = p;
    }
    *out = g_scratch[dev];
    return 0;
}

// Clears the status words and counters (the fixed prefix) when the error word is set.
__global__ void static_recover_kernel(unsigned char *scratch) {
    __shared__ int s_err;
    if (threadIdx.x == 0) s_err = *reinterpret_cast<volatile int *>(scratch + offsetof(nb::DecHdr, error));
    __syncthreads();
    if (!s_err) return;
    int4 *p = reinterpret_cast<int4 *>(scratch);
    for (size_t i = threadIdx.x; i < nb::kPrefixBytes / sizeof(int4); i += blockDim.x) p[i] = make_int4(0, 0, 0, 0);
}

}  // namespace

extern "C" int qg_moe_routed_static(float *out, const float *x, const int *ids, const float *weights, int tokens,
                                    const void *gate, int gate_type, const void *up, int up_type, const void *down,
                                    int down_type, int hidden, int ffn) {
    size_t need = 0;
    int rc = qg_moe_workspace_bytes(tokens, hidden, ffn, &need);
    if (rc) return rc;
    if (need > kStaticScratchBytes) return cudaErrorInvalidValue;  // too large for the static scratch
    void *ws = nullptr;
    if ((rc = device_scratch(&ws))) return rc;
    static_recover_kernel<<<1, 256, 0, nb::launch_stream>>>(static_cast<unsigned char *>(ws));
    if ((rc = cudaGetLastError())) return rc;
    return qg_moe_routed(out, x, ids, weights, tokens, gate, gate_type, up, up_type, down, down_type, hidden, ffn,
                         ws);
}
