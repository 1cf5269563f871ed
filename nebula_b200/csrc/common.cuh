// Shared helpers for the sm_100a routed-MoE library: the thread-local launch
// stream, GGML row sizes, fp16 decode, and the PTX wrappers for TMA bulk
// copies and mbarriers that the staged kernels use.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
// Entry points keep default visibility; everything else is hidden (-fvisibility=hidden).
#pragma GCC visibility push(default)
#include "../../include/gpu.h"
#pragma GCC visibility pop

namespace nb {

// Launch stream of the calling host thread: 0 (legacy default stream) unless a
// qg_graph_begin capture is active on this thread (reference qwen/gpu.cu:10).
// Its symbol is fixed (nebula_launch_stream) so that code linked into the same
// library - the reference's non-MoE kernels in the qwen.c integration build -
// can launch on the same per-thread stream and join the same captures.
extern thread_local cudaStream_t launch_stream asm("nebula_launch_stream");

constexpr int kExperts = 512;
constexpr int kTop = 10;
constexpr int kMaxTokens = 8192;

// Bytes of one GGML row of `cols` values (reference qwen/gpu.cu:105-113 and
// qwen/cpu.c:17-30). Zero for an unsupported type or a ragged block.
__host__ __device__ inline size_t row_bytes(int type, int cols) {
    if (cols < 1) return 0;
    switch (type) {
    case 0: return (size_t)cols * 4;
    case 1: case 30: return (size_t)cols * 2;
    case 2: case 20: return cols % 32 ? 0 : (size_t)cols / 32 * 18;
    case 6: return cols % 32 ? 0 : (size_t)cols / 32 * 22;
    case 7: return cols % 32 ? 0 : (size_t)cols / 32 * 24;
    case 8: return cols % 32 ? 0 : (size_t)cols / 32 * 34;
    case 12: return cols % 256 ? 0 : (size_t)cols / 256 * 144;
    case 13: return cols % 256 ? 0 : (size_t)cols / 256 * 176;
    case 14: return cols % 256 ? 0 : (size_t)cols / 256 * 210;
    default: return 0;
    }
}

__device__ __forceinline__ float half_at(const unsigned char *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}
__device__ __forceinline__ float half_bits(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xffffu)));
}

// SiLU and sigmoid exactly as the reference writes them (qwen/gpu.cu:88,
// qwen/cpu.c:216): 1/(1+expf(-x)).
__device__ __forceinline__ float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---- PTX wrappers ------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make the initialised barrier visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// One-dimensional TMA bulk copy global -> this CTA's shared memory. dst, src
// and bytes must all be multiples of 16.
__device__ __forceinline__ void tma_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about hint_ns elapse, so waiting warps take no issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Every wait on another role or another CTA gives up after this long.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kWaitHintNs = 20000;
// Bounded wait on an mbarrier phase: a lost completion becomes an error flag
// instead of a hang. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    do {
        if (mbar_try_wait_sleep(bar, parity, kWaitHintNs)) return true;
    } while (global_ns() - t0 < kWaitLimitNs);
    if (err_flag) atomicOr(err_flag, 1);
    return false;
}

}  // namespace nb

#define NB_CHECK_LAUNCH() return (int)cudaGetLastError()
