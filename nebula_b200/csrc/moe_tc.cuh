// Tensor-core (tcgen05) expert kernel for Q4_K experts: interface.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace nb {

constexpr int kTcTok = 64;     // tokens per sub-job (token tile of one expert)
constexpr int kTcRows = 128;   // weight rows per tile (MMA M)

// One token tile of one expert. expert < 0 is the shared expert, whose tokens
// are tok0 .. tok0+n-1; a routed sub-job covers pairs[first .. first+n).
struct SubJob {
    int expert, first, n, tok0;
};

struct TcArgs {
    int T, H, F;
    const unsigned char *gate, *up, *down, *sg, *su, *sd;  // Q4_K experts (+ shared), gate/up rows hold H values
    size_t grb, drb;
    const __half *x16;     // [T][2][H]: x*s hi, (x*s - hi)*2048 lo, s a power of two per token
    const float *xinv;     // [T]: 1/s
    const float *xsum;     // [T][H/32]: 32-value group sums of x
    const SubJob *sub;     // shared sub-jobs first, then routed
    const int *n_sub;      // device count of sub-jobs
    int shared_subs;       // number of shared sub-jobs (known before routing)
    const int *pairs;      // expert-major slot list (t*10+k)
    const float *wts;      // [T*10]
    const int *ids;        // [T*10]
    const int *expect;     // [T]: contributions per token (| bad bit)
    const float *sgate;    // [T] shared-gate logits, or null
    float *mid;            // [(T*10+T)][F] fp32: routed pair p -> row p, shared token t -> row T*10+t
    __half *mid16;         // [(T*10+T)][2][F]
    float *midinv, *msum;  // [(T*10+T)], [(T*10+T)][F/32]
    float *slots;          // [T*10][H]
    float *shout;          // [T][H]
    float *out;            // [T][H]
    int *queue;            // zero between calls (reset by the kernel's last CTA)
    int *tc_ticket;        // zero between calls
    int *gu_done;          // [n_sub], zeroed by the planner
    int *tilecnt;          // [T][H/128], zeroed by the planner
    int *err;
};

struct TcMaps {
    CUtensorMap gate, up, down, sg, su, sd;
};

bool tc_supported(int H, int F, int QG, int QD);
size_t tc_smem_bytes();
int tc_make_maps(const TcArgs &a, TcMaps &m);
int tc_launch(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl);
// x16 / xinv / xsum for T tokens (one CTA per token)
int tc_prep_launch(const float *x, int T, int H, __half *x16, float *xinv, float *xsum, cudaStream_t st);

// Per-token preparation shared by the decode router kernel and the prep kernel:
// scale to max|x*s| in [2^13, 2^14), split into fp16 hi/lo, 32-value group sums.
__device__ inline void tc_prep_token(const float *x, int H, __half *x16, float *xinv, float *xsum) {
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float m = 0.0f;
    for (int i = tid; i < H; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
#pragma unroll
    for (int d = 16; d; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = 0.0f;
    for (int w = 0; w < nw; w++) m = fmaxf(m, red[w]);
    __syncthreads();
    int e = 0;
    if (m > 0.0f && isfinite(m)) frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
    const float s = (m > 0.0f && isfinite(m)) ? ldexpf(1.0f, 14 - e) : 1.0f;
    if (tid == 0) *xinv = 1.0f / s;
    for (int i = tid; i < H; i += blockDim.x) {
        const float v = x[i] * s;
        const __half hi = __float2half_rn(v);
        const __half lo = __float2half_rn((v - __half2float(hi)) * 2048.0f);
        x16[i] = hi;
        x16[H + i] = lo;
    }
    for (int g = warp; g < H / 32; g += nw) {
        float v = x[g * 32 + lane];
#pragma unroll
        for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
        if (lane == 0) xsum[g] = v;
    }
}

}  // namespace nb
