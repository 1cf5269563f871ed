// Tensor-core (tcgen05) expert kernel for Q4_K and IQ4_NL experts: interface.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace nb {

constexpr int kTcTok = 48;     // tokens per sub-job (token tile of one expert)
constexpr int kTcTokSmall = 24;  // decode tiles with the Q4_K min term on the tensor cores
constexpr int kTcRows = 128;   // weight rows per tile (MMA M)
constexpr int kMaxRanks = 8;   // expert-parallel ranks (GPUs of one box)
constexpr int kMaxParts = 3;   // K parts of one gate/up tile (balanced gate/up work)

// One token tile of one expert. expert < 0 is the shared expert, whose tokens
// are tok0 .. tok0+n-1; a routed sub-job covers pairs[first .. first+n).
struct SubJob {
    int expert, first, n, tok0;
};

struct TcArgs {
    int T, H, F;
    // gate/up rows of H values, Q4_K or (gu_iq4, decode tiles, with IQ4_NL
    // down) IQ4_NL; down rows of F values, Q4_K or (dn_iq4) IQ4_NL; the shared
    // expert (sg/su/sd) in the same formats
    const unsigned char *gate, *up, *down, *sg, *su, *sd;
    size_t grb, drb;
    int gu_iq4, dn_iq4;
    // Gate/up activations: either per token (all_tok = 1: every gate/up tile
    // multiplies all T <= tile tokens and keeps its own columns) or per routed
    // row (rows as for the SwiGLU outputs below, filled by tc_prep_rows_launch).
    int all_tok;
    const __half *x16;     // [T or rows][2][H]: x*s hi, (x*s - hi)*2048 lo, s a power of two per row
    const float *xinv;     // [T or rows][4]: 1/s in element 0
    const float *xsum;     // [T or rows][H/32]: 32-value group sums of x
    const __half *xs16;    // [T][2][H/32] (24-token decode tiles): group sums * s/32, hi and lo as x16
    const SubJob *sub;     // shared sub-jobs first, then routed
    const int *n_sub;      // device count of sub-jobs
    int shared_subs;       // number of shared sub-jobs (known before routing)
    const int *pairs;      // expert-major slot list (t*10+k)
    const float *wts;      // [T*10]
    const int *ids;        // [T*10]
    const int *expect;     // [T]: contributions per token (| bad bit)
    const float *sgate;    // [T] shared-gate logits, or null
    // SwiGLU outputs, one row per routed pair p (row p) and shared token t (row T*10+t):
    __half *mid16;         // [rows][2][F]: v*s hi, (v*s - hi)*2048 lo, s per 128-value tile
    float *midinv;         // [rows][mi_stride]: 1/s per 128-value tile
    int mi_stride;         // F/128 rounded up to a multiple of 4
    float *msum;           // [rows][F/32]: 32-value group sums of v
    float *slots;          // [T*10][H]
    float *shout;          // [T][H]
    float *out;            // [T][H]; null: down tiles only store slot/shared rows (combined by a later kernel)
    int *queue;            // zero between calls (reset by the kernel's last CTA)
    int *tc_ticket;        // zero between calls
    int *gu_done;          // [n_sub] finished gate/up tiles, zeroed by the planner
    int *tilecnt;          // [T][H/128], zeroed by the planner
    int *err;
    int n_experts;         // experts held in gate/up/down
    // Expert parallelism (ep_ranks > 0): the down tiles write their weighted
    // rows into every rank's buffers (peer memory) instead of combining, and
    // the last CTA raises this rank's flag in every rank; a separate combine
    // kernel reduces. ep_cap > 0: the buffers hold two sets of ep_cap tokens'
    // rows and a call uses the set of its epoch's parity; ep_cap = 0: one set
    // indexed by the call's own tokens.
    int ep_ranks, ep_rank, ep_cap;
    // ep_block > 0 (large batches): token t belongs to rank t / ep_block, and a
    // down tile stores each row only into its owner's buffers.
    int ep_block;
    // The shared expert's tokens: [sh_t0, sh_t1), in sub-jobs of the tile size.
    int sh_t0, sh_t1;
    // Balanced gate/up work (gu_part non-null): the routed gate/up superblocks
    // are dealt to the CTAs in equal contiguous ranges, so a tile may be split
    // along K into up to kMaxParts items. Each writes fp32 partial sums
    // [row][kMaxParts][gate|up][F] into gu_part, and the last to finish - counted
    // in gu_pcnt[sub * F/128 + row tile], zero between calls - sums them in part
    // order and finishes the tile. Null: whole tiles only.
    float *gu_part;
    int *gu_pcnt;
    float *ep_slots[kMaxRanks];   // per rank: [2][ep_cap*10][H], or [T*10][H] when ep_cap = 0
    float *ep_shout[kMaxRanks];   // per rank: [2][ep_cap][H], or [T][H]
    int *ep_flags[kMaxRanks];     // per rank: [kMaxRanks] epoch reached by each source rank
    const int *ep_epoch;          // this rank's call epoch (advanced by the combine)
};

struct TcMaps {
    CUtensorMap gate, up, down, sg, su, sd;  // raw Q4_K rows, one superblock x 128 rows per box (down/sd unused for IQ4_NL)
    CUtensorMap bx_hi, bx_lo, bm_hi, bm_lo;  // B rows (activations, SwiGLU outputs), 64 values x tile rows, 128B swizzle
    CUtensorMap sx, sm, ix, im;              // their group sums (8 x tile rows) and scales (4 x tile rows)
    CUtensorMap gx_hi, gx_lo;                // xs16 hi and lo planes (8 x tile rows, no swizzle)
};

// Q4_K gate/up (hidden a multiple of 256, ffn of 128) with Q4_K down (ffn a
// multiple of 256) or IQ4_NL down (ffn up to 640); IQ4_NL gate/up with IQ4_NL
// down for launches whose token tiles are at most 32 (decode).
bool tc_supported(int H, int F, int QG, int QD, int max_tile = kTcTok);
int tc_make_maps(const TcArgs &a, TcMaps &m, int max_tile);
// max_tile: the largest token tile of the launch (sub-jobs, and the split of
// the shared expert's tokens: shared sub-job i covers tokens i*max_tile ..).
int tc_launch(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl, int max_tile);
// x16 / xinv / xsum for T tokens (one CTA per token)
int tc_prep_launch(const float *x, int T, int H, __half *x16, float *xinv, float *xsum, cudaStream_t st);
// The same per routed row: rows [0, *n_pairs) take token pairs[row]/10, rows
// T*10 + t (when shared) token t.
int tc_prep_rows_launch(const float *x, int T, int H, const int *pairs, const int *n_pairs, bool shared, __half *x16,
                        float *xinv, float *xsum, cudaStream_t st);

// Power of two s with max|v*s| in [2^13, 2^14) for mx = max|v| (s = 1 when
// mx is zero, subnormal-small or not finite), and 1/s, both built from the
// exponent bits.
__device__ __forceinline__ void pow2_scale(float mx, float &s, float &inv) {
    const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);  // mx in [2^(E-127), 2^(E-126))
    if (E >= 14 && E <= 254) {
        s = __uint_as_float((uint32_t)(267 - E) << 23);  // 2^(140-E)
        inv = __uint_as_float((uint32_t)(E - 13) << 23);  // 2^(E-140)
    } else {
        s = inv = 1.0f;
    }
}

// Per-token preparation shared by the decode router kernel and the prep kernel:
// scale to max|x*s| in [2^13, 2^14), split into fp16 hi/lo, 32-value group sums
// (and, when xs16 is given, the group sums times s/32 split into fp16 hi/lo).
__device__ inline void tc_prep_token(const float *x, int H, __half *x16, float *xinv, float *xsum,
                                     __half *xs16 = nullptr) {
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
    float s, inv;
    pow2_scale(m, s, inv);
    if (tid == 0) *xinv = inv;
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
        if (lane == 0) {
            xsum[g] = v;
            if (xs16) {
                const float w = v * s * 0.03125f;
                const __half hi = __float2half_rn(w);
                xs16[g] = hi;
                xs16[H / 32 + g] = __float2half_rn((w - __half2float(hi)) * 2048.0f);
            }
        }
    }
}

// The same preparation by one warp (H a multiple of 128): lane l holds values
// 128i + 4l .. 4l+3; a 32-value group spans eight lanes.
__device__ inline void tc_prep_token_warp(const float *x, int H, __half *x16, float *xinv, float *xsum) {
    const int lane = threadIdx.x & 31;
    float m = 0.0f;
    for (int i = 0; i < H / 128; i++) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x + 128 * i) + lane);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    float s, inv;
    pow2_scale(m, s, inv);
    if (lane == 0) *xinv = inv;
    for (int i = 0; i < H / 128; i++) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x + 128 * i) + lane);
        const float f[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
        __half hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            hi[j] = __float2half_rn(f[j]);
            lo[j] = __float2half_rn((f[j] - __half2float(hi[j])) * 2048.0f);
        }
        *reinterpret_cast<uint2 *>(x16 + 128 * i + 4 * lane) = *reinterpret_cast<uint2 *>(hi);
        *reinterpret_cast<uint2 *>(x16 + H + 128 * i + 4 * lane) = *reinterpret_cast<uint2 *>(lo);
        float g = (v.x + v.y) + (v.z + v.w);
#pragma unroll
        for (int d = 4; d; d >>= 1) g += __shfl_xor_sync(0xffffffffu, g, d);
        if ((lane & 7) == 0) xsum[4 * i + (lane >> 3)] = g;
    }
}

}  // namespace nb
