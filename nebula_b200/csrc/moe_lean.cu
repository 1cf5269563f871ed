// Lean decode layer for batches of 1 or 2 tokens at hidden 2048 / ffn 512 with
// Q4_K experts, and of 1 to 4 tokens at Nebula's 2560 / 640 with Q4_K gate/up and
// IQ4_NL down: the whole routed-MoE layer
// (router GEMV, top-10, gate/up + SwiGLU, down x route weight, combine and the
// gated shared expert) in ONE cooperative kernel of one CTA per SM.
//
// At these batch sizes the tensor cores have nothing to multiply (N = T), and
// the general decode path's time is its chain of hand-offs: the router kernel,
// the plan, the work queue, per-chunk role hand-offs and per-tile tails. Here
// every warp streams weight rows with all of a row's loads issued at once, and
// the phases are separated by two grid-wide barriers:
//   1. the router GEMV (512 rows + the shared-gate row), one warp per row, in the
//      reference's 32-lane order, so the logits and expert ids are bit-exact;
//   2. every CTA computes the top-10 of each token itself (identical results),
//      and gate/up + SwiGLU rows are dealt to all warps: (token, slot, row) of
//      each routed pair and of the shared expert -> mid;
//   3. each warp takes output rows: for one token and one row it reads the ten
//      routed experts' down rows and the shared expert's down row, and sums
//      w_k * (down_k . mid_k) plus sigmoid(gate) * (shared . mid) - the combine
//      happens in the same pass, with no slot rows.
// Each weight row is copied into the warp's shared memory with 16-byte loads
// (all of a row's loads in flight at once), then lane j multiplies byte j of
// every 32-byte block of quantized values, so the activations the lanes read
// are consecutive (no bank conflicts). Expert outputs match the reference within
// the float tolerance of the path (each weight is d*sc*q - dmin*m with one
// rounding, summed in another order than the reference's); routing is bitwise
// the reference's.
//
// The barriers are waits on other CTAs, so the kernel is launched cooperatively
// (every CTA resident) and each wait gives up after a bound, raising the error
// word instead of hanging; after such an error the workspace must be zeroed
// again (as after any error), which also restarts the barrier counter.
#include "moe_decode.cuh"
#include "quant.cuh"
#include "route.cuh"

using namespace nb;

namespace {


constexpr int cmax(int a, int b) { return a > b ? a : b; }
// One instantiation's shape: hidden H, ffn F, Q4_K gate/up, down Q4_K (QD 12) or IQ4_NL (QD 20).
template <int H, int F, int QD>
struct LeanShape {
    // threads per CTA (one CTA per SM): 512 for Q4_K down, whose items are short; 768 for
    // IQ4_NL down, whose per-value decoding gains from more warps to hide latency (measured:
    // 768 threads made the 2560/640 layer 18% faster at T=1 and the 2048/512 one 5% slower)
    static constexpr int kThreads = QD == 20 ? 768 : 512, kWarps = kThreads / 32;
    // tokens the layer takes here: 4 for the 2560/640 mix, 2 for 2048/512, where the
    // tensor-core decode path is faster from 3 tokens on. Each shape has an instance
    // for up to 2 tokens and the mix one for 3 or 4 (kernel parameter MT): sized for
    // 4, the T = 1 and 2 launches measured 2-3 % slower
    static constexpr int kMaxT = QD == 20 ? 4 : 2;
    static constexpr int kSbH = H / 256, kChH = kSbH * 9;  // gate/up: Q4_K superblocks, 16-byte chunks per row
    static constexpr int kDnRow = QD == 12 ? F / 256 * 144 : F / 32 * 18;  // bytes of a down row
    static constexpr int kSbF = QD == 12 ? F / 256 : 0;     // Q4_K superblocks per down row
    // down rows are copied 16 bytes at a time (Q4_K), or 8 (IQ4_NL rows are only 8-byte aligned)
    static constexpr int kDnUnit = QD == 12 ? 16 : 8, kChF = kDnRow / kDnUnit;
    // gate/up: the two rows' chunks over 32 lanes; down: eleven rows' units
    static constexpr int kGuPer = (2 * kChH + 31) / 32, kDnPer = (11 * kChF + 31) / 32;
    // shared memory: activations (x [T][H], then mid [P][F]) for the launch's T tokens,
    // then one region per warp. Each launch asks for only what its T needs: the rest of
    // the SM's 256 KB stays L1, which holds the weight loads in flight
    static constexpr __host__ __device__ int act_floats(int t) { return cmax(t * H, (t * kTop + t) * F); }
    // a warp's region holds its item's weight rows, then their Q4_K superblock scales
    // (gate/up and down items never overlap in time, so the two phases share it)
    static constexpr int kGuRows = 2 * kChH * 16, kDnRows = 11 * kDnRow;
    static constexpr int kWBuf = (cmax(kGuRows + 2 * kSbH * 64, kDnRows + 11 * kSbF * 64) + 127) / 128 * 128;
    static constexpr __host__ __device__ int smem(int t) { return act_floats(t) * 4 + kWarps * kWBuf; }
    static_assert(kGuRows % 16 == 0 && (kDnRows % 16 == 0 || QD == 20), "scales 16-byte aligned");
    static_assert(smem(kMaxT) <= 226 * 1024, "one CTA per SM, with room for the static arrays");
    static_assert(H % 32 == 0 && F % 32 == 0, "warp regions 128-byte aligned for every T");
    static_assert(H % 256 == 0 && F % 256 == 0 || QD == 20, "Q4_K rows");
    static_assert(kDnRow % kDnUnit == 0 && (2 * kChH * 16) % 16 == 0, "copy units");
};

// Grid-wide barrier over the resident CTAs (cooperative launch) on one 64-bit
// counter that only grows: every CTA adds 1 per barrier with a non-returning
// release add (no serialised returning atomics), and barrier k of a launch is
// passed once the counter reaches base + k * grid. A launch makes exactly two
// barriers, so base = the counter rounded down to a multiple of 2 * grid when the
// CTA starts (the counter then holds at most grid - 1 arrivals of this launch).
// Bounded: false (and error bit 4) after kWaitLimitNs.
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ bool grid_barrier(unsigned long long *ctr, unsigned long long target, int *err, volatile int *s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
        if (ld_acquire_u64(ctr) < target) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_u64(ctr) < target) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(err, 4);
                    *s_ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return *s_ok != 0;
}

// (d*sc, dmin*m) of every sub-block of nh superblocks whose rows sit in the
// warp's buffer (row r of `rb` bytes, sbs superblocks each), one (superblock,
// sub-block) per lane and step: scl[h*8 + g] for superblock h = r*sbs + sb.
__device__ __forceinline__ void q4k_scales(const unsigned char *buf, int rb, int sbs, int nh, float2 *scl) {
    for (int pg = threadIdx.x & 31; pg < nh * 8; pg += 32) {
        const int h = pg >> 3, g = pg & 7, j = g & 3;
        const unsigned char *hd = buf + (h / sbs) * rb + (h % sbs) * 144;
        // the 6-bit scale and min of sub-block g (k_scale_min's layout), selected without branches
        const int b0 = hd[4 + j], b4 = hd[8 + j], b8 = hd[12 + j];
        const int sc = g < 4 ? (b0 & 63) : ((b8 & 15) | ((b0 >> 6) << 4));
        const int m = g < 4 ? (b4 & 63) : ((b8 >> 4) | ((b4 >> 6) << 4));
        scl[pg] = make_float2(half_at(hd) * static_cast<float>(sc), half_at(hd + 2) * static_cast<float>(m));
    }
}

// Two Q4_K values of byte b (low nibble: sub-block 2i, high: 2i+1) as exact floats.
__device__ __forceinline__ float2 nibbles(unsigned b) {
    return __fadd2_rn(make_float2(__uint_as_float((b & 15u) | 0x4B000000u), __uint_as_float((b >> 4) | 0x4B000000u)),
                      make_float2(-8388608.0f, -8388608.0f));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

}  // namespace

namespace {

// Router GEMV (and the shared-gate row) for NT tokens: warp gw takes rows gw, gw + nw, ...;
// lane j adds k = j, j+32, ... in order and the lanes are summed by lane_tree, the
// reference's order (qwen/gpu.cu:89-92).
template <int NT, int H>
__device__ __forceinline__ void router_rows(const DecArgs &a, const float *act, int gw, int nw, int lane) {
    const int rrows = kExperts + (a.s_router ? 1 : 0);
    for (int row = gw; row < rrows; row += nw) {
        const float *w = row < kExperts ? a.router + (size_t)row * H : a.s_router;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        constexpr int kIter = H / 32;  // columns per lane
#pragma unroll
        for (int h = 0; h < kIter; h += 64) {
            float wv[64];  // up to 64 of a row's loads in flight before the first multiply-add
#pragma unroll
            for (int i = 0; i < 64; i++)
                if (h + i < kIter) wv[i] = __ldg(w + (h + i) * 32 + lane);
#pragma unroll
            for (int i = 0; i < 64; i++) {
                if (h + i < kIter) {
                    const int k = (h + i) * 32 + lane;
#pragma unroll
                    for (int t = 0; t < NT; t++) acc[t] = __fmaf_rn(wv[i], act[t * H + k], acc[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float s = lane_tree(acc[t]);
            if (lane == 0) {
                if (row < kExperts) a.logits[t * kExperts + row] = s;
                else a.sgate[t] = s;
            }
        }
    }
}

// router_rows<T> for the runtime T in 1..NT
template <int NT, int H>
__device__ __forceinline__ void router_rows_upto(const DecArgs &a, const float *act, int T, int gw, int nw, int lane) {
    if constexpr (NT > 1) {
        if (T < NT) {
            router_rows_upto<NT - 1, H>(a, act, T, gw, nw, lane);
            return;
        }
    }
    router_rows<NT, H>(a, act, gw, nw, lane);
}

template <int H, int F, int QD, int MT>
__global__ void __launch_bounds__(LeanShape<H, F, QD>::kThreads, 1) lean_moe_kernel(DecArgs a) {
    using S = LeanShape<H, F, QD>;
    constexpr int kLeanThreads = S::kThreads, kLeanWarps = S::kWarps;
    constexpr int kLeanH = H, kLeanF = F, kSbH = S::kSbH, kChH = S::kChH, kSbF = S::kSbF, kChF = S::kChF,
                  kGuPer = S::kGuPer, kDnPer = S::kDnPer,
                  kWBuf = S::kWBuf;
    extern __shared__ __align__(16) float lsm[];
    float *act = lsm;
    static_assert(MT >= 1 && MT <= S::kMaxT, "token limit of the instance");
    constexpr int kLeanMaxT = MT;
    unsigned char *wbuf = reinterpret_cast<unsigned char *>(lsm + S::act_floats(a.T)) + (threadIdx.x >> 5) * kWBuf;
    float2 *wscl_gu = reinterpret_cast<float2 *>(wbuf + S::kGuRows);  // scales after the rows of each phase
    float2 *wscl_dn = reinterpret_cast<float2 *>(wbuf + S::kDnRows);
    __shared__ int s_ids[kLeanMaxT * kTop];
    __shared__ float s_w[kLeanMaxT * kTop], s_sig[kLeanMaxT];
    __shared__ int s_ok;
    __shared__ float s_lut[16];  // IQ4_NL code book
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < 16) s_lut[tid] = static_cast<float>(kIq4nl[tid]);
    const int T = a.T, gw = blockIdx.x * kLeanWarps + warp, nw = gridDim.x * kLeanWarps;
    const bool shared = a.sg != nullptr;
    unsigned long long *ctr = &a.ctr->lean_barrier;
    int *err = &a.hdr->error;
    __shared__ unsigned long long s_base;
    if (tid == 0) {
        s_ok = 1;
        const unsigned long long c0 = ld_acquire_u64(ctr), round = 2ull * gridDim.x;
        s_base = c0 - c0 % round;
    }
    for (int i = tid; i < T * kLeanH / 4; i += kLeanThreads)
        reinterpret_cast<float4 *>(act)[i] = __ldg(reinterpret_cast<const float4 *>(a.x) + i);
    __syncthreads();

    // 1. router GEMV (and the shared-gate row), compiled for the launch's token count
    router_rows_upto<MT, H>(a, act, T, gw, nw, lane);
    if (!grid_barrier(ctr, s_base + gridDim.x, err, &s_ok)) return;

    // 2. top-10 of every token, in every CTA
    if (warp < T) route_token_warp(a.logits + warp * kExperts, a.bias, s_ids + warp * kTop, s_w + warp * kTop);
    if (tid < T && shared) s_sig[tid] = sigmoidf_ref(__ldcg(a.sgate + tid));
    __syncthreads();
    if (blockIdx.x == 0) {
        if (tid < T * kTop) {
            a.ids[tid] = s_ids[tid];
            a.wts[tid] = s_w[tid];
        }
        if (warp == 0) {  // status words: pairs computed, distinct experts, tokens with NaN rows
            int first = 0;    // ids that no earlier slot holds, one slot per lane and step
            for (int i = lane; i < T * kTop; i += 32) {
                const int e = s_ids[i];
                bool f = e >= 0;
                for (int j = 0; j < i && f; j++) f = s_ids[j] != e;
                first += f;
            }
            const int used = (int)__reduce_add_sync(0xffffffffu, (unsigned)first);
            if (lane == 0) {
                int pairs = 0, bad = 0;
                for (int t = 0; t < T; t++) {
                    if (s_ids[t * kTop] < 0) bad++;
                    else pairs += kTop;
                }
                a.hdr->n_pairs = pairs;
                a.hdr->n_used = used;
                a.hdr->invalid_tokens = bad;
            }
        }
    }
    //    gate/up + SwiGLU: item = (pair p, row); pairs 0..10T-1 routed, 10T.. the shared expert's
    const int P = T * kTop + (shared ? T : 0);
    // items in order it = gw, gw + nw, ...; the next item's loads are issued before
    // this item's multiply-adds, so its latency overlaps them
    auto gu_src = [&](int it, const unsigned char *&g, const unsigned char *&u, int &t) {
        const int p = it / kLeanF, row = it % kLeanF;
        if (p < T * kTop) {
            t = p / kTop;
            const int e = s_ids[p];
            if (e < 0) return false;  // a token whose logits were not finite: no contributions
            g = a.gate + ((size_t)e * kLeanF + row) * a.grb;
            u = a.up + ((size_t)e * kLeanF + row) * a.grb;
        } else {
            t = p - T * kTop;
            g = a.sg + (size_t)row * a.grb;
            u = a.su + (size_t)row * a.grb;
        }
        return true;
    };
    auto gu_load = [&](const unsigned char *g, const unsigned char *u, uint4 (&v)[kGuPer]) {
#pragma unroll
        for (int i = 0; i < kGuPer; i++) {
            const int f = lane + 32 * i;
            if (f < 2 * kChH) v[i] = __ldg(reinterpret_cast<const uint4 *>(f < kChH ? g : u) + (f < kChH ? f : f - kChH));
        }
    };
    const int total = P * kLeanF;
    int it = gw, t = 0;
    const unsigned char *g = nullptr, *u = nullptr;
    while (it < total && !gu_src(it, g, u, t)) it += nw;
    uint4 v[kGuPer];
    if (it < total) gu_load(g, u, v);
    while (it < total) {
#pragma unroll
        for (int i = 0; i < kGuPer; i++) {
            const int f = lane + 32 * i;
            if (f < 2 * kChH) reinterpret_cast<uint4 *>(wbuf)[f] = v[i];  // gate row at byte 0, up row at kChH*16
        }
        const int p = it / kLeanF, row = it % kLeanF;
        int nx = it + nw, tn = 0;
        while (nx < total && !gu_src(nx, g, u, tn)) nx += nw;
        if (nx < total) gu_load(g, u, v);
        __syncwarp();
        q4k_scales(wbuf, kChH * 16, kSbH, 2 * kSbH, wscl_gu);
        __syncwarp();
        // lane j takes byte j of every 32-byte q block: its activations are consecutive
        // across lanes, and each is loaded once for the gate and the up row
        const float *xt = act + t * kLeanH;
        float2 ag = make_float2(0.0f, 0.0f), au = make_float2(0.0f, 0.0f);
#pragma unroll 2
        for (int sb = 0; sb < kSbH; sb++) {
            const unsigned char *qg = wbuf + sb * 144 + 16, *qu = qg + kChH * 16;
            const float4 *sg = reinterpret_cast<const float4 *>(wscl_gu + sb * 8);
            const float4 *su = reinterpret_cast<const float4 *>(wscl_gu + (kSbH + sb) * 8);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 x = make_float2(xt[sb * 256 + 64 * i + lane], xt[sb * 256 + 64 * i + 32 + lane]);
                const float4 s = sg[i], z = su[i];  // d*sc, dmin*m of sub-blocks 2i and 2i+1
                const float2 wg = __ffma2_rn(make_float2(s.x, s.z), nibbles(qg[32 * i + lane]), make_float2(-s.y, -s.w));
                const float2 wu = __ffma2_rn(make_float2(z.x, z.z), nibbles(qu[32 * i + lane]), make_float2(-z.y, -z.w));
                ag = __ffma2_rn(wg, x, ag);
                au = __ffma2_rn(wu, x, au);
            }
        }
        const float gs = warp_sum(ag.x + ag.y), us = warp_sum(au.x + au.y);
        if (lane == 0) a.mid[(size_t)p * kLeanF + row] = (gs * sigmoidf_ref(gs)) * us;
        __syncwarp();  // the buffer and the scales are rewritten by the next item
        it = nx;
        t = tn;
    }
    if (!grid_barrier(ctr, s_base + 2ull * gridDim.x, err, &s_ok)) return;

    // 3. down rows x route weights, summed over the ten experts, plus the gated shared expert
    for (int i = tid; i < P * kLeanF / 4; i += kLeanThreads)
        reinterpret_cast<float4 *>(act)[i] = __ldcg(reinterpret_cast<const float4 *>(a.mid) + i);
    __syncthreads();
    const int nk = kTop + (shared ? 1 : 0);
    for (int it = gw; it < T * kLeanH; it += nw) {
        const int t = it / kLeanH, row = it % kLeanH;
        if (s_ids[t * kTop] < 0) {
            if (lane == 0) a.out[(size_t)t * kLeanH + row] = __int_as_float(0x7fc00000);
            continue;
        }
        float acc = 0.0f;
        if constexpr (QD == 12) {
            uint4 v[kDnPer];
#pragma unroll
            for (int i = 0; i < kDnPer; i++) {
                const int f = lane + 32 * i;
                if (f < nk * kChF) {
                    const int k = f / kChF, c = f % kChF;
                    const unsigned char *rp = k < kTop ? a.down + ((size_t)s_ids[t * kTop + k] * kLeanH + row) * a.drb
                                                       : a.sd + (size_t)row * a.drb;
                    v[i] = __ldg(reinterpret_cast<const uint4 *>(rp) + c);
                    reinterpret_cast<uint4 *>(wbuf)[f] = v[i];  // row k at byte k*kChF*16
                }
            }
            __syncwarp();
            q4k_scales(wbuf, kChF * 16, kSbF, nk * kSbF, wscl_dn);
            __syncwarp();
            for (int k = 0; k < nk; k++) {
                const int pi = k < kTop ? t * kTop + k : T * kTop + t;
                const float wk = k < kTop ? s_w[t * kTop + k] : s_sig[t];
                const float *mt = act + pi * kLeanF;
                float2 a2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int sb = 0; sb < kSbF; sb++) {
                    const unsigned char *q = wbuf + k * kChF * 16 + sb * 144 + 16;
                    const float4 *sc = reinterpret_cast<const float4 *>(wscl_dn + (k * kSbF + sb) * 8);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 s = sc[i];
                        const float2 m = make_float2(mt[sb * 256 + 64 * i + lane], mt[sb * 256 + 64 * i + 32 + lane]);
                        const float2 w = __ffma2_rn(make_float2(s.x, s.z), nibbles(q[32 * i + lane]), make_float2(-s.y, -s.w));
                        a2 = __ffma2_rn(w, m, a2);
                    }
                }
                acc = __fmaf_rn(wk, a2.x + a2.y, acc);
            }
        } else {
            // IQ4_NL rows: 8-byte units. Half-warp h takes block 2m+h of each pair of
            // blocks; lane j of it reads code byte j (values j and j+16 of the block),
            // the two halves loading their activations in orders that use different banks
#pragma unroll
            for (int i = 0; i < kDnPer; i++) {
                const int f = lane + 32 * i;
                if (f < nk * kChF) {
                    const int k = f / kChF, c = f % kChF;
                    const unsigned char *rp = k < kTop ? a.down + ((size_t)s_ids[t * kTop + k] * kLeanH + row) * a.drb
                                                       : a.sd + (size_t)row * a.drb;
                    reinterpret_cast<uint2 *>(wbuf)[f] = __ldg(reinterpret_cast<const uint2 *>(rp) + c);
                }
            }
            __syncwarp();
            for (int k = 0; k < nk; k++) {
                const int pi = k < kTop ? t * kTop + k : T * kTop + t;
                const float wk = k < kTop ? s_w[t * kTop + k] : s_sig[t];
                const float *mt = act + pi * kLeanF;
                const unsigned char *rw = wbuf + k * S::kDnRow;
                float a2 = 0.0f;
                const int hb = lane >> 4, j = lane & 15;
#pragma unroll 5
                for (int m = 0; m < kLeanF / 64; m++) {
                    const int b = 2 * m + hb;
                    const unsigned char *blk = rw + b * 18;
                    const unsigned q = blk[2 + j];
                    const float d = half_at(blk);
                    // first the value at j + 16*hb (low nibble for h = 0, high for h = 1), then the other
                    const float w1 = d * s_lut[(q >> (4 * hb)) & 15u], w2 = d * s_lut[(q >> (4 - 4 * hb)) & 15u];
                    a2 = __fmaf_rn(w1, mt[b * 32 + j + 16 * hb], a2);
                    a2 = __fmaf_rn(w2, mt[b * 32 + j + 16 - 16 * hb], a2);
                }
                acc = __fmaf_rn(wk, a2, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) a.out[(size_t)t * kLeanH + row] = acc;
        __syncwarp();
    }
}

// Taken up to each shape's kMaxT tokens. On the 48-layer stack (2048/512, Q4_K,
// with the routing skew) it gives 706 / 938 tokens/s at T = 1 / 2 against 356 / 687
// for the tensor-core decode path, which stays faster at T = 3 and 4 there (1,000 /
// 1,296 tokens/s). A 4-token instance of this shape took 63.6 / 78.9 us per layer
// with unbiased routing, against 71.8 / 84.0 us on the tensor-core path; the skew
// leaves fewer distinct experts, which favours the tensor-core path. At 2560/640 it takes
// 42.9 / 71.9 / 102.5 / 119.6 us per layer at T = 1..4, against 98.7 / 100.5 /
// 128.8 / 156.5 us on the tensor-core path (8 rotated layers, graph replay).

bool lean_shape(const DecArgs &a, int &which) {
    if (a.QG != 12) return false;
    if (a.H == 2048 && a.F == 512 && a.QD == 12) which = 0;       // the benchmark configurations
    else if (a.H == 2560 && a.F == 640 && a.QD == 20) which = 1;  // Nebula's production mix
    else return false;
    return true;
}

template <int H, int F, int QD, int MT>
int lean_launch(const DecArgs &a, cudaStream_t st, int dev) {
    using S = LeanShape<H, F, QD>;
    auto k = lean_moe_kernel<H, F, QD, MT>;
    // once per device: the shared-memory attribute, and the grid (one CTA per SM, all
    // resident: the grid barriers wait on every CTA)
    static int grid[64];
    if (!grid[dev]) {
        int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::smem(MT));
        if (rc) return rc;
        int sms = 0, occ = 0;
        if ((rc = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return rc;
        if ((rc = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, S::kThreads, S::smem(MT)))) return rc;
        if (occ < 1) return cudaErrorCooperativeLaunchTooLarge;
        grid[dev] = sms;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid[dev]);
    cfg.blockDim = dim3(S::kThreads);
    cfg.dynamicSmemBytes = S::smem(a.T);  // 1 <= a.T <= MT (lean_run)
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace

namespace nb {

bool lean_supported(const DecArgs &a) {
    int which = 0;
    if (a.T < 1 || !lean_shape(a, which) || !a.router || a.ep_ranks || a.ep_local) return false;
    if (a.T > (which == 0 ? LeanShape<2048, 512, 12>::kMaxT : LeanShape<2560, 640, 20>::kMaxT)) return false;
    int dev = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    return coop != 0;
}

int lean_run(const DecArgs &a, cudaStream_t st) {
    int dev = 0, which = 0, rc = cudaGetDevice(&dev);
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!lean_shape(a, which)) return cudaErrorInvalidValue;
    if (a.T < 1 || a.T > (which == 0 ? LeanShape<2048, 512, 12>::kMaxT : LeanShape<2560, 640, 20>::kMaxT))
        return cudaErrorInvalidValue;
    if (which == 0) return lean_launch<2048, 512, 12, 2>(a, st, dev);
    return a.T <= 2 ? lean_launch<2560, 640, 20, 2>(a, st, dev) : lean_launch<2560, 640, 20, 4>(a, st, dev);
}

}  // namespace nb
