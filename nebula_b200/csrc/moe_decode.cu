// Decode / speculative-verify routed MoE (small token batches): two kernels
// per layer, chained with programmatic dependent launch.
//
//  K1 dec_router_kernel: one CTA per 4 router rows (+ one for the shared
//     gate row). Stages x and its rows in shared memory with TMA bulk copies
//     and computes logits in the reference's 32-lane order (bitwise equal to
//     qc_matmul, so expert ids are bit-exact). The last T CTAs to finish
//     (atomic ticket) each run the top-10 routing of one token
//     (qwen/gpu.cu:456-465 semantics) once all logits are in, and the last
//     of them builds the plan: per-expert token lists in ascending token
//     order, offsets, the used-expert list and per-token contribution counts.
//     The first T CTAs to finish each write one token's activations in the
//     layout the expert kernel reads (fp16 hi/lo or pair-interleaved, plus
//     32-value group sums). Without a router (qg_moe_routed) CTA t < T
//     writes x[t]'s activations and the last CTA plans from the given
//     ids/weights.
//
//  K2 dec_experts_kernel: persistent, one CTA per SM of eight warps. Thread 0
//     also produces: it claims work items from a device queue and streams
//     their weight tiles into a two-stage shared-memory ring with TMA bulk
//     copies (the first two tiles are fetched while K1 still runs), refilling
//     a stage as soon as all warps have released it. Items in
//     queue order: gate/up tiles of 32 gate + 32 up rows (shared expert
//     first), then down tiles of 128-256 rows. A gate/up tile writes
//     mid = SiLU(g)*u for every token of its expert (qwen/cpu.c:209-217); a
//     down tile waits for its expert's gate/up tiles, writes
//     w[t][k] * (W_down mid) into slot rows (qwen/cpu.c:219-225), and the
//     last contribution to a (token, row tile) sums the ten slots in rank
//     order and adds the gated shared expert (qwen/cpu.c:227-231,
//     qwen/gpu.cu:552).
//
// Dot products use the group-factored form sum_g d*sc_g*(sum q x) -
// dmin*m_g*(sum x) with packed f32x2 FMAs; results match the reference
// within float tolerance (the router stays bit-exact).
//
// Every wait is bounded: a timeout sets the sticky error word read by
// qg_moe_status rather than hanging. Counters are returned to zero by the
// last CTA of each kernel; the workspace must be zero-filled once after
// allocation.
#include <algorithm>
#include "quant.cuh"
#include "route.cuh"
#include "moe_decode.cuh"

using namespace nb;

namespace {

constexpr int kRouterRows = 4;   // router rows per K1 CTA
constexpr int kK1Threads = 512;  // one expert per thread in the plan
constexpr int kGuRows = 32;      // gate rows (and up rows) per gate/up tile
constexpr int kConsumers = 8;    // warps in K2; thread 0 also produces
constexpr int kK2Threads = kConsumers * 32;
constexpr int kStages = 2;
constexpr int kTP = 2;           // tokens per pass in K2
constexpr uint32_t kBadBit = 1u << 16;

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Position of value l (0..63) of a 64-value unit in the pair-interleaved
// layout: Q4_K pairs (l, l+32) share a byte; IQ4_NL pairs (j, j+16) inside
// each 32-value block.
template <int Q>
__device__ __forceinline__ int pair_pos(int l) {
    if (Q == 12) return l < 32 ? 2 * l : 2 * (l - 32) + 1;
    int blk = l >> 5, j = l & 31;
    return blk * 32 + (j < 16 ? 2 * j : 2 * (j - 16) + 1);
}

__device__ bool wait_geq(const int *p, int target, int *err) {
    const uint64_t t0 = global_ns();
    do {
        if (ld_acquire(p) >= target) return true;
        __nanosleep(64);
    } while (global_ns() - t0 < kWaitLimitNs);
    atomicOr(err, 2);
    return false;
}

// ------------------------------------------------------------------ K1
template <int QG, int TMAX>
__global__ void __launch_bounds__(kK1Threads) dec_router_kernel(DecArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    __shared__ int s_last;
    float *xs = reinterpret_cast<float *>(smem);  // [T][H]
    float *wr = xs + (size_t)a.T * a.H;           // [rows][H]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T, H = a.H;
    // token t's activations in the layout the expert kernel reads (src: x[t])
    auto prep_token = [&](int t, const float *src) {
        if (a.use_tc) {
            tc_prep_token(src, H, a.x16 + (size_t)t * 2 * H, a.xinv + (size_t)t * 4, a.xsum + (size_t)t * (H / 32),
                          a.xs16 + (size_t)t * (H / 16));
        } else {
            float *dst = a.xpair + (size_t)t * H;
            for (int i = tid; i < H; i += blockDim.x) dst[(i >> 6) * 64 + pair_pos<QG>(i & 63)] = src[i];
            for (int g = warp; g < H / 32; g += blockDim.x / 32) {
                float v = src[g * 32 + lane];
#pragma unroll
                for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
                if (lane == 0) a.xsum[t * (H / 32) + g] = v;
            }
        }
    };
    int row0 = 0, nrows = 0;
    if (a.router) {
        if (blockIdx.x < kExperts / kRouterRows) {
            row0 = blockIdx.x * kRouterRows;
            nrows = kRouterRows;
        } else if (a.s_router && blockIdx.x == kExperts / kRouterRows) {
            row0 = kExperts;
            nrows = 1;
        }
    }
    const bool stage_x = nrows > 0 || (int)blockIdx.x < T;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    grid_dep_wait();    // earlier kernels (the previous layer) are complete
    grid_dep_launch();  // the expert kernel may start prefetching weights
    bool ok = true;
    if (stage_x) {
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar, (uint32_t)((T + nrows) * H * 4));
            tma_load_1d(xs, a.x, (uint32_t)(T * H * 4), &bar);
            if (nrows) {
                const float *src = row0 < kExperts ? a.router + (size_t)row0 * H : a.s_router;
                tma_load_1d(wr, src, (uint32_t)(nrows * H * 4), &bar);
            }
        }
        ok = mbar_wait_bounded(&bar, 0, &a.hdr->error);
    }
    if (!__syncthreads_or(!ok)) {
        if (nrows > 0) {
            // warp w: staged row w%4 against tokens w/4, w/4+4, ...; lane j sums
            // k = j, j+32, ... in order (the reference's 32-lane order)
            constexpr int kTg = kK1Threads / 32 / kRouterRows;  // token groups
            constexpr int kTpw = (TMAX + kTg - 1) / kTg;
            const int r = warp % kRouterRows, tg = warp / kRouterRows;
            if (r < nrows) {
                float acc[kTpw];
#pragma unroll
                for (int i = 0; i < kTpw; i++) acc[i] = 0.0f;
                const float *w = wr + (size_t)r * H;
#pragma unroll 4
                for (int k = lane; k < H; k += 32) {
                    const float wv = w[k];
#pragma unroll
                    for (int i = 0; i < kTpw; i++) {
                        const int t = tg + kTg * i;
                        if (t < T) acc[i] = __fmaf_rn(wv, xs[(size_t)t * H + k], acc[i]);
                    }
                }
                const int row = row0 + r;
#pragma unroll
                for (int i = 0; i < kTpw; i++) {
                    const int t = tg + kTg * i;
                    if (t < T) {
                        const float s = lane_tree(acc[i]);
                        if (lane == 0) {
                            if (row < kExperts) a.logits[t * kExperts + row] = s;
                            else a.sgate[t] = s;
                        }
                    }
                }
            }
        }
        if ((int)blockIdx.x < T && !a.router) prep_token(blockIdx.x, xs + (size_t)blockIdx.x * H);
    }
    __threadfence();
    __syncthreads();
    const int G = gridDim.x;
    __shared__ int s_tk;
    if (tid == 0) s_tk = atomicAdd(&a.ctr->k1_ticket, 1);
    __syncthreads();
    if (a.router) {
        // The first T CTAs to finish write one token's activations each; the last T
        // route one token each, in parallel on their own SMs, once every CTA's logits
        // are in (all K1 CTAs are resident, so the bounded wait only spans the last
        // arrivals); the last of them plans. The grid has at least 128 CTAs and
        // T <= 32, so the two groups are disjoint.
        if (s_tk < T) {
            prep_token(s_tk, a.x + (size_t)s_tk * H);
            return;
        }
        const int t = s_tk - (G - T);
        if (t < 0) return;
        if (tid == 0) s_last = wait_geq(&a.ctr->k1_ticket, G, &a.hdr->error);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (warp == 0) route_token_warp(a.logits + t * kExperts, a.bias, a.ids + t * kTop, a.wts + t * kTop);
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&a.ctr->k1_routed, 1) == T - 1;
        __syncthreads();
        if (!s_last) return;
    } else if (s_tk != G - 1) {
        return;
    }
    __threadfence();

    // ---------------------------------------------------------- plan
    __shared__ int s_ids[kMaxDecodeTokens * kTop];
    __shared__ float s_w[kMaxDecodeTokens * kTop];
    __shared__ unsigned s_bm[kExperts];
    __shared__ int s_off[kExperts];
    __shared__ int s_bad[kMaxDecodeTokens];
    __shared__ int s_wt[kK1Threads / 32], s_wu[kK1Threads / 32], s_wm[kK1Threads / 32], s_inv[kK1Threads / 32];
    for (int i = tid; i < T * kTop; i += blockDim.x) {
        s_ids[i] = __ldcg(a.ids + i);
        s_w[i] = __ldcg(a.wts + i);
    }
    for (int e = tid; e < kExperts; e += blockDim.x) s_bm[e] = 0;
    __syncthreads();
    for (int t = tid; t < T; t += blockDim.x) {
        // qc_moe's route validation (qwen/cpu.c:241-246)
        bool good = true;
        for (int k = 0; k < kTop; k++) {
            const int e = s_ids[t * kTop + k];
            const float w = s_w[t * kTop + k];
            if (e <= -2 && e >= -kExperts - 1 && w == 0.0f) continue;
            if (e < 0 || e >= kExperts || !(w >= 0.0f) || isinf(w)) good = false;
            for (int j = 0; j < k; j++)
                if (s_ids[t * kTop + j] == e) good = false;
        }
        s_bad[t] = !good;
    }
    __syncthreads();
    for (int i = tid; i < T * kTop; i += blockDim.x) {
        const int t = i / kTop, e = s_ids[i];
        if (!s_bad[t] && e >= 0) atomicOr(&s_bm[e], 1u << t);
    }
    __syncthreads();
    {
        // one expert per thread: counts, exclusive offsets, ascending used list
        static_assert(kK1Threads == kExperts, "one expert per thread");
        const int e = tid;
        const int c = __popc(s_bm[e]), used = c > 0;
        const int loc = a.ep_local ? __ldg(a.ep_local + e) : e;  // index in gate/up/down, or -1
        const int mine = used && loc >= 0;
        int st = c, su = used, sm = mine;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int vt = __shfl_up_sync(0xffffffffu, st, d), vu = __shfl_up_sync(0xffffffffu, su, d),
                      vm = __shfl_up_sync(0xffffffffu, sm, d);
            if (lane >= d) {
                st += vt;
                su += vu;
                sm += vm;
            }
        }
        if (lane == 31) {
            s_wt[warp] = st;
            s_wu[warp] = su;
            s_wm[warp] = sm;
        }
        __syncthreads();
        int bt = 0, bu = 0, bmn = 0;
        for (int w = 0; w < warp; w++) {
            bt += s_wt[w];
            bu += s_wu[w];
            bmn += s_wm[w];
        }
        const int ot = bt + st - c, ou = bu + su - used, om = bmn + sm - mine;
        const int shared_sub = (a.sg && a.ep_shared_here) ? 1 : 0;
        s_off[e] = ot;
        a.off[e] = ot;
        if (c) a.used[ou] = e;
        if (mine && a.use_tc) a.sub[shared_sub + om] = SubJob{loc, ot, c, 0};
        if (tid == blockDim.x - 1) {  // totals: this thread's inclusive sums
            a.off[kExperts] = ot + c;
            a.hdr->n_pairs = ot + c;
            a.hdr->n_used = ou + used;
            if (a.use_tc) *a.n_sub = shared_sub + om + mine;
        }
    }
    __syncthreads();
    for (int i = tid; i < T * kTop; i += blockDim.x) {
        const int t = i / kTop, e = s_ids[i];
        if (s_bad[t] || e < 0) continue;
        a.pairs[s_off[e] + __popc(s_bm[e] & ((1u << t) - 1))] = i;
    }
    const int has_shared = a.sg != nullptr;
    if (a.use_tc) {
        // counters the tensor-core kernel counts up from zero
        for (int i = tid; i <= kExperts; i += blockDim.x) a.ctr->gu_done[i] = 0;
        for (int i = tid; i < T * (H / kTcRows); i += blockDim.x) a.ctr->tilecnt[i] = 0;
        if (tid == 0 && has_shared && a.ep_shared_here) a.sub[0] = SubJob{-1, 0, T, 0};
    }
    int invalid = 0;
    for (int t = tid; t < T; t += blockDim.x) {
        int n = 0;
        if (!s_bad[t])
            for (int k = 0; k < kTop; k++) n += s_ids[t * kTop + k] >= 0;
        const int expect = n + has_shared;
        a.expect[t] = expect | (s_bad[t] ? (int)kBadBit : 0);
        invalid += s_bad[t];
        if (expect == 0 && !a.ep_ranks) {  // no contribution will arrive: write the row here
            const float v = s_bad[t] ? __int_as_float(0x7fc00000) : 0.0f;
            for (int d = 0; d < H; d++) a.out[(size_t)t * H + d] = v;
        }
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) invalid += __shfl_xor_sync(0xffffffffu, invalid, d);
    if (lane == 0) s_inv[warp] = invalid;
    __syncthreads();
    if (tid == 0) {
        int inv = 0;
        for (int w = 0; w < kK1Threads / 32; w++) inv += s_inv[w];
        a.hdr->invalid_tokens = inv;
        a.ctr->k1_ticket = 0;
        a.ctr->k1_routed = 0;
    }
}

// ------------------------------------------------------------------ K2
enum ItemKind { kEnd = 0, kGateUp = 1, kDown = 2 };
struct Item {
    int kind, job, tile, n, first;  // job 0 is the shared expert when present
};

// Q4_K: byte b of w -> (low nibble, high nibble) as exact floats, by placing
// each nibble in the mantissa of a power of two and subtracting it.
__device__ __forceinline__ void q4k_word(uint32_t w, float2 (&q)[4]) {
    const uint32_t h = w >> 16;
    q[0] = __fadd2_rn(make_float2(__uint_as_float((w & 0xFu) | 0x4B000000u), __uint_as_float((w & 0xF0u) | 0x49000000u)),
                      make_float2(-8388608.0f, -524288.0f));
    q[1] = __fadd2_rn(make_float2(__uint_as_float((w & 0xF00u) | 0x47000000u), __uint_as_float((w & 0xF000u) | 0x45000000u)),
                      make_float2(-32768.0f, -2048.0f));
    q[2] = __fadd2_rn(make_float2(__uint_as_float((h & 0xFu) | 0x4B000000u), __uint_as_float((h & 0xF0u) | 0x49000000u)),
                      make_float2(-8388608.0f, -524288.0f));
    q[3] = __fadd2_rn(make_float2(__uint_as_float((h & 0xF00u) | 0x47000000u), __uint_as_float((h & 0xF000u) | 0x45000000u)),
                      make_float2(-32768.0f, -2048.0f));
}

// byte b of (lo4, hi4) -> exact code-book values (low nibble, high nibble)
__device__ __forceinline__ float2 iq4_pair(uint32_t lo4, uint32_t hi4, int b) {
    const uint32_t sel = 0x7650u | (uint32_t)b;  // byte b, then bytes 1..3 of 0x4B000000
    return __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo4, 0x4B000000u, sel)),
                                  __uint_as_float(__byte_perm(hi4, 0x4B000000u, sel))),
                      make_float2(-8388736.0f, -8388736.0f));  // -(2^23 + 128)
}

// y[r][t] += row_r(unit u) . v_t(unit u) for RM staged rows and kTP tokens
// whose 64-value unit is stored as 32 float2 pairs (+ 2 group sums for Q4_K).
template <int Q, int RM>
__device__ __forceinline__ void unit_rows(const unsigned char *const (&rows)[RM], int u, const float2 *const (&v)[kTP],
                                          const float *const (&vsum)[kTP], int nt, float (&y)[RM][kTP]) {
    float2 S[RM][kTP];
#pragma unroll
    for (int r = 0; r < RM; r++)
#pragma unroll
        for (int t = 0; t < kTP; t++) S[r][t] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int half = 0; half < 2; half++) {
        float2 xv[kTP][16];
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            const float4 *p = reinterpret_cast<const float4 *>(v[t] + u * 32 + half * 16);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 f = t < nt ? __ldcg(p + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                xv[t][2 * j] = make_float2(f.x, f.y);
                xv[t][2 * j + 1] = make_float2(f.z, f.w);
            }
        }
        if (Q == 12) {
            const int sb = u >> 2, i = u & 3;
#pragma unroll
            for (int r = 0; r < RM; r++) {
                const uint4 q4 = *reinterpret_cast<const uint4 *>(rows[r] + sb * 144 + 16 + 32 * i + 16 * half);
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    float2 q[4];
                    q4k_word((&q4.x)[w], q);
#pragma unroll
                    for (int b = 0; b < 4; b++)
#pragma unroll
                        for (int t = 0; t < kTP; t++) S[r][t] = __ffma2_rn(q[b], xv[t][4 * w + b], S[r][t]);
                }
            }
        } else {
#pragma unroll
            for (int r = 0; r < RM; r++) {
                const uint32_t *p = reinterpret_cast<const uint32_t *>(rows[r] + 36 * u);
                uint32_t W[5];
#pragma unroll
                for (int j = 0; j < 5; j++) W[j] = p[4 * half + j];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    // half 0: block 2u codes are bytes 2..17; half 1: block 2u+1 codes are bytes 20..35
                    const uint32_t word = half == 0 ? __byte_perm(W[w], W[w + 1], 0x5432) : W[w + 1];
                    const uint32_t lo4 = iq4_lut4(word & 0x0F0F0F0Fu), hi4 = iq4_lut4((word >> 4) & 0x0F0F0F0Fu);
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const float2 q = iq4_pair(lo4, hi4, b);
#pragma unroll
                        for (int t = 0; t < kTP; t++) S[r][t] = __ffma2_rn(q, xv[t][4 * w + b], S[r][t]);
                    }
                }
                if (half == 0) {  // fold block 2u with its scale and restart for block 2u+1
                    const float dA = half_bits(W[0]);
#pragma unroll
                    for (int t = 0; t < kTP; t++) {
                        y[r][t] = __fmaf_rn(dA, S[r][t].x + S[r][t].y, y[r][t]);
                        S[r][t] = make_float2(0.0f, 0.0f);
                    }
                } else {
                    const float dB = half_bits(W[0] >> 16);
#pragma unroll
                    for (int t = 0; t < kTP; t++) y[r][t] = __fmaf_rn(dB, S[r][t].x + S[r][t].y, y[r][t]);
                }
            }
        }
    }
    if (Q == 12) {
        const int sb = u >> 2, i = u & 3;
        float gl[kTP], gh[kTP];
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            gl[t] = t < nt ? __ldcg(vsum[t] + 2 * u) : 0.0f;
            gh[t] = t < nt ? __ldcg(vsum[t] + 2 * u + 1) : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < RM; r++) {
            const uint4 hd = *reinterpret_cast<const uint4 *>(rows[r] + sb * 144);
            const unsigned char *sc = reinterpret_cast<const unsigned char *>(&hd) + 4;
            int s0, m0, s1, m1;
            k_scale_min(sc, 2 * i, s0, m0);
            k_scale_min(sc, 2 * i + 1, s1, m1);
            const float d = half_bits(hd.x), dmin = half_bits(hd.x >> 16);
            const float ds0 = d * (float)s0, ds1 = d * (float)s1, dm0 = dmin * (float)m0, dm1 = dmin * (float)m1;
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                float acc = __fmaf_rn(ds0, S[r][t].x, ds1 * S[r][t].y);
                acc = __fmaf_rn(-dm0, gl[t], acc);
                y[r][t] += __fmaf_rn(-dm1, gh[t], acc);
            }
        }
    }
}

struct K2Shared {
    uint64_t full[kStages], empty[kStages];
    Item item[kStages];
    float red[kConsumers][2 * kGuRows][kTP];
    int combine[kTP];
    int n_combine;
};

template <int RM, int QD>
__device__ __forceinline__ void down_rows(const DecArgs &a, const Item &item, bool shared_job, const unsigned char *stage,
                                          int rows_per_warp, int warp, int lane, const float2 *const (&v)[kTP],
                                          const float *const (&vs)[kTP], int np, const int (&slot)[kTP]) {
    const int c = lane & 7, rs = lane >> 3;
    const unsigned char *rows[RM];
#pragma unroll
    for (int i = 0; i < RM; i++) rows[i] = stage + (size_t)(warp * rows_per_warp + rs + 4 * i) * a.drb;
    float y[RM][kTP];
#pragma unroll
    for (int r = 0; r < RM; r++)
#pragma unroll
        for (int t = 0; t < kTP; t++) y[r][t] = 0.0f;
    for (int u = c; u < a.F / 64; u += 8) unit_rows<QD, RM>(rows, u, v, vs, np, y);
#pragma unroll
    for (int r = 0; r < RM; r++)
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            float val = y[r][t];
            val += __shfl_xor_sync(0xffffffffu, val, 1);
            val += __shfl_xor_sync(0xffffffffu, val, 2);
            val += __shfl_xor_sync(0xffffffffu, val, 4);
            y[r][t] = val;
        }
    if (c == 0) {
#pragma unroll
        for (int i = 0; i < RM; i++) {
            const int row = item.tile * a.dn_rows + warp * rows_per_warp + rs + 4 * i;
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                if (t < np) {
                    if (shared_job) a.shout[(size_t)slot[t] * a.H + row] = y[i][t];
                    else a.slots[(size_t)slot[t] * a.H + row] = y[i][t] * __ldcg(a.wts + slot[t]);
                }
            }
        }
    }
}

template <int QG, int QD>
__global__ void __launch_bounds__(kK2Threads, 1) dec_experts_kernel(DecArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ K2Shared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T, H = a.H, F = a.F;
    const int gu_tiles = F / kGuRows, dn_tiles = H / a.dn_rows, shared_jobs = a.sg ? 1 : 0;
    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    grid_dep_launch();  // the next layer's router kernel may be scheduled
    const int S_gu = shared_jobs * gu_tiles, S_dn = shared_jobs * dn_tiles;

    // ---------------------------------------------------- producer (thread 0)
    bool planned = false, produced_end = false;
    int n_used = 0;
    auto produce = [&](int it) {
        const int s = it % kStages;
        const int idx = atomicAdd(&a.ctr->queue, 1);
        if (idx >= S_gu && !planned) {
            grid_dep_wait();  // K1's plan is complete and visible
            n_used = __ldcg(&a.hdr->n_used);
            planned = true;
        }
        const int R_gu = n_used * gu_tiles, R_dn = n_used * dn_tiles;
        Item item{kEnd, 0, 0, 0, 0};
        if (idx < S_gu) {
            item.kind = kGateUp, item.job = 0, item.tile = idx;
        } else if (idx < S_gu + R_gu) {
            const int j = idx - S_gu;
            item.kind = kGateUp, item.job = shared_jobs + j / gu_tiles, item.tile = j % gu_tiles;
        } else if (idx < S_gu + R_gu + S_dn) {
            item.kind = kDown, item.job = 0, item.tile = idx - S_gu - R_gu;
        } else if (idx < S_gu + R_gu + S_dn + R_dn) {
            const int j = idx - S_gu - R_gu - S_dn;
            item.kind = kDown, item.job = shared_jobs + j / dn_tiles, item.tile = j % dn_tiles;
        }
        unsigned char *dst = smem + (size_t)s * a.stage_bytes;
        if (item.kind == kEnd) {
            sh.item[s] = item;
            produced_end = true;
            mbar_arrive(&sh.full[s]);
            return;
        }
        const bool shared_job = shared_jobs && item.job == 0;
        int e = 0;
        if (shared_job) {
            item.n = T;
        } else {
            e = __ldcg(a.used + item.job - shared_jobs);
            item.first = __ldcg(a.off + e);
            item.n = __ldcg(a.off + e + 1) - item.first;
        }
        sh.item[s] = item;
        if (item.kind == kGateUp) {
            const size_t off = (size_t)item.tile * kGuRows * a.grb;
            const unsigned char *w0 = (shared_job ? a.sg : a.gate + (size_t)e * F * a.grb) + off;
            const unsigned char *w1 = (shared_job ? a.su : a.up + (size_t)e * F * a.grb) + off;
            mbar_arrive_expect_tx(&sh.full[s], 2u * kGuRows * (uint32_t)a.grb);
            for (int r = 0; r < kGuRows; r++)
                tma_load_1d(dst + r * a.gstride, w0 + r * a.grb, (uint32_t)a.grb, &sh.full[s]);
            for (int r = 0; r < kGuRows; r++)
                tma_load_1d(dst + (kGuRows + r) * a.gstride, w1 + r * a.grb, (uint32_t)a.grb, &sh.full[s]);
        } else {
            const unsigned char *w0 =
                (shared_job ? a.sd : a.down + (size_t)e * H * a.drb) + (size_t)item.tile * a.dn_rows * a.drb;
            const uint32_t bytes = (uint32_t)(a.dn_rows * a.drb);
            mbar_arrive_expect_tx(&sh.full[s], bytes);
            tma_load_1d(dst, w0, bytes, &sh.full[s]);
        }
    };
    if (tid == 0) {
        for (int it = 0; it < kStages && !produced_end; it++) produce(it);
    }
    {
        // ------------------------------------------------ consumers
        grid_dep_wait();  // x pairs, routing and plan from K1
        const int ctid = tid;
        for (int it = 0;; it++) {
            const int s = it % kStages;
            const bool ok = mbar_wait_bounded(&sh.full[s], (it / kStages) & 1, &a.hdr->error);
            const Item item = sh.item[s];
            if (!ok || item.kind == kEnd) break;
            const bool shared_job = shared_jobs && item.job == 0;
            const unsigned char *stage = smem + (size_t)s * a.stage_bytes;
            if (item.kind == kGateUp) {
                const int c = lane & 3, rs = lane >> 2;  // 4 unit slots x 8 row sets per warp
                const unsigned char *rows[8];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    rows[i] = stage + (size_t)(rs + 8 * i) * a.gstride;
                    rows[4 + i] = stage + (size_t)(kGuRows + rs + 8 * i) * a.gstride;
                }
                for (int p0 = 0; p0 < item.n; p0 += kTP) {
                    const int np = min(kTP, item.n - p0);
                    const float2 *v[kTP];
                    const float *vs[kTP];
#pragma unroll
                    for (int t = 0; t < kTP; t++) {
                        const int pi = p0 + min(t, np - 1);
                        const int tok = shared_job ? pi : __ldcg(a.pairs + item.first + pi) / kTop;
                        v[t] = reinterpret_cast<const float2 *>(a.xpair + (size_t)tok * H);
                        vs[t] = a.xsum + (size_t)tok * (H / 32);
                    }
                    float y[8][kTP];
#pragma unroll
                    for (int r = 0; r < 8; r++)
#pragma unroll
                        for (int t = 0; t < kTP; t++) y[r][t] = 0.0f;
                    for (int u = warp * 4 + c; u < H / 64; u += 4 * kConsumers) unit_rows<QG, 8>(rows, u, v, vs, np, y);
#pragma unroll
                    for (int r = 0; r < 8; r++)
#pragma unroll
                        for (int t = 0; t < kTP; t++) {
                            float val = y[r][t];
                            val += __shfl_xor_sync(0xffffffffu, val, 1);
                            val += __shfl_xor_sync(0xffffffffu, val, 2);
                            y[r][t] = val;
                        }
                    consumers_sync();  // the previous pass is done with sh.red
                    if (c == 0) {
#pragma unroll
                        for (int i = 0; i < 4; i++)
#pragma unroll
                            for (int t = 0; t < kTP; t++) {
                                sh.red[warp][rs + 8 * i][t] = y[i][t];
                                sh.red[warp][kGuRows + rs + 8 * i][t] = y[4 + i][t];
                            }
                    }
                    consumers_sync();
                    if (ctid < kGuRows * kTP) {  // warp t, lane = row
                        const int row = ctid % kGuRows, t = ctid / kGuRows;
                        float g = 0.0f, uu = 0.0f;
#pragma unroll
                        for (int w = 0; w < kConsumers; w++) {
                            g += sh.red[w][row][t];
                            uu += sh.red[w][kGuRows + row][t];
                        }
                        const float m = (g * sigmoidf_ref(g)) * uu;
                        float sum = m;
#pragma unroll
                        for (int d = 16; d; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
                        if (t < np) {
                            const int gr = item.tile * kGuRows + row;  // row of W_gate = value index of mid
                            const size_t mrow = shared_job ? (size_t)T * kTop + p0 + t : (size_t)(item.first + p0 + t);
                            a.mid[mrow * F + (gr >> 6) * 64 + pair_pos<QD>(gr & 63)] = m;
                            if (row == 0) a.msum[mrow * (F / 32) + item.tile] = sum;
                        }
                    }
                }
                __threadfence();
                consumers_sync();
                if (ctid == 0) atomicAdd(&a.ctr->gu_done[item.job], 1);
            } else {
                if (ctid == 0) wait_geq(&a.ctr->gu_done[item.job], gu_tiles, &a.hdr->error);
                consumers_sync();
                for (int p0 = 0; p0 < item.n; p0 += kTP) {
                    const int np = min(kTP, item.n - p0);
                    const float2 *v[kTP];
                    const float *vs[kTP];
                    int slot[kTP];
#pragma unroll
                    for (int t = 0; t < kTP; t++) {
                        const int pi = p0 + min(t, np - 1);
                        size_t mrow;
                        if (shared_job) {
                            mrow = (size_t)T * kTop + pi;
                            slot[t] = pi;
                        } else {
                            mrow = (size_t)(item.first + pi);
                            slot[t] = __ldcg(a.pairs + item.first + pi);
                        }
                        v[t] = reinterpret_cast<const float2 *>(a.mid + mrow * F);
                        vs[t] = a.msum + mrow * (F / 32);
                    }
                    if (a.dn_rows == 256)
                        down_rows<8, QD>(a, item, shared_job, stage, 32, warp, lane, v, vs, np, slot);
                    else
                        down_rows<4, QD>(a, item, shared_job, stage, 16, warp, lane, v, vs, np, slot);
                    // publish the rows, then count this (token, row tile) contribution
                    __threadfence();
                    consumers_sync();
                    if (ctid == 0) sh.n_combine = 0;
                    consumers_sync();
                    if (ctid < np) {
                        const int t = shared_job ? slot[ctid] : slot[ctid] / kTop;
                        int *cnt = a.ctr->tilecnt + t * 64 + item.tile;
                        const int expect = __ldcg(a.expect + t) & 0xffff;
                        if (atomicAdd(cnt, 1) == expect - 1) {
                            *cnt = 0;  // ready for the next call
                            sh.combine[atomicAdd(&sh.n_combine, 1)] = t;
                        }
                    }
                    consumers_sync();
                    const int nc = sh.n_combine;
                    if (nc) {
                        __threadfence();
                        for (int ci = 0; ci < nc; ci++) {
                            const int t = sh.combine[ci];
                            const bool bad = (__ldcg(a.expect + t) & kBadBit) != 0;
                            int ids[kTop];
#pragma unroll
                            for (int k = 0; k < kTop; k++) ids[k] = __ldcg(a.ids + t * kTop + k);
                            const float gate = a.sg ? sigmoidf_ref(__ldcg(a.sgate + t)) : 0.0f;
                            for (int r = ctid; r < a.dn_rows; r += kConsumers * 32) {
                                const int row = item.tile * a.dn_rows + r;
                                float sum = 0.0f;
#pragma unroll
                                for (int k = 0; k < kTop; k++)
                                    sum += ids[k] >= 0 ? __ldcg(a.slots + ((size_t)t * kTop + k) * H + row) : 0.0f;
                                if (a.sg) sum = __fmaf_rn(__ldcg(a.shout + (size_t)t * H + row), gate, sum);
                                a.out[(size_t)t * H + row] = bad ? __int_as_float(0x7fc00000) : sum;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
            if (tid == 0 && !produced_end) {
                mbar_wait_bounded(&sh.empty[s], (it / kStages) & 1, &a.hdr->error);  // every warp released it
                produce(it + kStages);
            }
        }
    }
    // the last CTA resets the queue and the per-job counters for the next call
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&a.ctr->k2_ticket, 1) == (int)gridDim.x - 1) {
            __threadfence();
            const int jobs = min(shared_jobs + __ldcg(&a.hdr->n_used), kExperts + 1);
            for (int j = 0; j < jobs; j++) a.ctr->gu_done[j] = 0;
            a.ctr->queue = 0;
            a.ctr->k2_ticket = 0;
        }
    }
}

template <typename K, typename... Args>
int launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int QG, int TMAX>
int launch_k1(const DecArgs &a, cudaStream_t st, size_t smem) {
    auto k = dec_router_kernel<QG, TMAX>;
    int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (rc) return rc;
    return launch_pdl(k, dim3(a.k1_ctas), dim3(kK1Threads), smem, st, true, a);
}

template <int QG, int QD>
int launch_k2(const DecArgs &a, cudaStream_t st, int ctas, bool pdl) {
    auto k = dec_experts_kernel<QG, QD>;
    const size_t smem = (size_t)kStages * a.stage_bytes;
    int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (rc) return rc;
    return launch_pdl(k, dim3(ctas), dim3(kK2Threads), smem, st, pdl, a);
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

}  // namespace

namespace nb {

DecLayout dec_layout(int T, int H, int F, size_t start) {
    DecLayout L{};
    size_t p = start;
    auto take = [&](size_t bytes) {
        size_t at = p;
        p = (p + bytes + 255) & ~size_t(255);
        return at;
    };
    L.logits = take(sizeof(float) * T * kExperts);
    L.sgate = take(sizeof(float) * T);
    L.ids = take(sizeof(int) * T * kTop);
    L.wts = take(sizeof(float) * T * kTop);
    L.xpair = take(sizeof(float) * T * H);
    L.xsum = take(sizeof(float) * T * (H / 32));
    L.off = take(sizeof(int) * (kExperts + 1));
    L.used = take(sizeof(int) * kExperts);
    L.pairs = take(sizeof(int) * T * kTop);
    L.expect = take(sizeof(int) * T);
    L.mid = take(sizeof(float) * (T * kTop + T) * F);
    L.msum = take(sizeof(float) * (T * kTop + T) * (F / 32));
    L.slots = take(sizeof(float) * T * kTop * H);
    L.shout = take(sizeof(float) * T * H);
    L.x16 = take(sizeof(__half) * T * 2 * H);
    L.xinv = take(sizeof(float) * T * 4);
    L.xs16 = take(sizeof(__half) * T * 2 * (H / 32));
    L.sub = take(sizeof(SubJob) * (kExperts + 1));
    L.nsub = take(sizeof(int));
    L.mid16 = take(sizeof(__half) * (T * kTop + T) * 2 * F);
    L.midinv = take(sizeof(float) * (T * kTop + T) * (((F / 128) + 3) & ~3));
    L.part = take(sizeof(float) * (T * kTop + T) * kMaxParts * 2 * F);  // gate/up K-part sums
    L.total = p;
    return L;
}

bool dec_supported(int T, int H, int F, int QG, int QD) {
    if (T < 1 || T > kMaxDecodeTokens || H % 256 || F % 64 || F % kGuRows) return false;
    if ((QG != 12 && QG != 20) || (QD != 12 && QD != 20)) return false;
    if (!row_bytes(QG, H) || !row_bytes(QD, F)) return false;
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    // K1 holds all token vectors plus four router rows
    if ((size_t)(T + kRouterRows) * H * 4 + 4096 > (size_t)optin) return false;
    const size_t grb = row_bytes(QG, H), drb = row_bytes(QD, F);
    if (grb % 16 || (128 * drb) % 16) return false;
    const int gstride = (int)((grb + 127) / 128 * 128 + 16);
    if ((size_t)kStages * 2 * kGuRows * gstride + 8192 > (size_t)optin) return false;
    return true;
}

int dec_run(const DecArgs &in, cudaStream_t st, cudaEvent_t split) {
    DecArgs a = in;
    a.use_tc = tc_supported(a.H, a.F, a.QG, a.QD, kMaxDecodeTokens) && a.H / kTcRows <= 64;
    const size_t grb = a.grb, drb = a.drb;
    a.gstride = (int)((grb + 127) / 128 * 128 + 16);  // rows start 16 bytes apart modulo 128
    const int gu_bytes = 2 * kGuRows * a.gstride;
    a.dn_rows = (size_t)256 * drb <= (size_t)gu_bytes ? 256 : 128;
    if (a.H % a.dn_rows) a.dn_rows = 128;
    if (a.H % a.dn_rows || ((size_t)a.dn_rows * drb) % 16) return cudaErrorInvalidValue;
    a.stage_bytes = std::max(gu_bytes, (int)(a.dn_rows * drb));
    a.stage_bytes = (a.stage_bytes + 127) / 128 * 128;
    a.k1_ctas = a.router ? kExperts / kRouterRows + (a.s_router ? 1 : 0) : a.T;
    a.k1_ctas = std::max(a.k1_ctas, a.T);
    const size_t k1_smem = (size_t)(a.T + (a.router ? kRouterRows : 0)) * a.H * 4;
    int rc;
    const int tmax = a.T <= 4 ? 4 : a.T <= 8 ? 8 : a.T <= 17 ? 17 : 32;
#define NB_K1(Q, TM) rc = launch_k1<Q, TM>(a, st, k1_smem)
    if (a.QG == 12) {
        if (tmax == 4) NB_K1(12, 4); else if (tmax == 8) NB_K1(12, 8); else if (tmax == 17) NB_K1(12, 17); else NB_K1(12, 32);
    } else {
        if (tmax == 4) NB_K1(20, 4); else if (tmax == 8) NB_K1(20, 8); else if (tmax == 17) NB_K1(20, 17); else NB_K1(20, 32);
    }
#undef NB_K1
    if (rc) return rc;
    // profiling: an event between the two kernels, which then run without overlap
    const bool pdl = split == nullptr;
    if (split && (rc = cudaEventRecord(split, st))) return rc;
    if (a.use_tc) {
        TcArgs t{};
        t.T = a.T, t.H = a.H, t.F = a.F;
        t.gate = a.gate, t.up = a.up, t.down = a.down, t.sg = a.sg, t.su = a.su, t.sd = a.sd;
        t.grb = a.grb, t.drb = a.drb, t.gu_iq4 = a.QG == 20, t.dn_iq4 = a.QD == 20;
        t.all_tok = 1;
        t.x16 = a.x16, t.xinv = a.xinv, t.xsum = a.xsum, t.xs16 = a.xs16;
        t.mi_stride = ((a.F / 128) + 3) & ~3;
        t.sub = a.sub, t.n_sub = a.n_sub, t.shared_subs = (a.sg && a.ep_shared_here) ? 1 : 0;
        t.sh_t0 = 0, t.sh_t1 = a.T;
        t.pairs = a.pairs, t.wts = a.wts, t.ids = a.ids, t.expect = a.expect, t.sgate = a.sg ? a.sgate : nullptr;
        t.mid16 = a.mid16, t.midinv = a.midinv, t.msum = a.msum;
        t.slots = a.slots, t.shout = a.shout, t.out = a.out;
        t.queue = &a.ctr->tc_queue, t.tc_ticket = &a.ctr->tc_ticket;
        t.gu_done = a.ctr->gu_done, t.tilecnt = a.ctr->tilecnt, t.err = &a.hdr->error;
        t.n_experts = a.n_experts;
        t.ep_ranks = a.ep_ranks, t.ep_rank = a.ep_rank, t.ep_cap = a.ep_cap, t.ep_epoch = a.ep_epoch;
        if (a.F / kTcRows <= kMaxGuTiles) t.gu_part = a.gu_part, t.gu_pcnt = a.ctr->gu_pcnt;
        for (int p = 0; p < kMaxRanks; p++)
            t.ep_slots[p] = a.ep_slots[p], t.ep_shout[p] = a.ep_shout[p], t.ep_flags[p] = a.ep_flags[p];
        TcMaps maps;
        const int tile = a.T <= kTcTokSmall ? kTcTokSmall : kMaxDecodeTokens;  // tokens per tile (all T)
        if ((rc = tc_make_maps(t, maps, tile))) return rc;
        return tc_launch(t, maps, st, pdl, tile);
    }
    const int ctas = sm_count();
    if (a.QG == 12 && a.QD == 12) return launch_k2<12, 12>(a, st, ctas, pdl);
    if (a.QG == 12 && a.QD == 20) return launch_k2<12, 20>(a, st, ctas, pdl);
    if (a.QG == 20 && a.QD == 12) return launch_k2<20, 12>(a, st, ctas, pdl);
    return launch_k2<20, 20>(a, st, ctas, pdl);
}

}  // namespace nb
