// All-resident routed MoE for sm_100a: qg_moe_workspace_bytes, qg_moe_routed,
// qg_moe_layer, qg_moe_status.
//
// One layer is a fixed sequence of kernels on the caller's stream, with no
// host synchronisation (graph-capturable):
//   plan     - one CTA validates the routes, counts tokens per expert and
//              builds the expert-major pair list (ascending token order),
//              replacing the host read of route ids (qwen/qwen.c:649-655) and
//              the moe_map kernel (qwen/gpu.cu:489-505).
//   gate_up  - grid (F/16 row tiles) x (used experts [+ shared]); each CTA
//              stages 16 gate rows and 16 up rows of one expert in shared
//              memory with TMA bulk copies and produces mid = SiLU(g)*u for
//              every token routed to that expert (qwen/cpu.c:209-217).
//   down     - grid (H/64 row tiles) x (used experts [+ shared]); weighted
//              slot rows slots[t*10+k] = w[t][k] * (W_down mid)
//              (qwen/cpu.c:219-225).
//   combine  - out[t] = sum_{k=0..9} slots (rank order, from +0.0f), then the
//              gated shared expert (qwen/cpu.c:227-231, qwen/gpu.cu:552).
//
// Dequant-dot formulation (both Q4_K and IQ4_NL): the scale of each 32-value
// group is applied once per group instead of once per weight,
//   sum_k w_k x_k = sum_g [ d*sc_g * sum_l q_l x_l  -  dmin*m_g * sum_l x_l ]
// with the 4-bit codes q_l converted exactly. The per-group sums of x are
// computed once per staged token. This is not the reference's summation
// order, so routed outputs match qc_moe within the float tolerance rather
// than bitwise; the router (ids) and qg_matmul stay bit-exact.
#include <algorithm>
#include <cstddef>
#include <utility>
#include <cstring>
#include <vector>
#include "quant.cuh"
#include "moe_decode.cuh"

using namespace nb;

namespace nb {
int launch_matmul(float *o, const void *w, int type, int rows, int cols, const float *x, int nt, cudaStream_t st);
int launch_route(int *ids, float *weights, const float *logits, const float *bias, int nt, cudaStream_t st);
}  // namespace nb

namespace {

// ---------------------------------------------------------------- profiling
// Optional CUDA-event timing of each phase of the MoE layer (qg_moe_profile).
// Only eager launches on the legacy stream are timed; graph captures are not.
// kExpertsFused: one kernel doing gate/up, SwiGLU, down and the combine;
// kDecodeRouter: one kernel doing the router GEMV, top-10 and the plan.
// kLean: the whole layer in one kernel (batches of 1 to 4 tokens).
enum Phase { kRouter, kRoute, kPlan, kGateUp, kDown, kCombine, kExpertsFused, kDecodeRouter, kLean, kPhases };
struct Profiler {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> spans;
    size_t next = 0;
    cudaEvent_t take() {
        if (next == pool.size()) {
            cudaEvent_t e = nullptr;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            pool.push_back(e);
        }
        return pool[next++];
    }
};
Profiler g_prof;

// Decode path: the router/plan kernel and the expert kernel timed separately.
int dec_run_timed(const DecArgs &a, cudaStream_t st) {
    cudaEvent_t e0, e1, e2;
    if (!g_prof.on || st != 0 || !(e0 = g_prof.take()) || !(e1 = g_prof.take()) || !(e2 = g_prof.take()))
        return dec_run(a, st);
    cudaEventRecord(e0, st);
    int rc = dec_run(a, st, e1);
    cudaEventRecord(e2, st);
    g_prof.spans.push_back({kDecodeRouter, {e0, e1}});
    g_prof.spans.push_back({kExpertsFused, {e1, e2}});
    return rc;
}

struct Span {
    int phase;
    cudaEvent_t a = nullptr, b = nullptr;
    cudaStream_t st;
    Span(int p, cudaStream_t s) : phase(p), st(s) {
        if (g_prof.on && st == 0 && (a = g_prof.take()) && (b = g_prof.take())) cudaEventRecord(a, st);
    }
    ~Span() {
        if (a && b) {
            cudaEventRecord(b, st);
            g_prof.spans.push_back({phase, {a, b}});
        }
    }
};

constexpr int kThreads = 256;
constexpr int kTP = 4;               // tokens per pass
constexpr int kGateUpRows = 16;      // rows of gate (and of up) per CTA
constexpr int kDownRows = 64;        // rows of down per CTA
constexpr int kPlanChunk = 512;      // tokens per bitmap chunk in the plan kernel
constexpr int kPC = 128;             // tokens per CTA of the multi-CTA plan (large batches)
constexpr int kPlanMultiMin = 256;   // batches from this size plan with several CTAs

// ---------------------------------------------------------------- workspace
struct Layout {
    size_t hdr, counts, off, used, pairs, bad, logits, ids, wts, mid, slots, shared;
    size_t x16, xinv, xsum, sub, nsub, mid16, midinv, msum, gudone, tilecnt, expect;  // tensor-core path
    size_t pcnt, total;  // multi-CTA plan: per chunk of kPC tokens, per-expert counts then offsets, + invalid
};

inline int max_subjobs(int T) { return (T + kTcTok - 1) / kTcTok + kExperts + (T * kTop + kTcTok - 1) / kTcTok; }

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Regions from `start`: the status words and decode-path counters (the fixed
// prefix) come first; expert parallelism also puts its fixed block before start.
Layout layout(int T, int H, int F, size_t start = kPrefixBytes) {
    Layout L{};
    size_t p = start;
    auto take = [&](size_t bytes) {
        size_t at = p;
        p = align256(p + bytes);
        return at;
    };
    L.hdr = 0;
    L.counts = take(sizeof(int) * kExperts);
    L.off = take(sizeof(int) * (kExperts + 1));
    L.used = take(sizeof(int) * kExperts);
    L.pairs = take(sizeof(int) * (size_t)T * kTop);
    L.bad = take(sizeof(int) * (size_t)T);
    L.logits = take(sizeof(float) * (size_t)T * (kExperts + 1));
    L.ids = take(sizeof(int) * (size_t)T * kTop);
    L.wts = take(sizeof(float) * (size_t)T * kTop);
    L.mid = take(sizeof(float) * ((size_t)T * kTop + T) * F);
    L.slots = take(sizeof(float) * (size_t)T * kTop * H);
    L.shared = take(sizeof(float) * (size_t)T * H);
    // tensor-core gate/up activations: per token (T <= one token tile) or per routed row
    const size_t rows = (size_t)T * kTop + T;
    L.x16 = take(sizeof(__half) * rows * 2 * H);
    L.xinv = take(sizeof(float) * rows * 4);
    L.xsum = take(sizeof(float) * rows * (H / 32));
    L.sub = take(sizeof(SubJob) * (size_t)max_subjobs(T));
    L.nsub = take(sizeof(int));
    L.mid16 = take(sizeof(__half) * ((size_t)T * kTop + T) * 2 * F);
    L.midinv = take(sizeof(float) * rows * (((F / 128) + 3) & ~3));
    L.msum = take(sizeof(float) * ((size_t)T * kTop + T) * (F / 32));
    L.gudone = take(sizeof(int) * (size_t)max_subjobs(T));
    L.tilecnt = take(sizeof(int) * (size_t)T * (H / kTcRows));
    L.expect = take(sizeof(int) * (size_t)T);
    L.pcnt = take(sizeof(int) * (size_t)((T + kPC - 1) / kPC) * (kExperts + 1));
    L.total = p;
    return L;
}

// Status words at the start of the workspace.
struct Header {
    int invalid_tokens;  // tokens given NaN output rows
    int n_pairs;         // routed (token, expert) pairs computed
    int n_used;          // distinct experts used
    int error;           // bounded-wait timeouts or internal errors
};

struct Plan {
    Header *hdr;
    int *counts, *off, *used, *pairs, *bad;
};

Plan plan_ptrs(void *ws, const Layout &L) {
    char *b = static_cast<char *>(ws);
    return Plan{reinterpret_cast<Header *>(b + L.hdr), reinterpret_cast<int *>(b + L.counts),
                reinterpret_cast<int *>(b + L.off),   reinterpret_cast<int *>(b + L.used),
                reinterpret_cast<int *>(b + L.pairs), reinterpret_cast<int *>(b + L.bad)};
}

// ---------------------------------------------------------------- plan
// Validation follows qc_moe (qwen/cpu.c:241-246): an omitted route is an id
// in [-513,-2] with weight exactly 0; otherwise the id must be in [0,512),
// the weight finite and >= 0, and the id must not repeat within the token.
__global__ void __launch_bounds__(1024) plan_kernel(const int *ids, const float *wts, int nt, Plan pl) {
    __shared__ int cnt[kExperts];
    __shared__ int run[kExperts];
    __shared__ unsigned bm[kExperts * (kPlanChunk / 32)];
    __shared__ int warp_tot[32];
    __shared__ int s_invalid;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < kExperts; e += blockDim.x) cnt[e] = 0;
    if (tid == 0) s_invalid = 0;
    __syncthreads();
    // A: validate tokens and count routes per expert.
    for (int t = tid; t < nt; t += blockDim.x) {
        bool ok = true;
        int e_k[kTop];
#pragma unroll
        for (int k = 0; k < kTop; k++) {
            int e = ids[t * kTop + k];
            float w = wts[t * kTop + k];
            e_k[k] = e;
            bool omitted = e <= -2 && e >= -kExperts - 1 && w == 0.0f;
            if (omitted) {
                e_k[k] = -1;
                continue;
            }
            if (e < 0 || e >= kExperts || !(w >= 0.0f) || isinf(w)) ok = false;
#pragma unroll
            for (int j = 0; j < k; j++)
                if (ids[t * kTop + j] == e) ok = false;
        }
        pl.bad[t] = ok ? 0 : 1;
        if (ok) {
#pragma unroll
            for (int k = 0; k < kTop; k++)
                if (e_k[k] >= 0) atomicAdd(&cnt[e_k[k]], 1);
        } else {
            atomicAdd(&s_invalid, 1);
        }
    }
    __syncthreads();
    // B: exclusive scan of counts (512 entries, 16 warps of 32).
    int c = 0, incl = 0;
    if (tid < kExperts) {
        c = cnt[tid];
        incl = c;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += v;
        }
        if (lane == 31) warp_tot[warp] = incl;
    }
    __syncthreads();
    if (tid < 32) {
        int v = tid < kExperts / 32 ? warp_tot[tid] : 0, s = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            int o = __shfl_up_sync(0xffffffffu, s, d);
            if (tid >= d) s += o;
        }
        warp_tot[tid] = s - v;  // exclusive prefix of warp totals
    }
    __syncthreads();
    if (tid < kExperts) {
        int excl = warp_tot[warp] + incl - c;
        pl.off[tid] = excl;
        pl.counts[tid] = c;
        run[tid] = excl;
        if (tid == kExperts - 1) {
            pl.off[kExperts] = excl + c;
            pl.hdr->n_pairs = excl + c;
        }
    }
    // used experts list (ascending): rank = number of used experts below e.
    __syncthreads();
    if (tid < kExperts) {
        unsigned m = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) warp_tot[warp] = __popc(m);
    }
    __syncthreads();
    if (tid < kExperts) {
        unsigned m = __ballot_sync(0xffffffffu, c > 0);
        int before = __popc(m & ((1u << lane) - 1));
        for (int w = 0; w < warp; w++) before += warp_tot[w];
        if (c > 0) pl.used[before] = tid;
        if (tid == kExperts - 1) pl.hdr->n_used = before + (c > 0);
    }
    if (tid == 0) pl.hdr->invalid_tokens = s_invalid;
    // C: placement, one bitmap chunk of tokens at a time, ascending tokens: a
    // pair's slot is its expert's running offset plus the chunk's tokens of that
    // expert before it (set bits below it in the expert's bitmap).
    constexpr int W = kPlanChunk / 32;
    for (int c0 = 0; c0 < nt; c0 += kPlanChunk) {
        __syncthreads();
        for (int i = tid; i < kExperts * W; i += blockDim.x) bm[i] = 0;
        __syncthreads();
        const int c1 = min(nt, c0 + kPlanChunk);
        for (int t = c0 + tid; t < c1; t += blockDim.x) {
            if (pl.bad[t]) continue;
            for (int k = 0; k < kTop; k++) {
                const int e = ids[t * kTop + k];
                if (e >= 0) atomicOr(&bm[e * W + (t - c0) / 32], 1u << ((t - c0) & 31));
            }
        }
        __syncthreads();
        for (int t = c0 + tid; t < c1; t += blockDim.x) {
            if (pl.bad[t]) continue;
            const int wd = (t - c0) / 32;
            const unsigned below = (1u << ((t - c0) & 31)) - 1u;
            for (int k = 0; k < kTop; k++) {
                const int e = ids[t * kTop + k];
                if (e < 0) continue;
                int pos = run[e] + __popc(bm[e * W + wd] & below);
                for (int w2 = 0; w2 < wd; w2++) pos += __popc(bm[e * W + w2]);
                pl.pairs[pos] = t * kTop + k;
            }
        }
        __syncthreads();
        for (int e = tid; e < kExperts; e += blockDim.x) {
            int total = 0;
            for (int w2 = 0; w2 < W; w2++) total += __popc(bm[e * W + w2]);
            run[e] += total;
        }
    }
}

// Multi-CTA plan for large batches: the same validation, offsets and pair
// order (ascending tokens within each expert) as plan_kernel, in three steps.
// Validation follows qc_moe (qwen/cpu.c:241-246); e_k gets -1 for an omitted route.
__device__ __forceinline__ bool plan_validate(const int *ids, const float *wts, int t, int (&e_k)[kTop]) {
    bool ok = true;
#pragma unroll
    for (int k = 0; k < kTop; k++) {
        const int e = ids[t * kTop + k];
        const float w = wts[t * kTop + k];
        e_k[k] = e;
        if (e <= -2 && e >= -kExperts - 1 && w == 0.0f) {
            e_k[k] = -1;
            continue;
        }
        if (e < 0 || e >= kExperts || !(w >= 0.0f) || isinf(w)) ok = false;
#pragma unroll
        for (int j = 0; j < k; j++)
            if (ids[t * kTop + j] == e) ok = false;
    }
    return ok;
}

// Step 1 (CTA c: tokens [c*kPC, (c+1)*kPC)): validation, and the chunk's count
// per expert and of invalid tokens into pcnt[c][0..512].
__global__ void __launch_bounds__(512) plan_count_kernel(const int *ids, const float *wts, int nt, Plan pl, int *pcnt) {
    constexpr int W = kPC / 32;
    __shared__ unsigned bm[kExperts * W];
    __shared__ int s_inv;
    const int tid = threadIdx.x, c0 = blockIdx.x * kPC, c1 = min(nt, c0 + kPC);
    for (int i = tid; i < kExperts * W; i += blockDim.x) bm[i] = 0;
    if (tid == 0) s_inv = 0;
    __syncthreads();
    for (int t = c0 + tid; t < c1; t += blockDim.x) {
        int e_k[kTop];
        const bool ok = plan_validate(ids, wts, t, e_k);
        pl.bad[t] = ok ? 0 : 1;
        if (ok) {
#pragma unroll
            for (int k = 0; k < kTop; k++)
                if (e_k[k] >= 0) atomicOr(&bm[e_k[k] * W + (t - c0) / 32], 1u << ((t - c0) & 31));
        } else {
            atomicAdd(&s_inv, 1);
        }
    }
    __syncthreads();
    int *row = pcnt + (size_t)blockIdx.x * (kExperts + 1);
    for (int e = tid; e < kExperts; e += blockDim.x) {
        int n = 0;
#pragma unroll
        for (int w = 0; w < W; w++) n += __popc(bm[e * W + w]);
        row[e] = n;
    }
    if (tid == 0) row[kExperts] = s_inv;
}

// Step 2 (one CTA, thread e = expert): totals, offsets, the used-expert list and
// the header; pcnt[c][e] becomes the first pair position of chunk c's tokens of e.
__global__ void __launch_bounds__(kExperts) plan_scan_kernel(int nchunks, Plan pl, int *pcnt) {
    __shared__ int warp_tot[32];
    const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
    int c = 0;
    for (int ch = 0; ch < nchunks; ch++) {
        int *v = pcnt + (size_t)ch * (kExperts + 1) + e;
        const int n = *v;
        *v = c;
        c += n;
    }
    int incl = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (e < 32) {
        const int v = e < kExperts / 32 ? warp_tot[e] : 0;
        int s2 = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, s2, d);
            if (e >= d) s2 += o;
        }
        warp_tot[e] = s2 - v;
    }
    __syncthreads();
    const int excl = warp_tot[warp] + incl - c;
    pl.off[e] = excl;
    pl.counts[e] = c;
    if (e == kExperts - 1) {
        pl.off[kExperts] = excl + c;
        pl.hdr->n_pairs = excl + c;
    }
    for (int ch = 0; ch < nchunks; ch++) pcnt[(size_t)ch * (kExperts + 1) + e] += excl;
    __syncthreads();
    {
        const unsigned m = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) warp_tot[warp] = __popc(m);
    }
    __syncthreads();
    {
        const unsigned m = __ballot_sync(0xffffffffu, c > 0);
        int before = __popc(m & ((1u << lane) - 1));
        for (int w = 0; w < warp; w++) before += warp_tot[w];
        if (c > 0) pl.used[before] = e;
        if (e == kExperts - 1) pl.hdr->n_used = before + (c > 0);
    }
    if (e == 0) {
        int inv = 0;
        for (int ch = 0; ch < nchunks; ch++) inv += pcnt[(size_t)ch * (kExperts + 1) + kExperts];
        pl.hdr->invalid_tokens = inv;
    }
}

// Step 3 (CTA c): each valid pair's position is its chunk's start for the expert
// plus the chunk's earlier tokens of that expert (set bits below it).
__global__ void __launch_bounds__(512) plan_place_kernel(const int *ids, int nt, Plan pl, const int *pcnt) {
    constexpr int W = kPC / 32;
    __shared__ unsigned bm[kExperts * W];
    const int tid = threadIdx.x, c0 = blockIdx.x * kPC, c1 = min(nt, c0 + kPC);
    for (int i = tid; i < kExperts * W; i += blockDim.x) bm[i] = 0;
    __syncthreads();
    for (int t = c0 + tid; t < c1; t += blockDim.x) {
        if (pl.bad[t]) continue;
        for (int k = 0; k < kTop; k++) {
            const int e = ids[t * kTop + k];
            if (e >= 0) atomicOr(&bm[e * W + (t - c0) / 32], 1u << ((t - c0) & 31));
        }
    }
    __syncthreads();
    const int *start = pcnt + (size_t)blockIdx.x * (kExperts + 1);
    for (int t = c0 + tid; t < c1; t += blockDim.x) {
        if (pl.bad[t]) continue;
        const int wd = (t - c0) / 32;
        const unsigned below = (1u << ((t - c0) & 31)) - 1u;
        for (int k = 0; k < kTop; k++) {
            const int e = ids[t * kTop + k];
            if (e < 0) continue;
            int pos = start[e] + __popc(bm[e * W + wd] & below);
            for (int w2 = 0; w2 < wd; w2++) pos += __popc(bm[e * W + w2]);
            pl.pairs[pos] = t * kTop + k;
        }
    }
}

// ---------------------------------------------------------------- staging
// Shared-memory row stride for staged weight rows: padded so consecutive
// rows start 16 bytes apart modulo 128 (no bank conflicts between the rows
// a warp reads together).
__host__ __device__ inline int padded(int bytes) {
    int r = bytes % 128;
    return bytes + ((16 - r) + 128) % 128;
}

// Rows are copied in groups of G consecutive rows so that every TMA bulk copy
// has a 16-byte-multiple size and a 16-byte-aligned source.
__host__ __device__ inline int row_group(size_t rb) {
    int g = 1;
    while ((g * rb) % 16) g *= 2;
    return g;
}

struct Tile {
    int rb;      // bytes of one row
    int G;       // rows per bulk copy
    int gstride; // shared-memory bytes per row group
    __device__ const unsigned char *row(const unsigned char *base, int r) const {
        return base + (r / G) * gstride + (r % G) * rb;
    }
};

__host__ __device__ inline Tile make_tile(size_t rb) {
    Tile t;
    t.rb = (int)rb;
    t.G = row_group(rb);
    t.gstride = padded(t.G * (int)rb);
    return t;
}

// Issue the bulk copies of `rows` consecutive rows starting at src into dst.
__device__ inline void tile_load(unsigned char *dst, const unsigned char *src, int rows, const Tile &t,
                                 uint64_t *bar) {
    for (int g = 0; g < rows / t.G; g++)
        tma_load_1d(dst + g * t.gstride, src + (size_t)g * t.G * t.rb, (uint32_t)(t.G * t.rb), bar);
}

// x staging: each 64-value unit u of a token vector is stored as 32 float2
// pairs matching the byte layout of the weights, plus the two 32-value
// group sums (Q4_K min term). The unit stride is padded by 16 bytes.
constexpr int kUnitFloats = 64 + 4;  // 32 pairs + 2 group sums (+2 pad) = 272 bytes

template <int QT>
__device__ inline void stage_tokens(float *xs, const float *const *src, int n, int K) {
    // one warp per (token, unit); lane l writes pair l of that unit
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int units = K / 64;
    for (int job = warp; job < kTP * units; job += nwarps) {
        int tp = job / units, u = job % units;
        float a = 0.0f, b = 0.0f;
        if (tp < n) {
            const float *v = src[tp] + u * 64;
            int ia, ib;
            if (QT == 12) {
                ia = lane;
                ib = lane + 32;
            } else {  // IQ4_NL: blocks of 32 with byte j holding values j and j+16
                int blk = lane >> 4, j = lane & 15;
                ia = blk * 32 + j;
                ib = blk * 32 + 16 + j;
            }
            a = v[ia];
            b = v[ib];
        }
        float *dst = xs + ((size_t)tp * units + u) * kUnitFloats;
        reinterpret_cast<float2 *>(dst)[lane] = make_float2(a, b);
        if (QT == 12) {
            // group sums: values 0..31 (the "a" of every lane) and 32..63 (the "b")
            float sa = a, sb = b;
#pragma unroll
            for (int d = 16; d; d >>= 1) {
                sa += __shfl_xor_sync(0xffffffffu, sa, d);
                sb += __shfl_xor_sync(0xffffffffu, sb, d);
            }
            if (lane == 0) {
                dst[64] = sa;
                dst[65] = sb;
            }
        }
    }
}

__device__ __forceinline__ float code_f(uint32_t v) { return static_cast<float>(v); }

// Accumulate one 64-value unit u of RM staged rows against the staged
// tokens: y[rm][tp] += dot(row rm unit u, token tp unit u).
template <int QT, int RM>
__device__ inline void unit_dot(const unsigned char *const (&rows)[RM], int u, const float *xs, int units,
                                const float *lut, float (&y)[RM][kTP]) {
    if (QT == 12) {
        const int sb = u >> 2, i = u & 3;
        float ds_lo[RM], ds_hi[RM], dm_lo[RM], dm_hi[RM];
        uint4 qa[RM], qb[RM];
#pragma unroll
        for (int r = 0; r < RM; r++) {
            const unsigned char *p = rows[r] + sb * 144;
            const uint4 h = *reinterpret_cast<const uint4 *>(p);
            const unsigned char *sc = reinterpret_cast<const unsigned char *>(&h) + 4;
            int s0, m0, s1, m1;
            k_scale_min(sc, 2 * i, s0, m0);
            k_scale_min(sc, 2 * i + 1, s1, m1);
            float d = half_bits(h.x), dmin = half_bits(h.x >> 16);
            ds_lo[r] = d * (float)s0;
            ds_hi[r] = d * (float)s1;
            dm_lo[r] = dmin * (float)m0;
            dm_hi[r] = dmin * (float)m1;
            qa[r] = *reinterpret_cast<const uint4 *>(p + 16 + 32 * i);
            qb[r] = *reinterpret_cast<const uint4 *>(p + 32 + 32 * i);
        }
        float s_lo[RM][kTP], s_hi[RM][kTP];
#pragma unroll
        for (int r = 0; r < RM; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) s_lo[r][t] = s_hi[r][t] = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            float2 xv[kTP][4];
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                const float4 *src = reinterpret_cast<const float4 *>(xs + ((size_t)t * units + u) * kUnitFloats) + 2 * w;
                float4 A = src[0], B = src[1];
                xv[t][0] = make_float2(A.x, A.y);
                xv[t][1] = make_float2(A.z, A.w);
                xv[t][2] = make_float2(B.x, B.y);
                xv[t][3] = make_float2(B.z, B.w);
            }
#pragma unroll
            for (int r = 0; r < RM; r++) {
                uint32_t word = w < 4 ? (&qa[r].x)[w] : (&qb[r].x)[w - 4];
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    float ql = code_f((word >> (8 * b)) & 15u), qh = code_f((word >> (8 * b + 4)) & 15u);
#pragma unroll
                    for (int t = 0; t < kTP; t++) {
                        s_lo[r][t] = __fmaf_rn(ql, xv[t][b].x, s_lo[r][t]);
                        s_hi[r][t] = __fmaf_rn(qh, xv[t][b].y, s_hi[r][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            const float *g = xs + ((size_t)t * units + u) * kUnitFloats + 64;
            float glo = g[0], ghi = g[1];
#pragma unroll
            for (int r = 0; r < RM; r++) {
                float v = __fmaf_rn(ds_lo[r], s_lo[r][t], ds_hi[r] * s_hi[r][t]);
                v = __fmaf_rn(-dm_lo[r], glo, v);
                v = __fmaf_rn(-dm_hi[r], ghi, v);
                y[r][t] += v;
            }
        }
    } else {  // IQ4_NL: blocks 2u and 2u+1, 36 bytes at offset 36u
        float dA[RM], dB[RM];
        uint32_t q[RM][8];
#pragma unroll
        for (int r = 0; r < RM; r++) {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(rows[r] + 36 * u);
            uint32_t W[9];
#pragma unroll
            for (int j = 0; j < 9; j++) W[j] = p[j];
            dA[r] = half_bits(W[0]);
            dB[r] = half_bits(W[4] >> 16);
#pragma unroll
            for (int j = 0; j < 4; j++) q[r][j] = __byte_perm(W[j], W[j + 1], 0x5432);
#pragma unroll
            for (int j = 0; j < 4; j++) q[r][4 + j] = W[5 + j];
        }
        float sA[RM][kTP], sB[RM][kTP];
#pragma unroll
        for (int r = 0; r < RM; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) sA[r][t] = sB[r][t] = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            float2 xv[kTP][4];
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                const float4 *src = reinterpret_cast<const float4 *>(xs + ((size_t)t * units + u) * kUnitFloats) + 2 * w;
                float4 A = src[0], B = src[1];
                xv[t][0] = make_float2(A.x, A.y);
                xv[t][1] = make_float2(A.z, A.w);
                xv[t][2] = make_float2(B.x, B.y);
                xv[t][3] = make_float2(B.z, B.w);
            }
#pragma unroll
            for (int r = 0; r < RM; r++) {
                uint32_t word = q[r][w];
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    float ql = lut[(word >> (8 * b)) & 15u], qh = lut[(word >> (8 * b + 4)) & 15u];
#pragma unroll
                    for (int t = 0; t < kTP; t++) {
                        float acc = w < 4 ? sA[r][t] : sB[r][t];
                        acc = __fmaf_rn(ql, xv[t][b].x, acc);
                        acc = __fmaf_rn(qh, xv[t][b].y, acc);
                        if (w < 4) sA[r][t] = acc; else sB[r][t] = acc;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RM; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) y[r][t] += __fmaf_rn(dA[r], sA[r][t], dB[r] * sB[r][t]);
    }
}

__device__ inline void fill_lut(float *lut) {
    if (threadIdx.x < 16) lut[threadIdx.x] = (float)kIq4nl[threadIdx.x];
}

// ---------------------------------------------------------------- gate/up
struct GateUpArgs {
    const float *x;
    int nt, H, F;
    const unsigned char *gate, *up;  // routed experts
    const unsigned char *sgate, *sup;  // shared expert or null
    Tile tile;
    Plan pl;
    float *mid;  // [(T*10 + T)][F]: pair rows, then shared rows
    int max_jobs;
};

template <int QT>
__global__ void __launch_bounds__(kThreads) gate_up_kernel(GateUpArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    __shared__ float lut[16];
    __shared__ float red[kThreads / 32][kGateUpRows][2][kTP];
    const int job = blockIdx.y;
    const bool shared_job = a.sgate && job == a.max_jobs;
    int e = 0, first = 0, n = 0;
    if (shared_job) {
        n = a.nt;
    } else {
        if (job >= a.pl.hdr->n_used) return;
        e = a.pl.used[job];
        first = a.pl.off[e];
        n = a.pl.off[e + 1] - first;
    }
    const int r0 = blockIdx.x * kGateUpRows;
    const Tile &tl = a.tile;
    const int tile_bytes = (kGateUpRows / tl.G) * tl.gstride;
    unsigned char *sg = smem, *su = smem + tile_bytes;
    float *xs = reinterpret_cast<float *>(smem + 2 * tile_bytes);
    const int units = a.H / 64;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (QT == 20) fill_lut(lut);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned char *gsrc = (shared_job ? a.sgate : a.gate + (size_t)e * a.F * tl.rb) + (size_t)r0 * tl.rb;
        const unsigned char *usrc = (shared_job ? a.sup : a.up + (size_t)e * a.F * tl.rb) + (size_t)r0 * tl.rb;
        mbar_arrive_expect_tx(&bar, 2u * kGateUpRows * tl.rb);
        tile_load(sg, gsrc, kGateUpRows, tl, &bar);
        tile_load(su, usrc, kGateUpRows, tl, &bar);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = lane & 3, rg = lane >> 2;  // 4 unit slots x 8 row pairs per warp
    const int slot = warp * 4 + c;           // unit slot 0..31
    const unsigned char *rows[4] = {tl.row(sg, 2 * rg), tl.row(sg, 2 * rg + 1), tl.row(su, 2 * rg),
                                    tl.row(su, 2 * rg + 1)};
    bool loaded = false;
    for (int p0 = 0; p0 < n; p0 += kTP) {
        const int np = min(kTP, n - p0);
        const float *src[kTP];
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            int pi = min(t, np - 1);
            int tok = shared_job ? p0 + pi : a.pl.pairs[first + p0 + pi] / kTop;
            src[t] = a.x + (size_t)tok * a.H;
        }
        __syncthreads();  // previous pass finished reading xs / red
        stage_tokens<QT>(xs, src, np, a.H);
        __syncthreads();
        if (!loaded) {
            bool ok = mbar_wait_bounded(&bar, 0, &a.pl.hdr->error);
            if (__syncthreads_or(!ok)) return;  // every thread leaves together on a timeout
            loaded = true;
        }
        float y[4][kTP];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) y[r][t] = 0.0f;
        for (int u = slot; u < units; u += 32) unit_dot<QT, 4>(rows, u, xs, units, lut, y);
        // reduce the 4 unit slots of this warp, then across warps in fixed order
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                float v = y[r][t];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                y[r][t] = v;
            }
        if (c == 0) {
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                red[warp][2 * rg][0][t] = y[0][t];
                red[warp][2 * rg + 1][0][t] = y[1][t];
                red[warp][2 * rg][1][t] = y[2][t];
                red[warp][2 * rg + 1][1][t] = y[3][t];
            }
        }
        __syncthreads();
        if (threadIdx.x < kGateUpRows * kTP) {
            const int row = threadIdx.x / kTP, t = threadIdx.x % kTP;
            if (t < np) {
                float g = 0.0f, uu = 0.0f;
#pragma unroll
                for (int w = 0; w < kThreads / 32; w++) {
                    g += red[w][row][0][t];
                    uu += red[w][row][1][t];
                }
                float m = (g * sigmoidf_ref(g)) * uu;
                size_t mrow = shared_job ? (size_t)a.nt * kTop + p0 + t : (size_t)(first + p0 + t);
                a.mid[mrow * a.F + r0 + row] = m;
            }
        }
    }
}

// ---------------------------------------------------------------- down
struct DownArgs {
    int nt, H, F;
    const unsigned char *down, *sdown;
    const float *wts;
    Tile tile;
    Plan pl;
    const float *mid;
    float *slots, *shared;
    int max_jobs;
};

template <int QT>
__global__ void __launch_bounds__(kThreads) down_kernel(DownArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    __shared__ float lut[16];
    const int job = blockIdx.y;
    const bool shared_job = a.sdown && job == a.max_jobs;
    int e = 0, first = 0, n = 0;
    if (shared_job) {
        n = a.nt;
    } else {
        if (job >= a.pl.hdr->n_used) return;
        e = a.pl.used[job];
        first = a.pl.off[e];
        n = a.pl.off[e + 1] - first;
    }
    const int r0 = blockIdx.x * kDownRows;
    const Tile &tl = a.tile;
    const int tile_bytes = (kDownRows / tl.G) * tl.gstride;
    unsigned char *sd = smem;
    float *xs = reinterpret_cast<float *>(smem + tile_bytes);
    const int units = a.F / 64;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (QT == 20) fill_lut(lut);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned char *src = (shared_job ? a.sdown : a.down + (size_t)e * a.H * tl.rb) + (size_t)r0 * tl.rb;
        mbar_arrive_expect_tx(&bar, (uint32_t)kDownRows * tl.rb);
        tile_load(sd, src, kDownRows, tl, &bar);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = lane & 7, rg = warp * 4 + (lane >> 3);  // 8 unit slots x 32 row pairs
    const unsigned char *rows[2] = {tl.row(sd, 2 * rg), tl.row(sd, 2 * rg + 1)};
    bool loaded = false;
    for (int p0 = 0; p0 < n; p0 += kTP) {
        const int np = min(kTP, n - p0);
        const float *src[kTP];
        int slot_of[kTP];
#pragma unroll
        for (int t = 0; t < kTP; t++) {
            int pi = min(t, np - 1);
            size_t mrow;
            if (shared_job) {
                mrow = (size_t)a.nt * kTop + p0 + pi;
                slot_of[t] = p0 + pi;
            } else {
                mrow = (size_t)(first + p0 + pi);
                slot_of[t] = a.pl.pairs[first + p0 + pi];
            }
            src[t] = a.mid + mrow * a.F;
        }
        __syncthreads();
        stage_tokens<QT>(xs, src, np, a.F);
        __syncthreads();
        if (!loaded) {
            bool ok = mbar_wait_bounded(&bar, 0, &a.pl.hdr->error);
            if (__syncthreads_or(!ok)) return;  // every thread leaves together on a timeout
            loaded = true;
        }
        float y[2][kTP];
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) y[r][t] = 0.0f;
        for (int u = c; u < units; u += 8) unit_dot<QT, 2>(rows, u, xs, units, lut, y);
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                float v = y[r][t];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                y[r][t] = v;
            }
        if (c == 0) {
#pragma unroll
            for (int t = 0; t < kTP; t++) {
                if (t >= np) break;
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    int row = r0 + 2 * rg + r;
                    if (shared_job)
                        a.shared[(size_t)slot_of[t] * a.H + row] = y[r][t];
                    else
                        a.slots[(size_t)slot_of[t] * a.H + row] = y[r][t] * a.wts[slot_of[t]];
                }
            }
        }
    }
}

// ---------------------------------------------------------------- combine
__global__ void combine_kernel(float *out, const float *slots, const int *ids, const float *wts, const int *bad,
                               const float *shared, const float *sgate, int sgate_stride, int nt, int H) {
    const int t = blockIdx.y;
    const int d4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (d4 * 4 >= H) return;
    float4 *o = reinterpret_cast<float4 *>(out + (size_t)t * H) + d4;
    if (bad[t]) {
        *o = make_float4(NAN, NAN, NAN, NAN);
        return;
    }
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < kTop; k++) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (ids[t * kTop + k] >= 0) v = reinterpret_cast<const float4 *>(slots + ((size_t)t * kTop + k) * H)[d4];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
    }
    if (shared) {
        float g = sigmoidf_ref(sgate[(size_t)t * sgate_stride]);
        float4 v = reinterpret_cast<const float4 *>(shared + (size_t)t * H)[d4];
        s.x = __fmaf_rn(v.x, g, s.x);
        s.y = __fmaf_rn(v.y, g, s.y);
        s.z = __fmaf_rn(v.z, g, s.z);
        s.w = __fmaf_rn(v.w, g, s.w);
    }
    *o = s;
}

// ---------------------------------------------------------------- tensor-core planning
// Turns the per-expert token lists into token tiles of at most 64 tokens
// (shared expert first), per-token contribution counts (| bad bit), and
// zeroes the counters the tensor-core kernel counts up.
// Expert parallelism: ep_local (else null) maps each expert to its index on this
// rank or -1, and the shared expert covers tokens [sh_t0, sh_t1) only; out is
// null there (the combine kernel writes every row of the rank's tokens).
__global__ void __launch_bounds__(1024) tc_plan_kernel(Plan pl, const int *ids, int T, int H, int has_shared,
                                                      SubJob *sub, int *n_sub, int *expect, int *gu_done,
                                                      int *tilecnt, float *out, const int *ep_local, int sh_t0,
                                                      int sh_t1) {
    __shared__ int s_pre[kExperts];
    __shared__ int s_wt[32];
    __shared__ int s_total;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = has_shared ? (sh_t1 - sh_t0 + kTcTok - 1) / kTcTok : 0;
    const int n_used = pl.hdr->n_used;
    for (int i = tid; i < S; i += blockDim.x)
        sub[i] = SubJob{-1, 0, min(kTcTok, sh_t1 - sh_t0 - i * kTcTok), sh_t0 + i * kTcTok};
    int tiles = 0;
    if (tid < kExperts && tid < n_used && (!ep_local || __ldg(ep_local + pl.used[tid]) >= 0))
        tiles = (pl.counts[pl.used[tid]] + kTcTok - 1) / kTcTok;
    int incl = tiles;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) s_wt[warp] = incl;
    __syncthreads();
    if (tid < 32) {
        int v = tid < kExperts / 32 ? s_wt[tid] : 0, t = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, t, d);
            if (lane >= d) t += o;
        }
        s_wt[tid] = t - v;
        if (tid == 31) s_total = t;
    }
    __syncthreads();
    if (tid < kExperts) s_pre[tid] = s_wt[warp] + incl - tiles;
    __syncthreads();
    if (tid < kExperts && tid < n_used) {
        const int e = pl.used[tid], n = pl.counts[e], first = pl.off[e];
        const int loc = ep_local ? __ldg(ep_local + e) : e;
        for (int i = 0; i < tiles; i++)
            sub[S + s_pre[tid] + i] = SubJob{loc, first + i * kTcTok, min(kTcTok, n - i * kTcTok), 0};
    }
    const int total = S + s_total;
    if (tid == 0) *n_sub = total;
    for (int i = tid; i < total; i += blockDim.x) gu_done[i] = 0;
    const int dn_mt = H / kTcRows;
    for (int i = tid; i < T * dn_mt; i += blockDim.x) tilecnt[i] = 0;
    for (int t = tid; t < T; t += blockDim.x) {
        int n = 0;
        const bool bad = pl.bad[t] != 0;
        if (!bad)
            for (int k = 0; k < kTop; k++) n += ids[t * kTop + k] >= 0;
        const int e = n + has_shared;
        expect[t] = e | (bad ? 0x10000 : 0);
        if (e == 0 && out) {
            const float v = bad ? __int_as_float(0x7fc00000) : 0.0f;
            for (int d = 0; d < H; d++) out[(size_t)t * H + d] = v;
        }
    }
}

// ---------------------------------------------------------------- host side
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct Shape {
    int T, H, F;
};

int check_shape(int T, int H, int F) {
    if (T < 1 || T > kMaxTokens || H < 64 || F < 64 || H % 64 || F % 64) return cudaErrorInvalidValue;
    if (F % kGateUpRows || H % kDownRows) return cudaErrorInvalidValue;
    return 0;
}

int smem_gate_up(const Tile &t) { return 2 * (kGateUpRows / t.G) * t.gstride; }
int smem_down(const Tile &t) { return (kDownRows / t.G) * t.gstride; }

template <int QT>
int launch_gate_up(const GateUpArgs &a, cudaStream_t st) {
    int bytes = smem_gate_up(a.tile) + kTP * (a.H / 64) * kUnitFloats * 4;
    int rc = cudaFuncSetAttribute(gate_up_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (rc) return rc;
    dim3 grid(a.F / kGateUpRows, a.max_jobs + (a.sgate ? 1 : 0));
    gate_up_kernel<QT><<<grid, kThreads, bytes, st>>>(a);
    return cudaGetLastError();
}

template <int QT>
int launch_down(const DownArgs &a, cudaStream_t st) {
    int bytes = smem_down(a.tile) + kTP * (a.F / 64) * kUnitFloats * 4;
    int rc = cudaFuncSetAttribute(down_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (rc) return rc;
    dim3 grid(a.H / kDownRows, a.max_jobs + (a.sdown ? 1 : 0));
    down_kernel<QT><<<grid, kThreads, bytes, st>>>(a);
    return cudaGetLastError();
}

// Routed experts (+ optional shared expert) from device ids/weights.
// Expert parallelism over a large batch (run_experts): this rank's experts and
// token block [t0, t1) (tokens of rank r: r*block ..), and the ranks' buffers.
struct EpRun {
    const int *local;  // [512] each expert's index on this rank, or -1
    int n_local, ranks, rank, block, t0, t1;
    size_t start;      // offset of the per-call regions in the workspace
    float *slots[kMaxRanks], *shout[kMaxRanks];
    int *flags[kMaxRanks];
    int *epoch;
};

int run_experts(float *out, const float *x, const int *ids, const float *wts, int T, const void *gate, int gt,
                const void *up, int ut, const void *down, int dt, const void *sg, int sgt, const void *su, int sut,
                const void *sd, int sdt, const float *sgate, int sgate_stride, int H, int F, void *ws,
                cudaStream_t st, const EpRun *ep = nullptr) {
    if (int rc = check_shape(T, H, F)) return rc;
    if (!out || !x || !ids || !wts || !gate || !up || !down || !ws) return cudaErrorInvalidValue;
    if (gt != ut || (gt != 12 && gt != 20) || (dt != 12 && dt != 20)) return cudaErrorInvalidValue;
    size_t grb = row_bytes(gt, H), drb = row_bytes(dt, F);
    if (!grb || !drb) return cudaErrorInvalidValue;
    if (!aligned16(gate) || !aligned16(up) || !aligned16(down) || !aligned16(x) || !aligned16(out))
        return cudaErrorInvalidValue;
    const bool has_shared = sg != nullptr;
    if (has_shared) {
        if (!su || !sd || !sgate || sgt != gt || sut != gt || sdt != dt) return cudaErrorInvalidValue;
        if (!aligned16(sg) || !aligned16(su) || !aligned16(sd)) return cudaErrorInvalidValue;
    }
    Layout L = layout(T, H, F, ep ? ep->start : kPrefixBytes);
    char *base = static_cast<char *>(ws);
    if (!aligned16(base)) return cudaErrorInvalidValue;
    Plan pl = plan_ptrs(ws, L);
    float *mid = reinterpret_cast<float *>(base + L.mid);
    float *slots = reinterpret_cast<float *>(base + L.slots);
    float *shared = reinterpret_cast<float *>(base + L.shared);
    const int max_jobs = std::min(T * kTop, kExperts);

    {
        Span sp(kPlan, st);
        if (T >= kPlanMultiMin) {
            const int nch = (T + kPC - 1) / kPC;
            int *pcnt = reinterpret_cast<int *>(base + L.pcnt);
            plan_count_kernel<<<nch, 512, 0, st>>>(ids, wts, T, pl, pcnt);
            plan_scan_kernel<<<1, kExperts, 0, st>>>(nch, pl, pcnt);
            plan_place_kernel<<<nch, 512, 0, st>>>(ids, T, pl, pcnt);
        } else {
            plan_kernel<<<1, 1024, 0, st>>>(ids, wts, T, pl);
        }
    }
    if (int rc = cudaGetLastError()) return rc;
    if (tc_supported(H, F, gt, dt)) {
        // tensor-core path: token tiles, fp16 hi/lo activations, tcgen05 experts
        TcArgs t{};
        t.T = T, t.H = H, t.F = F;
        t.gate = static_cast<const unsigned char *>(gate), t.up = static_cast<const unsigned char *>(up);
        t.down = static_cast<const unsigned char *>(down);
        t.sg = static_cast<const unsigned char *>(sg), t.su = static_cast<const unsigned char *>(su);
        t.sd = static_cast<const unsigned char *>(sd);
        t.grb = grb, t.drb = drb, t.gu_iq4 = gt == 20, t.dn_iq4 = dt == 20;
        t.all_tok = T <= kTcTok;
        t.x16 = reinterpret_cast<__half *>(base + L.x16);
        t.xinv = reinterpret_cast<float *>(base + L.xinv);
        t.xsum = reinterpret_cast<float *>(base + L.xsum);
        t.mi_stride = ((F / 128) + 3) & ~3;
        t.sub = reinterpret_cast<SubJob *>(base + L.sub);
        t.n_sub = reinterpret_cast<int *>(base + L.nsub);
        t.sh_t0 = ep ? ep->t0 : 0, t.sh_t1 = ep ? ep->t1 : T;
        t.shared_subs = has_shared ? (t.sh_t1 - t.sh_t0 + kTcTok - 1) / kTcTok : 0;
        t.pairs = pl.pairs, t.wts = wts, t.ids = ids;
        t.expect = reinterpret_cast<int *>(base + L.expect);
        t.sgate = has_shared ? sgate : nullptr;
        t.mid16 = reinterpret_cast<__half *>(base + L.mid16);
        t.midinv = reinterpret_cast<float *>(base + L.midinv);
        t.msum = reinterpret_cast<float *>(base + L.msum);
        // small batches combine in the expert kernel (last contribution per row tile);
        // large ones store the weighted rows and reduce them in a combine kernel after
        // it, which keeps the per-token fences and counts out of the down tiles' tails
        const bool fused = t.all_tok || ep;
        t.slots = slots, t.shout = shared, t.out = fused ? out : nullptr;
        DecCtr *ctr = reinterpret_cast<DecCtr *>(base + kHdrBytes);
        t.queue = &ctr->tc_queue, t.tc_ticket = &ctr->tc_ticket;
        t.gu_done = reinterpret_cast<int *>(base + L.gudone);
        t.tilecnt = reinterpret_cast<int *>(base + L.tilecnt);
        t.err = &pl.hdr->error;
        t.n_experts = ep ? ep->n_local : kExperts;
        if (ep) {
            t.ep_ranks = ep->ranks, t.ep_rank = ep->rank, t.ep_block = ep->block, t.ep_epoch = ep->epoch;
            t.ep_cap = 0;  // one set of rows: a peer stores a call's rows only after this rank sent its routes
            for (int r = 0; r < kMaxRanks; r++)
                t.ep_slots[r] = ep->slots[r], t.ep_shout[r] = ep->shout[r], t.ep_flags[r] = ep->flags[r];
        }
        TcMaps maps;
        if (int rc = tc_make_maps(t, maps, kTcTok)) return rc;
        {
            Span sp(kPlan, st);
            tc_plan_kernel<<<1, 1024, 0, st>>>(pl, ids, T, H, has_shared ? 1 : 0, const_cast<SubJob *>(t.sub),
                                               const_cast<int *>(t.n_sub), const_cast<int *>(t.expect), t.gu_done,
                                               t.tilecnt, (ep || !fused) ? nullptr : out, ep ? ep->local : nullptr, t.sh_t0,
                                               t.sh_t1);
            if (int rc = cudaGetLastError()) return rc;
            const int rc = t.all_tok ? tc_prep_launch(x, T, H, const_cast<__half *>(t.x16), const_cast<float *>(t.xinv),
                                                      const_cast<float *>(t.xsum), st)
                                     : tc_prep_rows_launch(x, T, H, pl.pairs, &pl.hdr->n_pairs, has_shared,
                                                           const_cast<__half *>(t.x16), const_cast<float *>(t.xinv),
                                                           const_cast<float *>(t.xsum), st);
            if (rc) return rc;
        }
        {
            Span sp(kExpertsFused, st);
            if (int rc = tc_launch(t, maps, st, false, kTcTok)) return rc;
        }
        if (!fused) {
            Span sp(kCombine, st);
            combine_kernel<<<dim3((H / 4 + 127) / 128, T), 128, 0, st>>>(out, slots, ids, wts, pl.bad,
                                                                        has_shared ? shared : nullptr, sgate,
                                                                        sgate_stride, T, H);
        }
        return cudaGetLastError();
    }

    GateUpArgs ga{x, T, H, F, static_cast<const unsigned char *>(gate), static_cast<const unsigned char *>(up),
                  static_cast<const unsigned char *>(sg), static_cast<const unsigned char *>(su), make_tile(grb),
                  pl, mid, max_jobs};
    int rc;
    {
        Span sp(kGateUp, st);
        rc = gt == 12 ? launch_gate_up<12>(ga, st) : launch_gate_up<20>(ga, st);
    }
    if (rc) return rc;
    DownArgs da{T, H, F, static_cast<const unsigned char *>(down), static_cast<const unsigned char *>(sd), wts,
                make_tile(drb), pl, mid, slots, shared, max_jobs};
    {
        Span sp(kDown, st);
        rc = dt == 12 ? launch_down<12>(da, st) : launch_down<20>(da, st);
    }
    if (rc) return rc;
    {
        Span sp(kCombine, st);
        combine_kernel<<<dim3((H / 4 + 127) / 128, T), 128, 0, st>>>(out, slots, ids, wts, pl.bad,
                                                                    has_shared ? shared : nullptr, sgate,
                                                                    sgate_stride, T, H);
    }
    return cudaGetLastError();
}

}  // namespace

extern "C" int qg_moe_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes) {
    if (!bytes || check_shape(tokens, hidden, ffn)) return cudaErrorInvalidValue;
    // every smaller batch fits too (both layouts grow with the token count)
    size_t n = layout(tokens, hidden, ffn).total;
    n = std::max(n, dec_layout(std::min(tokens, kMaxDecodeTokens), hidden, ffn).total);
    *bytes = n;
    return 0;
}

namespace {
// Decode-path arguments over the workspace; ids/wts point at the routing.
DecArgs dec_args(int T, int H, int F, int gt, int dt, const float *x, float *out, int *ids, float *wts, void *ws,
                 size_t start = kPrefixBytes) {
    DecArgs a{};
    DecLayout L = dec_layout(T, H, F, start);
    char *b = static_cast<char *>(ws);
    a.T = T, a.H = H, a.F = F, a.QG = gt, a.QD = dt;
    a.x = x;
    a.out = out;
    a.ids = ids;
    a.wts = wts;
    a.grb = row_bytes(gt, H);
    a.drb = row_bytes(dt, F);
    a.hdr = reinterpret_cast<DecHdr *>(b);
    a.ctr = reinterpret_cast<DecCtr *>(b + kHdrBytes);
    a.logits = reinterpret_cast<float *>(b + L.logits);
    a.sgate = reinterpret_cast<float *>(b + L.sgate);
    a.xpair = reinterpret_cast<float *>(b + L.xpair);
    a.xsum = reinterpret_cast<float *>(b + L.xsum);
    a.mid = reinterpret_cast<float *>(b + L.mid);
    a.msum = reinterpret_cast<float *>(b + L.msum);
    a.slots = reinterpret_cast<float *>(b + L.slots);
    a.shout = reinterpret_cast<float *>(b + L.shout);
    a.off = reinterpret_cast<int *>(b + L.off);
    a.used = reinterpret_cast<int *>(b + L.used);
    a.pairs = reinterpret_cast<int *>(b + L.pairs);
    a.expect = reinterpret_cast<int *>(b + L.expect);
    a.x16 = reinterpret_cast<__half *>(b + L.x16);
    a.xinv = reinterpret_cast<float *>(b + L.xinv);
    a.sub = reinterpret_cast<SubJob *>(b + L.sub);
    a.n_sub = reinterpret_cast<int *>(b + L.nsub);
    a.mid16 = reinterpret_cast<__half *>(b + L.mid16);
    a.midinv = reinterpret_cast<float *>(b + L.midinv);
    a.xs16 = reinterpret_cast<__half *>(b + L.xs16);
    a.gu_part = reinterpret_cast<float *>(b + L.part);
    a.n_experts = kExperts;
    a.ep_shared_here = 1;
    return a;
}

bool dec_pointers_ok(const void *gate, const void *up, const void *down, const float *x, const float *out,
                     const void *ws) {
    return aligned16(gate) && aligned16(up) && aligned16(down) && aligned16(x) && aligned16(out) && aligned16(ws);
}
}  // namespace

extern "C" int qg_moe_routed(float *out, const float *x, const int *ids, const float *weights, int tokens,
                             const void *gate, int gt, const void *up, int ut, const void *down, int dt, int hidden,
                             int ffn, void *workspace) {
    if (check_shape(tokens, hidden, ffn) || !out || !x || !ids || !weights || !gate || !up || !down || !workspace)
        return cudaErrorInvalidValue;
    if (gt == ut && dec_supported(tokens, hidden, ffn, gt, dt)) {
        if (!dec_pointers_ok(gate, up, down, x, out, workspace)) return cudaErrorInvalidValue;
        DecArgs a = dec_args(tokens, hidden, ffn, gt, dt, x, out, const_cast<int *>(ids),
                             const_cast<float *>(weights), workspace);
        a.gate = static_cast<const unsigned char *>(gate);
        a.up = static_cast<const unsigned char *>(up);
        a.down = static_cast<const unsigned char *>(down);
        return dec_run_timed(a, launch_stream);
    }
    return run_experts(out, x, ids, weights, tokens, gate, gt, up, ut, down, dt, nullptr, 0, nullptr, 0, nullptr, 0,
                       nullptr, 0, hidden, ffn, workspace, launch_stream);
}

extern "C" int qg_moe_layer(float *out, int *ids_out, float *weights_out, const float *x, int tokens,
                            const float *router, const float *logit_bias, const void *gate, int gt, const void *up, int ut, const void *down,
                            int dt, const void *sg, int sgt, const void *su, int sut, const void *sd, int sdt,
                            const float *s_router, int hidden, int ffn, void *workspace) {
    if (check_shape(tokens, hidden, ffn) || !router || !workspace || (sg && !s_router)) return cudaErrorInvalidValue;
    cudaStream_t st = launch_stream;
    if (gt == ut && dec_supported(tokens, hidden, ffn, gt, dt) && (!sg || (sgt == gt && sut == gt && sdt == dt))) {
        if (!out || !x || !gate || !up || !down || !dec_pointers_ok(gate, up, down, x, out, workspace) ||
            !aligned16(router) || (sg && (!su || !sd || !aligned16(sg) || !aligned16(su) || !aligned16(sd) ||
                                          !aligned16(s_router))))
            return cudaErrorInvalidValue;
        DecLayout DL = dec_layout(tokens, hidden, ffn);
        char *b = static_cast<char *>(workspace);
        int *ids = ids_out ? ids_out : reinterpret_cast<int *>(b + DL.ids);
        float *wts = weights_out ? weights_out : reinterpret_cast<float *>(b + DL.wts);
        DecArgs a = dec_args(tokens, hidden, ffn, gt, dt, x, out, ids, wts, workspace);
        a.router = router;
        a.bias = logit_bias;
        a.s_router = sg ? s_router : nullptr;
        a.gate = static_cast<const unsigned char *>(gate);
        a.up = static_cast<const unsigned char *>(up);
        a.down = static_cast<const unsigned char *>(down);
        a.sg = static_cast<const unsigned char *>(sg);
        a.su = static_cast<const unsigned char *>(su);
        a.sd = static_cast<const unsigned char *>(sd);
        if (lean_supported(a)) {
            Span sp(kLean, st);
            const int rc = lean_run(a, st);
            // a device that cannot hold every CTA of the cooperative launch at once takes
            // the multi-kernel path below instead
            if (rc != cudaErrorCooperativeLaunchTooLarge) return rc;
            (void)cudaGetLastError();
        }
        return dec_run_timed(a, st);
    }
    Layout L = layout(tokens, hidden, ffn);
    char *base = static_cast<char *>(workspace);
    float *logits = reinterpret_cast<float *>(base + L.logits);
    int *ids = ids_out ? ids_out : reinterpret_cast<int *>(base + L.ids);
    float *wts = weights_out ? weights_out : reinterpret_cast<float *>(base + L.wts);
    float *sgate = logits + (size_t)tokens * kExperts;  // [T] shared-gate logits after the router block
    int rc;
    {
        Span sp(kRouter, st);
        rc = launch_matmul(logits, router, 0, kExperts, hidden, x, tokens, st);
        if (!rc && sg) rc = launch_matmul(sgate, s_router, 0, 1, hidden, x, tokens, st);
    }
    if (rc) return rc;
    {
        Span sp(kRoute, st);
        rc = launch_route(ids, wts, logits, logit_bias, tokens, st);
    }
    if (rc) return rc;
    return run_experts(out, x, ids, wts, tokens, gate, gt, up, ut, down, dt, sg, sgt, su, sut, sd, sdt, sgate, 1,
                       hidden, ffn, workspace, st);
}

extern "C" int qg_moe_status(const void *workspace, int *invalid_tokens, int *selected, int *experts) {
    if (!workspace) return cudaErrorInvalidValue;
    Header h{};
    int rc = cudaDeviceSynchronize();
    if (rc) return rc;
    if ((rc = cudaMemcpy(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost))) return rc;
    if (h.error) {  // sticky until read here
        const int zero = 0;
        if ((rc = cudaMemcpy(static_cast<char *>(const_cast<void *>(workspace)) + offsetof(Header, error), &zero,
                             sizeof(zero), cudaMemcpyHostToDevice)))
            return rc;
    }
    if (invalid_tokens) *invalid_tokens = h.invalid_tokens;
    if (selected) *selected = h.n_pairs;
    if (experts) *experts = h.n_used;
    return h.error ? cudaErrorLaunchTimeout : 0;
}

extern "C" int qg_moe_profile(int enable) {
    g_prof.on = enable != 0;
    g_prof.spans.clear();
    g_prof.next = 0;
    return 0;
}

extern "C" int qg_moe_profile_read(int phase, double *total_ms, int *launches) {
    if (phase < 0 || phase >= kPhases || !total_ms || !launches) return cudaErrorInvalidValue;
    int rc = cudaDeviceSynchronize();
    if (rc) return rc;
    double sum = 0;
    int n = 0;
    for (auto &sp : g_prof.spans) {
        if (sp.first != phase) continue;
        float ms = 0;
        if ((rc = cudaEventElapsedTime(&ms, sp.second.first, sp.second.second))) return rc;
        sum += ms;
        n++;
    }
    *total_ms = sum;
    *launches = n;
    return 0;
}

// ------------------------------------------------------------------ expert parallelism
// One process per GPU. Every rank routes the same tokens (the router is
// replicated and bit-exact, so all ranks agree on every id), runs the tiles of
// the experts it holds, and writes each weighted slot row (and, on one rank,
// the shared expert's rows) straight into every rank's workspace over NVLink.
// Its last CTA then raises its flag in every rank. Each rank's combine kernel
// waits for all flags of the call (bounded), reduces in router-rank order and
// advances the call epoch.
//
// Workspace: everything kept from call to call and everything a peer writes
// before this rank has finished its previous call sits at offsets that do not
// depend on the call's token count, so one workspace serves batches of any
// size up to the one it was sized for, in any order:
//   fixed prefix (status words, decode counters)
//   fixed block: flags, epoch, route flags, the route table (8192 tokens), and
//                the decode batches' slot/shared rows, two sets of 32 tokens
//                (a rank one call ahead writes the other parity's set, never
//                rows a peer is still combining)
//   per-call regions of this rank (dec_layout / layout from the block's end)
//   large batches: one set of slot/shared rows after those (a peer stores a
//                call's rows only after every rank has sent that call's routes,
//                i.e. after this rank's previous combine has finished)
namespace {

struct EpFixed {
    size_t flags, epoch, rflags, rids, rwts, dslots, dshout, start;
};

EpFixed ep_fixed(int H) {
    EpFixed E{};
    size_t p = kPrefixBytes;
    auto take = [&](size_t bytes) {
        size_t at = p;
        p = align256(p + bytes);
        return at;
    };
    E.flags = take(sizeof(int) * kMaxRanks);   // epoch reached by each source rank
    E.epoch = take(sizeof(int) * 2);           // call epoch, combine ticket
    E.rflags = take(sizeof(int) * kMaxRanks);  // epoch whose routes each rank has sent
    E.rids = take(sizeof(int) * (size_t)kMaxTokens * kTop);  // large batches: every rank's routes
    E.rwts = take(sizeof(float) * (size_t)kMaxTokens * kTop);
    E.dslots = take(sizeof(float) * 2 * (size_t)kMaxDecodeTokens * kTop * H);  // [2][32*10][H]
    E.dshout = take(sizeof(float) * 2 * (size_t)kMaxDecodeTokens * H);         // [2][32][H]
    E.start = p;
    return E;
}

// Large batches: this rank's slot rows [T*10][H] and shared rows [T][H] after
// the per-call regions; returns the end of the workspace.
struct EpLarge {
    size_t slots, shout, total;
};

EpLarge ep_large(int T, int H, int F) {
    EpLarge E{};
    E.slots = align256(layout(T, H, F, ep_fixed(H).start).total);
    E.shout = align256(E.slots + sizeof(float) * (size_t)T * kTop * H);
    E.total = align256(E.shout + sizeof(float) * (size_t)T * H);
    return E;
}

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// grid (H/256, tokens from t0): out[t] = sum_k (rank order) slots[t][k] +
// sigmoid(g_t) * shared[t] once every rank has raised its flag for this call.
// cap > 0: the rows sit in the set of the epoch's parity (two sets of cap
// tokens); cap = 0: one set. A wait that runs out sets error bit 8 and gives
// the tokens NaN rows.
__global__ void ep_combine_kernel(float *out, const float *slots, const float *shout, const int *ids,
                                  const int *expect, const float *sgate, int has_shared, int T, int H, int ranks,
                                  const int *flags, int *epoch, int *err, int t0, int cap) {
    __shared__ int s_ok;
    const int t = t0 + blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
    const int e = __ldcg(epoch);
    if (threadIdx.x == 0) {
        int ok = 1;
        const uint64_t t0 = global_ns();
        for (int p = 0; p < ranks && ok; p++)
            while (ld_acquire_sys(flags + p) < e + 1) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(err, 8);
                    ok = 0;
                    break;
                }
                __nanosleep(100);
            }
        s_ok = ok;
    }
    __syncthreads();
    if (d < H && !s_ok) {
        out[(size_t)t * H + d] = __int_as_float(0x7fc00000);
    } else if (d < H) {
        const size_t pt = (cap ? (size_t)(e & 1) * cap : 0) + t;
        const bool bad = (__ldcg(expect + t) & (1 << 16)) != 0;
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < kTop; k++) {
            const int id = __ldcg(ids + t * kTop + k);
            sum += id >= 0 ? __ldcg(slots + (pt * kTop + k) * H + d) : 0.0f;
        }
        if (has_shared) sum = __fmaf_rn(__ldcg(shout + pt * H + d), sigmoidf_ref(__ldcg(sgate + t)), sum);
        out[(size_t)t * H + d] = bad ? __int_as_float(0x7fc00000) : sum;
    }
    // the epoch advances once every CTA has read it
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(epoch + 1, 1) == (int)(gridDim.x * gridDim.y) - 1) {
            epoch[1] = 0;
            __threadfence();
            epoch[0] = e + 1;
        }
    }
}

// Large-batch expert parallelism: each rank routes its own token block and
// shares the ids and weights. CTA p copies rows [t0, t1) into rank p's route
// table, then raises this rank's route flag there for this call (system-scope
// release after a system fence, as for the slot rows).
struct EpRoutes {
    int *rids[kMaxRanks];
    float *rwts[kMaxRanks];
    int *rflags[kMaxRanks];
};

__global__ void ep_routes_send_kernel(const int *ids, const float *wts, int t0, int t1, EpRoutes pr, int rank,
                                      const int *epoch) {
    const int p = blockIdx.x;
    int *dids = pr.rids[p];
    float *dwts = pr.rwts[p];
    for (int i = t0 * kTop + (int)threadIdx.x; i < t1 * kTop; i += blockDim.x) {
        dids[i] = ids[i];
        dwts[i] = wts[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const int e = __ldcg(epoch) + 1;
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(pr.rflags[p] + rank), "r"(e) : "memory");
    }
}

// Waits (bounded: error bit 8, and ids -1 so every token is reported invalid)
// until every rank's routes of this call are in this rank's table, then copies
// the whole table to ids / wts.
__global__ void ep_routes_recv_kernel(int *ids, float *wts, const int *rids, const float *rwts, int T, int ranks,
                                      const int *rflags, const int *epoch, int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        const int e = __ldcg(epoch);
        int ok = 1;
        const uint64_t t0 = global_ns();
        for (int p = 0; p < ranks && ok; p++)
            while (ld_acquire_sys(rflags + p) < e + 1) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(err, 8);
                    ok = 0;
                    break;
                }
                __nanosleep(100);
            }
        s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T * kTop; i += gridDim.x * blockDim.x) {
        ids[i] = ok ? __ldcg(rids + i) : -1;
        wts[i] = ok ? __ldcg(rwts + i) : 0.0f;
    }
}

}  // namespace

extern "C" int qg_ep_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes) {
    if (!bytes || check_shape(tokens, hidden, ffn)) return cudaErrorInvalidValue;
    // every smaller batch fits too (each part grows with the token count)
    const size_t start = ep_fixed(hidden).start;
    size_t n = dec_layout(std::min(tokens, kMaxDecodeTokens), hidden, ffn, start).total;
    if (tokens > kMaxDecodeTokens) n = std::max(n, ep_large(tokens, hidden, ffn).total);
    *bytes = align256(n);
    return 0;
}

extern "C" int qg_ep_ipc_handle(void *workspace, void *handle) {
    if (!workspace || !handle) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    int rc = cudaIpcGetMemHandle(&h, workspace);
    if (rc) return rc;
    memcpy(handle, &h, sizeof(h));
    return 0;
}

extern "C" int qg_ep_ipc_open(const void *handle, void **ptr) {
    if (!handle || !ptr) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" int qg_ep_ipc_close(void *ptr) { return ptr ? cudaIpcCloseMemHandle(ptr) : cudaErrorInvalidValue; }

extern "C" int qg_moe_layer_ep(float *out, int *ids_out, float *weights_out, const float *x, int tokens,
                               const float *router, const float *logit_bias, const void *gate, int gt, const void *up,
                               int ut, const void *down, int dt, int n_local, const int *expert_local, const void *sg,
                               int sgt, const void *su, int sut, const void *sd, int sdt, const float *s_router,
                               int shared_rank, int hidden, int ffn, int rank, int ranks, void *const *workspaces) {
    if (check_shape(tokens, hidden, ffn) || !router || !workspaces || !expert_local || (sg && !s_router))
        return cudaErrorInvalidValue;
    if (ranks < 1 || ranks > kMaxRanks || rank < 0 || rank >= ranks || shared_rank < 0 || shared_rank >= ranks ||
        n_local < 1 || n_local > kExperts)
        return cudaErrorInvalidValue;
    const bool large = tokens > kMaxDecodeTokens;
    // the tensor-core path: Q4_K gate/up, Q4_K or IQ4_NL down (the shared expert alike)
    if (gt != 12 || ut != 12 || (dt != 12 && dt != 20) || (sg && (sgt != 12 || sut != 12 || sdt != dt)) ||
        (!large && !dec_supported(tokens, hidden, ffn, gt, dt)) || !tc_supported(hidden, ffn, gt, dt))
        return cudaErrorNotSupported;
    void *workspace = workspaces[rank];
    for (int p = 0; p < ranks; p++)
        if (!workspaces[p]) return cudaErrorInvalidValue;
    if (!out || !x || !gate || !up || !down || !dec_pointers_ok(gate, up, down, x, out, workspace) ||
        !aligned16(router) || (sg && (!su || !sd || !aligned16(sg) || !aligned16(su) || !aligned16(sd) ||
                                      !aligned16(s_router))))
        return cudaErrorInvalidValue;
    cudaStream_t st = launch_stream;
    if (large) {
        // Large batch: rank r owns tokens [r*block, (r+1)*block). It computes their
        // router logits and top-10 and sends the ids and weights to every rank, so
        // each rank holds all routes without repeating the router; it then runs
        // its experts on the pairs routed to them and the shared expert on its own
        // tokens, stores each weighted row into the buffers of the token's rank,
        // and combines its own tokens once every rank has finished.
        const EpFixed EF = ep_fixed(hidden);
        const Layout L = layout(tokens, hidden, ffn, EF.start);
        const EpLarge EL = ep_large(tokens, hidden, ffn);
        char *b = static_cast<char *>(workspace);
        float *logits = reinterpret_cast<float *>(b + L.logits);
        float *sgate = logits + (size_t)tokens * kExperts;
        int *ids = ids_out ? ids_out : reinterpret_cast<int *>(b + L.ids);
        float *wts = weights_out ? weights_out : reinterpret_cast<float *>(b + L.wts);
        const int block = (tokens + ranks - 1) / ranks;
        const int t0 = std::min(tokens, rank * block), t1 = std::min(tokens, t0 + block), nb = t1 - t0;
        int rc = 0;
        if (nb > 0) {
            Span sp(kRouter, st);
            const float *xb = x + (size_t)t0 * hidden;
            rc = launch_matmul(logits + (size_t)t0 * kExperts, router, 0, kExperts, hidden, xb, nb, st);
            if (!rc && sg) rc = launch_matmul(sgate + t0, s_router, 0, 1, hidden, xb, nb, st);
        }
        if (rc) return rc;
        int *epoch = reinterpret_cast<int *>(b + EF.epoch);
        {
            Span sp(kRoute, st);
            if (nb > 0 &&
                (rc = launch_route(ids + (size_t)t0 * kTop, wts + (size_t)t0 * kTop, logits + (size_t)t0 * kExperts,
                                   logit_bias, nb, st)))
                return rc;
            EpRoutes pr;
            for (int p = 0; p < ranks; p++) {
                char *pb = static_cast<char *>(workspaces[p]);
                pr.rids[p] = reinterpret_cast<int *>(pb + EF.rids);
                pr.rwts[p] = reinterpret_cast<float *>(pb + EF.rwts);
                pr.rflags[p] = reinterpret_cast<int *>(pb + EF.rflags);
            }
            ep_routes_send_kernel<<<ranks, 256, 0, st>>>(ids, wts, t0, t1, pr, rank, epoch);
            ep_routes_recv_kernel<<<16, 256, 0, st>>>(ids, wts, pr.rids[rank], pr.rwts[rank], tokens, ranks,
                                                       pr.rflags[rank], epoch,
                                                       &reinterpret_cast<Header *>(b + L.hdr)->error);
            if ((rc = cudaGetLastError())) return rc;
        }
        EpRun ep{};
        ep.local = expert_local, ep.n_local = n_local, ep.ranks = ranks, ep.rank = rank;
        ep.block = block, ep.t0 = t0, ep.t1 = t1, ep.start = EF.start;
        for (int p = 0; p < ranks; p++) {
            char *pb = static_cast<char *>(workspaces[p]);
            ep.slots[p] = reinterpret_cast<float *>(pb + EL.slots);
            ep.shout[p] = reinterpret_cast<float *>(pb + EL.shout);
            ep.flags[p] = reinterpret_cast<int *>(pb + EF.flags);
        }
        ep.epoch = epoch;
        if ((rc = run_experts(out, x, ids, wts, tokens, gate, gt, up, ut, down, dt, sg, sgt, su, sut, sd, sdt, sgate, 1,
                              hidden, ffn, workspace, st, &ep)))
            return rc;
        if (ep.t1 > ep.t0) {
            Span sp(kCombine, st);
            ep_combine_kernel<<<dim3((hidden + 255) / 256, ep.t1 - ep.t0), 256, 0, st>>>(
                out, ep.slots[rank], ep.shout[rank], ids, reinterpret_cast<const int *>(b + L.expect), sgate,
                sg != nullptr, tokens, hidden, ranks, ep.flags[rank], ep.epoch,
                &reinterpret_cast<Header *>(b + L.hdr)->error, ep.t0, 0);
        } else {  // no tokens here: still advance the call epoch after every rank's rows are in
            ep_combine_kernel<<<dim3(1, 1), 32, 0, st>>>(out, ep.slots[rank], ep.shout[rank], ids,
                                                         reinterpret_cast<const int *>(b + L.expect), sgate, 0, tokens,
                                                         0, ranks, ep.flags[rank], ep.epoch,
                                                         &reinterpret_cast<Header *>(b + L.hdr)->error, 0, 0);
        }
        return cudaGetLastError();
    }
    const EpFixed EF = ep_fixed(hidden);
    const DecLayout DL = dec_layout(tokens, hidden, ffn, EF.start);
    char *b = static_cast<char *>(workspace);
    int *ids = ids_out ? ids_out : reinterpret_cast<int *>(b + DL.ids);
    float *wts = weights_out ? weights_out : reinterpret_cast<float *>(b + DL.wts);
    DecArgs a = dec_args(tokens, hidden, ffn, gt, dt, x, out, ids, wts, workspace, EF.start);
    a.router = router;
    a.bias = logit_bias;
    a.s_router = sg ? s_router : nullptr;
    a.gate = static_cast<const unsigned char *>(gate);
    a.up = static_cast<const unsigned char *>(up);
    a.down = static_cast<const unsigned char *>(down);
    a.sg = static_cast<const unsigned char *>(sg);
    a.su = static_cast<const unsigned char *>(su);
    a.sd = static_cast<const unsigned char *>(sd);
    a.ep_local = expert_local;
    a.n_experts = n_local;
    a.ep_shared_here = rank == shared_rank;
    a.ep_ranks = ranks, a.ep_rank = rank, a.ep_cap = kMaxDecodeTokens;
    for (int p = 0; p < ranks; p++) {
        char *pb = static_cast<char *>(workspaces[p]);
        a.ep_slots[p] = reinterpret_cast<float *>(pb + EF.dslots);
        a.ep_shout[p] = reinterpret_cast<float *>(pb + EF.dshout);
        a.ep_flags[p] = reinterpret_cast<int *>(pb + EF.flags);
    }
    a.ep_epoch = reinterpret_cast<int *>(b + EF.epoch);
    int rc = dec_run_timed(a, st);
    if (rc) return rc;
    Span sp(kCombine, st);  // includes the wait for the peers' rows
    ep_combine_kernel<<<dim3((hidden + 255) / 256, tokens), 256, 0, st>>>(
        out, reinterpret_cast<const float *>(b + EF.dslots), reinterpret_cast<const float *>(b + EF.dshout), ids,
        a.expect, a.sgate, sg != nullptr, tokens, hidden, ranks, reinterpret_cast<const int *>(b + EF.flags),
        reinterpret_cast<int *>(b + EF.epoch), &a.hdr->error, 0, kMaxDecodeTokens);
    return cudaGetLastError();
}
