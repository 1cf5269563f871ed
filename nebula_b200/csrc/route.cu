// Routing and the per-expert MoE primitives of the qwen/gpu.h ABI:
// qg_route, qg_prune_routes, qg_moe_map/gather/scatter/reduce, qg_mtp_moe.
//
// Results are identical to the reference kernels (qwen/gpu.cu:456-551); the
// implementations are warp-parallel where the reference is serial (top-10 is
// a warp argmax per pass instead of one thread scanning 512 logits ten times;
// the expert map is a ballot/popcount compaction per expert).
#include "quant.cuh"

using namespace nb;

#include "route.cuh"

namespace {
__global__ void route_kernel(int *ids, float *weights, const float *logits, const float *bias, int nt) {
    int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= nt) return;
    route_token_warp(logits + (size_t)t * kExperts, bias, ids + t * kTop, weights + t * kTop);
}

__global__ void prune_kernel(int *ids, float *weights, const unsigned char *resident, int nt, double threshold,
                             qg_prune_stats *stats) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nt) return;
    int missing = 0;
    double mass = 0;
    for (int k = 0; k < kTop; k++) {
        int e = ids[t * kTop + k];
        if (e < 0 || e >= kExperts) return;  // invalid distributions are left to the caller
        if (!resident[e]) {
            missing++;
            mass += (double)weights[t * kTop + k];
        }
    }
    atomicAdd(reinterpret_cast<unsigned long long *>(&stats->token_layers), 1ULL);
    atomicAdd(reinterpret_cast<unsigned long long *>(&stats->missing_selections), (unsigned long long)missing);
    if (missing && threshold > 0 && mass < threshold) {
        for (int k = 0; k < kTop; k++) {
            int e = ids[t * kTop + k];
            if (!resident[e]) {
                ids[t * kTop + k] = -e - 2;  // keeps the omitted id recoverable; -1 stays "invalid"
                weights[t * kTop + k] = 0.0f;
            }
        }
        atomicAdd(reinterpret_cast<unsigned long long *>(&stats->skipped_selections), (unsigned long long)missing);
        atomicAdd(reinterpret_cast<unsigned long long *>(&stats->avoided_token_handoffs), 1ULL);
        atomicAdd(&stats->skipped_mass, mass);
    }
}

// One warp per expert; tokens in chunks of 32, compacted with ballot/popc so
// each expert's list stays in ascending token order.
__global__ void moe_map_kernel(int *map, const int *ids, int nt) {
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (e >= kExperts) return;
    int base = 0;
    for (int t0 = 0; t0 < nt; t0 += 32) {
        int t = t0 + lane;
        bool sel = false;
        if (t < nt)
#pragma unroll
            for (int k = 0; k < kTop; k++) sel |= ids[t * kTop + k] == e;
        unsigned mask = __ballot_sync(0xffffffffu, sel);
        if (sel) map[(size_t)e * nt + base + __popc(mask & ((1u << lane) - 1))] = t;
        base += __popc(mask);
    }
}

constexpr int kLegacyWidth = 2560, kLegacyFfn = 640;

__global__ void moe_gather_kernel(float *out, const float *x, const int *map) {
    int rank = blockIdx.x, t = map[rank];
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * kLegacyWidth);
    float4 *dst = reinterpret_cast<float4 *>(out + (size_t)rank * kLegacyWidth);
    for (int d = threadIdx.x; d < kLegacyWidth / 4; d += blockDim.x) dst[d] = src[d];
}

__global__ void moe_scatter_kernel(float *slots, const float *x, const float *w, const int *ids, const int *map,
                                   int expert) {
    __shared__ int slot;
    int rank = blockIdx.x, t = map ? map[rank] : rank;
    if (!threadIdx.x) {
        slot = -1;
        for (int k = 0; k < kTop; k++)
            if (ids[t * kTop + k] == expert) slot = k;
    }
    __syncthreads();
    if (slot < 0) return;
    float scale = w[t * kTop + slot];
    float *dst = slots + ((size_t)t * kTop + slot) * kLegacyWidth;
    const float *src = x + (size_t)rank * kLegacyWidth;
    for (int d = threadIdx.x; d < kLegacyWidth; d += blockDim.x) dst[d] = src[d] * scale;
}

__global__ void moe_reduce_kernel(float *out, const float *slots, int nt) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nt * kLegacyWidth) return;
    int t = i / kLegacyWidth, d = i % kLegacyWidth;
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kTop; k++) sum += slots[((size_t)t * kTop + k) * kLegacyWidth + d];
    out[i] = sum;
}

// MTP path (qwen/gpu.cu:528-551): one warp per (row, rank, token) in the
// reference lane order, so gate/up/down dot products are bitwise equal to
// the reference's.
template <int GT, int UT>
__global__ void mtp_gate_up_kernel(float *mid, const float *x, const int *ids, const unsigned char *g, int gt,
                                   size_t gs, const unsigned char *u, int ut, size_t us) {
    int row = blockIdx.x * 8 + (threadIdx.x >> 5), rank = blockIdx.y, t = blockIdx.z;
    int e = ids[t * kTop + rank];
    if (row >= kLegacyFfn) return;
    if (e < 0 || e >= kExperts) {
        if ((threadIdx.x & 31) == 0) mid[(t * kTop + rank) * kLegacyFfn + row] = NAN;
        return;
    }
    const float *xs[1] = {x + (size_t)t * kLegacyWidth};
    float sg[1] = {0.0f}, su[1] = {0.0f};
    const unsigned char *grow = g + ((size_t)e * kLegacyFfn + row) * gs, *urow = u + ((size_t)e * kLegacyFfn + row) * us;
    if constexpr (GT >= 0) lane_dot<GT, 1>(grow, kLegacyWidth, xs, 1, sg);
    else lane_dot_generic<1>(grow, gt, kLegacyWidth, xs, 1, sg);
    if constexpr (UT >= 0) lane_dot<UT, 1>(urow, kLegacyWidth, xs, 1, su);
    else lane_dot_generic<1>(urow, ut, kLegacyWidth, xs, 1, su);
    float a = lane_tree(sg[0]), b = lane_tree(su[0]);
    if ((threadIdx.x & 31) == 0) mid[(t * kTop + rank) * kLegacyFfn + row] = (a * sigmoidf_ref(a)) * b;
}

template <int DT>
__global__ void mtp_down_kernel(float *slots, const float *mid, const int *ids, const float *weights,
                                const unsigned char *d, int dt, size_t stride) {
    int row = blockIdx.x * 8 + (threadIdx.x >> 5), rank = blockIdx.y, t = blockIdx.z;
    int e = ids[t * kTop + rank];
    if (row >= kLegacyWidth) return;
    if (e < 0 || e >= kExperts) {
        if ((threadIdx.x & 31) == 0) slots[(t * kTop + rank) * kLegacyWidth + row] = NAN;
        return;
    }
    const float *xs[1] = {mid + (size_t)(t * kTop + rank) * kLegacyFfn};
    float acc[1] = {0.0f};
    const unsigned char *drow = d + ((size_t)e * kLegacyWidth + row) * stride;
    if constexpr (DT >= 0) lane_dot<DT, 1>(drow, kLegacyFfn, xs, 1, acc);
    else lane_dot_generic<1>(drow, dt, kLegacyFfn, xs, 1, acc);
    float s = lane_tree(acc[0]);
    if ((threadIdx.x & 31) == 0) slots[(t * kTop + rank) * kLegacyWidth + row] = s * weights[t * kTop + rank];
}

template <int GT, int UT, int DT>
int launch_mtp(float *slots, float *mid, const float *x, const int *ids, const float *weights, const void *g,
               int gt, size_t gs, const void *u, int ut, size_t us, const void *d, int dt, size_t ds, int nt) {
    mtp_gate_up_kernel<GT, UT><<<dim3(kLegacyFfn / 8, kTop, nt), 256, 0, launch_stream>>>(
        mid, x, ids, static_cast<const unsigned char *>(g), gt, gs, static_cast<const unsigned char *>(u), ut, us);
    int rc = cudaGetLastError();
    if (rc) return rc;
    mtp_down_kernel<DT><<<dim3(kLegacyWidth / 8, kTop, nt), 256, 0, launch_stream>>>(
        slots, mid, ids, weights, static_cast<const unsigned char *>(d), dt, ds);
    return cudaGetLastError();
}
}  // namespace

namespace nb {
int launch_route(int *ids, float *weights, const float *logits, const float *bias, int nt, cudaStream_t st) {
    if (!ids || !weights || !logits || nt < 1 || nt > kMaxTokens) return cudaErrorInvalidValue;
    route_kernel<<<(nt + 7) / 8, 256, 0, st>>>(ids, weights, logits, bias, nt);
    return cudaGetLastError();
}
}  // namespace nb

extern "C" int qg_route(int *ids, float *weights, const float *logits, int nt) {
    return launch_route(ids, weights, logits, nullptr, nt, launch_stream);
}

extern "C" int qg_prune_routes(int *ids, float *weights, const unsigned char *resident, int nt, double threshold,
                               qg_prune_stats *stats) {
    if (!ids || !weights || !resident || !stats || nt < 1 || nt > kMaxTokens || threshold < 0 || threshold > 0.1 ||
        !isfinite(threshold))
        return cudaErrorInvalidValue;
    prune_kernel<<<(nt + 127) / 128, 128, 0, launch_stream>>>(ids, weights, resident, nt, threshold, stats);
    return cudaGetLastError();
}

extern "C" int qg_moe_map(int *map, const int *ids, int nt) {
    if (!map || !ids || nt < 1 || nt > kMaxTokens) return cudaErrorInvalidValue;
    moe_map_kernel<<<kExperts / 8, 256, 0, launch_stream>>>(map, ids, nt);
    return cudaGetLastError();
}

extern "C" int qg_moe_gather(float *o, const float *x, const int *map, int selected) {
    if (selected < 0 || (selected && (!o || !x || !map))) return cudaErrorInvalidValue;
    if (!selected) return 0;
    moe_gather_kernel<<<selected, 128, 0, launch_stream>>>(o, x, map);
    return cudaGetLastError();
}

extern "C" int qg_moe_scatter(float *o, const float *x, const float *w, const int *ids, const int *map, int expert,
                              int selected) {
    if (selected < 0 || (selected && (!o || !x || !w || !ids))) return cudaErrorInvalidValue;
    if (!selected) return 0;
    moe_scatter_kernel<<<selected, 256, 0, launch_stream>>>(o, x, w, ids, map, expert);
    return cudaGetLastError();
}

extern "C" int qg_moe_reduce(float *out, const float *slots, int nt) {
    if (!out || !slots || nt < 1) return cudaErrorInvalidValue;
    moe_reduce_kernel<<<(nt * kLegacyWidth + 255) / 256, 256, 0, launch_stream>>>(out, slots, nt);
    return cudaGetLastError();
}

extern "C" int qg_mtp_moe(float *slots, float *mid, const float *x, const int *ids, const float *weights,
                          const void *g, int gt, const void *u, int ut, const void *d, int dt, int nt) {
    size_t gs = row_bytes(gt, kLegacyWidth), us = row_bytes(ut, kLegacyWidth), ds = row_bytes(dt, kLegacyFfn);
    // Catch-up replays the anchor plus sixteen accepted proposals (qwen/gpu.cu:546-547).
    if (!gs || !us || !ds || nt < 1 || nt > 17 || !slots || !mid || !x || !ids || !weights || !g || !u || !d)
        return cudaErrorInvalidValue;
#define NB_MTP(G, U, D) launch_mtp<G, U, D>(slots, mid, x, ids, weights, g, gt, gs, u, ut, us, d, dt, ds, nt)
    if (gt == 12 && ut == 12 && dt == 20) return NB_MTP(12, 12, 20);
    if (gt == 12 && ut == 12 && dt == 12) return NB_MTP(12, 12, 12);
    if (gt == 20 && ut == 20 && dt == 20) return NB_MTP(20, 20, 20);
    // Other format mixes go through the per-element decoder.
    return NB_MTP(-1, -1, -1);
#undef NB_MTP
}
