// Warp-parallel top-10-of-512 routing shared by qg_route and the MoE layer.
#pragma once
#include "common.cuh"

namespace nb {
// Order-preserving map of finite floats to unsigned keys (and back).
__device__ __forceinline__ uint32_t float_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Top-10 of 512 for one token, run by a full warp. Reference semantics
// (qwen/gpu.cu:456-465): any non-finite logit -> ids -1, weights 0; ten
// argmax passes with lowest-index tie break; w = expf(s - max), divided by
// their sum taken in rank order. Lane 0 writes the results.
// `bias` (optional, [512]) is added to the logits first.
__device__ __forceinline__ void route_token_warp(const float *logits, const float *bias, int *ids, float *weights) {
    const int lane = threadIdx.x & 31;
    float v[16];
    bool bad = false;
#pragma unroll
    for (int m = 0; m < 16; m++) {
        v[m] = __ldcg(logits + m * 32 + lane);  // index m*32+lane; L2 read (other CTAs may have written it)
        if (bias) v[m] += __ldg(bias + m * 32 + lane);
        bad |= !isfinite(v[m]);
    }
    bad = __any_sync(0xffffffffu, bad);
    if (bad) {
        if (lane < kTop) {
            ids[lane] = -1;
            weights[lane] = 0.0f;
        }
        return;
    }
    // Each lane keeps the best of its 16 values as an order-preserving key; a
    // pick is two warp reductions: the largest key, then the lowest index among
    // the lanes holding it. Only the winning lane rescans its values (a taken
    // mask, so everything stays in registers). Lane k keeps pick k; every lane
    // sums the weights in rank order.
    uint32_t key[16];
#pragma unroll
    for (int m = 0; m < 16; m++) key[m] = float_key(v[m] + 0.0f);  // -0 ties with +0, as in the comparison
    uint32_t taken = 0, bk = key[0];
    int bm = 0;
#pragma unroll
    for (int m = 1; m < 16; m++)
        if (key[m] > bk) bk = key[m], bm = m;
    float largest = 0.0f, total = 0.0f, my_w = 0.0f;
    int my_id = -1;
#pragma unroll 1
    for (int k = 0; k < kTop; k++) {
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const int bi = (int)__reduce_min_sync(0xffffffffu, bk == mk ? (uint32_t)(bm * 32 + lane) : 0xFFFFu);
        const float bv = key_float(mk);
        if (k == 0) largest = bv;  // the first pick is the maximum of all 512
        const float w = expf(bv - largest);
        total += w;
        if (lane == k) my_id = bi, my_w = w;
        if ((bi & 31) == lane) {
            taken |= 1u << (bi >> 5);
            bk = 0, bm = 0;
#pragma unroll
            for (int m = 0; m < 16; m++)
                if (!((taken >> m) & 1u) && key[m] > bk) bk = key[m], bm = m;
        }
    }
    if (lane < kTop) {
        ids[lane] = my_id;
        weights[lane] = my_w / total;
    }
}
}  // namespace nb
