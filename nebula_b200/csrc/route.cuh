// Warp-parallel top-10-of-512 routing shared by qg_route and the MoE layer.
#pragma once
#include "common.cuh"

namespace nb {
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
    float sel_w[kTop];
    int sel_id[kTop];
    float largest = 0.0f;
#pragma unroll
    for (int k = 0; k < kTop; k++) {
        // lane-local best: highest value, then lowest index (indices grow with m)
        float bv = v[0];
        int bm = 0;
#pragma unroll
        for (int m = 1; m < 16; m++)
            if (v[m] > bv) {
                bv = v[m];
                bm = m;
            }
        int bi = bm * 32 + lane;
#pragma unroll
        for (int d = 16; d; d >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, d);
            int oi = __shfl_xor_sync(0xffffffffu, bi, d);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (k == 0) largest = bv;  // the first pick is the maximum of all 512
        sel_id[k] = bi;
        sel_w[k] = expf(bv - largest);
        if ((bi & 31) == lane) {
#pragma unroll
            for (int m = 0; m < 16; m++)
                if (m == (bi >> 5)) v[m] = -INFINITY;
        }
    }
    if (lane == 0) {
        float total = 0.0f;
#pragma unroll
        for (int k = 0; k < kTop; k++) total += sel_w[k];
#pragma unroll
        for (int k = 0; k < kTop; k++) {
            ids[k] = sel_id[k];
            weights[k] = sel_w[k] / total;
        }
    }
}
}  // namespace nb
