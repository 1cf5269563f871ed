// Per-element decoding of the GGML block formats the reference supports, and
// the 32-lane dot-product order that makes GPU and CPU results bitwise equal.
//
// The block layouts are GGML's (they are the on-disk format of the weights);
// the per-element arithmetic below is arranged so that every decoded weight
// equals the reference's value bit for bit (qwen/cpu.c:43-67,
// qwen/gpu.cu:121-153): each decoded value is either exact in fp32 or, for
// Q4_K/Q5_K, a single rounding of an exact d*sc*q - dmin*m.
#pragma once
#include "common.cuh"

namespace nb {

// IQ4_NL non-linear code book (GGML's kvalues_iq4nl).
static __constant__ const signed char kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                             1,    13,   25,  38,  53,  69,  89,  113};

// IQ4_NL: four codes (one per byte of q, each < 16) -> code-book value + 128
// per byte, selected with byte permutes from two 8-entry halves.
__device__ __forceinline__ uint32_t iq4_lut4(uint32_t q) {
    // code book + 128: 1,24,45,63,79,93,106,118 | 129,141,153,166,181,197,217,241
    constexpr uint32_t T0 = 0x3F2D1801u, T1 = 0x766A5D4Fu, T2 = 0xA6998D81u, T3 = 0xF1D9C5B5u;
    const uint32_t s = q & 0x07070707u;
    const uint32_t n = s | (s >> 4);
    const uint32_t sel = __byte_perm(n, 0, 0x0020);
    const uint32_t lo = __byte_perm(T0, T1, sel), hi = __byte_perm(T2, T3, sel);
    uint32_t mask;  // 0xFF where the code is >= 8: prmt replicates bit 7 of each byte (selector msb set)
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(mask) : "r"(q << 4), "r"(0xBA98u));
    return (hi & mask) | (lo & ~mask);
}
// Q4_K / Q5_K 6-bit scale and min of sub-block g from the 12 packed bytes.
__device__ __forceinline__ void k_scale_min(const unsigned char *sc, int g, int &s, int &m) {
    if (g < 4) {
        s = sc[g] & 63;
        m = sc[g + 4] & 63;
    } else {
        s = (sc[g + 4] & 15) | ((sc[g - 4] >> 6) << 4);
        m = (sc[g + 4] >> 4) | ((sc[g] >> 6) << 4);
    }
}

// Value i of a packed row of GGML type t.
__device__ inline float decode_at(const unsigned char *row, int t, int i) {
    switch (t) {
    case 0: return reinterpret_cast<const float *>(row)[i];
    case 1: return half_at(row + 2 * i);
    case 30: return __uint_as_float(static_cast<unsigned>(reinterpret_cast<const unsigned short *>(row)[i]) << 16);
    case 8: {
        const unsigned char *p = row + (i / 32) * 34;
        return half_at(p) * static_cast<float>(reinterpret_cast<const signed char *>(p + 2)[i % 32]);
    }
    case 2: case 6: case 7: case 20: {
        int bytes = t == 7 ? 24 : t == 6 ? 22 : 18, j = i % 32, off = t == 7 ? 8 : t == 6 ? 6 : 2;
        const unsigned char *p = row + (i / 32) * bytes;
        int q = (p[off + j % 16] >> ((j / 16) * 4)) & 15;
        if (t == 6 || t == 7) {
            const unsigned char *h = p + (t == 7 ? 4 : 2);
            unsigned high = h[0] | (h[1] << 8) | (h[2] << 16) | (static_cast<unsigned>(h[3]) << 24);
            q |= ((high >> j) & 1) << 4;
        }
        if (t == 20) return half_at(p) * static_cast<float>(kIq4nl[q]);
        if (t == 7) return __fmaf_rn(half_at(p), static_cast<float>(q), half_at(p + 2));
        return half_at(p) * static_cast<float>(q - (t == 2 ? 8 : 16));
    }
    case 14: {
        int k = i % 256, h = k / 128, s = (k % 128) / 32, l = k % 32;
        const unsigned char *p = row + (i / 256) * 210;
        int lo = (p[h * 64 + (s % 2) * 32 + l] >> ((s / 2) * 4)) & 15;
        int hi = (p[128 + h * 32 + l] >> (s * 2)) & 3;
        int scale = reinterpret_cast<const signed char *>(p + 192)[h * 8 + s * 2 + l / 16];
        return half_at(p + 208) * static_cast<float>(scale) * static_cast<float>((lo | (hi << 4)) - 32);
    }
    case 12: case 13: {
        int k = i % 256, g = k / 32, l = k % 32;
        const unsigned char *p = row + (i / 256) * (t == 12 ? 144 : 176);
        int s, m;
        k_scale_min(p + 4, g, s, m);
        int q = (p[(t == 12 ? 16 : 48) + (g / 2) * 32 + l] >> ((g % 2) * 4)) & 15;
        if (t == 13) q |= ((p[16 + l] >> g) & 1) << 4;
        return __fmaf_rn(half_at(p) * static_cast<float>(s), static_cast<float>(q),
                         -(half_at(p + 2) * static_cast<float>(m)));
    }
    default: return 0.0f;
    }
}

// Butterfly 16/8/4/2/1 with __shfl_down: lane 0 ends with the reference's
// reduction tree (qwen/gpu.cu:89-92; _mm512_reduce_add_ps in qwen/cpu.c:139).
__device__ __forceinline__ float lane_tree(float v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_down_sync(0xffffffffu, v, d);
    return v;
}

// Accumulates one weight row against NT token vectors in the reference's
// 32-lane order: lane j owns columns k = j (mod 32) in increasing k, one
// fused multiply-add per element. Results stay per-lane (call lane_tree).
template <int T, int NT>
__device__ __forceinline__ void lane_dot(const unsigned char *row, int cols, const float *const *xs, int n,
                                         float (&acc)[NT]) {
    const int lane = threadIdx.x & 31;
    if (T == 0) {
        const float *w = reinterpret_cast<const float *>(row);
        for (int k = lane; k < cols; k += 32) {
            float a = __ldg(w + k);
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t < n) acc[t] = __fmaf_rn(a, __ldg(xs[t] + k), acc[t]);
        }
    } else if (T == 12) {
        for (int sb = 0; sb < cols / 256; sb++) {
            const unsigned char *p = row + sb * 144;
            // lanes 0..7 decode (d*sc, dmin*m) of sub-block `lane`; everyone reads them back.
            float ds = 0, dm = 0;
            if (lane < 8) {
                int s, m;
                k_scale_min(p + 4, lane, s, m);
                ds = half_at(p) * static_cast<float>(s);
                dm = half_at(p + 2) * static_cast<float>(m);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                unsigned b = __ldg(p + 16 + 32 * i + lane);
                float ds0 = __shfl_sync(0xffffffffu, ds, 2 * i), dm0 = __shfl_sync(0xffffffffu, dm, 2 * i);
                float ds1 = __shfl_sync(0xffffffffu, ds, 2 * i + 1), dm1 = __shfl_sync(0xffffffffu, dm, 2 * i + 1);
                float w0 = __fmaf_rn(ds0, static_cast<float>(b & 15), -dm0);
                float w1 = __fmaf_rn(ds1, static_cast<float>(b >> 4), -dm1);
                int k0 = sb * 256 + 64 * i + lane;
#pragma unroll
                for (int t = 0; t < NT; t++)
                    if (t < n) acc[t] = __fmaf_rn(w0, __ldg(xs[t] + k0), acc[t]);
#pragma unroll
                for (int t = 0; t < NT; t++)
                    if (t < n) acc[t] = __fmaf_rn(w1, __ldg(xs[t] + k0 + 32), acc[t]);
            }
        }
    } else if (T == 20) {
        for (int b = 0; b < cols / 32; b++) {
            const unsigned char *p = row + b * 18;
            unsigned byte = __ldg(p + 2 + (lane & 15));
            int q = lane < 16 ? (byte & 15) : (byte >> 4);
            float a = half_at(p) * static_cast<float>(kIq4nl[q]);
            int k = b * 32 + lane;
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t < n) acc[t] = __fmaf_rn(a, __ldg(xs[t] + k), acc[t]);
        }
    } else {
        for (int k = lane; k < cols; k += 32) {
            float a = decode_at(row, T, k);
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t < n) acc[t] = __fmaf_rn(a, __ldg(xs[t] + k), acc[t]);
        }
    }
}

// Runtime-type version of lane_dot for the less common formats.
template <int NT>
__device__ __forceinline__ void lane_dot_generic(const unsigned char *row, int type, int cols,
                                                 const float *const *xs, int n, float (&acc)[NT]) {
    const int lane = threadIdx.x & 31;
    for (int k = lane; k < cols; k += 32) {
        float a = decode_at(row, type, k);
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < n) acc[t] = __fmaf_rn(a, __ldg(xs[t] + k), acc[t]);
    }
}

}  // namespace nb
