// Synthetic weights and activations for tests and benchmarks (qg_synth_*).
//
// Values are approximately N(0, stddev) from a counter-based generator: the
// sum of eight 16-bit uniforms taken from two splitmix64 hashes of the seed
// and the element index (Irwin-Hall with n = 8, support +-4.9 stddev),
// centred and scaled. Any slice can be regenerated independently and
// identically. Quantisation is this library's own simple round-to-nearest
// scheme for the GGML Q4_K and IQ4_NL layouts; the reference used llama.cpp's
// searched quantiser, which is not available here. Kernel parity never
// depends on it: the checkers read back the exact bytes the device produced.
//
// Every floating-point step is a single correctly rounded operation (integer
// sums, int->float conversion, one multiply, IEEE divide, fp16 round to
// nearest even; products that feed an add are written with __fmul_rn so no
// multiply-add is contracted), so a host restatement reproduces the bytes
// bit for bit.
#include "quant.cuh"

using namespace nb;

namespace {
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

// 1 / standard deviation of 2*S - 8*65535 for S a sum of eight uniform
// 16-bit integers: 1 / (65536 * sqrt(8/3)).
constexpr float kIhInvStd = 9.3440618e-06f;

// Element i of the stream `seed`.
__device__ inline float normal_at(uint64_t seed, uint64_t i, float stddev) {
    const uint64_t k = seed * 0xd1342543de82ef95ULL;
    const uint64_t h1 = mix64(k ^ mix64(2 * i)), h2 = mix64(k ^ mix64(2 * i + 1));
    int64_t s = 0;
    for (int j = 0; j < 4; j++) s += (int64_t)((h1 >> (16 * j)) & 0xffff) + (int64_t)((h2 >> (16 * j)) & 0xffff);
    const int c = (int)(2 * s - 8 * 65535);  // odd, |c| < 2^20: exact as a float
    return __fmul_rn(__int2float_rn(c), __fmul_rn(stddev, kIhInvStd));
}

__global__ void normal_kernel(float *dst, size_t n, uint64_t seed, float stddev) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = normal_at(seed, i, stddev);
}

__device__ inline unsigned short f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// One Q4_K superblock (256 values) per thread.
__global__ void q4k_kernel(unsigned char *dst, int rows, int cols, uint64_t seed, float stddev) {
    const int sbs = cols / 256;
    const size_t nsb = (size_t)rows * sbs;
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nsb; b += (size_t)gridDim.x * blockDim.x) {
        const size_t r = b / sbs, sb = b % sbs;
        const uint64_t first = r * (uint64_t)cols + sb * 256;
        float scale[8], minv[8];
        float smax = 0.0f, mmax = 0.0f;
        for (int g = 0; g < 8; g++) {
            float lo = 0.0f, hi = 0.0f;  // the range always contains 0, so mins are >= 0
            for (int l = 0; l < 32; l++) {
                float v = normal_at(seed, first + g * 32 + l, stddev);
                lo = fminf(lo, v);
                hi = fmaxf(hi, v);
            }
            scale[g] = (hi - lo) / 15.0f;
            minv[g] = -lo;
            smax = fmaxf(smax, scale[g]);
            mmax = fmaxf(mmax, minv[g]);
        }
        unsigned short dh = f16_bits(smax / 63.0f), mh = f16_bits(mmax / 63.0f);
        float d = __half2float(__ushort_as_half(dh)), dmin = __half2float(__ushort_as_half(mh));
        int sc[8], mc[8];
        for (int g = 0; g < 8; g++) {
            sc[g] = d > 0 ? min(63, max(0, __float2int_rn(scale[g] / d))) : 0;
            mc[g] = dmin > 0 ? min(63, max(0, __float2int_rn(minv[g] / dmin))) : 0;
        }
        unsigned char *p = dst + b * 144;
        p[0] = dh & 255;
        p[1] = dh >> 8;
        p[2] = mh & 255;
        p[3] = mh >> 8;
        for (int j = 0; j < 4; j++) {
            p[4 + j] = (unsigned char)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            p[8 + j] = (unsigned char)((mc[j] & 63) | ((mc[j + 4] >> 4) << 6));
            p[12 + j] = (unsigned char)((sc[j + 4] & 15) | ((mc[j + 4] & 15) << 4));
        }
        for (int i = 0; i < 4; i++) {
            const int g0 = 2 * i, g1 = 2 * i + 1;
            const float ds0 = __fmul_rn(d, (float)sc[g0]), dm0 = __fmul_rn(dmin, (float)mc[g0]);
            const float ds1 = __fmul_rn(d, (float)sc[g1]), dm1 = __fmul_rn(dmin, (float)mc[g1]);
            for (int l = 0; l < 32; l++) {
                float v0 = normal_at(seed, first + g0 * 32 + l, stddev);
                float v1 = normal_at(seed, first + g1 * 32 + l, stddev);
                int q0 = ds0 > 0 ? min(15, max(0, __float2int_rn((v0 + dm0) / ds0))) : 0;
                int q1 = ds1 > 0 ? min(15, max(0, __float2int_rn((v1 + dm1) / ds1))) : 0;
                p[16 + 32 * i + l] = (unsigned char)(q0 | (q1 << 4));
            }
        }
    }
}

// One IQ4_NL block (32 values) per thread: d = (signed extreme)/(-127), each
// value to the nearest code-book entry.
__global__ void iq4nl_kernel(unsigned char *dst, int rows, int cols, uint64_t seed, float stddev) {
    const int bpr = cols / 32;
    const size_t nb_ = (size_t)rows * bpr;
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb_; b += (size_t)gridDim.x * blockDim.x) {
        const size_t r = b / bpr, blk = b % bpr;
        const uint64_t first = r * (uint64_t)cols + blk * 32;
        float ext = 0.0f;
        for (int l = 0; l < 32; l++) {
            float v = normal_at(seed, first + l, stddev);
            if (fabsf(v) > fabsf(ext)) ext = v;
        }
        unsigned short dh = f16_bits(ext / -127.0f);
        float d = __half2float(__ushort_as_half(dh));
        unsigned char q[32];
        for (int l = 0; l < 32; l++) {
            float v = normal_at(seed, first + l, stddev);
            int best = 0;
            float err = INFINITY;
            for (int c = 0; c < 16; c++) {
                float e = fabsf(__fmul_rn(d, (float)kIq4nl[c]) - v);
                if (e < err) {
                    err = e;
                    best = c;
                }
            }
            q[l] = (unsigned char)best;
        }
        // the 18-byte block as nine little-endian 16-bit words (blocks start on even
        // addresses): d, then code bytes j = 0..15 holding values j (low nibble) and
        // j+16 (high nibble)
        unsigned short *p16 = reinterpret_cast<unsigned short *>(dst + b * 18);
        p16[0] = dh;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const unsigned lo = q[2 * i] | (q[2 * i + 16] << 4), hi = q[2 * i + 1] | (q[2 * i + 17] << 4);
            p16[1 + i] = (unsigned short)(lo | (hi << 8));
        }
    }
}
}  // namespace

extern "C" int qg_synth_normal(float *dst, size_t count, uint64_t seed, float stddev) {
    if (!dst) return cudaErrorInvalidValue;
    if (!count) return 0;
    normal_kernel<<<1184, 256, 0, launch_stream>>>(dst, count, seed, stddev);
    return cudaGetLastError();
}

extern "C" int qg_synth_weights(void *dst, int type, int rows, int cols, uint64_t seed, float stddev) {
    if (!dst || rows < 1 || !row_bytes(type, cols)) return cudaErrorInvalidValue;
    if (type == 20 && (reinterpret_cast<uintptr_t>(dst) & 1)) return cudaErrorInvalidValue;  // 16-bit stores
    unsigned char *p = static_cast<unsigned char *>(dst);
    if (type == 0) {
        normal_kernel<<<1184, 256, 0, launch_stream>>>(reinterpret_cast<float *>(p), (size_t)rows * cols, seed, stddev);
    } else if (type == 12) {
        q4k_kernel<<<1184, 128, 0, launch_stream>>>(p, rows, cols, seed, stddev);
    } else if (type == 20) {
        iq4nl_kernel<<<1184, 128, 0, launch_stream>>>(p, rows, cols, seed, stddev);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}
