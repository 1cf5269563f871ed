/* TEST INFRASTRUCTURE ONLY - host restatement of the library's synthetic
 * weight and activation generator (qg_synth_weights / qg_synth_normal in
 * nebula_b200/csrc/synth.cu), bit for bit.
 *
 * The CPU baseline and the reference arm of bench.py use it to build the same
 * layers the GPU arm builds on the device, without calling the product
 * library. tests/test_gpu_ops.py checks the bytes against the device's.
 *
 * Values: the sum of eight 16-bit uniforms from two splitmix64 hashes of the
 * seed and the element index, centred (2*S - 8*65535, an odd integer below
 * 2^20) and multiplied by stddev / (65536*sqrt(8/3)) - integer arithmetic
 * plus two correctly rounded float multiplies. Quantisers: the Q4_K and
 * IQ4_NL round-to-nearest schemes of synth.cu, one correctly rounded float
 * operation per step (compiled with -ffp-contract=off so no multiply-add is
 * fused), fp16 conversion with round to nearest even (_Float16).
 *
 * Rows [row0, row0 + nrows) of a rows x cols matrix are written to dst (the
 * start of row row0), so a caller can generate only the experts it needs.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float kIhInvStd = 9.3440618e-06f;
static const int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static float normal_at(uint64_t seed, uint64_t i, float stddev) {
    const uint64_t k = seed * 0xd1342543de82ef95ULL;
    const uint64_t h1 = mix64(k ^ mix64(2 * i)), h2 = mix64(k ^ mix64(2 * i + 1));
    int64_t s = 0;
    for (int j = 0; j < 4; j++) s += (int64_t)((h1 >> (16 * j)) & 0xffff) + (int64_t)((h2 >> (16 * j)) & 0xffff);
    const int c = (int)(2 * s - 8 * 65535);
    const float scale = stddev * kIhInvStd;
    return (float)c * scale;
}

static uint16_t f16_bits(float v) {
    _Float16 h = (_Float16)v;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

static float f16_value(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }
static int rne(float v) { return (int)rintf(v); }

static void q4k_block(unsigned char *p, uint64_t first, uint64_t seed, float stddev) {
    float scale[8], minv[8], smax = 0.0f, mmax = 0.0f;
    for (int g = 0; g < 8; g++) {
        float lo = 0.0f, hi = 0.0f;
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
    uint16_t dh = f16_bits(smax / 63.0f), mh = f16_bits(mmax / 63.0f);
    float d = f16_value(dh), dmin = f16_value(mh);
    int sc[8], mc[8];
    for (int g = 0; g < 8; g++) {
        sc[g] = d > 0 ? clampi(rne(scale[g] / d), 0, 63) : 0;
        mc[g] = dmin > 0 ? clampi(rne(minv[g] / dmin), 0, 63) : 0;
    }
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
        const float ds0 = d * (float)sc[g0], dm0 = dmin * (float)mc[g0];
        const float ds1 = d * (float)sc[g1], dm1 = dmin * (float)mc[g1];
        for (int l = 0; l < 32; l++) {
            float v0 = normal_at(seed, first + g0 * 32 + l, stddev);
            float v1 = normal_at(seed, first + g1 * 32 + l, stddev);
            int q0 = ds0 > 0 ? clampi(rne((v0 + dm0) / ds0), 0, 15) : 0;
            int q1 = ds1 > 0 ? clampi(rne((v1 + dm1) / ds1), 0, 15) : 0;
            p[16 + 32 * i + l] = (unsigned char)(q0 | (q1 << 4));
        }
    }
}

static void iq4nl_block(unsigned char *p, uint64_t first, uint64_t seed, float stddev) {
    float ext = 0.0f;
    for (int l = 0; l < 32; l++) {
        float v = normal_at(seed, first + l, stddev);
        if (fabsf(v) > fabsf(ext)) ext = v;
    }
    uint16_t dh = f16_bits(ext / -127.0f);
    float d = f16_value(dh);
    p[0] = dh & 255;
    p[1] = dh >> 8;
    unsigned char q[32];
    for (int l = 0; l < 32; l++) {
        float v = normal_at(seed, first + l, stddev);
        int best = 0;
        float err = INFINITY;
        for (int c = 0; c < 16; c++) {
            float e = fabsf(d * (float)kIq4nl[c] - v);
            if (e < err) {
                err = e;
                best = c;
            }
        }
        q[l] = (unsigned char)best;
    }
    for (int j = 0; j < 16; j++) p[2 + j] = (unsigned char)(q[j] | (q[j + 16] << 4));
}

/* x[i] = value i of stream `seed`, i in [first, first + count). */
void or_synth_normal(float *dst, uint64_t first, uint64_t count, uint64_t seed, float stddev) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)count; i++) dst[i] = normal_at(seed, first + (uint64_t)i, stddev);
}

/* Rows [row0, row0+nrows) of a type-0/12/20 matrix of `cols` values per row. */
int or_synth_weights(unsigned char *dst, int type, int cols, uint64_t seed, float stddev, int64_t row0,
                     int64_t nrows) {
    if (!dst || cols < 1 || row0 < 0 || nrows < 0) return -1;
    if (type == 0) {
        or_synth_normal((float *)dst, (uint64_t)row0 * cols, (uint64_t)nrows * cols, seed, stddev);
        return 0;
    }
    const int block = type == 12 ? 256 : type == 20 ? 32 : 0, bytes = type == 12 ? 144 : 18;
    if (!block || cols % block) return -1;
    const int64_t per_row = cols / block, n = nrows * per_row;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < n; b++) {
        const int64_t r = row0 + b / per_row, k = b % per_row;
        const uint64_t first = (uint64_t)r * (uint64_t)cols + (uint64_t)k * block;
        if (type == 12) q4k_block(dst + b * bytes, first, seed, stddev);
        else iq4nl_block(dst + b * bytes, first, seed, stddev);
    }
    return 0;
}
