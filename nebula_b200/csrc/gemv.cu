// Dense projections and element-wise operators of the qwen/gpu.h ABI:
// qg_matmul, qg_gather, qg_dequant, qg_unary, qg_binary, qg_shared_add.
//
// qg_matmul keeps the reference's 32-lane accumulation order (lane j owns
// columns j mod 32, then the 16/8/4/2/1 tree), so its output is bitwise equal
// to qc_matmul (qwen/cpu.c:119-148): a staged kernel (chunks of rows and token
// vectors copied into shared memory, one warp per two rows), a tiled kernel
// for fp32 rows against 64 or more tokens, and one warp per row for shapes
// neither takes, all with the same order per output. The router GEMV that
// feeds top-10 selection relies on this for bit-exact expert ids.
#include "quant.cuh"

using namespace nb;

namespace {
constexpr int kRowsPerCta = 4;  // one warp per row
constexpr int kTokTile = 16;    // token vectors per pass, kept in registers

template <int T>
__global__ void __launch_bounds__(kRowsPerCta * 32) matmul_kernel(float *out, const unsigned char *w, int type,
                                                                  int rows, int cols, const float *x, int nt,
                                                                  size_t stride) {
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    const int first = blockIdx.y * kTokTile;
    if (row >= rows) return;
    const int n = min(kTokTile, nt - first);
    const float *xs[kTokTile];
#pragma unroll
    for (int t = 0; t < kTokTile; t++) xs[t] = x + (size_t)(first + min(t, n - 1)) * cols;
    float acc[kTokTile];
#pragma unroll
    for (int t = 0; t < kTokTile; t++) acc[t] = 0.0f;
    const unsigned char *r = w + (size_t)row * stride;
    if (T >= 0)
        lane_dot<T, kTokTile>(r, cols, xs, n, acc);
    else
        lane_dot_generic<kTokTile>(r, type, cols, xs, n, acc);
#pragma unroll
    for (int t = 0; t < kTokTile; t++) {
        if (t < n) {
            float s = lane_tree(acc[t]);
            if ((threadIdx.x & 31) == 0) out[(size_t)(first + t) * rows + row] = s;
        }
    }
}

// fp32 weights, large batches: a CTA computes TR rows x TT tokens (32 x 32, or
// 8 x 16 for a handful of rows such as the shared-expert gate). Lane j of
// every warp holds the partial sums over k = j (mod 32) of an 8-row x 8-token
// tile, accumulated in increasing k with fused multiply-adds from 256-column
// chunks of the rows and token vectors staged in shared memory, then the same
// 16/8/4/2/1 tree: bitwise the order of one warp per row above.
constexpr int kTK = 256;
template <int TR, int TT>
constexpr int tiled_smem() { return 2 * (TR + TT) * kTK * 4; }  // two stages of row and token chunks
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// The chunks are staged with cp.async into two alternating buffers, so the
// next chunk's copies overlap this chunk's multiply-adds.
template <int kTR, int kTT>
__global__ void __launch_bounds__(kTR * kTT / 2) matmul_f32_tiled_kernel(float *out, const float *w, int rows, int cols,
                                                                         const float *x, int nt) {
    constexpr int kTThreads = kTR * kTT / 2;  // one warp per 8 x 8 tile
    extern __shared__ __align__(16) float tsm[];
    float(*ws)[kTR][kTK] = reinterpret_cast<float(*)[kTR][kTK]>(tsm);
    float(*xs)[kTT][kTK] = reinterpret_cast<float(*)[kTT][kTK]>(tsm + 2 * kTR * kTK);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row0 = blockIdx.x * kTR, tok0 = blockIdx.y * kTT;
    const int wr = (warp / (kTT / 8)) * 8, wt = (warp % (kTT / 8)) * 8;  // this warp's rows and tokens
    auto stage = [&](int b, int kc) {
        const int kn = min(kTK, cols - kc);  // a multiple of 32
        for (int i = tid; i < kTR * (kTK / 4); i += kTThreads) {
            const int r = i / (kTK / 4), c = (i % (kTK / 4)) * 4;
            float *dst = &ws[b][r][c];
            if (row0 + r < rows && c < kn) cp_async16(dst, w + (size_t)(row0 + r) * cols + kc + c);
            else *reinterpret_cast<float4 *>(dst) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        for (int i = tid; i < kTT * (kTK / 4); i += kTThreads) {
            const int t = i / (kTK / 4), c = (i % (kTK / 4)) * 4;
            float *dst = &xs[b][t][c];
            if (tok0 + t < nt && c < kn) cp_async16(dst, x + (size_t)(tok0 + t) * cols + kc + c);
            else *reinterpret_cast<float4 *>(dst) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        cp_async_commit();
    };
    // acc[r][p] holds tokens 2p and 2p+1 of row r: paired fused multiply-adds,
    // each half the same rounding as a scalar one
    float2 acc[8][4];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int p = 0; p < 4; p++) acc[r][p] = make_float2(0.0f, 0.0f);
    stage(0, 0);
    int b = 0;
    for (int kc = 0; kc < cols; kc += kTK, b ^= 1) {
        const int kn = min(kTK, cols - kc);
        if (kc + kTK < cols) {
            stage(b ^ 1, kc + kTK);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        for (int k = lane; k < kn; k += 32) {
            float wv[8];
            float2 xv[4];
#pragma unroll
            for (int r = 0; r < 8; r++) wv[r] = ws[b][wr + r][k];
#pragma unroll
            for (int p = 0; p < 4; p++) xv[p] = make_float2(xs[b][wt + 2 * p][k], xs[b][wt + 2 * p + 1][k]);
#pragma unroll
            for (int r = 0; r < 8; r++) {
                const float2 w2 = make_float2(wv[r], wv[r]);
#pragma unroll
                for (int p = 0; p < 4; p++) acc[r][p] = __ffma2_rn(w2, xv[p], acc[r][p]);
            }
        }
        __syncthreads();  // buffer b is restaged two chunks later
    }
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int t = 0; t < 8; t++) {
            const float s = lane_tree((t & 1) ? acc[r][t >> 1].y : acc[r][t >> 1].x);
            const int row = row0 + wr + r, tok = tok0 + wt + t;
            if (lane == 0 && row < rows && tok < nt) out[(size_t)tok * rows + row] = s;
        }
}

// Staged GEMV for batches the tiled kernel does not take: a CTA of kGvWarps
// warps owns 2 rows per warp (4 for 8 or more tokens). Each 256-column chunk of those rows and of
// the token vectors is copied into shared memory (two stages: the next chunk's
// copies are in flight while one is multiplied), so a chunk's loads
// are all issued at once instead of one dependent load per lane step. Lane j then
// multiplies columns j, j+32, ... of the chunk in increasing order with one
// fused multiply-add per element, continuing the same per-lane sums across
// chunks: the order of matmul_kernel, so the results are bitwise the same.
constexpr int kGvWarps = 8, kGvK = 256;

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

// Rows per warp of the staged kernel for a token tile of NT.
template <int NT>
constexpr int gv_rows() { return NT >= 8 ? 4 : 2; }

// Lane columns of one staged chunk of nr rows (row r's bytes at rows + r*pitch)
// against n token vectors xs[t][kGvK], tokens in pairs: acc[r][p] holds tokens
// 2p and 2p+1, each half a fused multiply-add with the rounding of a scalar one,
// in increasing column order. T >= 0: that format; T < 0: `type`, per element.
template <int T, int NT, int R>
__device__ __forceinline__ void gv_chunk(const unsigned char *rows, int pitch, int nr, int type, const float *xs,
                                         int kn, int n, const float *lut, float2 *gv_scales,
                                         float2 (&acc)[R][(NT + 1) / 2]) {
    constexpr int NP = (NT + 1) / 2;
    const int lane = threadIdx.x & 31;
    auto load_x = [&](int k, float2 (&xv)[NP]) {
#pragma unroll
        for (int p = 0; p < NP; p++)
            xv[p] = make_float2(2 * p < n ? xs[2 * p * kGvK + k] : 0.0f, 2 * p + 1 < n ? xs[(2 * p + 1) * kGvK + k] : 0.0f);
    };
    if (T == 12) {  // one Q4_K superblock per chunk (kn = 256)
        // (d*sc, -dmin*m) of the 8 sub-blocks of each row, decoded by lanes 0..7 and
        // read back as broadcasts; nibbles become exact floats through the exponent
        // field (q + 2^23 - 2^23); w = d*sc*q - dmin*m with one rounding, in pairs
        float2 *scl = gv_scales + (threadIdx.x >> 5) * (R * 8);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (r < nr && lane < 8) {
                const unsigned char *p = rows + r * pitch;
                int s, m;
                k_scale_min(p + 4, lane, s, m);
                scl[r * 8 + lane] = make_float2(half_at(p) * static_cast<float>(s),
                                                -(half_at(p + 2) * static_cast<float>(m)));
            }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k0 = 64 * i + lane;  // sub-block 2i; sub-block 2i+1 at k0 + 32
            float2 x0[NP], x1[NP];
            if constexpr (NT == 1) {  // one token: scalar multiply-adds on .x
                x0[0].x = xs[k0];
                x1[0].x = xs[k0 + 32];
            } else {
                load_x(k0, x0);
                load_x(k0 + 32, x1);
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (r < nr) {
                    const float4 sc = *reinterpret_cast<const float4 *>(scl + r * 8 + 2 * i);  // ds0, -dm0, ds1, -dm1
                    const unsigned b = rows[r * pitch + 16 + 32 * i + lane];
                    const float2 q = __fadd2_rn(make_float2(__uint_as_float((b & 15u) | 0x4B000000u),
                                                            __uint_as_float((b >> 4) | 0x4B000000u)),
                                                make_float2(-8388608.0f, -8388608.0f));
                    const float2 wv = __ffma2_rn(make_float2(sc.x, sc.z), q, make_float2(sc.y, sc.w));
                    if constexpr (NT == 1) {
                        acc[r][0].x = __fmaf_rn(wv.x, x0[0].x, acc[r][0].x);
                        acc[r][0].x = __fmaf_rn(wv.y, x1[0].x, acc[r][0].x);
                    } else {
                        const float2 w0 = make_float2(wv.x, wv.x), w1 = make_float2(wv.y, wv.y);
#pragma unroll
                        for (int p = 0; p < NP; p++) acc[r][p] = __ffma2_rn(w0, x0[p], acc[r][p]);
#pragma unroll
                        for (int p = 0; p < NP; p++) acc[r][p] = __ffma2_rn(w1, x1[p], acc[r][p]);
                    }
                }
            }
        }
        __syncwarp();  // the scales are rewritten for the next chunk
        return;
    }
#pragma unroll(NT == 1 ? 8 : 1)
    for (int m = 0; m < kn / 32; m++) {
        const int k = 32 * m + lane;
        float2 xv[NP];
        if constexpr (NT == 1) xv[0].x = xs[k];  // one token: scalar multiply-adds on .x
        else load_x(k, xv);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (r >= nr) break;
            const unsigned char *p = rows + r * pitch;
            float a;
            if (T == 0) {
                a = reinterpret_cast<const float *>(p)[k];
            } else if (T == 8) {  // Q8_0: 34-byte blocks, the lane's value is byte 2 + lane
                const unsigned char *b = p + m * 34;
                a = half_at(b) * static_cast<float>(reinterpret_cast<const signed char *>(b + 2)[lane]);
            } else if (T == 20) {  // IQ4_NL: 18-byte blocks
                const unsigned char *b = p + m * 18;
                const unsigned q = b[2 + (lane & 15)];
                a = half_at(b) * lut[lane < 16 ? (q & 15) : (q >> 4)];
            } else {
                a = decode_at(p, T < 0 ? type : T, k);
            }
            if constexpr (NT == 1) {
                acc[r][0].x = __fmaf_rn(a, xv[0].x, acc[r][0].x);
            } else {
                const float2 a2 = make_float2(a, a);
#pragma unroll
                for (int p2 = 0; p2 < NP; p2++) acc[r][p2] = __ffma2_rn(a2, xv[p2], acc[r][p2]);
            }
        }
    }
}

// cb / cb_tail: bytes of a row's full chunk and of its last chunk; pitch: a
// staged row's size (cb rounded up to 16); mode: copy width 16 or 4 (cp.async)
// or 2 (plain loads), chosen by the host from the alignment of rows and chunks.
// Two stages: deeper rings measured no faster (the kernel is bound by its
// instruction issue at small batches) and cost fp32 rows occupancy.
template <int NT>
constexpr int gv_stages() { return 2; }
template <int T, int NT>
__global__ void __launch_bounds__(kGvWarps * 32) gemv_staged_kernel(float *out, const unsigned char *w, int type,
                                                                    int rows, int cols, const float *x, int nt,
                                                                    size_t stride, int cb, int cb_tail, int pitch,
                                                                    int mode) {
    extern __shared__ __align__(16) unsigned char gsm[];
    __shared__ float lut[16];
    constexpr int R = gv_rows<NT>(), kRowsCta = kGvWarps * R, NP = (NT + 1) / 2;
    __shared__ __align__(16) float2 scales[kGvWarps * R * 8];  // Q4_K sub-block scales per warp and row
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row0 = blockIdx.x * kRowsCta, first = blockIdx.y * NT;
    const int n = min(NT, nt - first), nrows = min(kRowsCta, rows - row0);
    const int stage_sz = kRowsCta * pitch + NT * kGvK * 4;
    if (tid < 16) lut[tid] = static_cast<float>(kIq4nl[tid]);
    auto stage = [&](int buf, int kc) {
        unsigned char *ws = gsm + buf * stage_sz;
        float *xs = reinterpret_cast<float *>(ws + kRowsCta * pitch);
        const int kn = min(kGvK, cols - kc), bytes = kn == kGvK ? cb : cb_tail;
        const size_t off = (size_t)(kc / kGvK) * cb;
        // warp w copies rows w, w+8, ... and token vectors w, w+8, ...; lanes across the bytes
        for (int r = warp; r < nrows; r += kGvWarps) {
            unsigned char *d = ws + r * pitch;
            const unsigned char *src = w + (size_t)(row0 + r) * stride + off;
            if (mode == 16)
                for (int o = lane * 16; o < bytes; o += 32 * 16) cp_async16(d + o, src + o);
            else if (mode == 4)
                for (int o = lane * 4; o < bytes; o += 32 * 4) cp_async4(d + o, src + o);
            else
                for (int o = lane * 2; o < bytes; o += 32 * 2)
                    *reinterpret_cast<unsigned short *>(d + o) = __ldg(reinterpret_cast<const unsigned short *>(src + o));
        }
        for (int t = warp; t < n; t += kGvWarps) {
            const float *src = x + (size_t)(first + t) * cols + kc;
            for (int o = lane * 4; o < kn; o += 32 * 4) cp_async16(xs + t * kGvK + o, src + o);
        }
        cp_async_commit();
    };
    float2 acc[R][NP];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int p = 0; p < NP; p++) acc[r][p] = make_float2(0.0f, 0.0f);
    const int r0 = warp * R, nr = min(R, nrows - r0);  // this warp's rows (nr <= 0: none)
    constexpr int S = gv_stages<NT>();
    const int nch = (cols + kGvK - 1) / kGvK;
    // one copy group per chunk (empty past the end), so group c is chunk c's
#pragma unroll
    for (int c = 0; c < S - 1; c++) {
        if (c < nch) stage(c, c * kGvK);
        else cp_async_commit();
    }
    for (int c = 0; c < nch; c++) {
        cp_async_wait<S - 2>();  // chunk c's copies have landed
        __syncthreads();         // ... for every thread; and chunk c-1's buffer is free again
        if (c + S - 1 < nch) stage((c + S - 1) % S, (c + S - 1) * kGvK);
        else cp_async_commit();
        const unsigned char *ws = gsm + (c % S) * stage_sz;
        if (nr > 0)
            gv_chunk<T, NT, R>(ws + r0 * pitch, pitch, nr, type,
                               reinterpret_cast<const float *>(ws + kRowsCta * pitch), min(kGvK, cols - c * kGvK), n,
                            lut, scales, acc);
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
        if (r >= nr) break;
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < n) {
                const float s = lane_tree((t & 1) ? acc[r][t >> 1].y : acc[r][t >> 1].x);
                if (lane == 0) out[(size_t)(first + t) * rows + row0 + r0 + r] = s;
            }
        }
    }
}

template <int TR, int TT>
int launch_tiled(float *o, const float *w, int rows, int cols, const float *x, int nt, cudaStream_t st) {
    auto k = matmul_f32_tiled_kernel<TR, TT>;
    if (int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tiled_smem<TR, TT>())) return rc;
    k<<<dim3((rows + TR - 1) / TR, (nt + TT - 1) / TT), TR * TT / 2, tiled_smem<TR, TT>(), st>>>(o, w, rows, cols, x, nt);
    return cudaGetLastError();
}

template <int T, int NT>
int launch_gv(float *o, const unsigned char *w, int type, int rows, int cols, const float *x, int nt, size_t stride,
              int cb, int cbt, int pitch, int mode, cudaStream_t st) {
    auto k = gemv_staged_kernel<T, NT>;
    constexpr int kRowsCta = kGvWarps * gv_rows<NT>();
    const int smem = gv_stages<NT>() * (kRowsCta * pitch + NT * kGvK * 4);
    // the attribute is raised once per device, when a launch first needs more than the default
    static int max_smem[64];
    int dev = 0;
    if (int rc = cudaGetDevice(&dev)) return rc;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && smem > max_smem[dev]) {
        if (int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return rc;
        max_smem[dev] = smem;
    }
    k<<<dim3((rows + kRowsCta - 1) / kRowsCta, (nt + NT - 1) / NT), kGvWarps * 32, smem, st>>>(
        o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode);
    return cudaGetLastError();
}

template <int T>
int launch_gv_nt(float *o, const unsigned char *w, int type, int rows, int cols, const float *x, int nt,
                 size_t stride, int cb, int cbt, int pitch, int mode, cudaStream_t st) {
    if (nt == 1) return launch_gv<T, 1>(o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
    if (nt <= 4) return launch_gv<T, 4>(o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
    if (nt <= 8) return launch_gv<T, 8>(o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
    if (nt == 17 || nt == 18) return launch_gv<T, 18>(o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
    return launch_gv<T, 16>(o, w, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
}

__global__ void gather_kernel(float *out, const unsigned char *w, int type, int n, size_t stride, int row) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = decode_at(w + (size_t)row * stride, type, i);
}

__global__ void dequant_kernel(float *o, const unsigned char *w, int type, int rows, int cols, size_t stride) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)rows * cols) o[i] = decode_at(w + (i / cols) * stride, type, (int)(i % cols));
}

__global__ void unary_kernel(float *o, const float *x, int n, int op, float s) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float a = x[i] * s;
        o[i] = op == 0 ? a * sigmoidf_ref(a) : op == 1 ? sigmoidf_ref(a) : a;
    }
}

__global__ void binary_kernel(float *o, const float *a, const float *b, int n, int op) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) o[i] = op == 0 ? a[i] + b[i] : a[i] * b[i];
}

__global__ void shared_add_kernel(float *o, const float *x, const float *g, int nt, int width) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nt * width) o[i] = __fmaf_rn(x[i], sigmoidf_ref(g[i / width]), o[i]);
}

bool valid_cols(int type, int cols) {
    if (type == 12 || type == 13 || type == 14) return cols % 256 == 0;
    if (type == 2 || type == 6 || type == 7 || type == 8 || type == 20) return cols % 32 == 0;
    return true;
}
}  // namespace

namespace nb {
// Bit-exact GEMV launch shared with the MoE layer's router.
int launch_matmul(float *o, const void *w, int type, int rows, int cols, const float *x, int nt, cudaStream_t st) {
    size_t stride = row_bytes(type, cols);
    if (!o || !w || !x || !stride || rows < 1 || cols < 1 || nt < 1 || nt > kMaxTokens || !valid_cols(type, cols))
        return cudaErrorInvalidValue;
    if (type == 0 && nt >= 64 && cols % 32 == 0 && !(reinterpret_cast<uintptr_t>(w) & 15) &&
        !(reinterpret_cast<uintptr_t>(x) & 15)) {  // fp32 rows against a large batch: tiled
        const float *wf = static_cast<const float *>(w);
        if (rows >= 32) return launch_tiled<32, 32>(o, wf, rows, cols, x, nt, st);
        return launch_tiled<8, 16>(o, wf, rows, cols, x, nt, st);
    }
    const unsigned char *wb = static_cast<const unsigned char *>(w);
    if (cols % 32 == 0 && !(reinterpret_cast<uintptr_t>(x) & 15)) {
        // staged kernel: chunks of kGvK columns (the last may be shorter), copied as wide as
        // the rows' and chunks' alignment allows
        const int cb = (int)row_bytes(type, kGvK), cbt = (int)row_bytes(type, cols % kGvK ? cols % kGvK : kGvK);
        auto aligned = [&](int a) {
            return reinterpret_cast<uintptr_t>(w) % a == 0 && stride % a == 0 && cb % a == 0 && cbt % a == 0;
        };
        const int mode = aligned(16) ? 16 : aligned(4) ? 4 : aligned(2) ? 2 : 0;
        if (mode && cb > 0 && cbt > 0) {
            const int pitch = (cb + 15) & ~15;
            switch (type) {
            case 0: return launch_gv_nt<0>(o, wb, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
            case 8: return launch_gv_nt<8>(o, wb, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
            case 12: return launch_gv_nt<12>(o, wb, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
            case 20: return launch_gv_nt<20>(o, wb, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
            default: return launch_gv_nt<-1>(o, wb, type, rows, cols, x, nt, stride, cb, cbt, pitch, mode, st);
            }
        }
    }
    dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta, (nt + kTokTile - 1) / kTokTile);
    switch (type) {
    case 0: matmul_kernel<0><<<grid, kRowsPerCta * 32, 0, st>>>(o, wb, type, rows, cols, x, nt, stride); break;
    case 12: matmul_kernel<12><<<grid, kRowsPerCta * 32, 0, st>>>(o, wb, type, rows, cols, x, nt, stride); break;
    case 20: matmul_kernel<20><<<grid, kRowsPerCta * 32, 0, st>>>(o, wb, type, rows, cols, x, nt, stride); break;
    default: matmul_kernel<-1><<<grid, kRowsPerCta * 32, 0, st>>>(o, wb, type, rows, cols, x, nt, stride); break;
    }
    return cudaGetLastError();
}
}  // namespace nb

extern "C" int qg_matmul(float *o, const void *w, int type, int rows, int cols, const float *x, int nt) {
    return launch_matmul(o, w, type, rows, cols, x, nt, launch_stream);
}

extern "C" int qg_gather(float *o, const void *w, int type, int cols, int row) {
    size_t stride = row_bytes(type, cols);
    if (!o || !w || !stride || row < 0 || !valid_cols(type, cols)) return cudaErrorInvalidValue;
    gather_kernel<<<(cols + 255) / 256, 256, 0, launch_stream>>>(o, static_cast<const unsigned char *>(w), type,
                                                                  cols, stride, row);
    return cudaGetLastError();
}

extern "C" int qg_dequant(float *o, const void *w, int type, int rows, int cols) {
    size_t stride = row_bytes(type, cols);
    if (!o || !w || !stride || rows < 1 || !valid_cols(type, cols)) return cudaErrorInvalidValue;
    size_t n = (size_t)rows * cols;
    dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, launch_stream>>>(o, static_cast<const unsigned char *>(w),
                                                                           type, rows, cols, stride);
    return cudaGetLastError();
}

extern "C" int qg_unary(float *o, const float *x, int n, int op, float s) {
    if (n < 0) return cudaErrorInvalidValue;
    if (!n) return 0;
    unary_kernel<<<(n + 255) / 256, 256, 0, launch_stream>>>(o, x, n, op, s);
    return cudaGetLastError();
}

extern "C" int qg_binary(float *o, const float *a, const float *b, int n, int op) {
    if (n < 0) return cudaErrorInvalidValue;
    if (!n) return 0;
    binary_kernel<<<(n + 255) / 256, 256, 0, launch_stream>>>(o, a, b, n, op);
    return cudaGetLastError();
}

// Width 2560 is part of this entry point's contract (qwen/gpu.cu:552-553).
extern "C" int qg_shared_add(float *o, const float *x, const float *g, int nt) {
    if (nt < 1) return cudaErrorInvalidValue;
    shared_add_kernel<<<(nt * 2560 + 255) / 256, 256, 0, launch_stream>>>(o, x, g, nt, 2560);
    return cudaGetLastError();
}
