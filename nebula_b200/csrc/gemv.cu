// Dense projections and element-wise operators of the qwen/gpu.h ABI:
// qg_matmul, qg_gather, qg_dequant, qg_unary, qg_binary, qg_shared_add.
//
// qg_matmul keeps the reference's 32-lane accumulation order (lane j owns
// columns j mod 32, then the 16/8/4/2/1 tree), so its output is bitwise equal
// to qc_matmul (qwen/cpu.c:119-148): one warp per weight row, or for fp32 rows
// against 64 or more tokens a tiled kernel with the same order per output. The router GEMV
// that feeds top-10 selection relies on this for bit-exact expert ids.
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

template <int TR, int TT>
int launch_tiled(float *o, const float *w, int rows, int cols, const float *x, int nt, cudaStream_t st) {
    auto k = matmul_f32_tiled_kernel<TR, TT>;
    if (int rc = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tiled_smem<TR, TT>())) return rc;
    k<<<dim3((rows + TR - 1) / TR, (nt + TT - 1) / TT), TR * TT / 2, tiled_smem<TR, TT>(), st>>>(o, w, rows, cols, x, nt);
    return cudaGetLastError();
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
    dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta, (nt + kTokTile - 1) / kTokTile);
    const unsigned char *wb = static_cast<const unsigned char *>(w);
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
