// Tensor-core (tcgen05) expert kernel for Q4_K routed experts and the shared
// expert, used by both the decode and the prefill paths.
//
// Work items (claimed from a device queue, shared expert first): a gate/up
// tile = 128 rows of W_gate and of W_up of one expert x one token tile of up
// to 64 tokens; a down tile = 128 rows of W_down x the same token tile.
//
// The contraction runs on the 5th-generation tensor cores:
//   A = sc_g * q_k    fp16, exact (integers <= 945), decoded from the raw Q4_K
//                     bytes by four converter warps into the UMMA K-major
//                     no-swizzle layout (8x8 core matrices);
//   B = [x_hi | x_lo] fp16, x*s = x_hi + x_lo/2048 with a per-token power of
//                     two s (22-bit precision), copied from a prepared buffer;
//   D = A B^T         fp32 in tensor memory, accumulated per 256-value Q4_K
//                     superblock into one of two TMEM buffers.
// Eight epilogue warps read each superblock's D back (tcgen05.ld), apply the
// superblock scale d and the dmin*m_g*sum(x) term in fp32 and accumulate in
// registers; gate/up tiles finish with SiLU(g)*u, down tiles with the route
// weight, and the last contribution to a (token, 128-row tile) sums the ten
// slots in router-rank order plus the gated shared expert
// (qwen/cpu.c:209-231, qwen/gpu.cu:552).
//
// Raw weight bytes stream with 2-D TMA tensor copies (a 144-byte x 128-row
// box = one superblock of 128 rows) into a two-stage ring. Warp roles:
//   warp 0 lane 0   producer: claims items, issues TMA
//   warp 1          TMEM owner; lane 0 issues tcgen05.mma and commits
//   warps 2-5       converters (thread = weight row): A tiles, B copies
//   warps 6-13      epilogue (warp w reads TMEM lanes 32*(w%4).., half the
//                   tokens each)
// Every wait is bounded; on a timeout the CTA raises the error word, stops
// taking work, drains its copies and MMAs, frees TMEM and exits.
#include <algorithm>
#include "moe_tc.cuh"
#include "quant.cuh"

using namespace nb;

namespace {

constexpr int kWarps = 14, kThreads = kWarps * 32;
constexpr int kConvWarp0 = 2, kEpiWarp0 = 6;
constexpr int kSbBytes = kTcRows * 144;          // one superblock of 128 Q4_K rows
constexpr int kRawStage = 2 * kSbBytes;          // gate + up
constexpr int kABytes = kTcRows * 64 * 2;        // 128 rows x 64 halves
constexpr int kBBytes = 2 * kTcTok * 64 * 2;     // up to 128 B rows x 64 halves
constexpr int kScRows = 2 * kTcRows * 16;        // d, dmin, m[8] per row per matrix
constexpr int kScSlot = kScRows + 8 * kTcTok * 4; // + the superblock's 8 group sums per token
constexpr int kOffRaw = 0, kOffA = kOffRaw + 2 * kRawStage, kOffB = kOffA + 2 * 2 * kABytes,
              kOffSc = kOffB + 2 * kBBytes, kSmem = kOffSc + 4 * kScSlot;
constexpr uint32_t kBad = 1u << 16;

enum { kEnd = 0, kGU = 1, kDN = 2 };
struct Item {
    int kind, sub, mt, expert, first, n, tok0;
};

struct Bars {
    uint64_t item_full[4], item_empty[4];
    uint64_t raw_full[2], raw_empty[2];
    uint64_t ab_full[2], ab_empty[2];
    uint64_t d_full[2], d_empty[2];
    uint64_t sc_full[4], sc_empty[4];
    uint64_t mma_done;
};

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void bar_named(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Bounded wait used by every role; `abort` is the CTA-wide stop flag.
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    for (int i = 0; i < (1 << 21); i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    atomicOr(err, 4);
    return false;
}

// Bounded wait that ignores the stop flag: used to drain work already in flight.
__device__ __forceinline__ bool wait_drain(uint64_t *bar, uint32_t parity) {
    for (int i = 0; i < (1 << 21); i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ bool wait_geq_int(const int *p, int target, int *err) {
    for (int i = 0; i < (1 << 22); i++) {
        if (ld_acquire(p) >= target) return true;
        __nanosleep(64);
    }
    atomicOr(err, 4);
    return false;
}

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// UMMA shared-memory descriptor, K-major, no swizzle: 8x8 core matrices of
// 128 contiguous bytes; LBO = distance between the two K-halves of one MMA,
// SBO = distance between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both K-major.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t addr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Q4_K: decode unit c (values 64c..64c+63 of a superblock) of one 144-byte
// row into four 16-byte A rows (k-slots 8kb..8kb+7 for kb = 0..7, value
// 64c + k). Low nibbles of bytes 0..31 are values 0..31 (scale sc[2c]), high
// nibbles are values 32..63 (scale sc[2c+1]); each half is sc*q exactly.
__device__ __forceinline__ void q4k_unit_to_a(const unsigned char *row, int c, unsigned char *a_row, int a_kstride) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(row);
    const unsigned char *sc = reinterpret_cast<const unsigned char *>(&hd) + 4;
    int s0, m0, s1, m1;
    k_scale_min(sc, 2 * c, s0, m0);
    k_scale_min(sc, 2 * c + 1, s1, m1);
    (void)m0;
    (void)m1;
    const __half2 sc_lo = __half2half2(__int2half_rn(s0)), neg_lo = __half2half2(__int2half_rn(-1024 * s0));
    const __half2 sc_hi = __half2half2(__float2half_rn((float)s1 * 0.0625f)), neg_hi = __half2half2(__int2half_rn(-64 * s1));
    const uint4 q0 = *reinterpret_cast<const uint4 *>(row + 16 + 32 * c);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(row + 32 + 32 * c);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int kb = 0; kb < 4; kb++) {
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t word = w[2 * kb + h];
            const uint32_t t01 = __byte_perm(word, 0, 0x4140), t23 = __byte_perm(word, 0, 0x4342);
            const uint32_t ts[2] = {t01, t23};
#pragma unroll
            for (int p = 0; p < 2; p++) {
                uint32_t vl = (ts[p] & 0x000F000Fu) | 0x64006400u;  // 1024 + q
                uint32_t vh = (ts[p] & 0x00F000F0u) | 0x64006400u;  // 1024 + 16 q
                __half2 rl = __hfma2(*reinterpret_cast<__half2 *>(&vl), sc_lo, neg_lo);
                __half2 rh = __hfma2(*reinterpret_cast<__half2 *>(&vh), sc_hi, neg_hi);
                lo[2 * h + p] = *reinterpret_cast<uint32_t *>(&rl);
                hi[2 * h + p] = *reinterpret_cast<uint32_t *>(&rh);
            }
        }
        *reinterpret_cast<uint4 *>(a_row + kb * a_kstride) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4 *>(a_row + (kb + 4) * a_kstride) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

// d, dmin and the eight 6-bit mins of one 144-byte superblock row.
__device__ __forceinline__ uint4 q4k_row_scales(const unsigned char *row) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(row);
    const unsigned char *sc = reinterpret_cast<const unsigned char *>(&hd) + 4;
    uint32_t m4[2] = {0, 0};
#pragma unroll
    for (int g = 0; g < 8; g++) {
        int s, m;
        k_scale_min(sc, g, s, m);
        m4[g >> 2] |= (uint32_t)m << (8 * (g & 3));
    }
    const float d = half_bits(hd.x), dmin = half_bits(hd.x >> 16);
    return make_uint4(__float_as_uint(d), __float_as_uint(dmin), m4[0], m4[1]);
}

// Per-item token table, filled once per item (shared by all roles).
struct __align__(16) TokTab {
    int tok[kTcTok];   // token index
    int src[kTcTok];   // B source row, in halves: x16 row (gate/up) or mid16 row (down)
    int mrow[kTcTok];  // mid row written (gate/up) or read (down)
    int slot[kTcTok];  // routed slot t*10+k (down)
    float w[kTcTok];   // route weight (down)
    float inv[kTcTok]; // 1/s of the B row (filled by the converters)
};

__device__ __forceinline__ void tmem_ld8_nw(uint32_t addr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1) tc_experts_kernel(const TcArgs a, const __grid_constant__ TcMaps maps) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ Bars bars;
    __shared__ Item items[4];
    __shared__ TokTab tabs[4];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ int s_flag;
    __shared__ int s_combine[kTcTok];
    __shared__ int s_ncombine;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, H = a.H, F = a.F;
    const int gu_mt = F / kTcRows, dn_mt = H / kTcRows;
    const int gu_sb = H / 256, dn_sb = F / 256;
    if (tid == 0) {
        for (int i = 0; i < 4; i++) {
            mbar_init(&bars.item_full[i], 1);
            mbar_init(&bars.item_empty[i], 4 + 1 + 8);
            mbar_init(&bars.sc_full[i], 4);
            mbar_init(&bars.sc_empty[i], 8);
        }
        mbar_init(&bars.mma_done, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars.raw_full[i], 1);
            mbar_init(&bars.raw_empty[i], 4);
            mbar_init(&bars.ab_full[i], 4);
            mbar_init(&bars.ab_empty[i], 1);
            mbar_init(&bars.d_full[i], 1);
            mbar_init(&bars.d_empty[i], 8);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = tmem_base;
    int *err = a.err;

    if (warp == 0) {
        // ------------------------------------------------------ producer warp
        bool planned = false;
        int nsub = a.shared_subs;
        int gsb = 0;
        const int S_gu = a.shared_subs * gu_mt;
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            int idx = 1 << 30;
            if (lane == 0) {
                bool ok = seq < 4 || wait_phase(&bars.item_empty[slot], ((seq >> 2) - 1) & 1, &abort_flag, err);
                if (ok && !abort_flag) idx = atomicAdd(a.queue, 1);
                if (idx >= S_gu && idx != (1 << 30) && !planned) {
                    grid_dep_wait();
                    nsub = __ldcg(a.n_sub);
                    planned = true;
                }
            }
            idx = __shfl_sync(0xffffffffu, idx, 0);
            nsub = __shfl_sync(0xffffffffu, nsub, 0);
            if (idx >= S_gu && idx != (1 << 30)) grid_dep_wait();
            Item it{kEnd, 0, 0, -1, 0, 0, 0};
            const int total_gu = nsub * gu_mt, total_dn = nsub * dn_mt;
            if (idx < total_gu) {
                it.kind = kGU, it.sub = idx / gu_mt, it.mt = idx % gu_mt;
            } else if (idx < total_gu + total_dn) {
                it.kind = kDN, it.sub = (idx - total_gu) / dn_mt, it.mt = (idx - total_gu) % dn_mt;
            }
            if (it.kind != kEnd) {
                if (it.sub < a.shared_subs) {  // known without the routing
                    it.expert = -1, it.tok0 = it.sub * kTcTok, it.n = min(kTcTok, T - it.tok0), it.first = 0;
                } else {
                    it.expert = __ldcg(&a.sub[it.sub].expert);
                    it.first = __ldcg(&a.sub[it.sub].first);
                    it.n = __ldcg(&a.sub[it.sub].n);
                }
                TokTab &tb = tabs[slot];
                for (int j = lane; j < it.n; j += 32) {
                    const bool sh = it.expert < 0;
                    const int sl = sh ? 0 : __ldcg(a.pairs + it.first + j);
                    const int tok = sh ? it.tok0 + j : sl / kTop;
                    const int mrow = sh ? T * kTop + it.tok0 + j : it.first + j;
                    tb.tok[j] = tok;
                    tb.mrow[j] = mrow;
                    tb.src[j] = it.kind == kGU ? tok * 2 * H : mrow * 2 * F;
                    tb.slot[j] = sl;
                    tb.w[j] = (sh || it.kind == kGU) ? 0.0f : __ldcg(a.wts + sl);
                }
            }
            __syncwarp();
            if (lane == 0) {
                items[slot] = it;
                arrive(&bars.item_full[slot]);
                if (it.kind != kEnd) {
                    const int nsb = it.kind == kGU ? gu_sb : dn_sb;
                    for (int sb = 0; sb < nsb; sb++, gsb++) {
                        const int st = gsb & 1;
                        if (gsb >= 2 && !wait_phase(&bars.raw_empty[st], ((gsb >> 1) - 1) & 1, &abort_flag, err)) break;
                        unsigned char *dst = smem + kOffRaw + st * kRawStage;
                        if (it.kind == kGU) {
                            const int y = (it.expert < 0 ? 0 : it.expert * F) + it.mt * kTcRows;
                            mbar_arrive_expect_tx(&bars.raw_full[st], 2 * kSbBytes);
                            tma_2d(dst, it.expert < 0 ? &maps.sg : &maps.gate, sb * 144, y, &bars.raw_full[st]);
                            tma_2d(dst + kSbBytes, it.expert < 0 ? &maps.su : &maps.up, sb * 144, y, &bars.raw_full[st]);
                        } else {
                            const int y = (it.expert < 0 ? 0 : it.expert * H) + it.mt * kTcRows;
                            mbar_arrive_expect_tx(&bars.raw_full[st], kSbBytes);
                            tma_2d(dst, it.expert < 0 ? &maps.sd : &maps.down, sb * 144, y, &bars.raw_full[st]);
                        }
                    }
                }
            }
            __syncwarp();
            if (it.kind == kEnd || abort_flag) break;
        }
        if (lane == 0)  // the last copies issued have landed before the CTA may exit
            for (int k = max(0, gsb - 2); k < gsb; k++) wait_drain(&bars.raw_full[k & 1], (k >> 1) & 1);
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int gsb = 0, gch = 0;
            const uint32_t a_base = smem_u32(smem + kOffA), b_base = smem_u32(smem + kOffB);
            for (int seq = 0;; seq++) {
                const int slot = seq & 3;
                if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
                const Item it = items[slot];
                if (it.kind == kEnd) break;
                const int n_pad = (it.n + 15) & ~15, N = 2 * n_pad;
                const uint32_t idesc = idesc_f16(kTcRows, N);
                const int mats = it.kind == kGU ? 2 : 1;
                const int nsb = it.kind == kGU ? gu_sb : dn_sb;
                bool ok = true;
                for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                    const int db = gsb & 1;
                    if (gsb >= 2 && !(ok = wait_phase(&bars.d_empty[db], ((gsb >> 1) - 1) & 1, &abort_flag, err))) break;
                    tc_fence_after();
                    for (int c = 0; c < 4; c++, gch++) {
                        const int ab = gch & 1;
                        if (!(ok = wait_phase(&bars.ab_full[ab], (gch >> 1) & 1, &abort_flag, err))) break;
                        tc_fence_after();
                        for (int s = 0; s < 4; s++) {
                            const uint64_t bd = umma_desc(b_base + ab * kBBytes + 2 * s * 128, 128, 1024);
                            for (int m = 0; m < mats; m++) {
                                const uint64_t ad = umma_desc(a_base + (ab * 2 + m) * kABytes + 2 * s * 128, 128, 1024);
                                mma_f16(tmem + (uint32_t)((db * 2 + m) * 128), ad, bd, idesc, (c | s) != 0);
                            }
                        }
                        mma_commit(&bars.ab_empty[ab]);
                    }
                    if (ok) mma_commit(&bars.d_full[db]);
                }
                arrive(&bars.item_empty[slot]);
                if (!ok) break;
            }
            // every MMA issued by this thread completes before TMEM is released
            mma_commit(&bars.mma_done);
            wait_drain(&bars.mma_done, 0);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------ converters
        grid_dep_wait();  // activations, routing and plan come from the preceding kernel
        const int ct = tid - kConvWarp0 * 32;  // weight row of the tile
        int gsb = 0, gch = 0;
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
            const Item it = items[slot];
            if (it.kind == kEnd) break;
            TokTab &tb = tabs[slot];
            const int n_pad = (it.n + 15) & ~15, N = 2 * n_pad;
            const int mats = it.kind == kGU ? 2 : 1;
            const int nsb = it.kind == kGU ? gu_sb : dn_sb;
            const int K = it.kind == kGU ? H : F;
            const int ngroups = K / 32;
            const __half *bsrc = it.kind == kGU ? a.x16 : a.mid16;
            const float *gsums = it.kind == kGU ? a.xsum : a.msum;
            if (it.kind == kDN) {
                // the token tile's mid must be complete and converted (gu_done = gu_mt + 1)
                if (ct == 0 && !wait_geq_int(a.gu_done + it.sub, gu_mt + 1, err)) abort_flag = 1;
                bar_named(2, 128);
            }
            if (ct < kTcTok)  // padding tokens get 0 so their (discarded) columns stay finite
                tb.inv[ct] = ct >= it.n ? 0.0f : it.kind == kGU ? __ldcg(a.xinv + tb.tok[ct]) : __ldcg(a.midinv + tb.mrow[ct]);
            const int grow = ct < it.n ? (it.kind == kGU ? tb.tok[ct] : tb.mrow[ct]) : 0;  // group-sum row
            bar_named(2, 128);
            bool ok = !abort_flag;
            for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                const int st = gsb & 1, sc_slot = gsb & 3;
                if (!(ok = wait_phase(&bars.raw_full[st], (gsb >> 1) & 1, &abort_flag, err))) break;
                const unsigned char *raw = smem + kOffRaw + st * kRawStage;
                if (gsb >= 4 && !(ok = wait_phase(&bars.sc_empty[sc_slot], ((gsb >> 2) - 1) & 1, &abort_flag, err)))
                    break;
                unsigned char *scb = smem + kOffSc + sc_slot * kScSlot;
                uint4 *scs = reinterpret_cast<uint4 *>(scb);
                float *xs = reinterpret_cast<float *>(scb + kScRows);  // [8][64]
                for (int m = 0; m < mats; m++) scs[m * kTcRows + ct] = q4k_row_scales(raw + m * kSbBytes + ct * 144);
                if (ct < kTcTok) {
                    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
                    if (ct < it.n) {
                        const float4 *gp = reinterpret_cast<const float4 *>(gsums + (size_t)grow * ngroups + sb * 8);
                        v0 = __ldcg(gp);
                        v1 = __ldcg(gp + 1);
                    }
                    xs[0 * kTcTok + ct] = v0.x, xs[1 * kTcTok + ct] = v0.y, xs[2 * kTcTok + ct] = v0.z;
                    xs[3 * kTcTok + ct] = v0.w, xs[4 * kTcTok + ct] = v1.x, xs[5 * kTcTok + ct] = v1.y;
                    xs[6 * kTcTok + ct] = v1.z, xs[7 * kTcTok + ct] = v1.w;
                }
                __syncwarp();
                if (lane == 0) arrive(&bars.sc_full[sc_slot]);
                for (int c = 0; c < 4; c++, gch++) {
                    const int ab = gch & 1;
                    if (gch >= 2 && !(ok = wait_phase(&bars.ab_empty[ab], ((gch >> 1) - 1) & 1, &abort_flag, err)))
                        break;
                    // B rows: token j hi -> row j, lo -> row n_pad + j; k-slots = values 64u .. 64u+63.
                    // Eight consecutive threads fill the eight rows of one core matrix (128 B).
                    const int u = sb * 4 + c;
                    unsigned char *bt = smem + kOffB + ab * kBBytes;
                    for (int sgi = ct; sgi < N * 8; sgi += 128) {
                        const int rr = sgi & 7, kb = (sgi >> 3) & 7, row = (sgi >> 6) * 8 + rr;
                        const int j = row < n_pad ? row : row - n_pad, hl = row < n_pad ? 0 : 1;
                        unsigned char *dst = bt + ((row >> 3) * 8 + kb) * 128 + rr * 16;
                        if (j < it.n)
                            cp_async16(dst, bsrc + (size_t)tb.src[j] + hl * K + u * 64 + kb * 8);
                        else
                            *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
                    }
                    for (int m = 0; m < mats; m++) {
                        unsigned char *at = smem + kOffA + (ab * 2 + m) * kABytes + ((ct >> 3) * 8) * 128 + (ct & 7) * 16;
                        q4k_unit_to_a(raw + m * kSbBytes + ct * 144, c, at, 128);
                    }
                    cp_async_wait_all();
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) arrive(&bars.ab_full[ab]);
                }
                __syncwarp();
                if (lane == 0) arrive(&bars.raw_empty[st]);
            }
            __syncwarp();
            if (lane == 0) arrive(&bars.item_empty[slot]);
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------------ epilogue
        grid_dep_wait();
        const int ew = warp - kEpiWarp0;         // 0..7
        const int q = warp & 3;                  // TMEM lane quarter
        const int r = 32 * q + lane;             // row within the tile
        const int half = ew >> 2;                // token half
        const int et = tid - kEpiWarp0 * 32;     // 0..255
        int gsb = 0;
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
            const Item it = items[slot];
            if (it.kind == kEnd) break;
            const TokTab &tb = tabs[slot];
            const int n_pad = (it.n + 15) & ~15, hw = n_pad >> 1;  // tokens per half (multiple of 8)
            const int j0 = half * hw;
            const int mats = it.kind == kGU ? 2 : 1;
            const int nsb = it.kind == kGU ? gu_sb : dn_sb;
            float2 acc[2][16];
#pragma unroll
            for (int m = 0; m < 2; m++)
#pragma unroll
                for (int p = 0; p < 16; p++) acc[m][p] = make_float2(0.0f, 0.0f);
            bool ok = true;
            for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                const int db = gsb & 1, sc_slot = gsb & 3;
                if (!(ok = wait_phase(&bars.d_full[db], (gsb >> 1) & 1, &abort_flag, err))) break;
                if (!(ok = wait_phase(&bars.sc_full[sc_slot], (gsb >> 2) & 1, &abort_flag, err))) break;
                tc_fence_after();
                const unsigned char *scb = smem + kOffSc + sc_slot * kScSlot;
                const uint4 *scs = reinterpret_cast<const uint4 *>(scb);
                const float *xs = reinterpret_cast<const float *>(scb + kScRows);
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    if (m >= mats) break;
                    const uint4 sv = scs[m * kTcRows + r];
                    const float2 d2 = make_float2(__uint_as_float(sv.x), __uint_as_float(sv.x));
                    const float2 nm2 = make_float2(-__uint_as_float(sv.y), -__uint_as_float(sv.y));
                    float mg[8];
#pragma unroll
                    for (int g = 0; g < 8; g++) mg[g] = (float)(((g < 4 ? sv.z : sv.w) >> (8 * (g & 3))) & 0xFFu);
                    const uint32_t col0 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((db * 2 + m) * 128);
#pragma unroll
                    for (int cb = 0; cb < 4; cb++) {
                        if (cb * 8 >= hw) break;
                        uint32_t rh[8], rl[8];
                        tmem_ld8_nw(col0 + j0 + cb * 8, rh);
                        tmem_ld8_nw(col0 + n_pad + j0 + cb * 8, rl);
                        tmem_wait_ld();
#pragma unroll
                        for (int pp = 0; pp < 4; pp++) {
                            const int j = j0 + cb * 8 + 2 * pp;
                            const float2 hi = make_float2(__uint_as_float(rh[2 * pp]), __uint_as_float(rh[2 * pp + 1]));
                            const float2 lo = make_float2(__uint_as_float(rl[2 * pp]), __uint_as_float(rl[2 * pp + 1]));
                            const float2 inv = *reinterpret_cast<const float2 *>(&tb.inv[j]);
                            const float2 dot = __fmul2_rn(__ffma2_rn(lo, make_float2(1.0f / 2048.0f, 1.0f / 2048.0f), hi), inv);
                            float2 mt = make_float2(0.0f, 0.0f);
#pragma unroll
                            for (int g = 0; g < 8; g++)
                                mt = __ffma2_rn(make_float2(mg[g], mg[g]), *reinterpret_cast<const float2 *>(&xs[g * kTcTok + j]), mt);
                            float2 &ac = acc[m][cb * 4 + pp];
                            ac = __ffma2_rn(d2, dot, ac);
                            ac = __ffma2_rn(nm2, mt, ac);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    arrive(&bars.d_empty[db]);
                    arrive(&bars.sc_empty[sc_slot]);
                }
            }
            if (ok) {
                if (it.kind == kGU) {
#pragma unroll
                    for (int p = 0; p < 16; p++) {
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int jj = 2 * p + e, j = j0 + jj;
                            if (jj < hw && j < it.n) {
                                const float g = e ? acc[0][p].y : acc[0][p].x, uu = e ? acc[1][p].y : acc[1][p].x;
                                a.mid[(size_t)tb.mrow[j] * F + it.mt * kTcRows + r] = (g * sigmoidf_ref(g)) * uu;
                            }
                        }
                    }
                    __threadfence();
                    bar_named(3, 256);
                    if (et == 0) s_flag = atomicAdd(a.gu_done + it.sub, 1) == gu_mt - 1;
                    bar_named(3, 256);
                    if (s_flag) {
                        // last gate/up tile of this token tile: fp16 hi/lo copies of its mid rows
                        __threadfence();
                        for (int j = ew; j < it.n; j += 8) {
                            const size_t mrow = (size_t)tb.mrow[j];
                            const float *src = a.mid + mrow * F;
                            float mx = 0.0f;
                            for (int i = lane; i < F; i += 32) mx = fmaxf(mx, fabsf(__ldcg(src + i)));
#pragma unroll
                            for (int dd = 16; dd; dd >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, dd));
                            int e = 0;
                            if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);
                            const float s = (mx > 0.0f && isfinite(mx)) ? ldexpf(1.0f, 14 - e) : 1.0f;
                            __half *dst = a.mid16 + mrow * 2 * F;
                            for (int i = lane; i < F; i += 32) {
                                const float v = __ldcg(src + i) * s;
                                const __half hi = __float2half_rn(v);
                                dst[i] = hi;
                                dst[F + i] = __float2half_rn((v - __half2float(hi)) * 2048.0f);
                            }
                            for (int g = 0; g < F / 32; g++) {
                                float v = __ldcg(src + g * 32 + lane);
#pragma unroll
                                for (int dd = 16; dd; dd >>= 1) v += __shfl_xor_sync(0xffffffffu, v, dd);
                                if (lane == 0) a.msum[mrow * (F / 32) + g] = v;
                            }
                            if (lane == 0) a.midinv[mrow] = 1.0f / s;
                        }
                        __threadfence();
                        bar_named(3, 256);
                        if (et == 0) atomicAdd(a.gu_done + it.sub, 1);
                    }
                } else {
                    const int row = it.mt * kTcRows + r;
#pragma unroll
                    for (int p = 0; p < 16; p++) {
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int jj = 2 * p + e, j = j0 + jj;
                            if (jj < hw && j < it.n) {
                                const float y = e ? acc[0][p].y : acc[0][p].x;
                                if (it.expert < 0) a.shout[(size_t)tb.tok[j] * H + row] = y;
                                else a.slots[(size_t)tb.slot[j] * H + row] = y * tb.w[j];
                            }
                        }
                    }
                    __threadfence();
                    bar_named(3, 256);
                    if (et == 0) s_ncombine = 0;
                    bar_named(3, 256);
                    if (et < it.n) {
                        const int t = tb.tok[et];
                        int *cnt = a.tilecnt + (size_t)t * dn_mt + it.mt;
                        const int expect = __ldcg(a.expect + t) & 0xffff;
                        if (atomicAdd(cnt, 1) == expect - 1) {
                            *cnt = 0;
                            s_combine[atomicAdd(&s_ncombine, 1)] = t;
                        }
                    }
                    bar_named(3, 256);
                    const int nc = s_ncombine;
                    if (nc) {
                        __threadfence();
                        for (int ci = et >> 7; ci < nc; ci += 2) {
                            const int t = s_combine[ci];
                            const int rr = it.mt * kTcRows + (et & 127);
                            const bool bad = (__ldcg(a.expect + t) & (int)kBad) != 0;
                            float sum = 0.0f;
#pragma unroll
                            for (int k = 0; k < kTop; k++) {
                                const int id = __ldcg(a.ids + t * kTop + k);
                                sum += id >= 0 ? __ldcg(a.slots + ((size_t)t * kTop + k) * H + rr) : 0.0f;
                            }
                            if (a.sg) sum = __fmaf_rn(__ldcg(a.shout + (size_t)t * H + rr), sigmoidf_ref(__ldcg(a.sgate + t)), sum);
                            a.out[(size_t)t * H + rr] = bad ? __int_as_float(0x7fc00000) : sum;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) arrive(&bars.item_empty[slot]);
            if (!ok) break;
        }
    }
    // ---------------------------------------------------------- teardown
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.tc_ticket, 1) == (int)gridDim.x - 1) {
            __threadfence();
            *a.queue = 0;
            *a.tc_ticket = 0;
        }
    }
}

__global__ void tc_prep_kernel(const float *x, int H, __half *x16, float *xinv, float *xsum) {
    const int t = blockIdx.x;
    tc_prep_token(x + (size_t)t * H, H, x16 + (size_t)t * 2 * H, xinv + t, xsum + (size_t)t * (H / 32));
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

// 2-D byte tensor [rows][row_bytes] read in boxes of one Q4_K superblock
// (144 bytes) by 128 rows.
int make_map(CUtensorMap *m, const void *base, size_t rows, size_t row_bytes) {
    EncodeTiled fn = encoder();
    if (!fn) return cudaErrorNotSupported;
    if (!base || (reinterpret_cast<uintptr_t>(base) & 15) || row_bytes % 16) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {row_bytes, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {144, (cuuint32_t)kTcRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}

int sm_count_tc() {
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

bool tc_supported(int H, int F, int QG, int QD) {
    return QG == 12 && QD == 12 && H % 256 == 0 && F % 256 == 0 && H >= 256 && F >= 256 && encoder() != nullptr;
}

size_t tc_smem_bytes() { return kSmem; }

int tc_make_maps(const TcArgs &a, TcMaps &m) {
    const size_t E = kExperts;
    int rc = make_map(&m.gate, a.gate, E * a.F, a.grb);
    if (!rc) rc = make_map(&m.up, a.up, E * a.F, a.grb);
    if (!rc) rc = make_map(&m.down, a.down, E * a.H, a.drb);
    if (!rc && a.sg) rc = make_map(&m.sg, a.sg, a.F, a.grb);
    if (!rc && a.sg) rc = make_map(&m.su, a.su, a.F, a.grb);
    if (!rc && a.sg) rc = make_map(&m.sd, a.sd, a.H, a.drb);
    if (!rc && !a.sg) {
        m.sg = m.gate;
        m.su = m.up;
        m.sd = m.down;
    }
    return rc;
}

int tc_launch(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl) {
    int rc = cudaFuncSetAttribute(tc_experts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count_tc());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tc_experts_kernel, a, m);
}

int tc_prep_launch(const float *x, int T, int H, __half *x16, float *xinv, float *xsum, cudaStream_t st) {
    tc_prep_kernel<<<T, 256, 0, st>>>(x, H, x16, xinv, xsum);
    return cudaGetLastError();
}

}  // namespace nb
