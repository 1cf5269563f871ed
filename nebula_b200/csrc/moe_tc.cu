// Tensor-core (tcgen05) expert kernel for Q4_K routed experts and the shared
// expert, used by both the decode and the prefill paths. The down weights may
// instead be IQ4_NL (the production mix: Q4_K gate/up, IQ4_NL down, ffn 640):
// see the IQ4_NL notes below.
//
// Work items (claimed from a device queue, shared expert first): a gate/up
// tile = 128 rows of W_gate and of W_up of one expert x one token tile of up
// to 48 tokens; a down tile = 128 rows of W_down x the same token tile.
//
// The contraction runs on the 5th-generation tensor cores:
//   A = sc_g * q_k    fp16, exact (integers <= 945), decoded from the raw Q4_K
//                     bytes by four converter warps straight into tensor
//                     memory (tcgen05.st; lane = weight row), so A never
//                     crosses shared memory;
//   B = [v_hi | v_lo] fp16 in shared memory (UMMA K-major, 128B swizzle),
//                     v*s = v_hi + v_lo/2048 with a power of two s (22-bit
//                     precision): the token's activations (one s per token)
//                     for gate/up, the SwiGLU output (one s per token and
//                     128-value tile) for down;
//   D = A B^T         fp32 in tensor memory, accumulated per 256-value Q4_K
//                     superblock (down: per 128-value half, one per scale)
//                     into one of two TMEM buffers.
// A tcgen05.mma with N <= 64 costs about the same issue time whatever N is, so
// two threads issue them: one for W_gate (or the first half of a down
// superblock), one for W_up (or the second half).
// Eight epilogue warps read each superblock's D back (tcgen05.ld), apply the
// superblock scale d and the dmin*m_g*sum(v) term in fp32 and accumulate in
// registers. A gate/up tile ends with SiLU(g)*u, whose fp16 hi/lo split, scale
// and 32-value group sums it writes directly for the down tiles; a down tile
// ends with the route weight, and the last contribution to a (token, 128-row
// tile) sums the ten slots in router-rank order plus the gated shared expert
// (qwen/cpu.c:209-231, qwen/gpu.cu:552).
//
// Raw weight bytes stream with 2-D TMA tensor copies (a 144-byte x 128-row
// box = one superblock of 128 rows) into a three-stage ring; B rows (128B
// swizzled, hi rows then lo rows), group sums and scales stream with 2-D TMA
// copies issued by their own warp into four- and four-slot rings. Roles:
//   warp 0 lane 0   producer: claims items, issues TMA
//   warp 1          TMEM owner; lane 0 issues the gate (first-half) MMAs
//   warp 2          B stager: token table, B rows, per-superblock group sums
//   warp 3 lane 0   issues the up (second-half) MMAs
//   warps 4-11      converters (thread = weight row; warps 4-7 the low
//                   nibbles and the row scales, warps 8-11 the high nibbles)
//   warps 12-19     epilogue (warp w reads TMEM lanes 32*(w%4).., half the
//                   tokens each); a tile's per-token outputs go through a
//                   shared buffer so the per-token loops stay short
// IQ4_NL down (DIQ): each 32-value block's fp16 scale d is folded into A as
// two fp16 planes, hi = fp16(d*c) and lo = d*c - hi (exact), issued as two
// MMAs into the same accumulator; the epilogue then applies only the B scale.
// A down tile's 128 rows (ffn/32 blocks of 18 bytes each, not a multiple of
// 16 bytes) arrive in one bulk copy, and an ffn of 640 ends in a half step of
// 128 values.
// Every wait is bounded; on a timeout the CTA raises the error word, stops
// taking work, drains its copies and MMAs, frees TMEM and exits.
#include <algorithm>
#include <cstring>
#include "moe_tc.cuh"
#include "quant.cuh"

using namespace nb;

namespace {

constexpr int kWarps = 20, kThreads = kWarps * 32;
constexpr int kProdWarp = 0, kMmaWarp = 1, kStageWarp = 2, kMma2Warp = 3, kConvWarp0 = 4, kEpiWarp0 = 12;
constexpr int kConvWarps = 8, kEpiWarps = 8;
// Registers: launched at 96 per thread (20 warps x 32 x 96 = 61440); warpgroups
// 0-2 (producer, issuers, stager, converters) give theirs down to 64 and the
// two epilogue warpgroups take them up to 144: 12*32*64 + 8*32*144 = 61440.
constexpr int kRegsLaunch = 96, kRegsLow = 64, kRegsEpi = 144;
static_assert((kWarps - kEpiWarps) * kRegsLow + kEpiWarps * kRegsEpi == kWarps * kRegsLaunch, "register split");
static_assert(kEpiWarp0 % 4 == 0 && kEpiWarps % 4 == 0, "register split is per warpgroup");
constexpr int kSbBytes = kTcRows * 144;           // one superblock of 128 Q4_K rows
constexpr int kOffRaw = 0;
constexpr int kScRows = 2 * kTcRows * 16;         // d, dmin, m[8] per row per matrix
// IQ4_NL down rows (ffn/32 blocks of 18 bytes) need not be a multiple of 16
// bytes long, so a down tile's 128 rows arrive whole in one bulk copy: up to
// ffn = 640 (46,080 bytes).
constexpr int kDiqMaxFfn = 640;
constexpr int kDiqRawStage = kTcRows * kDiqMaxFfn / 32 * 18;
// Layout of one instantiation for token tiles of up to TOK tokens; DIQ: the
// down weights are IQ4_NL; GIQ: the gate/up weights too (decode tiles only).
template <int TOK, bool DIQ = false, bool GIQ = false>
struct Cfg {
    static_assert(!GIQ || (DIQ && TOK <= 32), "IQ4_NL gate/up: with IQ4_NL down, decode tiles");
    // raw weight ring: a gate + up superblock, or (DIQ) a whole down tile
    static constexpr int kRawStage = DIQ ? kDiqRawStage : 2 * kSbBytes;
    static constexpr int kRawStages = (DIQ && TOK > 32) ? 2 : 3;
    // Decode tiles of kTcTokSmall tokens run the gate/up Q4_K min term
    // dmin*sum_g m_g*sum(x over g) on the tensor cores: per superblock one more
    // K=16 MMA per matrix, A'' = dmin*m_g*2^8 split hi/lo (exact in 22 bits), B'' =
    // the 8 group sums of x*s/32 split hi/lo, accumulated over the whole item in
    // D2 (read once per item) instead of per-superblock epilogue arithmetic.
    static constexpr bool kMinD2 = TOK == kTcTokSmall && !GIQ;
    static constexpr int kBBytes = 2 * TOK * 128;             // B: TOK hi rows, then TOK lo rows, 128 B each
    static constexpr int kB2Bytes = kMinD2 ? 64 * TOK : 0;    // B'': two K halves x [hi rows | lo rows] x 16 B
    static constexpr int kBSlot = (kBBytes + kB2Bytes + 1023) & ~1023;
    static constexpr int kBStages = TOK <= 32 ? 4 : 3;        // B ring depth
    static constexpr int kScXs = 8 * TOK * 4;                 // the superblock's 8 group sums per row [row][8]
    static constexpr int kScSlot = kScRows + kScXs + 4 * TOK * 4;  // + scales [row][4]
    static constexpr int kVBytes = 2 * TOK * kTcRows * 4;     // one tile's outputs [plane][slot][row] (gate/up: g, u)
    static constexpr int kOffB = kRawStages * kRawStage, kOffSc = kOffB + kBStages * kBSlot,
                         kOffV = kOffSc + 4 * kScSlot, kSmem = kOffV + kVBytes;
    // Tensor memory (512 columns): D[db][m] at (db*2+m)*kDCols; with the min term
    // D2[m] at kD2Col + m*kDCols and A''[buf][m] (8 columns) at kA2Col +
    // (buf*2+m)*8; A stage ab at kACol0 + ab*kAStride, its 32-column blocks (64
    // fp16 of one 64-value chunk) at (m*2+p)*32 for matrix m and plane p (an
    // IQ4_NL gate/up stage holds both planes of both matrices; a Q4_K stage
    // matrix m at m*32; an IQ4_NL down stage plane p at p*32).
    static constexpr int kDCols = 2 * TOK;
    static constexpr int kD2Col = 4 * kDCols, kA2Col = kD2Col + 2 * kDCols;
    static constexpr int kACol0 = kMinD2 ? kA2Col + 32 : 4 * kDCols;
    static constexpr int kAStride = GIQ ? 128 : 64;
    static constexpr int kAStages = (512 - kACol0) / kAStride >= 4 ? 4 : (512 - kACol0) / kAStride;
    static_assert(kAStages >= 2 && kACol0 + kAStages * kAStride <= 512, "tensor memory budget");
    static_assert(kSmem % 16 == 0 && kScSlot % 16 == 0 && kOffB % 1024 == 0 && kBBytes % 1024 == 0 &&
                      kBSlot % 1024 == 0 && (TOK * 128) % 1024 == 0 && (16 * TOK) % 128 == 0, "alignment");
    // 227 KB per CTA, less about 4 KB of static shared memory (barriers, tables)
    static_assert(kSmem <= 232448 - 4096, "shared memory budget");
};
constexpr int kTokDecode = 32;  // decode: every token tile has at most kMaxDecodeTokens tokens
static_assert(kTokDecode <= kTcTok, "tile sizes");
constexpr uint32_t kBad = 1u << 16;

enum { kEnd = 0, kGU = 1, kDN = 2 };
// A gate/up item covers superblocks k0 .. k0+nk-1 of its tile, part kq of np
// (np > 1: the tile is split along K between items; see the producer).
struct Item {
    int kind, sub, mt, expert, first, n, tok0, k0, nk, kq, np;
};

struct Bars {
    uint64_t item_full[4], item_empty[4], tab_full[4];
    uint64_t raw_full[3], raw_empty[3];  // up to three raw stages
    uint64_t a_full[4], a_empty[4];
    uint64_t b_full[8], b_empty[8];
    uint64_t d_full[2], d_empty[2];
    uint64_t sc_full[4], sc_empty[4];
    uint64_t mma_done[2];
    uint64_t d2_empty;  // the epilogue has read D2 (gate/up items, min term on the tensor cores)
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
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow)); }
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpi)); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Bounded wait used by every role; `abort` is the CTA-wide stop flag. Kept
// small (it is inlined at every hand-off): up to 2^17 sleeping attempts, each
// suspending until the phase completes or for at most a 20 us hint, so a lost
// completion ends the wait with an error within about 2.6 s.
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    for (int i = 0; i < (1 << 17); i++) {
        if (mbar_try_wait_sleep(bar, parity, kWaitHintNs)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    atomicOr(err, 4);
    return false;
}

// Bounded wait that ignores the stop flag: used to drain work already in flight.
__device__ __forceinline__ bool wait_drain(uint64_t *bar, uint32_t parity) {
    for (int i = 0; i < (1 << 17); i++)
        if (mbar_try_wait_sleep(bar, parity, kWaitHintNs)) return true;
    return false;
}

// Bounded wait on a counter written by other CTAs.
__device__ bool wait_geq_int(const int *p, int target, int *err) {
    const uint64_t t0 = global_ns();
    do {
        if (ld_acquire(p) >= target) return true;
        __nanosleep(64);
    } while (global_ns() - t0 < kWaitLimitNs);
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
// SBO = distance between 8-row groups. Adding n to the descriptor advances
// its start address by 16*n bytes.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// The same for a K-major tile with 128-byte swizzle (rows of 64 fp16 = 128 B,
// 8-row atoms 1024 B apart; the tile starts on a 1024-byte boundary). Moving
// to the next 16-value step adds 32 B (2 units) to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both K-major.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D (tmem) [+]= A (tmem) * B (smem descriptor)^T
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_ts1(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;" ::"r"(d), "r"(a), "l"(b), "r"(idesc)
                 : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8_nw(uint32_t addr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(addr));
}
__device__ __forceinline__ void tmem_ld4_nw(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t addr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(addr));
    return r;
}
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Named barrier over n threads that also ANDs a predicate across them.
__device__ __forceinline__ bool bar_all(int id, int n, bool ok) {
    int r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.b32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"((int)ok), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Q4_K: decode half `nib` of unit c of one 144-byte row into 16 tensor-memory
// columns. Unit c holds values 64c..64c+63: the low nibbles of its 32 bytes
// are values 64c+l (scale sc[2c]), the high nibbles 64c+32+l (scale sc[2c+1]).
// Column i of the unit holds values 64c+2i (low half) and 64c+2i+1, so half 0
// fills columns 0..15 and half 1 columns 16..31. Each value is sc*q exactly:
// (1024 + q) or (1024 + 16 q) come out of the nibbles as fp16 bit patterns
// and one half-precision FMA per pair removes the offset and applies sc.
__device__ __forceinline__ void q4k_half_cols(const unsigned char *row, int c, int nib, uint32_t (&r)[16]) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(row);
    const unsigned char *sc = reinterpret_cast<const unsigned char *>(&hd) + 4;
    int s, m;
    k_scale_min(sc, 2 * c + nib, s, m);
    (void)m;
    const __half2 mul = __half2half2(nib ? __float2half_rn((float)s * 0.0625f) : __int2half_rn(s));
    const __half2 off = __half2half2(__int2half_rn(nib ? -64 * s : -1024 * s));
    const uint32_t mask = nib ? 0x00F000F0u : 0x000F000Fu;
    const uint4 q0 = *reinterpret_cast<const uint4 *>(row + 16 + 32 * c);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(row + 32 + 32 * c);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t t01 = __byte_perm(w[i], 0, 0x4140), t23 = __byte_perm(w[i], 0, 0x4342);
        uint32_t v0 = (t01 & mask) | 0x64006400u, v1 = (t23 & mask) | 0x64006400u;
        __half2 h0 = __hfma2(*reinterpret_cast<__half2 *>(&v0), mul, off);
        __half2 h1 = __hfma2(*reinterpret_cast<__half2 *>(&v1), mul, off);
        r[2 * i] = *reinterpret_cast<uint32_t *>(&h0);
        r[2 * i + 1] = *reinterpret_cast<uint32_t *>(&h1);
    }
}

// IQ4_NL: one 32-value block (fp16 d, then 16 code bytes: low nibbles are
// values 0..15, high nibbles 16..31) of one row as 16 tensor-memory columns
// per plane, column i holding values 2i and 2i+1: hi = fp16(d*c) and
// lo = fp16(d*c - hi) for the code-book integer c. d*c has at most 18
// significant bits and is a multiple of 2^-24, so lo is exact and
// hi + lo == d*c (for |d| < 512, where d*c stays finite in fp16).
__device__ __forceinline__ void iq4_block_cols(const unsigned char *blk, uint32_t (&hi)[16], uint32_t (&lo)[16]) {
    const unsigned short *p16 = reinterpret_cast<const unsigned short *>(blk);  // blocks start on even bytes
    const __half2 d2 = __half2half2(__ushort_as_half(p16[0]));
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480u));  // 1152 = 1024 + 128
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t w = (uint32_t)p16[1 + 2 * i] | ((uint32_t)p16[2 + 2 * i] << 16);  // code bytes 4i..4i+3
#pragma unroll
        for (int h = 0; h < 2; h++) {  // low nibbles: values 4i..4i+3; high nibbles: 16+4i..16+4i+3
            const uint32_t cb = iq4_lut4(h ? (w >> 4) & 0x0F0F0F0Fu : w & 0x0F0F0F0Fu);  // code + 128 per byte
#pragma unroll
            for (int k = 0; k < 2; k++) {
                // two codes as the fp16 pair (1024 + code + 128), then exact code-book values
                uint32_t v = __byte_perm(cb, 0x64646464u, k ? 0x4342u : 0x4140u);
                const __half2 c2 = __hsub2(*reinterpret_cast<const __half2 *>(&v), bias);
                const __half2 h2 = __hmul2_rn(c2, d2);
                const __half2 l2 = __hfma2(c2, d2, __hneg2(h2));
                const int col = 8 * h + 2 * i + k;
                hi[col] = *reinterpret_cast<const uint32_t *>(&h2);
                lo[col] = *reinterpret_cast<const uint32_t *>(&l2);
            }
        }
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

// The min term of one superblock row as a K=16 A operand (8 tensor-memory
// columns): values 0..7 are the fp16 hi parts of dmin*m_g*2^8 for g = 0..7,
// values 8..15 the lo parts (v - hi; v has at most 17 significant bits, so the
// pair is exact unless dmin is below about 2^-16). The B operand pairs both
// halves with the same group sums.
__device__ __forceinline__ void q4k_min_a(const unsigned char *row, uint32_t (&o)[8]) {
    const uint4 rs = q4k_row_scales(row);  // d, dmin, m[8]
    const float dm = __uint_as_float(rs.y) * 256.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int g0 = 2 * i, g1 = 2 * i + 1;
        const float v0 = dm * (float)(((g0 < 4 ? rs.z : rs.w) >> (8 * (g0 & 3))) & 0xFFu);
        const float v1 = dm * (float)(((g1 < 4 ? rs.z : rs.w) >> (8 * (g1 & 3))) & 0xFFu);
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
        o[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        o[4 + i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
}

// sum_g m_g * xs[row][g] for rows j0 and j1 (xs: 8 group sums per row)
__device__ __forceinline__ float2 mterm2(const float (&mg)[8], const float *xs, int j0, int j1) {
    const float4 a0 = *reinterpret_cast<const float4 *>(xs + j0 * 8), a1 = *reinterpret_cast<const float4 *>(xs + j0 * 8 + 4);
    const float4 b0 = *reinterpret_cast<const float4 *>(xs + j1 * 8), b1 = *reinterpret_cast<const float4 *>(xs + j1 * 8 + 4);
    float2 t = __fmul2_rn(make_float2(mg[0], mg[0]), make_float2(a0.x, b0.x));
    t = __ffma2_rn(make_float2(mg[1], mg[1]), make_float2(a0.y, b0.y), t);
    t = __ffma2_rn(make_float2(mg[2], mg[2]), make_float2(a0.z, b0.z), t);
    t = __ffma2_rn(make_float2(mg[3], mg[3]), make_float2(a0.w, b0.w), t);
    t = __ffma2_rn(make_float2(mg[4], mg[4]), make_float2(a1.x, b1.x), t);
    t = __ffma2_rn(make_float2(mg[5], mg[5]), make_float2(a1.y, b1.y), t);
    t = __ffma2_rn(make_float2(mg[6], mg[6]), make_float2(a1.z, b1.z), t);
    t = __ffma2_rn(make_float2(mg[7], mg[7]), make_float2(a1.w, b1.w), t);
    return t;
}

// Per-item token table, filled by the B stager once per item.
template <int TOK>
struct __align__(16) TokTab {
    int tok[TOK];   // token index
    int mrow[TOK];  // SwiGLU-output row written (gate/up) or read (down)
    int slot[TOK];  // routed slot t*10+k (down)
    float w[TOK];   // route weight (down)
    float xi[TOK];  // 1/s of each D column's activation row (gate/up with the min term on the tensor cores)
    int ex[TOK];    // expected contributions of the token (down; combine counting)
};

template <int TOK, bool DIQ, bool GIQ>
__global__ void __launch_bounds__(kThreads, 1) tc_experts_kernel(const TcArgs a, const __grid_constant__ TcMaps maps) {
    using C = Cfg<TOK, DIQ, GIQ>;
    constexpr int kTok = TOK, kBBytes = C::kBBytes, kScXs = C::kScXs, kScSlot = C::kScSlot, kOffB = C::kOffB,
                  kOffSc = C::kOffSc, kOffV = C::kOffV, kDCols = C::kDCols, kACol0 = C::kACol0,
                  kAStages = C::kAStages, kBStages = C::kBStages, kRawStage = C::kRawStage,
                  kRawStages = C::kRawStages, kAStride = C::kAStride;
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ Bars bars;
    __shared__ Item items[4];
    __shared__ TokTab<TOK> tabs[4];
    __shared__ float s_scale[kTok];  // power-of-two scale per token of one gate/up tile
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ int s_combine[kTok];
    __shared__ int s_ncombine;
    __shared__ int s_last;  // this K part is the last of its gate/up tile
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, H = a.H, F = a.F;
    const int gu_mt = F / kTcRows, dn_mt = H / kTcRows;
    // superblocks (K steps of 256 values) of a whole gate/up tile, of a down tile
    // (IQ4_NL down: ffn may end in a half step of 128 values)
    const int nsbk = H / 256, dn_sb = (F + 255) / 256;
    // 64-value chunks of step sb of a down tile
    auto dn_chunks = [&](int sb) { return DIQ ? min(4, (F - 256 * sb) / 64) : 4; };
    if (tid == 0) {
        for (int i = 0; i < 4; i++) {
            mbar_init(&bars.item_full[i], 1);
            mbar_init(&bars.item_empty[i], 2 + 1 + kConvWarps + kEpiWarps);  // issuers, stager, converters, epilogue
            mbar_init(&bars.tab_full[i], 1);
            mbar_init(&bars.sc_full[i], kConvWarps + 1);  // converters (row scales), stager (group sums, 1/s)
            mbar_init(&bars.sc_empty[i], kEpiWarps);
        }
        for (int i = 0; i < kRawStages; i++) {
            mbar_init(&bars.raw_full[i], 1);
            mbar_init(&bars.raw_empty[i], kConvWarps);
        }
        for (int i = 0; i < kAStages; i++) {
            mbar_init(&bars.a_full[i], kConvWarps);
            mbar_init(&bars.a_empty[i], 2);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars.d_full[i], 2);
            mbar_init(&bars.d_empty[i], kEpiWarps);
            mbar_init(&bars.mma_done[i], 1);
        }
        mbar_init(&bars.d2_empty, kEpiWarps);
        for (int i = 0; i < kBStages; i++) {
            mbar_init(&bars.b_full[i], 1);
            mbar_init(&bars.b_empty[i], 2);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = tmem_base;
    int *err = a.err;

    if (warp == kProdWarp) {
        // ------------------------------------------------------ producer
        regs_dec();
        if (lane == 0) {
            // Claim order: the shared expert's gate/up tiles (whole; known before the
            // routing), then the routed gate/up superblocks in ranges of q, then the
            // down tiles. With gu_part, q spreads the routed tiles' superblocks
            // evenly over the CTAs left (q >= half a tile keeps a tile in at most
            // kMaxParts ranges); a range that crosses tile boundaries becomes one
            // item per tile piece, and pieces of one tile are summed in part order.
            bool planned = false;
            int nsub = a.shared_subs, gsb = 0;
            const int S_gu = a.shared_subs * gu_mt;
            int q = nsbk, n_rng = 0, U = 0;  // routed range length, ranges, superblocks
            int r_beg = 0, r_end = 0, r_id = 0;  // the claimed range's superblocks not yet emitted
            for (int seq = 0;; seq++) {
                const int slot = seq & 3;
                const bool ok = seq < 4 || wait_phase(&bars.item_empty[slot], ((seq >> 2) - 1) & 1, &abort_flag, err);
                Item it{kEnd, 0, 0, -1, 0, 0, 0, 0, 0, 0, 1};
                if (ok && !abort_flag) {
                    if (r_beg >= r_end) {
                        const int idx = atomicAdd(a.queue, 1);
                        if (idx >= S_gu && !planned) {
                            grid_dep_wait();  // routed work: the plan comes from the preceding kernel
                            nsub = __ldcg(a.n_sub);
                            planned = true;
                            U = (nsub - a.shared_subs) * gu_mt * nsbk;
                            if (a.gu_part && U > 0) {
                                const int g2 = max(1, (int)gridDim.x - S_gu);
                                q = max((nsbk + 1) / 2, (U + g2 - 1) / g2);
                            }
                            n_rng = (U + q - 1) / q;
                        }
                        const int total_dn = nsub * dn_mt;
                        if (idx < S_gu) {
                            it.kind = kGU, it.sub = idx / gu_mt, it.mt = idx % gu_mt, it.nk = nsbk;
                        } else if (idx < S_gu + n_rng) {
                            r_id = idx - S_gu, r_beg = r_id * q, r_end = min(U, r_beg + q);
                        } else if (idx < S_gu + n_rng + total_dn) {
                            const int d = idx - S_gu - n_rng;
                            it.kind = kDN, it.sub = d / dn_mt, it.mt = d % dn_mt;
                        }
                    }
                    if (r_beg < r_end) {  // the range's piece within its next tile
                        const int tile = r_beg / nsbk, k0 = r_beg % nsbk, nk = min(nsbk - k0, r_end - r_beg);
                        const int f = tile * nsbk / q, l = ((tile + 1) * nsbk - 1) / q;
                        it.kind = kGU, it.sub = a.shared_subs + tile / gu_mt, it.mt = tile % gu_mt;
                        it.k0 = k0, it.nk = nk, it.kq = r_id - f, it.np = l - f + 1;
                        r_beg += nk;
                    }
                }
                if (it.kind != kEnd) {
                    if (it.sub < a.shared_subs) {  // known without the routing
                        it.expert = -1, it.tok0 = a.sh_t0 + it.sub * kTok, it.n = min(kTok, a.sh_t1 - it.tok0), it.first = 0;
                    } else {
                        it.expert = __ldcg(&a.sub[it.sub].expert);
                        it.first = __ldcg(&a.sub[it.sub].first);
                        it.n = __ldcg(&a.sub[it.sub].n);
                    }
                }
                items[slot] = it;
                arrive(&bars.item_full[slot]);
                if (it.kind == kEnd) break;
                // raw units: one per superblock, or (IQ4_NL down) the whole tile
                const int nraw = it.kind == kGU ? it.nk : DIQ ? 1 : dn_sb;
                for (int sb = 0; sb < nraw; sb++, gsb++) {
                    const int st = gsb % kRawStages;
                    if (gsb >= kRawStages &&
                        !wait_phase(&bars.raw_empty[st], (gsb / kRawStages - 1) & 1, &abort_flag, err))
                        break;
                    unsigned char *dst = smem + kOffRaw + st * kRawStage;
                    if (it.kind == kGU) {
                        const int y = (it.expert < 0 ? 0 : it.expert * F) + it.mt * kTcRows;
                        mbar_arrive_expect_tx(&bars.raw_full[st], 2 * kSbBytes);
                        const int x = (it.k0 + sb) * 144;
                        tma_2d(dst, it.expert < 0 ? &maps.sg : &maps.gate, x, y, &bars.raw_full[st]);
                        tma_2d(dst + kSbBytes, it.expert < 0 ? &maps.su : &maps.up, x, y, &bars.raw_full[st]);
                    } else if (DIQ) {  // 128 whole rows: 128 * drb <= kRawStage bytes, 16-byte aligned
                        const size_t row = (size_t)(it.expert < 0 ? 0 : it.expert * H) + it.mt * kTcRows;
                        const uint32_t bytes = (uint32_t)(kTcRows * a.drb);
                        mbar_arrive_expect_tx(&bars.raw_full[st], bytes);
                        tma_load_1d(dst, (it.expert < 0 ? a.sd : a.down) + row * a.drb, bytes, &bars.raw_full[st]);
                    } else {
                        const int y = (it.expert < 0 ? 0 : it.expert * H) + it.mt * kTcRows;
                        mbar_arrive_expect_tx(&bars.raw_full[st], kSbBytes);
                        tma_2d(dst, it.expert < 0 ? &maps.sd : &maps.down, sb * 144, y, &bars.raw_full[st]);
                    }
                }
                if (abort_flag) break;
            }
            // the last copies issued have landed before the CTA may exit
            for (int k = max(0, gsb - kRawStages); k < gsb; k++)
                wait_drain(&bars.raw_full[k % kRawStages], (k / kRawStages) & 1);
        }
    } else if (warp == kMmaWarp || warp == kMma2Warp) {
        // ------------------------------------------------------ MMA issuers
        regs_dec();
        // issuer mi: gate/up tiles -> matrix mi; down tiles -> chunks 2mi, 2mi+1
        if (lane == 0) {
            const int mi = warp == kMmaWarp ? 0 : 1;
            int gsb = 0, gch = 0, gu_items = 0;
            const uint64_t b_desc0 = umma_desc_sw128(smem_u32(smem + kOffB));
            const uint64_t b2_desc0 = umma_desc(smem_u32(smem + kOffB + kBBytes), 32 * kTok, 128);
            const uint32_t idesc = idesc_f16(kTcRows, 2 * kTok);  // hi and lo rows of every tile row
            for (int seq = 0;; seq++) {
                const int slot = seq & 3;
                if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
                const Item it = items[slot];
                if (it.kind == kEnd) break;
                const bool gu = it.kind == kGU;
                const int nsb = gu ? it.nk : dn_sb;
                bool ok = true;
                for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                    const int db = gsb & 1;
                    if (gsb >= 2 && !(ok = wait_phase(&bars.d_empty[db], ((gsb >> 1) - 1) & 1, &abort_flag, err))) break;
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)((db * 2 + mi) * kDCols);
                    const int nch = gu ? 4 : dn_chunks(sb);
                    for (int c = 0; c < nch; c++, gch++) {
                        const int ab = gch % kAStages, bs = gch % kBStages;
                        if (!(ok = wait_phase(&bars.a_full[ab], (gch / kAStages) & 1, &abort_flag, err))) break;
                        if (!(ok = wait_phase(&bars.b_full[bs], (gch / kBStages) & 1, &abort_flag, err))) break;
                        if (gu || (c >> 1) == mi) {
                            tc_fence_after();
                            const uint32_t ac =
                                tmem + (uint32_t)(kACol0 + ab * kAStride + (gu ? mi * (GIQ ? 64 : 32) : 0));
                            const uint64_t bd = b_desc0 + (uint64_t)((bs * C::kBSlot) >> 4);
                            mma_ts(d, ac, bd, idesc, gu ? c != 0 : (c & 1) != 0);
                            mma_ts1(d, ac + 8, bd + 2, idesc);
                            mma_ts1(d, ac + 16, bd + 4, idesc);
                            mma_ts1(d, ac + 24, bd + 6, idesc);
                            if (gu ? GIQ : DIQ) {  // IQ4_NL: the lo plane of A into the same D
                                mma_ts1(d, ac + 32, bd, idesc);
                                mma_ts1(d, ac + 40, bd + 2, idesc);
                                mma_ts1(d, ac + 48, bd + 4, idesc);
                                mma_ts1(d, ac + 56, bd + 6, idesc);
                            }
                            if constexpr (C::kMinD2) {
                                if (gu && c == 3) {  // min term into D2 (the item's first superblock starts it)
                                    if (sb == 0 && gu_items > 0 &&
                                        !(ok = wait_phase(&bars.d2_empty, (gu_items - 1) & 1, &abort_flag, err)))
                                        break;
                                    tc_fence_after();
                                    mma_ts(tmem + (uint32_t)(C::kD2Col + mi * kDCols),
                                           tmem + (uint32_t)(C::kA2Col + ((gsb & 1) * 2 + mi) * 8),
                                           b2_desc0 + (uint64_t)((bs * C::kBSlot) >> 4), idesc, sb != 0);
                                }
                            }
                            mma_commit(&bars.a_empty[ab]);
                            mma_commit(&bars.b_empty[bs]);
                        } else {  // the other issuer's chunk: nothing read here
                            arrive(&bars.a_empty[ab]);
                            arrive(&bars.b_empty[bs]);
                        }
                    }
                    if (ok) mma_commit(&bars.d_full[db]);
                }
                if (gu) gu_items++;
                arrive(&bars.item_empty[slot]);
                if (!ok) break;
            }
            // every MMA issued by this thread completes before TMEM is released
            mma_commit(&bars.mma_done[mi]);
            wait_drain(&bars.mma_done[mi], 0);
        }
    } else if (warp == kStageWarp) {
        // ------------------------------------------------------ B stager
        regs_dec();
        grid_dep_wait();  // activations, routing and plan come from the preceding kernel
        int gsb = 0, gch = 0;
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
            const Item it = items[slot];
            if (it.kind == kEnd) break;
            TokTab<TOK> &tb = tabs[slot];
            const bool gu = it.kind == kGU, sh = it.expert < 0;
            const int n_pad = min(kTok, (it.n + 15) & ~15);  // table entries filled (padding repeats row 0)
            const int row0 = sh ? T * kTop + it.tok0 : it.first;  // first SwiGLU-output row of the tile
            for (int j = lane; j < n_pad; j += 32) {
                const int jv = j < it.n ? j : 0;
                const int sl = sh ? 0 : __ldcg(a.pairs + it.first + jv);
                tb.tok[j] = sh ? it.tok0 + jv : sl / kTop;
                tb.mrow[j] = row0 + jv;
                tb.slot[j] = sl;
                tb.w[j] = (sh || gu) ? 0.0f : __ldcg(a.wts + sl);
            }
            __syncwarp();
            // values the epilogue's tail would otherwise fetch from L2 on its critical path
            if (C::kMinD2 && gu) {
                const int ncol = a.all_tok ? T : it.n, xrow0 = a.all_tok ? 0 : row0;
                for (int c = lane; c < ncol; c += 32) tb.xi[c] = __ldcg(a.xinv + (size_t)(xrow0 + c) * 4);
            } else if (!gu && !a.ep_ranks) {
                for (int j = lane; j < it.n; j += 32) tb.ex[j] = __ldcg(a.expect + tb.tok[j]);
            }
            bool ok = true;
            if (!gu) {  // the token tile's SwiGLU outputs: every gate/up tile of this sub-job has finished
                if (lane == 0 && !wait_geq_int(a.gu_done + it.sub, gu_mt, err)) abort_flag = 1;
                __syncwarp();
                ok = !abort_flag;
            }
            __syncwarp();
            if (lane == 0) {
                arrive(&bars.tab_full[slot]);
                // B tile rows: all T tokens (per-token activations) or the tile's own rows
                const int brow = (gu && a.all_tok) ? 0 : row0;
                const CUtensorMap *bh = gu ? &maps.bx_hi : &maps.bm_hi, *bl = gu ? &maps.bx_lo : &maps.bm_lo;
                const CUtensorMap *gs = gu ? &maps.sx : &maps.sm, *iv = gu ? &maps.ix : &maps.im;
                const int nsb = gu ? it.nk : dn_sb;
                for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                    const int sc_slot = gsb & 3;
                    if (gsb >= 4 && !(ok = wait_phase(&bars.sc_empty[sc_slot], ((gsb >> 2) - 1) & 1, &abort_flag, err)))
                        break;
                    unsigned char *scb = smem + kOffSc + sc_slot * kScSlot;
                    mbar_arrive_expect_tx(&bars.sc_full[sc_slot], kScXs + 4 * kTok * 4);
                    const int gsbk = gu ? it.k0 + sb : sb;  // superblock index along K
                    tma_2d(scb + kScRows, gs, gsbk * 8, brow, &bars.sc_full[sc_slot]);
                    tma_2d(scb + kScRows + kScXs, iv, gu ? 0 : (2 * sb) & ~3, brow, &bars.sc_full[sc_slot]);
                    const int nch = gu ? 4 : dn_chunks(sb);
                    for (int c = 0; c < nch; c++, gch++) {
                        const int bs = gch % kBStages;
                        if (gch >= kBStages &&
                            !(ok = wait_phase(&bars.b_empty[bs], (gch / kBStages - 1) & 1, &abort_flag, err)))
                            break;
                        unsigned char *bt = smem + kOffB + bs * C::kBSlot;
                        const bool b2 = C::kMinD2 && gu && c == 3;  // with the superblock's min-term B
                        mbar_arrive_expect_tx(&bars.b_full[bs], kBBytes + (b2 ? C::kB2Bytes : 0));
                        tma_2d(bt, bh, (gsbk * 4 + c) * 64, brow, &bars.b_full[bs]);
                        tma_2d(bt + kTok * 128, bl, (gsbk * 4 + c) * 64, brow, &bars.b_full[bs]);
                        if (b2) {  // [K half][hi rows | lo rows] x 8 group sums, both halves the same
                            for (int kh = 0; kh < 2; kh++) {
                                tma_2d(bt + kBBytes + kh * 32 * kTok, &maps.gx_hi, gsbk * 8, brow, &bars.b_full[bs]);
                                tma_2d(bt + kBBytes + kh * 32 * kTok + 16 * kTok, &maps.gx_lo, gsbk * 8, brow,
                                       &bars.b_full[bs]);
                            }
                        }
                    }
                }
                arrive(&bars.item_empty[slot]);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
        if (lane == 0)  // copies still in flight land before the CTA may exit
            for (int k = max(0, gch - kBStages); k < gch; k++) wait_drain(&bars.b_full[k % kBStages], (k / kBStages) & 1);
    } else if (warp >= kConvWarp0 && warp < kEpiWarp0) {
        // ------------------------------------------------------ converters
        regs_dec();
        const int ct = 32 * (warp & 3) + lane;           // weight row of the tile = TMEM lane
        const int nib = (warp - kConvWarp0) >> 2;        // 0: low nibbles + row scales, 1: high nibbles
        const uint32_t a_lanes = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kACol0 + nib * 16;
        int gsb = 0, gch = 0, graw = 0;  // superblocks, chunks, raw units
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            if (!wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err)) break;
            const Item it = items[slot];
            if (it.kind == kEnd) break;
            const int mats = it.kind == kGU ? 2 : 1;
            const int nsb = it.kind == kGU ? it.nk : dn_sb;
            // IQ4_NL down: one raw unit holds the whole tile; this thread's row
            const bool diq = DIQ && it.kind == kDN;
            bool ok = true;
            int st = graw % kRawStages;
            if (diq) ok = wait_phase(&bars.raw_full[st], (graw / kRawStages) & 1, &abort_flag, err);
            for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                const int sc_slot = gsb & 3;
                if (!diq) {
                    st = graw % kRawStages;
                    if (!(ok = wait_phase(&bars.raw_full[st], (graw / kRawStages) & 1, &abort_flag, err))) break;
                }
                const unsigned char *raw = smem + kOffRaw + st * kRawStage;
                // row scales: matrix nib (gate by the low-nibble warps, up by the high-nibble ones)
                if (gsb >= 4 && !(ok = wait_phase(&bars.sc_empty[sc_slot], ((gsb >> 2) - 1) & 1, &abort_flag, err)))
                    break;
                if (nib < mats && !diq && !GIQ) {
                    uint4 *scs = reinterpret_cast<uint4 *>(smem + kOffSc + sc_slot * kScSlot);
                    scs[nib * kTcRows + ct] = q4k_row_scales(raw + nib * kSbBytes + ct * 144);
                }
                __syncwarp();
                if (lane == 0) arrive(&bars.sc_full[sc_slot]);
                // kGrp chunks per store-completion wait (half the A ring)
                constexpr int kGrp = kAStages >= 4 ? 2 : 1;
                const int nch = diq ? dn_chunks(sb) : 4;
                for (int c = 0; c < nch && ok; c += kGrp, gch += kGrp) {
                    for (int h = 0; h < kGrp; h++) {
                        const int g = gch + h, ab = g % kAStages;
                        if (g >= kAStages &&
                            !(ok = wait_phase(&bars.a_empty[ab], (g / kAStages - 1) & 1, &abort_flag, err)))
                            break;
                    }
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < kGrp; h++) {
                        const int ab = (gch + h) % kAStages;
                        if (DIQ && diq) {  // block 2*chunk + nib of the row: hi plane, lo plane
                            uint32_t rh[16], rl[16];
                            iq4_block_cols(raw + ct * a.drb + (size_t)(2 * (4 * sb + c + h) + nib) * 18, rh, rl);
                            tmem_st16(a_lanes + (uint32_t)(ab * kAStride), rh);
                            tmem_st16(a_lanes + (uint32_t)(ab * kAStride + 32), rl);
                        } else if (GIQ) {  // gate/up: block 2*chunk + nib of each matrix's row (144 B per 8 blocks)
                            for (int m = 0; m < 2; m++) {
                                uint32_t rh[16], rl[16];
                                iq4_block_cols(raw + m * kSbBytes + ct * 144 + (2 * (c + h) + nib) * 18, rh, rl);
                                tmem_st16(a_lanes + (uint32_t)(ab * kAStride + m * 64), rh);
                                tmem_st16(a_lanes + (uint32_t)(ab * kAStride + m * 64 + 32), rl);
                            }
                        } else {
                            for (int m = 0; m < mats; m++) {
                                uint32_t r[16];
                                q4k_half_cols(raw + m * kSbBytes + ct * 144, c + h, nib, r);
                                tmem_st16(a_lanes + (uint32_t)(ab * kAStride + m * 32), r);
                            }
                        }
                    }
                    if constexpr (C::kMinD2) {
                        if (mats == 2 && c + kGrp > 3) {  // with chunk 3: matrix nib's min-term A for this superblock
                            uint32_t o[8];
                            q4k_min_a(raw + nib * kSbBytes + ct * 144, o);
                            tmem_st8(tmem + ((uint32_t)(32 * (warp & 3)) << 16) +
                                         (uint32_t)(C::kA2Col + ((gsb & 1) * 2 + nib) * 8),
                                     o);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        for (int h = 0; h < kGrp; h++) arrive(&bars.a_full[(gch + h) % kAStages]);
                }
                if (!diq) {
                    __syncwarp();
                    if (lane == 0) arrive(&bars.raw_empty[st]);
                    graw++;
                }
            }
            if (diq) {
                __syncwarp();
                if (lane == 0) arrive(&bars.raw_empty[st]);
                graw++;
            }
            __syncwarp();
            if (lane == 0) arrive(&bars.item_empty[slot]);
            if (!ok) break;
        }
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------------ epilogue
        regs_inc();
        grid_dep_wait();
        const int ew = warp - kEpiWarp0;         // 0..7
        const int q = warp & 3;                  // TMEM lane quarter
        const int r = 32 * q + lane;             // row within the tile
        const int half = ew >> 2;                // token half
        const int et = tid - kEpiWarp0 * 32;     // 0..255
        constexpr int kHalf = (kTok / 2 + 7) / 8 * 8;  // token slots per half, at most (multiple of 8)
        int gsb = 0;
        for (int seq = 0;; seq++) {
            const int slot = seq & 3;
            bool ok = wait_phase(&bars.item_full[slot], (seq >> 2) & 1, &abort_flag, err);
            const Item it = items[slot];
            if (!bar_all(3, 256, ok) || it.kind == kEnd) break;
            const TokTab<TOK> &tb = tabs[slot];
            const bool gu = it.kind == kGU;
            // D columns c (hi) and kTok + c (lo): token c of all T tokens (gate/up on
            // per-token activations) or row c of the tile
            const bool by_tok = gu && a.all_tok;
            // token slots j (the item's tokens, in order) split in two halves of hw
            // (even) slots; slot j reads D column j, or column tok_j when the tile
            // multiplied all T tokens
            const int hw = ((it.n + 3) >> 2) << 1;
            const int j0 = half * hw;
            const int nsb = gu ? it.nk : dn_sb;
            float2 acc[2][kHalf / 2];
#pragma unroll
            for (int m = 0; m < 2; m++)
#pragma unroll
                for (int p = 0; p < kHalf / 2; p++) acc[m][p] = make_float2(0.0f, 0.0f);
            // min term on the tensor cores (gate/up): thread = row x matrix `half`, one
            // sum per D column (token of all T, or row of the tile)
            const int ncol = by_tok ? T : it.n;
            float acc2[C::kMinD2 ? kTok : 1];
#pragma unroll
            for (int i = 0; i < (C::kMinD2 ? kTok : 1); i++) acc2[i] = 0.0f;
            for (int sb = 0; sb < nsb && ok; sb++, gsb++) {
                const int db = gsb & 1, sc_slot = gsb & 3;
                if (!(ok = wait_phase(&bars.d_full[db], (gsb >> 1) & 1, &abort_flag, err))) break;
                if (!(ok = wait_phase(&bars.sc_full[sc_slot], (gsb >> 2) & 1, &abort_flag, err))) break;
                tc_fence_after();
                const unsigned char *scb = smem + kOffSc + sc_slot * kScSlot;
                const uint4 *scs = reinterpret_cast<const uint4 *>(scb);
                const float *xs = reinterpret_cast<const float *>(scb + kScRows);
                const float *inv4 = reinterpret_cast<const float *>(scb + kScRows + kScXs);  // [row][4]
                const uint32_t lanes = tmem + ((uint32_t)(32 * q) << 16);
                const float2 k2048 = make_float2(1.0f / 2048.0f, 1.0f / 2048.0f);
                bool d_released = false;
                if (TOK == 48 && gu && !by_tok) {
                    // 48-token tiles of per-row activations (prefill): each 4-slot block loads
                    // both matrices' hi/lo columns with one wait, then runs 8 independent
                    // per-slot chains; the D buffer is released once its last load has landed.
                    // Slots between the item's rows and the block end read finite padding
                    // data and are never stored.
                    float dsc[2], nmn[2], mg[2][8];
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        const uint4 sv = scs[m * kTcRows + r];
                        dsc[m] = __uint_as_float(sv.x);
                        nmn[m] = -__uint_as_float(sv.y);
#pragma unroll
                        for (int g = 0; g < 8; g++) mg[m][g] = (float)(((g < 4 ? sv.z : sv.w) >> (8 * (g & 3))) & 0xFFu);
                    }
                    const uint32_t colg = lanes + (uint32_t)((db * 2) * kDCols), colu = colg + kDCols;
                    const int ncb = min(kHalf / 4, (hw + 3) >> 2);
#pragma unroll
                    for (int cb = 0; cb < kHalf / 4; cb++) {
                        if (cb >= ncb) break;
                        uint32_t gh[4], gl[4], uh[4], ul[4];
                        const uint32_t o = (uint32_t)(j0 + cb * 4);
                        tmem_ld4_nw(colg + o, gh);
                        tmem_ld4_nw(colg + kTok + o, gl);
                        tmem_ld4_nw(colu + o, uh);
                        tmem_ld4_nw(colu + kTok + o, ul);
                        tmem_wait_ld();
                        if (cb == ncb - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) arrive(&bars.d_empty[db]);
                            d_released = true;
                        }
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int j = j0 + cb * 4 + i;
                            const float inv = inv4[j * 4];
                            const float4 xa = *reinterpret_cast<const float4 *>(xs + j * 8);
                            const float4 xb = *reinterpret_cast<const float4 *>(xs + j * 8 + 4);
                            const float hv[2] = {__uint_as_float(gh[i]), __uint_as_float(uh[i])};
                            const float lv[2] = {__uint_as_float(gl[i]), __uint_as_float(ul[i])};
#pragma unroll
                            for (int m = 0; m < 2; m++) {
                                const float dot = __fmul_rn(__fmaf_rn(lv[m], 1.0f / 2048.0f, hv[m]), inv);
                                float t = __fmul_rn(mg[m][0], xa.x);
                                t = __fmaf_rn(mg[m][1], xa.y, t);
                                t = __fmaf_rn(mg[m][2], xa.z, t);
                                t = __fmaf_rn(mg[m][3], xa.w, t);
                                t = __fmaf_rn(mg[m][4], xb.x, t);
                                t = __fmaf_rn(mg[m][5], xb.y, t);
                                t = __fmaf_rn(mg[m][6], xb.z, t);
                                t = __fmaf_rn(mg[m][7], xb.w, t);
                                float2 &ac = acc[m][cb * 2 + (i >> 1)];
                                float &a1 = (i & 1) ? ac.y : ac.x;
                                a1 = __fmaf_rn(nmn[m], t, __fmaf_rn(dsc[m], dot, a1));
                            }
                        }
                    }
                } else if (C::kMinD2 && gu) {
                    if constexpr (C::kMinD2) {
                        const float dsc = __uint_as_float(scs[half * kTcRows + r].x);
                        const uint32_t col0 = lanes + (uint32_t)((db * 2 + half) * kDCols);
#pragma unroll
                        for (int cb = 0; cb < kTok / 8; cb++) {
                            if (cb * 8 < ncol) {
                                uint32_t rh[8], rl[8];
                                tmem_ld8_nw(col0 + cb * 8, rh);
                                tmem_ld8_nw(col0 + kTok + cb * 8, rl);
                                tmem_wait_ld();
#pragma unroll
                                for (int i = 0; i < 8; i++)
                                    acc2[cb * 8 + i] = __fmaf_rn(
                                        dsc, __fmaf_rn(__uint_as_float(rl[i]), 1.0f / 2048.0f, __uint_as_float(rh[i])),
                                        acc2[cb * 8 + i]);
                            }
                        }
                    }
                } else if (GIQ && gu) {
                    // IQ4_NL gate/up: the block scales are in A; only the token's B scale
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        const uint32_t col0 = lanes + (uint32_t)((db * 2 + m) * kDCols);
#pragma unroll
                        for (int cb = 0; cb < kHalf / 8; cb++) {
                            if (cb * 8 >= hw) break;
                            uint32_t rh[8], rl[8];
                            if (by_tok) {  // gather the slots' token columns
#pragma unroll
                                for (int i = 0; i < 8; i++) {
                                    const int c = tb.tok[min(j0 + cb * 8 + i, it.n - 1)];
                                    rh[i] = tmem_ld1(col0 + c);
                                    rl[i] = tmem_ld1(col0 + kTok + c);
                                }
                            } else {
                                tmem_ld8_nw(col0 + j0 + cb * 8, rh);
                                tmem_ld8_nw(col0 + kTok + j0 + cb * 8, rl);
                            }
                            tmem_wait_ld();
#pragma unroll
                            for (int pp = 0; pp < 4; pp++) {
                                if (cb * 8 + 2 * pp >= hw) break;
                                const int j = j0 + cb * 8 + 2 * pp;
                                const int c0 = by_tok ? tb.tok[min(j, it.n - 1)] : j;
                                const int c1 = by_tok ? tb.tok[min(j + 1, it.n - 1)] : j + 1;
                                const float2 hi = make_float2(__uint_as_float(rh[2 * pp]), __uint_as_float(rh[2 * pp + 1]));
                                const float2 lo = make_float2(__uint_as_float(rl[2 * pp]), __uint_as_float(rl[2 * pp + 1]));
                                float2 &ac = acc[m][cb * 4 + pp];
                                ac = __ffma2_rn(__ffma2_rn(lo, k2048, hi), make_float2(inv4[c0 * 4], inv4[c1 * 4]), ac);
                            }
                        }
                    }
                } else if (gu) {
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        const uint4 sv = scs[m * kTcRows + r];
                        const float2 d2 = make_float2(__uint_as_float(sv.x), __uint_as_float(sv.x));
                        const float2 nm2 = make_float2(-__uint_as_float(sv.y), -__uint_as_float(sv.y));
                        float mg[8];
#pragma unroll
                        for (int g = 0; g < 8; g++) mg[g] = (float)(((g < 4 ? sv.z : sv.w) >> (8 * (g & 3))) & 0xFFu);
                        const uint32_t col0 = lanes + (uint32_t)((db * 2 + m) * kDCols);
#pragma unroll
                        for (int cb = 0; cb < kHalf / 8; cb++) {
                            if (cb * 8 >= hw) break;
                            uint32_t rh[8], rl[8];
                            if (by_tok) {  // gather the slots' token columns
#pragma unroll
                                for (int i = 0; i < 8; i++) {
                                    const int c = tb.tok[min(j0 + cb * 8 + i, it.n - 1)];
                                    rh[i] = tmem_ld1(col0 + c);
                                    rl[i] = tmem_ld1(col0 + kTok + c);
                                }
                            } else {
                                tmem_ld8_nw(col0 + j0 + cb * 8, rh);
                                tmem_ld8_nw(col0 + kTok + j0 + cb * 8, rl);
                            }
                            tmem_wait_ld();
#pragma unroll
                            for (int pp = 0; pp < 4; pp++) {
                                if (cb * 8 + 2 * pp >= hw) break;
                                const int j = j0 + cb * 8 + 2 * pp;
                                const int c0 = by_tok ? tb.tok[min(j, it.n - 1)] : j;
                                const int c1 = by_tok ? tb.tok[min(j + 1, it.n - 1)] : j + 1;
                                const float2 hi = make_float2(__uint_as_float(rh[2 * pp]), __uint_as_float(rh[2 * pp + 1]));
                                const float2 lo = make_float2(__uint_as_float(rl[2 * pp]), __uint_as_float(rl[2 * pp + 1]));
                                const float2 inv = make_float2(inv4[c0 * 4], inv4[c1 * 4]);
                                const float2 dot = __fmul2_rn(__ffma2_rn(lo, k2048, hi), inv);
                                const float2 mt = mterm2(mg, xs, c0, c1);
                                float2 &ac = acc[m][cb * 4 + pp];
                                ac = __ffma2_rn(d2, dot, ac);
                                ac = __ffma2_rn(nm2, mt, ac);
                            }
                        }
                    }
                } else if (DIQ) {
                    // IQ4_NL down: the block scales are in A; D[db][h] holds 128-value half h
                    // of this step (a step at the end of ffn may have one half), each with
                    // its own B scale
                    const uint32_t c0 = lanes + (uint32_t)((db * 2) * kDCols);
                    const int ioff = (2 * sb) & 3, nh = min(2, (F - 256 * sb) / 128);
#pragma unroll
                    for (int cb = 0; cb < kHalf / 8; cb++) {
                        if (cb * 8 >= hw) break;
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            if (h >= nh) break;
                            uint32_t rh[8], rl[8];
                            tmem_ld8_nw(c0 + h * kDCols + j0 + cb * 8, rh);
                            tmem_ld8_nw(c0 + h * kDCols + kTok + j0 + cb * 8, rl);
                            tmem_wait_ld();
#pragma unroll
                            for (int pp = 0; pp < 4; pp++) {
                                if (cb * 8 + 2 * pp >= hw) break;
                                const int j = j0 + cb * 8 + 2 * pp;
                                const float2 v = __ffma2_rn(make_float2(__uint_as_float(rl[2 * pp]), __uint_as_float(rl[2 * pp + 1])), k2048,
                                                            make_float2(__uint_as_float(rh[2 * pp]), __uint_as_float(rh[2 * pp + 1])));
                                float2 &ac = acc[0][cb * 4 + pp];
                                ac = __ffma2_rn(v, make_float2(inv4[j * 4 + ioff + h], inv4[j * 4 + 4 + ioff + h]), ac);
                            }
                        }
                    }
                } else {
                    const uint4 sv = scs[r];
                    const float2 d2 = make_float2(__uint_as_float(sv.x), __uint_as_float(sv.x));
                    const float2 nm2 = make_float2(-__uint_as_float(sv.y), -__uint_as_float(sv.y));
                    float mg[8];
#pragma unroll
                    for (int g = 0; g < 8; g++) mg[g] = (float)(((g < 4 ? sv.z : sv.w) >> (8 * (g & 3))) & 0xFFu);
                    const uint32_t c0 = lanes + (uint32_t)((db * 2) * kDCols);
                    const int ioff = (2 * sb) & 3;  // this superblock's two scales within the loaded four
#pragma unroll
                    for (int cb = 0; cb < kHalf / 8; cb++) {
                        if (cb * 8 >= hw) break;
#pragma unroll
                        for (int h = 0; h < 2; h++) {  // the two 128-value halves, one B scale each
                            uint32_t rh[8], rl[8];
                            tmem_ld8_nw(c0 + h * kDCols + j0 + cb * 8, rh);
                            tmem_ld8_nw(c0 + h * kDCols + kTok + j0 + cb * 8, rl);
                            tmem_wait_ld();
#pragma unroll
                            for (int pp = 0; pp < 4; pp++) {
                                if (cb * 8 + 2 * pp >= hw) break;
                                const int j = j0 + cb * 8 + 2 * pp;
                                const float2 v = __ffma2_rn(make_float2(__uint_as_float(rl[2 * pp]), __uint_as_float(rl[2 * pp + 1])), k2048,
                                                            make_float2(__uint_as_float(rh[2 * pp]), __uint_as_float(rh[2 * pp + 1])));
                                const float2 dot = __fmul2_rn(v, make_float2(inv4[j * 4 + ioff + h], inv4[j * 4 + 4 + ioff + h]));
                                float2 &ac = acc[0][cb * 4 + pp];
                                ac = __ffma2_rn(d2, dot, ac);
                                if (h) ac = __ffma2_rn(nm2, mterm2(mg, xs, j, j + 1), ac);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (!d_released) arrive(&bars.d_empty[db]);
                    arrive(&bars.sc_empty[sc_slot]);
                }
            }
            if constexpr (C::kMinD2) {
                if (gu) {  // the item's min term: D2, complete once its last superblock's D is
                    if (ok) {
                        tc_fence_after();
                        const uint32_t c2 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(C::kD2Col + half * kDCols);
#pragma unroll
                        for (int cb = 0; cb < kTok / 8; cb++) {
                            if (cb * 8 < ncol) {
                                uint32_t rh[8], rl[8];
                                tmem_ld8_nw(c2 + cb * 8, rh);
                                tmem_ld8_nw(c2 + kTok + cb * 8, rl);
                                tmem_wait_ld();
#pragma unroll
                                for (int i = 0; i < 8; i++)
                                    acc2[cb * 8 + i] = __fmaf_rn(
                                        -0.125f, __fmaf_rn(__uint_as_float(rl[i]), 1.0f / 2048.0f, __uint_as_float(rh[i])),
                                        acc2[cb * 8 + i]);
                            }
                        }
                        tc_fence_before();
                    }
                    __syncwarp();
                    if (lane == 0) arrive(&bars.d2_empty);
                }
            }
            ok = ok && wait_phase(&bars.tab_full[slot], (seq >> 2) & 1, &abort_flag, err);
            if (!bar_all(3, 256, ok)) break;
            // the tile's outputs (SwiGLU for gate/up) to the shared buffer sv[slot][row]
            // (with the min term on the tensor cores: sv[matrix][column][row], scaled
            // back by the column's 1/s)
            float *sv = reinterpret_cast<float *>(smem + kOffV);
            const bool cols_tok = C::kMinD2 && gu && by_tok;  // gate/up planes indexed by token
            if (C::kMinD2 && gu) {
#pragma unroll
                for (int c = 0; c < (C::kMinD2 ? kTok : 1); c++)
                    if (c < ncol) sv[(half * kTok + c) * kTcRows + r] = acc2[c] * tb.xi[c];
            } else {
#pragma unroll
            for (int cb = 0; cb < kHalf / 8; cb++) {
                if (cb * 8 < hw) {
#pragma unroll
                    for (int pp = 0; pp < 4; pp++) {
                        if (cb * 8 + 2 * pp >= hw) break;  // the other half's slots
                        const float2 v = acc[0][cb * 4 + pp];
                        const int j = j0 + cb * 8 + 2 * pp;
                        sv[j * kTcRows + r] = v.x;
                        sv[(j + 1) * kTcRows + r] = v.y;
                        if (gu) {
                            const float2 u = acc[1][cb * 4 + pp];
                            sv[(kTok + j) * kTcRows + r] = u.x;
                            sv[(kTok + j + 1) * kTcRows + r] = u.y;
                        }
                    }
                }
            }
            }
            bar_named(3, 256);
            const int rr = et & 127;  // row handled by this thread in the per-token loops
            bool finish = true;
            if (gu && it.np > 1) {
                // this K part's partial sums; the last part of the tile adds them up in
                // part order and finishes it
                const size_t F2 = 2 * (size_t)F;
#pragma unroll 4
                for (int j = et >> 7; j < it.n; j += 2) {
                    const int cj = cols_tok ? tb.tok[j] : j;
                    float *pp = a.gu_part + ((size_t)tb.mrow[j] * kMaxParts + it.kq) * F2 + it.mt * kTcRows + rr;
                    pp[0] = sv[cj * kTcRows + rr];
                    pp[F] = sv[(kTok + cj) * kTcRows + rr];
                }
                // the CTA's stores, then one thread's fence and count (cumulative
                // through the barrier); the last part's fence orders its reads after
                bar_named(3, 256);
                if (et == 0) {
                    __threadfence();
                    int *cnt = a.gu_pcnt + it.sub * gu_mt + it.mt;
                    const int last = atomicAdd(cnt, 1) == it.np - 1;
                    if (last) *cnt = 0;
                    __threadfence();
                    s_last = last;
                }
                bar_named(3, 256);
                finish = s_last != 0;
                if (finish) {
#pragma unroll 4
                    for (int j = et >> 7; j < it.n; j += 2) {
                        const float *pp = a.gu_part + (size_t)tb.mrow[j] * kMaxParts * F2 + it.mt * kTcRows + rr;
                        float g = 0.0f, u = 0.0f;
#pragma unroll
                        for (int q = 0; q < kMaxParts; q++) {
                            if (q < it.np) {
                                g += __ldcg(pp + q * F2);
                                u += __ldcg(pp + q * F2 + F);
                            }
                        }
                        const int cj = cols_tok ? tb.tok[j] : j;
                        sv[cj * kTcRows + rr] = g;
                        sv[(kTok + cj) * kTcRows + rr] = u;
                    }
                }
                bar_named(3, 256);
            }
            if (gu && !finish) {
                // another K part finishes this tile
            } else if (gu) {
                // per token (one warp each): the four 32-row group sums and a power-of-two
                // scale from the tile's max |v|
#pragma unroll 3
                for (int j = ew; j < it.n; j += kEpiWarps) {
                    // SwiGLU of the token's 128 rows, kept in plane 0 for the split below
                    const int cj = cols_tok ? tb.tok[j] : j;
                    float *vj = sv + cj * kTcRows;
                    const float *uj = sv + (kTok + cj) * kTcRows;
                    float v[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float g = vj[32 * i + lane];
                        v[i] = (g * sigmoidf_ref(g)) * uj[32 * i + lane];
                        vj[32 * i + lane] = v[i];
                    }
                    const float v0 = v[0], v1 = v[1], v2 = v[2], v3 = v[3];
                    float s0 = v0, s1 = v1, s2 = v2, s3 = v3;
#pragma unroll
                    for (int dd = 16; dd; dd >>= 1) {
                        s0 += __shfl_xor_sync(0xffffffffu, s0, dd);
                        s1 += __shfl_xor_sync(0xffffffffu, s1, dd);
                        s2 += __shfl_xor_sync(0xffffffffu, s2, dd);
                        s3 += __shfl_xor_sync(0xffffffffu, s3, dd);
                    }
                    const float mx = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
                    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
                    if (lane == 0) {
                        float sc, inv;
                        pow2_scale(__uint_as_float(mb), sc, inv);
                        const size_t mrow = (size_t)tb.mrow[j];
                        *reinterpret_cast<float4 *>(a.msum + mrow * (F / 32) + it.mt * 4) = make_float4(s0, s1, s2, s3);
                        a.midinv[mrow * a.mi_stride + it.mt] = inv;
                        s_scale[j] = sc;
                    }
                }
                bar_named(3, 256);
                // fp16 hi/lo split of v*s for the down tiles
#pragma unroll 4
                for (int j = et >> 7; j < it.n; j += 2) {
                    const float v = sv[(cols_tok ? tb.tok[j] : j) * kTcRows + rr] * s_scale[j];
                    const __half hi = __float2half_rn(v);
                    const size_t base = (size_t)tb.mrow[j] * 2 * F + it.mt * kTcRows + rr;
                    a.mid16[base] = hi;
                    a.mid16[base + F] = __float2half_rn((v - __half2float(hi)) * 2048.0f);
                }
                bar_named(3, 256);
                if (et == 0) {
                    __threadfence();
                    atomicAdd(a.gu_done + it.sub, 1);
                }
            } else {
                const int row = it.mt * kTcRows + rr;
                if (a.ep_ranks) {
                    // every rank's buffers (this call's parity set when double-buffered);
                    // the combine kernel reduces
                    const size_t pbase = a.ep_cap ? (size_t)(__ldcg(a.ep_epoch) & 1) * a.ep_cap : 0;
#pragma unroll 4
                    for (int j = et >> 7; j < it.n; j += 2) {
                        const float y = sv[j * kTcRows + rr];
                        const size_t o = it.expert < 0 ? (pbase + tb.tok[j]) * H + row
                                                       : (pbase * kTop + tb.slot[j]) * H + row;
                        const float v = it.expert < 0 ? y : y * tb.w[j];
                        if (a.ep_block > 0) {  // the token's owner only
                            const int p = tb.tok[j] / a.ep_block;
                            (it.expert < 0 ? a.ep_shout[p] : a.ep_slots[p])[o] = v;
                        } else {
                            for (int p = 0; p < a.ep_ranks; p++) (it.expert < 0 ? a.ep_shout[p] : a.ep_slots[p])[o] = v;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) arrive(&bars.item_empty[slot]);
                    continue;
                }
#pragma unroll 4
                for (int j = et >> 7; j < it.n; j += 2) {
                    const float y = sv[j * kTcRows + rr];
                    if (it.expert < 0) a.shout[(size_t)tb.tok[j] * H + row] = y;
                    else a.slots[(size_t)tb.slot[j] * H + row] = y * tb.w[j];
                }
                if (!a.out) {  // large batches: a combine kernel after this one reduces the rows
                    __syncwarp();
                    if (lane == 0) arrive(&bars.item_empty[slot]);
                    continue;
                }
                if (et == 0) s_ncombine = 0;
                bar_named(3, 256);
                // per token: a fence (cumulative through the barrier) and the count; the
                // last contribution's fence orders the combine's reads after it
                if (et < it.n) {
                    const int t = tb.tok[et];
                    int *cnt = a.tilecnt + (size_t)t * dn_mt + it.mt;
                    const int expect = tb.ex[et] & 0xffff;
                    __threadfence();
                    if (atomicAdd(cnt, 1) == expect - 1) {
                        *cnt = 0;
                        __threadfence();
                        s_combine[atomicAdd(&s_ncombine, 1)] = t;
                    }
                }
                bar_named(3, 256);
                const int nc = s_ncombine;
                if (nc) {
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
            __syncwarp();
            if (lane == 0) arrive(&bars.item_empty[slot]);
        }
    }
    // ---------------------------------------------------------- teardown
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
    if (tid == 0) {
        if (a.ep_ranks) __threadfence_system();  // this CTA's peer stores before the ticket
        else __threadfence();
        if (atomicAdd(a.tc_ticket, 1) == (int)gridDim.x - 1) {
            __threadfence_system();
            *a.queue = 0;
            *a.tc_ticket = 0;
            if (a.ep_ranks) {  // every rank may now combine this rank's rows of this call
                grid_dep_wait();
                const int done = __ldcg(a.ep_epoch) + 1;
                for (int p = 0; p < a.ep_ranks; p++)
                    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(a.ep_flags[p] + a.ep_rank), "r"(done)
                                 : "memory");
            }
        }
    }
}

__global__ void tc_prep_kernel(const float *x, int H, __half *x16, float *xinv, float *xsum) {
    const int t = blockIdx.x;
    tc_prep_token(x + (size_t)t * H, H, x16 + (size_t)t * 2 * H, xinv + (size_t)t * 4, xsum + (size_t)t * (H / 32));
}

// One routed row per warp: rows [0, n_pairs) are the plan's (token, expert)
// pairs in expert order, rows T*10 + t the shared expert's tokens.
__global__ void __launch_bounds__(256) tc_prep_rows_kernel(const float *x, int T, int H, const int *pairs,
                                                           const int *n_pairs, int rows, __half *x16, float *xinv,
                                                           float *xsum) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    int tok;
    if (row < T * kTop) {
        if (row >= __ldcg(n_pairs)) return;
        tok = __ldcg(pairs + row) / kTop;
    } else {
        tok = row - T * kTop;
    }
    tc_prep_token_warp(x + (size_t)tok * H, H, x16 + (size_t)row * 2 * H, xinv + (size_t)row * 4,
                       xsum + (size_t)row * (H / 32));
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

// 2-D tensor [rows][inner] (row pitch in bytes) read in boxes of box_inner x box_rows.
int make_map_2d(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base, size_t inner, size_t rows,
                size_t pitch, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiled fn = encoder();
    if (!fn) return cudaErrorNotSupported;
    if (!base || (reinterpret_cast<uintptr_t>(base) & 15) || pitch % 16 || (box_inner * esize) % 16 || rows == 0)
        return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}

// Q4_K rows [rows][row_bytes] read one superblock (144 bytes) x 128 rows at a time.
int make_map(CUtensorMap *m, const void *base, size_t rows, size_t row_bytes) {
    if (row_bytes % 16) return cudaErrorInvalidValue;
    return make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, row_bytes, rows, row_bytes, 144, kTcRows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
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

bool tc_supported(int H, int F, int QG, int QD, int max_tile) {
    if (H % 256 || H < 256 || F % kTcRows || F < kTcRows || encoder() == nullptr) return false;
    if (QG == 12 && QD == 12) return F % 256 == 0;
    if (QG == 12 && QD == 20) return F <= kDiqMaxFfn;
    return QG == 20 && QD == 20 && F <= kDiqMaxFfn && max_tile <= kTokDecode;
}

int tc_make_maps(const TcArgs &a, TcMaps &m, int tok) {
    const size_t E = a.n_experts > 0 ? a.n_experts : kExperts, H = a.H, F = a.F;
    const size_t rows = (size_t)a.T * kTop + a.T;        // routed pairs + shared tokens
    const size_t xrows = a.all_tok ? (size_t)a.T : rows;  // rows of the gate/up activations
    const auto f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16, f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B, none = CU_TENSOR_MAP_SWIZZLE_NONE;
    // IQ4_NL down tiles arrive by plain bulk copies (rows need not be 16-byte multiples)
    if (a.dn_iq4) {
        if (a.F % kTcRows || a.F > kDiqMaxFfn || a.drb != (size_t)a.F / 32 * 18 ||
            (reinterpret_cast<uintptr_t>(a.down) & 15) || (a.sd && (reinterpret_cast<uintptr_t>(a.sd) & 15)))
            return cudaErrorInvalidValue;
        memset(&m.down, 0, sizeof(m.down));
        memset(&m.sd, 0, sizeof(m.sd));
    }
    int rc = make_map(&m.gate, a.gate, E * a.F, a.grb);
    if (!rc) rc = make_map(&m.up, a.up, E * a.F, a.grb);
    if (!rc && !a.dn_iq4) rc = make_map(&m.down, a.down, E * a.H, a.drb);
    if (!rc && a.sg) rc = make_map(&m.sg, a.sg, a.F, a.grb);
    if (!rc && a.sg) rc = make_map(&m.su, a.su, a.F, a.grb);
    if (!rc && a.sg && !a.dn_iq4) rc = make_map(&m.sd, a.sd, a.H, a.drb);
    if (!rc && !a.sg) {
        m.sg = m.gate;
        m.su = m.up;
        m.sd = m.down;
    }
    // activations and SwiGLU outputs: [row][2][K] fp16, hi plane then lo plane
    if (!rc) rc = make_map_2d(&m.bx_hi, f16, 2, a.x16, H, xrows, 4 * H, 64, tok, sw);
    if (!rc) rc = make_map_2d(&m.bx_lo, f16, 2, a.x16 + H, H, xrows, 4 * H, 64, tok, sw);
    if (!rc) rc = make_map_2d(&m.bm_hi, f16, 2, a.mid16, F, rows, 4 * F, 64, tok, sw);
    if (!rc) rc = make_map_2d(&m.bm_lo, f16, 2, a.mid16 + F, F, rows, 4 * F, 64, tok, sw);
    if (!rc) rc = make_map_2d(&m.sx, f32, 4, a.xsum, H / 32, xrows, H / 8, 8, tok, none);
    if (!rc && a.xs16) rc = make_map_2d(&m.gx_hi, f16, 2, a.xs16, H / 32, xrows, H / 8, 8, tok, none);
    if (!rc && a.xs16) rc = make_map_2d(&m.gx_lo, f16, 2, a.xs16 + H / 32, H / 32, xrows, H / 8, 8, tok, none);
    if (!rc && !a.xs16) m.gx_hi = m.gx_lo = m.sx;
    if (!rc && tok == kTcTokSmall && !a.gu_iq4 && !a.xs16) rc = cudaErrorInvalidValue;  // the min term needs the fp16 group sums
    if (!rc) rc = make_map_2d(&m.sm, f32, 4, a.msum, F / 32, rows, F / 8, 8, tok, none);
    if (!rc) rc = make_map_2d(&m.ix, f32, 4, a.xinv, 4, xrows, 16, 4, tok, none);
    if (!rc) rc = make_map_2d(&m.im, f32, 4, a.midinv, a.mi_stride, rows, 4 * (size_t)a.mi_stride, 4, tok, none);
    return rc;
}

template <int TOK, bool DIQ, bool GIQ>
int tc_launch_tok(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl) {
    constexpr int smem = Cfg<TOK, DIQ, GIQ>::kSmem;
    int rc = cudaFuncSetAttribute(tc_experts_kernel<TOK, DIQ, GIQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count_tc());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tc_experts_kernel<TOK, DIQ, GIQ>, a, m);
}

template <bool DIQ>
int tc_launch_fmt(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl, int max_tile) {
    if (max_tile <= kTcTokSmall) return tc_launch_tok<kTcTokSmall, DIQ, false>(a, m, st, pdl);
    if (max_tile <= kTokDecode) return tc_launch_tok<kTokDecode, DIQ, false>(a, m, st, pdl);
    if (max_tile <= kTcTok) return tc_launch_tok<kTcTok, DIQ, false>(a, m, st, pdl);
    return cudaErrorInvalidValue;
}

int tc_launch(const TcArgs &a, const TcMaps &m, cudaStream_t st, bool pdl, int max_tile) {
    if (a.gu_iq4) {  // IQ4_NL gate/up and down: decode tiles only
        if (!a.dn_iq4) return cudaErrorInvalidValue;
        if (max_tile <= kTcTokSmall) return tc_launch_tok<kTcTokSmall, true, true>(a, m, st, pdl);
        if (max_tile <= kTokDecode) return tc_launch_tok<kTokDecode, true, true>(a, m, st, pdl);
        return cudaErrorInvalidValue;
    }
    return a.dn_iq4 ? tc_launch_fmt<true>(a, m, st, pdl, max_tile) : tc_launch_fmt<false>(a, m, st, pdl, max_tile);
}

int tc_prep_launch(const float *x, int T, int H, __half *x16, float *xinv, float *xsum, cudaStream_t st) {
    tc_prep_kernel<<<T, 256, 0, st>>>(x, H, x16, xinv, xsum);
    return cudaGetLastError();
}

int tc_prep_rows_launch(const float *x, int T, int H, const int *pairs, const int *n_pairs, bool shared, __half *x16,
                        float *xinv, float *xsum, cudaStream_t st) {
    const int rows = T * kTop + (shared ? T : 0);
    if (H % 128) return cudaErrorInvalidValue;
    tc_prep_rows_kernel<<<(rows + 7) / 8, 256, 0, st>>>(x, T, H, pairs, n_pairs, rows, x16, xinv, xsum);
    return cudaGetLastError();
}

}  // namespace nb
