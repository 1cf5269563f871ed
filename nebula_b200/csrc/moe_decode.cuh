// Interface between the MoE entry points (moe.cu) and the decode kernels
// (moe_decode.cu), and the fixed workspace prefix both paths share.
#pragma once
#include <cstddef>
#include "common.cuh"
#include "moe_tc.cuh"

namespace nb {

constexpr int kMaxDecodeTokens = 32;
constexpr int kMaxGuTiles = 16;  // gate/up row tiles (ffn / 128) the balanced gate/up counters cover

// Workspace prefix: status words, then counters that every call leaves at
// zero for the next one. The general (large-batch) path never writes here.
struct DecHdr {
    int invalid_tokens, n_pairs, n_used, error;
};
struct DecCtr {
    int k1_ticket, queue, k2_ticket, tc_queue, tc_ticket, k1_routed, pad[8];
    unsigned long long lean_barrier;  // the lean kernel's grid barrier: arrivals, only growing
    int gu_done[kExperts + 1];
    int tilecnt[kMaxDecodeTokens * 64];
    int gu_pcnt[(kExperts + 1) * kMaxGuTiles];  // K parts finished per gate/up tile
};
static_assert(offsetof(DecCtr, lean_barrier) % 8 == 0, "64-bit barrier counter");
constexpr size_t kHdrBytes = 256;
constexpr size_t kPrefixBytes = (kHdrBytes + sizeof(DecCtr) + 255) & ~size_t(255);

struct DecLayout {
    size_t logits, sgate, ids, wts, xpair, xsum, off, used, pairs, expect, mid, msum, slots, shout;
    size_t x16, xinv, xs16, sub, nsub, mid16, midinv, part, total;  // tensor-core path
};
// Regions from `start` (the fixed prefix by default; expert parallelism puts its
// fixed cross-call block first and starts the per-call regions after it).
DecLayout dec_layout(int T, int H, int F, size_t start = kPrefixBytes);

struct DecArgs {
    int T, H, F, QG, QD;
    const float *x;
    const float *router, *bias, *s_router;  // router == null: ids/wts already hold the routing
    const unsigned char *gate, *up, *down, *sg, *su, *sd;
    size_t grb, drb;  // bytes of a gate/up row (hidden values) and of a down row (ffn values)
    float *out;
    int *ids;
    float *wts;
    DecHdr *hdr;
    DecCtr *ctr;
    float *logits, *sgate, *xpair, *xsum, *mid, *msum, *slots, *shout;
    int *off, *used, *pairs, *expect;
    // tensor-core path (Q4_K): fp16 hi/lo activations and sub-jobs
    int use_tc;
    __half *x16, *mid16, *xs16;
    float *xinv, *midinv;
    SubJob *sub;
    int *n_sub;
    // expert parallelism: ep_local[e] = index of expert e in gate/up/down on
    // this rank, or -1 (another rank's); null = all 512 here
    const int *ep_local;
    int n_experts;       // experts in gate/up/down
    int ep_shared_here;  // this rank computes the shared expert
    int ep_ranks, ep_rank;
    int ep_cap;  // tokens per parity buffer of the ranks' slot/shared rows
    float *ep_slots[kMaxRanks], *ep_shout[kMaxRanks];
    int *ep_flags[kMaxRanks];
    int *ep_epoch;
    float *gu_part;  // balanced gate/up work: K-part sums (TcArgs; counters in DecCtr)
    // filled by dec_run
    int gstride, dn_rows, stage_bytes, k1_ctas;
};

bool dec_supported(int T, int H, int F, int QG, int QD);
// split != null (profiling): recorded between the router/plan kernel and the
// expert kernel, which is then launched without programmatic overlap.
int dec_run(const DecArgs &a, cudaStream_t st, cudaEvent_t split = nullptr);
// The lean single-kernel layer (moe_lean.cu): router given, one GPU; 1 or 2
// tokens at hidden 2048 / ffn 512 with Q4_K experts, 1 to 4 at 2560 / 640 with
// Q4_K gate/up and IQ4_NL down.
bool lean_supported(const DecArgs &a);
int lean_run(const DecArgs &a, cudaStream_t st);

}  // namespace nb
