/* Expert parallelism driven from a plain C host: no Python, no torch, no MPI.
 *
 * The parent forks one process per GPU before any CUDA call. The ranks share an
 * anonymous mapping that carries each rank's 64-byte workspace handle
 * (qg_ep_ipc_handle) and a sense-free counting barrier with a bounded wait.
 * Rank r selects GPU r (cudaSetDevice: the library's calls follow the thread's
 * current device), builds the same synthetic layer as every other rank, keeps
 * the experts it owns (expert e belongs to rank e % ranks; a deal order, not a
 * ranking), opens the peers' workspaces (qg_ep_ipc_open) and runs
 * qg_moe_layer_ep on verify batches of 17, 5 and 17 tokens with one workspace.
 * Every call's ids must equal qg_moe_layer's on the full layer bit for bit and
 * its output match within rel-L2 1e-5 and max-abs 1e-4 * max|ref|.
 *
 * Usage: ep_c_host <ranks>. Exit 0 when every rank passed. */
#define _GNU_SOURCE
#include <math.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#include "gpu.h"

int cudaSetDevice(int device); /* CUDA runtime (libcudart) */

enum { H = 2048, F = 512, E = 512, MAXR = 8, TMAX = 17, Q4K = 12 };

typedef struct {
    atomic_int arrived;
    unsigned char handles[MAXR][64];
} shared_state;

static int barrier(shared_state *s, int ranks, int round) {
    atomic_fetch_add(&s->arrived, 1);
    const int target = ranks * round;
    struct timespec nap = {0, 1000000};
    for (int i = 0; i < 60000; i++) { /* at most about a minute */
        if (atomic_load(&s->arrived) >= target) return 0;
        nanosleep(&nap, NULL);
    }
    return -1;
}

#define CHECK(call)                                                               \
    do {                                                                          \
        int rc_ = (call);                                                         \
        if (rc_) {                                                                \
            fprintf(stderr, "rank %d: %s: %s\n", rank, #call, qg_error(rc_));     \
            return 1;                                                             \
        }                                                                         \
    } while (0)

static size_t q4k_row(int cols) { return (size_t)cols / 256 * 144; }

static int run_rank(shared_state *s, int rank, int ranks) {
    if (cudaSetDevice(rank)) {
        fprintf(stderr, "rank %d: cudaSetDevice failed\n", rank);
        return 1;
    }
    const size_t g_exp = F * q4k_row(H), d_exp = H * q4k_row(F);
    void *gate = qg_alloc(E * g_exp), *up = qg_alloc(E * g_exp), *down = qg_alloc(E * d_exp);
    void *router = qg_alloc((size_t)E * H * 4), *sg = qg_alloc(g_exp), *su = qg_alloc(g_exp), *sd = qg_alloc(d_exp);
    void *sr = qg_alloc(H * 4);
    if (!gate || !up || !down || !router || !sg || !su || !sd || !sr) return 1;
    CHECK(qg_synth_weights(gate, Q4K, E * F, H, 501, 0.02f));
    CHECK(qg_synth_weights(up, Q4K, E * F, H, 502, 0.02f));
    CHECK(qg_synth_weights(down, Q4K, E * H, F, 503, 0.02f));
    CHECK(qg_synth_weights(router, 0, E, H, 504, 0.02f));
    CHECK(qg_synth_weights(sg, Q4K, F, H, 505, 0.02f));
    CHECK(qg_synth_weights(su, Q4K, F, H, 506, 0.02f));
    CHECK(qg_synth_weights(sd, Q4K, H, F, 507, 0.02f));
    CHECK(qg_synth_weights(sr, 0, 1, H, 508, 0.02f));
    /* this rank's experts, in ascending order, and expert_local[512] */
    int local[E], n_local = 0;
    for (int e = 0; e < E; e++) local[e] = e % ranks == rank ? n_local++ : -1;
    void *lgate = qg_alloc(n_local * g_exp), *lup = qg_alloc(n_local * g_exp), *ldown = qg_alloc(n_local * d_exp);
    int *dlocal = qg_alloc(sizeof(local));
    if (!lgate || !lup || !ldown || !dlocal) return 1;
    for (int e = 0; e < E; e++) {
        if (local[e] < 0) continue;
        CHECK(qg_copy((char *)lgate + local[e] * g_exp, (char *)gate + e * g_exp, g_exp));
        CHECK(qg_copy((char *)lup + local[e] * g_exp, (char *)up + e * g_exp, g_exp));
        CHECK(qg_copy((char *)ldown + local[e] * d_exp, (char *)down + e * d_exp, d_exp));
    }
    CHECK(qg_write(dlocal, local, sizeof(local)));
    /* workspaces: this rank's, exported; the peers', mapped */
    size_t ep_bytes = 0, ws_bytes = 0;
    CHECK(qg_ep_workspace_bytes(TMAX, H, F, &ep_bytes));
    CHECK(qg_moe_workspace_bytes(TMAX, H, F, &ws_bytes));
    void *ews = qg_alloc(ep_bytes), *ws = qg_alloc(ws_bytes);
    if (!ews || !ws) return 1;
    CHECK(qg_zero(ews, ep_bytes));
    CHECK(qg_zero(ws, ws_bytes));
    CHECK(qg_sync());
    CHECK(qg_ep_ipc_handle(ews, s->handles[rank]));
    if (barrier(s, ranks, 1)) return 1;
    void *peers[MAXR];
    for (int p = 0; p < ranks; p++) {
        if (p == rank) peers[p] = ews;
        else CHECK(qg_ep_ipc_open(s->handles[p], &peers[p]));
    }
    const int sizes[3] = {17, 5, 17};
    float *x = qg_alloc(TMAX * H * 4), *out = qg_alloc(TMAX * H * 4), *ref = qg_alloc(TMAX * H * 4);
    int *ids = qg_alloc(TMAX * 10 * 4), *rids = qg_alloc(TMAX * 10 * 4);
    static float ho[TMAX * H], hr[TMAX * H];
    static int hi[TMAX * 10], hri[TMAX * 10];
    int failed = 0;
    for (int call = 0; call < 3; call++) {
        const int T = sizes[call];
        CHECK(qg_synth_normal(x, (size_t)T * H, 600 + call, 1.0f));
        CHECK(qg_moe_layer(ref, rids, NULL, x, T, router, NULL, gate, Q4K, up, Q4K, down, Q4K, sg, Q4K, su, Q4K,
                           sd, Q4K, sr, H, F, ws));
        CHECK(qg_moe_layer_ep(out, ids, NULL, x, T, router, NULL, lgate, Q4K, lup, Q4K, ldown, Q4K, n_local, dlocal,
                              sg, Q4K, su, Q4K, sd, Q4K, sr, call % ranks, H, F, rank, ranks, (void *const *)peers));
        CHECK(qg_read(ho, out, (size_t)T * H * 4));
        CHECK(qg_read(hr, ref, (size_t)T * H * 4));
        CHECK(qg_read(hi, ids, (size_t)T * 40));
        CHECK(qg_read(hri, rids, (size_t)T * 40));
        double num = 0, den = 0, mx = 0, mref = 0;
        int finite = 1;
        for (int i = 0; i < T * H; i++) {
            const double d = (double)ho[i] - hr[i];
            num += d * d;
            den += (double)hr[i] * hr[i];
            if (fabs(d) > mx) mx = fabs(d);
            if (fabs(hr[i]) > mref) mref = fabs(hr[i]);
            finite &= isfinite(ho[i]);
        }
        const double rel = sqrt(num / den);
        const int same_ids = !memcmp(hi, hri, (size_t)T * 40);
        const int ok = finite && same_ids && rel <= 1e-5 && mx <= 1e-4 * mref;
        printf("rank %d call %d (T=%d): ids %s, rel-L2 %.2e, max-abs %.2e (bound %.2e) %s\n", rank, call, T,
               same_ids ? "bit-exact" : "DIFFER", rel, mx, 1e-4 * mref, ok ? "ok" : "FAIL");
        failed |= !ok;
    }
    int inv = 0, sel = 0, used = 0;
    CHECK(qg_moe_status(ews, &inv, &sel, &used));
    if (barrier(s, ranks, 2)) return 1; /* every rank done before any unmaps */
    for (int p = 0; p < ranks; p++)
        if (p != rank) CHECK(qg_ep_ipc_close(peers[p]));
    if (barrier(s, ranks, 3)) return 1; /* unmapped everywhere before any frees */
    return failed;
}

int main(int argc, char **argv) {
    const int ranks = argc > 1 ? atoi(argv[1]) : 2;
    if (ranks < 1 || ranks > MAXR) return 2;
    shared_state *s = mmap(NULL, sizeof(shared_state), PROT_READ | PROT_WRITE, MAP_SHARED | MAP_ANONYMOUS, -1, 0);
    if (s == MAP_FAILED) return 2;
    memset(s, 0, sizeof(*s));
    pid_t pids[MAXR];
    for (int r = 0; r < ranks; r++) {
        pids[r] = fork(); /* before any CUDA call in this process */
        if (pids[r] < 0) return 2;
        if (pids[r] == 0) {
            const int rc = run_rank(s, r, ranks);
            fflush(stdout);
            _exit(rc);
        }
    }
    int failed = 0;
    for (int r = 0; r < ranks; r++) {
        int status = 0;
        waitpid(pids[r], &status, 0);
        failed |= !WIFEXITED(status) || WEXITSTATUS(status) != 0;
    }
    printf("%s\n", failed ? "FAILED" : "all ranks passed");
    return failed;
}
