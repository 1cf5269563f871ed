/* TEST INFRASTRUCTURE ONLY - the CPU checker for the routed-MoE path.
 *
 * Plain-C restatements of the reference's device-side routing steps, which
 * have no CPU implementation in the reference tree. The expert arithmetic
 * itself (qc_matmul / qc_moe) is not restated: the checker links the
 * reference's own qwen/cpu.c, compiled unmodified into oracle/_ref.
 *
 * Nothing in the product library links or calls this file. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Every function cites the reference lines it follows (paths relative to the
 * reference project root). Loops run in the reference's own order so that
 * integer outputs (ids, maps, counters) are bit-exact; floating-point results
 * use the host libm expf where the reference uses CUDA's expf (<=2 ulp apart).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { OR_EXPERTS = 512, OR_TOP = 10 };

/* qwen/gpu.cu:456-465 (route_kernel). Per token: any non-finite logit gives
 * ids=-1 and weights=0 for all ten slots. Otherwise ten argmax passes with a
 * strict '>' (lowest index wins ties), w_k = expf(s_k - max over all 512),
 * summed k=0..9 in order and divided by that sum. */
int or_route(int *ids, float *weights, const float *logits, int nt) {
    if (!ids || !weights || !logits || nt < 1) return -1;
    for (int t = 0; t < nt; t++) {
        float scores[OR_EXPERTS];
        memcpy(scores, logits + (size_t)t * OR_EXPERTS, sizeof(scores));
        int bad = 0;
        float largest = -INFINITY;
        for (int j = 0; j < OR_EXPERTS; j++) {
            if (!isfinite(scores[j])) { bad = 1; break; }
            largest = fmaxf(largest, scores[j]);
        }
        if (bad) {
            for (int k = 0; k < OR_TOP; k++) { ids[t * OR_TOP + k] = -1; weights[t * OR_TOP + k] = 0; }
            continue;
        }
        float total = 0;
        for (int k = 0; k < OR_TOP; k++) {
            int best = 0;
            for (int j = 1; j < OR_EXPERTS; j++) if (scores[j] > scores[best]) best = j;
            ids[t * OR_TOP + k] = best;
            weights[t * OR_TOP + k] = expf(scores[best] - largest);
            total += weights[t * OR_TOP + k];
            scores[best] = -INFINITY;
        }
        for (int k = 0; k < OR_TOP; k++) weights[t * OR_TOP + k] /= total;
    }
    return 0;
}

/* qwen/gpu.h:63-66 counter block, qwen/gpu.cu:467-483 (prune_routes_kernel).
 * A token whose ten ids are not all in [0,512) is left untouched and not
 * counted. Otherwise count it, count its missing selections, and when
 * 0 < mass(missing) < threshold rewrite each missing id e to -e-2 with weight
 * 0 (no renormalisation). Mass is accumulated in double in slot order. The
 * device version adds skipped_mass with atomics in an unspecified token order;
 * this restatement adds in token order. */
typedef struct {
    uint64_t token_layers, missing_selections, skipped_selections, avoided_token_handoffs;
    double skipped_mass;
} or_prune_stats;

int or_prune(int *ids, float *weights, const unsigned char *resident, int nt,
             double threshold, or_prune_stats *stats) {
    /* qwen/gpu.cu:486 argument checks. */
    if (nt < 1 || nt > 8192 || threshold < 0 || threshold > 0.1 || !isfinite(threshold)) return -1;
    for (int t = 0; t < nt; t++) {
        int missing = 0, valid = 1;
        double mass = 0;
        for (int k = 0; k < OR_TOP; k++) {
            int e = ids[t * OR_TOP + k];
            if (e < 0 || e >= OR_EXPERTS) { valid = 0; break; }
            if (!resident[e]) { missing++; mass += (double)weights[t * OR_TOP + k]; }
        }
        if (!valid) continue;
        stats->token_layers += 1;
        stats->missing_selections += (uint64_t)missing;
        if (missing && threshold > 0 && mass < threshold) {
            for (int k = 0; k < OR_TOP; k++) {
                int e = ids[t * OR_TOP + k];
                if (!resident[e]) { ids[t * OR_TOP + k] = -e - 2; weights[t * OR_TOP + k] = 0; }
            }
            stats->skipped_selections += (uint64_t)missing;
            stats->avoided_token_handoffs += 1;
            stats->skipped_mass += mass;
        }
    }
    return 0;
}

/* qwen/gpu.cu:489-505 (moe_map_kernel): for each expert e, map[e*nt + i] is
 * the i-th token (ascending) whose ten ids contain e. Entries past the
 * expert's count are left as they were. counts (optional) receives the count. */
int or_moe_map(int *map, int *counts, const int *ids, int nt) {
    if (!map || !ids || nt < 1 || nt > 8192) return -1;
    for (int e = 0; e < OR_EXPERTS; e++) {
        int n = 0;
        for (int t = 0; t < nt; t++) {
            int selected = 0;
            for (int k = 0; k < OR_TOP; k++) selected |= ids[t * OR_TOP + k] == e;
            if (selected) map[(size_t)e * nt + n++] = t;
        }
        if (counts) counts[e] = n;
    }
    return 0;
}

static float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

/* SwiGLU of the shared expert: qwen/qwen.c:709-710 runs qg_unary op 0 with
 * scale 1 (qwen/gpu.cu:215-216: a = x*1, a*sig(a)) then qg_binary op 1
 * (multiply). The routed path uses the same expression (qwen/cpu.c:216). */
void or_swiglu(float *mid, const float *gate, const float *up, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float a = gate[i] * 1.0f;
        mid[i] = (a * sigmoid(a)) * up[i];
    }
}

/* qwen/gpu.cu:552 (shared_add_kernel): out[t][d] += shared[t][d] *
 * sigmoid(gate[t]). nvcc contracts the multiply-add into one fused
 * operation, so the restatement uses fmaf. */
void or_shared_add(float *out, const float *shared, const float *gate, int nt, int width) {
    for (int t = 0; t < nt; t++) {
        float s = sigmoid(gate[t]);
        for (int d = 0; d < width; d++)
            out[(size_t)t * width + d] = fmaf(shared[(size_t)t * width + d], s, out[(size_t)t * width + d]);
    }
}

/* qwen/gpu.cu:521-524 (moe_reduce_kernel) and qwen/cpu.c:227-231: the
 * rank-order combine, out[t][d] = sum_{k=0..9} slots[t][k][d] from 0.0f. */
void or_moe_reduce(float *out, const float *slots, int nt, int width) {
    for (int t = 0; t < nt; t++)
        for (int d = 0; d < width; d++) {
            float sum = 0;
            for (int k = 0; k < OR_TOP; k++) sum += slots[((size_t)t * OR_TOP + k) * width + d];
            out[(size_t)t * width + d] = sum;
        }
}
