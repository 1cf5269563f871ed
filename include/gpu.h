#ifndef NEBULA_B200_GPU_H
#define NEBULA_B200_GPU_H
/* B200-native (sm_100a) routed-MoE operators behind Nebula's C ABI.
 *
 * Every declaration in the first part keeps the exact name, signature and
 * semantics of the reference header qwen/gpu.h (line numbers cited per entry)
 * so that qwen/qwen.c and the ctypes layers bind this library unchanged for
 * the MoE path. The second part appends new entry points; nothing existing
 * changed to make room for them.
 *
 * Conventions (qwen/gpu.h:4-10, qwen/gpu.cu:10,36-46):
 *  - int results are cudaError_t codes, 0 = success; argument validation
 *    happens before any launch and returns cudaErrorInvalidValue (1).
 *  - Device arrays are token-major. The caller allocates and owns every
 *    device buffer; the library allocates only its own objects (graphs,
 *    upload slabs, expert-parallel contexts).
 *  - Asynchronous work goes to the calling thread's capture stream: the
 *    legacy default stream normally, the capture stream between
 *    qg_graph_begin and qg_graph_end. qg_write/qg_read are synchronous.
 *  - Graphs contain only fixed-shape device work, never host routing
 *    decisions. A capture must be ended or aborted before any host
 *    transfer/synchronisation.
 */
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime (qwen/gpu.h:11-21,24,30-31) ---------------------------- */
void *qg_alloc(size_t bytes);                                   /* gpu.h:11 */
void qg_free(void *p);                                          /* gpu.h:12 */
int qg_write(void *dst, const void *src, size_t bytes);         /* gpu.h:13 */
int qg_read(void *dst, const void *src, size_t bytes);          /* gpu.h:14 */
int qg_copy(void *dst, const void *src, size_t bytes);          /* gpu.h:15 */
int qg_zero(void *dst, size_t bytes);                           /* gpu.h:16 */
int qg_sync(void);                                              /* gpu.h:17 */
int qg_graph_begin(void **graph);                               /* gpu.h:18 */
int qg_graph_end(void *graph);                                  /* gpu.h:19 */
int qg_graph_launch(void *graph);                               /* gpu.h:20 */
void qg_graph_destroy(void *graph);                             /* gpu.h:21 */
int qg_memory(size_t *free_bytes, size_t *total_bytes);         /* gpu.h:24 */
const char *qg_error(int error);                                /* gpu.h:30 */
/* GGML types: 0 F32, 1 F16, 30 BF16, 2 Q4_0, 6 Q5_0, 7 Q5_1, 8 Q8_0,
 * 12 Q4_K, 13 Q5_K, 14 Q6_K, 20 IQ4_NL. dims[0] is the row length. */
int qg_tensor_bytes(int type, const uint64_t dims[4], uint64_t *bytes); /* gpu.h:31 */

/* ---- expert uploads (qwen/gpu.h:32-36) ------------------------------ */
/* Two pinned slabs of expert_bytes each; packs gate|up|down contiguously into
 * dst on the legacy default stream. With every expert resident this becomes
 * the init-time bulk loader. */
void *qg_upload_create(size_t expert_bytes);                    /* gpu.h:32 */
void qg_upload_destroy(void *uploader);                         /* gpu.h:33 */
int qg_upload_expert(void *uploader, void *dst, const void *gate, size_t gate_bytes,
                     const void *up, size_t up_bytes, const void *down, size_t down_bytes); /* gpu.h:34-35 */
double qg_upload_seconds(void *uploader);                       /* gpu.h:36 */

/* ---- dense projections (qwen/gpu.h:37-38,42-43,77-78) --------------- */
/* out[t][row] = sum_k W[row][k]*x[t][k]; tokens <= 8192. Types 0, 12 and 20
 * keep the reference's 32-lane accumulation order (lane j owns k = j mod 32,
 * increasing k, then a 16/8/4/2/1 tree), so results are bitwise equal to
 * qc_matmul in qwen/cpu.c:119-148 and to the reference kernels. */
int qg_matmul(float *out, const void *w, int type, int rows, int cols,
              const float *x, int tokens);                      /* gpu.h:37-38 */
int qg_gather(float *out, const void *w, int type, int cols, int row); /* gpu.h:39 */
/* op 0: SiLU(x*scale), op 1: sigmoid(x*scale), otherwise x*scale. */
int qg_unary(float *out, const float *x, int count, int op, float scale); /* gpu.h:42 */
/* op 0: a+b, otherwise a*b. */
int qg_binary(float *out, const float *a, const float *b, int count, int op); /* gpu.h:43 */
int qg_dequant(float *out, const void *packed, int type, int rows, int cols); /* gpu.h:77 */
/* out[t][d] += shared[t][d]*sigmoid(gate[t]), width 2560. */
int qg_shared_add(float *out, const float *shared, const float *gate, int tokens); /* gpu.h:78 */

/* ---- routing and the per-expert MoE primitives (qwen/gpu.h:62-76) --- */
/* logits [t][512] -> ids [t][10] (rank order), weights [t][10]. A token with
 * any non-finite logit gets ids -1 and weights 0. Ties pick the lowest id. */
int qg_route(int *ids, float *weights, const float *logits, int tokens); /* gpu.h:62 */
typedef struct {
    uint64_t token_layers, missing_selections, skipped_selections, avoided_token_handoffs;
    double skipped_mass;
} qg_prune_stats;                                               /* gpu.h:63-66 */
/* Routes to non-resident experts whose total mass is below threshold
 * (0 < threshold <= 0.1) become -e-2 with weight 0, without renormalising. */
int qg_prune_routes(int *ids, float *weights, const unsigned char *resident,
                    int tokens, double threshold, qg_prune_stats *stats); /* gpu.h:67-68 */
/* map [512][tokens]: ascending token list per expert. */
int qg_moe_map(int *map, const int *ids, int tokens);           /* gpu.h:69 */
int qg_moe_gather(float *out, const float *x, const int *token_map, int selected_tokens); /* gpu.h:70 */
int qg_moe_scatter(float *slots, const float *expert, const float *weights, const int *ids,
                   const int *token_map, int expert_id, int selected_tokens); /* gpu.h:71-72 */
int qg_moe_reduce(float *out, const float *slots, int tokens);  /* gpu.h:73 */
/* Resident-expert MoE without host routing for tokens <= 17 at hidden 2560 /
 * ffn 640: mid [t][10][640], slots [t][10][2560] (weighted, unreduced).
 * Invalid ids give NaN rows. */
int qg_mtp_moe(float *slots, float *mid, const float *x, const int *ids, const float *weights,
               const void *gate, int gate_type, const void *up, int up_type,
               const void *down, int down_type, int tokens);    /* gpu.h:74-76 */

/* ===================================================================== *
 * Appended entry points (no counterpart in the reference header).       *
 * ===================================================================== */

/* Device workspace, in bytes, that qg_moe_routed / qg_moe_layer need for a
 * batch of up to `tokens` at the given shape. Replaces the per-layer host read of
 * route ids (qwen/qwen.c:649) and the per-expert launch loop
 * (qwen/qwen.c:680-698) with device-side grouping. Fill a new workspace with
 * zeros once (qg_zero): its counters start at zero and every call returns
 * them to zero for the next. Calls sharing a workspace must not overlap on
 * the device. After an error reported by qg_moe_status, zero it again. */
int qg_moe_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes);

/* All-resident routed MoE, one call per layer (replaces grouped_moe's GPU
 * branch, qwen/qwen.c:680-698, plus qg_moe_reduce, qwen/qwen.c:725):
 *   out[t] = sum_{k=0..9, rank order} weights[t][k] * E_{ids[t][k]}(x[t])
 *   E_e(x) = W_down[e] * (SiLU(W_gate[e] x) * (W_up[e] x))
 * Expert e's matrices sit at gate + e*ffn*row_bytes(gate_type, hidden) (rows
 * of `hidden` columns), likewise up, and down + e*hidden*row_bytes(down_type,
 * ffn) - the layout of ffn_{gate,up,down}_exps. gate/up/down types: 12 (Q4_K)
 * or 20 (IQ4_NL); gate and up share a type. Omitted routes (-e-2 with
 * weight 0, from qg_prune_routes) contribute +0. A token whose routes are
 * invalid (id -1, out-of-range id, duplicate id, negative or non-finite
 * weight) gets a NaN output row and is counted in qg_moe_status. No host
 * synchronisation; graph-capturable; tokens <= 8192; deterministic. */
int qg_moe_routed(float *out, const float *x, const int *ids, const float *weights, int tokens,
                  const void *gate, int gate_type, const void *up, int up_type,
                  const void *down, int down_type, int hidden, int ffn, void *workspace);

/* qg_moe_routed without a caller workspace (no counterpart in the reference):
 * for callers that cannot allocate device memory where they call, e.g. a
 * runtime whose device memory another allocator reserves in full up front.
 * The library keeps one static 8 MiB scratch per device: batches of up to 28
 * tokens at hidden 2048 / ffn 512 and up to 23 at 2560 / 640 fit (verify
 * batches of up to 17 fit both); shapes whose qg_moe_workspace_bytes exceed
 * it return cudaErrorInvalidValue before anything is launched. Nothing is
 * allocated. The first call on a device looks the scratch up and zeroes it
 * (and synchronises), so make it before any stream capture. Calls share the
 * scratch: calls that overlap on the device (other streams, other host
 * threads) race. There is no status readout: a call that finds the previous
 * call's bounded-wait timeout recorded in the scratch clears its counters
 * before running (the failed call's rows are not repaired); invalid routes
 * give NaN rows. cudaDeviceReset after using this entry point is not
 * supported. */
int qg_moe_routed_static(float *out, const float *x, const int *ids, const float *weights, int tokens,
                         const void *gate, int gate_type, const void *up, int up_type,
                         const void *down, int down_type, int hidden, int ffn);

/* One whole MoE layer (qwen/qwen.c:714-735): router GEMV against the F32
 * router [512][hidden] with the reference lane order (so ids are bit-exact),
 * plus logit_bias[512] when non-NULL (a per-expert routing bias; the
 * reference model has none, pass NULL), top-10 routing (qg_route
 * semantics), the routed experts as qg_moe_routed, and - when shared_gate is
 * non-NULL - the shared expert with its F32 [hidden] gate:
 * out[t] += shared(x[t]) * sigmoid(s_router . x[t]) (qwen/qwen.c:708-713).
 * The shared expert uses the routed experts' formats. ids_out/weights_out
 * (optional) receive the routing. */
int qg_moe_layer(float *out, int *ids_out, float *weights_out, const float *x, int tokens,
                 const float *router, const float *logit_bias,
                 const void *gate, int gate_type, const void *up, int up_type,
                 const void *down, int down_type,
                 const void *shared_gate, int shared_gate_type,
                 const void *shared_up, int shared_up_type,
                 const void *shared_down, int shared_down_type,
                 const float *shared_router, int hidden, int ffn, void *workspace);

/* Expert parallelism across the GPUs of one box (no counterpart in the
 * reference, which runs on one GPU): one process per GPU, every rank calls
 * qg_moe_layer_ep for the same tokens and layer. A workspace sized by
 * qg_ep_workspace_bytes for the largest batch serves every smaller batch, in
 * any order (verify batches change size from step to step): the state kept
 * between calls and the rows peers write sit at offsets independent of the
 * call's token count. Each rank holds n_local
 * experts (gate/up/down as for qg_moe_layer, n_local of them) and
 * expert_local[512] (device) gives each expert's index there, or -1 when
 * another rank holds it; one rank (shared_rank) computes the shared expert.
 * The router is replicated, so every rank derives the same ids; each rank
 * computes its experts' weighted rows and stores them into every rank's
 * workspace over NVLink, then every rank reduces all rows in router-rank
 * order. ids are bitwise those of qg_moe_layer; `out` matches it within the
 * float tolerance of the path (gate/up tiles are split along K across SMs
 * when each rank holds few experts, and the parts are added in fixed order).
 * workspaces[r] is rank r's workspace (qg_ep_workspace_bytes, zero-filled
 * once, allocated with qg_alloc) as seen from this process: this rank's own
 * pointer and the others mapped with qg_ep_ipc_open from the 64-byte handles
 * each rank exports with qg_ep_ipc_handle. Calls go in the same order on
 * every rank; a rank that stops makes the others' combines time out after
 * 2 s (error bit 8: qg_moe_status returns cudaErrorLaunchTimeout) with NaN
 * output rows instead of hanging; every rank then zeroes its workspace
 * before the next call. Q4_K gate/up with Q4_K or IQ4_NL down (the shared
 * expert in the same formats).
 * Large batches (tokens > 32): rank r owns tokens [r*B, (r+1)*B) with
 * B = ceil(tokens / ranks); each rank computes the router logits and top-10
 * of its own tokens and sends their ids and weights to every rank (ids_out
 * and weights_out receive all tokens on every rank), computes the shared
 * expert for its own tokens (shared_rank is not used), stores each weighted
 * row only into the owning rank's workspace, and writes only its own rows of
 * `out`. */
int qg_ep_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes);
int qg_ep_ipc_handle(void *workspace, void *handle);
int qg_ep_ipc_open(const void *handle, void **ptr);
int qg_ep_ipc_close(void *ptr);
int qg_moe_layer_ep(float *out, int *ids_out, float *weights_out, const float *x, int tokens,
                    const float *router, const float *logit_bias,
                    const void *gate, int gate_type, const void *up, int up_type,
                    const void *down, int down_type, int n_local, const int *expert_local,
                    const void *shared_gate, int shared_gate_type,
                    const void *shared_up, int shared_up_type,
                    const void *shared_down, int shared_down_type,
                    const float *shared_router, int shared_rank, int hidden, int ffn,
                    int rank, int ranks, void *const *workspaces);

/* Reads the status words the last MoE call left in `workspace`:
 * invalid_tokens = tokens given NaN rows, selected = (token, expert) pairs
 * computed, experts = distinct experts used. Synchronises the device. */
int qg_moe_status(const void *workspace, int *invalid_tokens, int *selected, int *experts);

/* Per-phase CUDA-event timing of the MoE entry points, for profiling.
 * qg_moe_profile(1) clears earlier records and starts recording events
 * around every eager launch on the legacy default stream (graph captures
 * are never timed); qg_moe_profile(0) stops. qg_moe_profile_read sums the
 * recorded durations of one phase - 0 router GEMV, 1 top-10, 2 plan,
 * 3 gate/up, 4 down, 5 combine, 6 fused expert kernel (gate/up, down and
 * combine in one launch), 7 fused router/top-10/plan kernel of the decode
 * path, 8 the single-kernel layer of small batches (1 or 2 tokens at
 * hidden 2048 / ffn 512, 1 to 4 at 2560 / 640) - and
 * synchronises the device. While profiling, the decode path's
 * two kernels run without programmatic overlap. */
int qg_moe_profile(int enable);
int qg_moe_profile_read(int phase, double *total_ms, int *launches);

/* ---- loading an all-resident model (no counterpart in the reference
 * header; the reference's loader is qwen/qwen.c:108-146,324-369) -------- */

/* Reads a COB_QWEN_INDEX_V1 weight index (the format and checks of
 * qwen/qwen.c:108-146) and maps its weight files read-only. Returns
 * cudaErrorFileNotFound for a missing index or weights file (or one of the
 * wrong size) and cudaErrorInvalidValue for a malformed index; `message`
 * (optional) receives a description. Host only. */
int qg_index_open(const char *path, void **index, char *message, size_t message_bytes);
void qg_index_close(void *index);
/* A tensor of the index by name (e.g. "blk.12.ffn_gate_exps.weight"): its
 * bytes in the mapped file, GGML type, dims (dims[0] = row length) and size.
 * cudaErrorInvalidValue when absent. */
int qg_index_tensor(const void *index, const char *name, const void **host, int *type, uint64_t dims[4],
                    uint64_t *bytes);
/* Bulk upload of whole experts of one matrix: expert experts[i] (or i when
 * experts is NULL), expert_bytes long at src + experts[i]*expert_bytes,
 * lands at dst + i*expert_bytes. Loads all 512 experts of a layer, or one
 * rank's experts under expert parallelism, through the uploader's pinned
 * blocks (expert_bytes <= the size given to qg_upload_create) on the legacy
 * default stream; returns once the last copy is queued. */
int qg_upload_experts(void *uploader, void *dst, const void *src, size_t expert_bytes, const int *experts,
                      int count);

/* QROUTE1 route traces (written by the reference's route profiler,
 * qwen/qwen.c:87-94,638-646): qg_route_trace_next reads the next record -
 * layer, target position, tokens, ids [tokens][10], weights [tokens][10] -
 * into caller buffers of `capacity` tokens; *tokens = 0 at the end of the
 * file; cudaErrorInvalidValue for a truncated record or more tokens than the
 * capacity (or 8192). Host only. */
int qg_route_trace_open(const char *path, void **trace);
int qg_route_trace_next(void *trace, int *layer, int *position, int *tokens, int *ids, float *weights,
                        int capacity);
void qg_route_trace_close(void *trace);

/* Synthetic weights for tests and benchmarks: rows x cols values drawn
 * N(0, stddev) from a counter-based generator keyed by seed, quantised on the
 * device to type 0, 12 (Q4_K) or 20 (IQ4_NL) with this library's own
 * quantiser (round-to-nearest block scales; not llama.cpp's search). */
int qg_synth_weights(void *dst, int type, int rows, int cols, uint64_t seed, float stddev);
/* x [count] fp32 N(0, stddev) from the same generator. */
int qg_synth_normal(float *dst, size_t count, uint64_t seed, float stddev);

#ifdef __cplusplus
}
#endif
#endif
