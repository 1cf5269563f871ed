/* All-resident routed MoE for the reference model runtime: the drop-in for
 * moe() in qwen/qwen.c:714-735.
 *
 * nebula_b200/integration/build.py compiles this file inside qwen.c's own
 * translation unit (it needs the model and layer structs there): the
 * reference's moe() is renamed moe_reference() and this file takes its place,
 * and qwen_close() is wrapped so the device copies made here are released.
 * Everything else in qwen.c is unchanged.
 *
 * Per layer call, instead of the router GEMV, qg_route, grouped_moe's host
 * read of the route ids (qwen/qwen.c:649), its per-expert launch loop
 * (qwen/qwen.c:680-698) or CPU hand-off, qg_moe_reduce and shared_direct
 * (qwen/qwen.c:708-713), one qg_moe_layer call computes on the device the
 * router GEMV (bit-exact with qg_matmul, so the ids are the reference's),
 * top-10, every routed expert with the router-rank-order combine and the
 * sigmoid-gated shared expert into m->moeout, with the routing in
 * m->route_ids / m->route_weights; qg_hc_write then adds it into the residual
 * stream exactly as shared_direct ends. Nothing is read back to the host
 * unless a route profile is being recorded (qwen_profile_routes), in which
 * case the QROUTE1 record is written as grouped_moe writes it.
 *
 * Residency: the first call for a layer copies its 512 experts (gate, up and
 * down, from the host copies the loader keeps, qwen/qwen.c:214-247) into
 * device memory with qg_upload_experts and keeps them there; a layer whose
 * expert tensors are already on the device (the MTP layer) is used in place.
 * The MoE workspace is allocated once, for the model's batch capacity. Host
 * copies on SSD (partial RAM storage) are not supported here: every expert
 * must be in host RAM at load time.
 */

/* Entry points this library appends to the qwen/gpu.h ABI (declared in
 * include/gpu.h, which cannot be included next to qwen/gpu.h: both define
 * qg_prune_stats). */
int qg_moe_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes);
int qg_moe_layer(float *out, int *ids_out, float *weights_out, const float *x, int tokens, const float *router,
                 const float *logit_bias, const void *gate, int gate_type, const void *up, int up_type,
                 const void *down, int down_type, const void *shared_gate, int shared_gate_type,
                 const void *shared_up, int shared_up_type, const void *shared_down, int shared_down_type,
                 const float *shared_router, int hidden, int ffn, void *workspace);
int qg_upload_experts(void *uploader, void *dst, const void *src, size_t expert_bytes, const int *experts,
                      int count);

static int moe_reference(qwen_model *m, layer *l, int nt, int mtp) __attribute__((unused));

enum { NEBULA_STAGE_BYTES = 16 << 20 };

static struct {
    qwen_model *model;           /* the model the state below belongs to */
    void *experts[NL + 1][3];    /* device gate / up / down copies made here */
    void *workspace;
    size_t workspace_bytes;
    void *uploader;
} nebula_moe_state;

static void nebula_moe_release(qwen_model *m) {
    if (!m || nebula_moe_state.model != m) return;
    qg_sync();
    for (int il = 0; il <= NL; il++)
        for (int k = 0; k < 3; k++) qg_free(nebula_moe_state.experts[il][k]);
    qg_free(nebula_moe_state.workspace);
    qg_upload_destroy(nebula_moe_state.uploader);
    memset(&nebula_moe_state, 0, sizeof(nebula_moe_state));
}

/* Device addresses of a layer's gate / up / down experts, uploading them on first use. */
static int nebula_resident_experts(qwen_model *m, layer *l, const void *dev[3]) {
    tensor *ts[3] = {l->eg, l->eu, l->ed};
    const int il = (int)(l - m->layers);
    if (nebula_moe_state.model != m) {
        nebula_moe_release(nebula_moe_state.model);
        nebula_moe_state.model = m;
    }
    for (int k = 0; k < 3; k++) {
        if (ts[k]->device) {
            dev[k] = ts[k]->device;
            continue;
        }
        void **copy = &nebula_moe_state.experts[il][k];
        if (!*copy) {
            if (!ts[k]->host) return fail("all-resident MoE: %s has no host copy", ts[k]->name);
            if (!nebula_moe_state.uploader && !(nebula_moe_state.uploader = qg_upload_create(NEBULA_STAGE_BYTES)))
                return fail("all-resident MoE: pinned staging allocation");
            const uint64_t per_expert = ts[k]->bytes / 512;
            if (per_expert > NEBULA_STAGE_BYTES) return fail("all-resident MoE: expert larger than a staging block");
            if (!(*copy = qg_alloc(ts[k]->bytes))) return fail("all-resident MoE: device copy of %s", ts[k]->name);
            GPU(qg_upload_experts(nebula_moe_state.uploader, *copy, ts[k]->host, per_expert, NULL, 512));
            GPU(qg_sync());
        }
        dev[k] = *copy;
    }
    return 0;
}

static int nebula_moe_workspace(qwen_model *m, int ffn, void **ws) {
    size_t need = 0;
    GPU(qg_moe_workspace_bytes(m->batch_capacity, D, ffn, &need));
    if (nebula_moe_state.workspace_bytes < need) {
        qg_free(nebula_moe_state.workspace);
        nebula_moe_state.workspace_bytes = 0;
        if (!(nebula_moe_state.workspace = qg_alloc(need))) return fail("all-resident MoE workspace allocation");
        GPU(qg_zero(nebula_moe_state.workspace, need));
        nebula_moe_state.workspace_bytes = need;
    }
    *ws = nebula_moe_state.workspace;
    return 0;
}

/* The QROUTE1 record grouped_moe writes while a route profile is open (qwen/qwen.c:638-646). */
static int nebula_profile_routes(qwen_model *m, layer *l, int nt) {
    static int ids[NT * 10];
    static float weights[NT * 10];
    const size_t n = (size_t)nt * 10;
    GPU(qg_read(ids, m->route_ids, n * sizeof(int)));
    GPU(qg_read(weights, m->route_weights, n * sizeof(float)));
    const uint32_t header[3] = {(uint32_t)(l - m->layers), (uint32_t)m->target_pos, (uint32_t)nt};
    if (fwrite(header, sizeof(uint32_t), 3, m->route_profile) != 3 || fwrite(ids, sizeof(int), n, m->route_profile) != n ||
        fwrite(weights, sizeof(float), n, m->route_profile) != n)
        return fail("write route profile");
    return 0;
}

static int moe(qwen_model *m, layer *l, int nt, int mtp) {
    m->cpu_reduced = 0;
    if (!l->router || l->router->type != 0 || !l->router->device || !l->sg || !l->su || !l->sd || !l->sr ||
        !l->sg->device || !l->su->device || !l->sd->device || !l->sr->device || l->sr->type != 0)
        return fail("all-resident MoE: layer %d lacks an F32 router or the shared expert on the device",
                    (int)(l - m->layers));
    if (m->ssd) return fail("all-resident MoE needs every expert in host RAM at load time");
    const int ffn = (int)l->eg->dim[1];
    const void *dev[3];
    void *ws = NULL;
    RUN(nebula_resident_experts(m, l, dev));
    RUN(nebula_moe_workspace(m, ffn, &ws));
    GPU(qg_moe_layer(m->moeout, m->route_ids, m->route_weights, m->x, nt, l->router->device, NULL, dev[0],
                     l->eg->type, dev[1], l->eu->type, dev[2], l->ed->type, l->sg->device, l->sg->type,
                     l->su->device, l->su->type, l->sd->device, l->sd->type, l->sr->device, D, ffn, ws));
    if (!mtp && m->route_profile) RUN(nebula_profile_routes(m, l, nt));
    GPU(qg_hc_write(m->h, m->moeout, m->inject, D, nt));
    return 0;
}
