/* GPU test entry into the all-resident MoE drop-in, built into
 * libqwen_moe_probe.so by nebula_b200/integration/build.py --harness.
 *
 * It includes the patched qwen.c (moe() replaced by
 * nebula_b200/integration/qwen_moe.c), opens one target layer through the
 * reference's own diagnostic loader (qwen_probe_layer_open: index parsing,
 * tensor binding, device upload, host expert copies; qwen/qwen.c:429-433) and
 * runs moe() alone on the given activations, twice in a row (the second call
 * reuses the experts made resident by the first). Only moe() and the
 * hyper-connection write after it run on the device; the layer's attention
 * is not executed. */
#include "qwen.c"

/* x [2][nt][2560] -> moeout [2][nt][2560], ids / weights [2][nt][10]. */
int nebula_probe_moe(const char *index_path, int il, int nt, const float *x, float *moeout, int *ids, float *weights,
                     double *upload_bytes) {
    qwen_model *m = qwen_probe_layer_open(index_path, il, nt);
    if (!m) return -1;
    layer *l = &m->layers[il];
    int rc = 0;
    for (int call = 0; call < 2 && !rc; call++) {
        const size_t off = (size_t)call * nt;
        if (qg_write(m->x, x + off * D, (size_t)nt * D * 4) || qg_zero(m->inject, (size_t)nt * 4 * 4) ||
            qg_zero(m->h, (size_t)nt * HD * 4)) {
            rc = fail("probe: input upload");
            break;
        }
        if ((rc = moe(m, l, nt, 0))) break;
        if (qg_read(moeout + off * D, m->moeout, (size_t)nt * D * 4) ||
            qg_read(ids + off * 10, m->route_ids, (size_t)nt * 10 * 4) ||
            qg_read(weights + off * 10, m->route_weights, (size_t)nt * 10 * 4))
            rc = fail("probe: result read");
    }
    if (upload_bytes) {
        *upload_bytes = 0;
        for (int k = 0; k < 3; k++)
            if (nebula_moe_state.experts[il][k]) *upload_bytes += (double)(k == 0 ? l->eg : k == 1 ? l->eu : l->ed)->bytes;
    }
    qwen_close(m);
    return rc;
}
