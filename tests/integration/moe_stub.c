/* The all-resident MoE drop-in inside the reference runtime, with inert GPU
 * stand-ins (the pattern of the reference's qwen/test_handoffs.c): compiled
 * with the patched qwen.c (moe() replaced by nebula_b200/integration/qwen_moe.c)
 * and checked on the CPU.
 *
 * Checks: one moe() call makes exactly one qg_moe_layer call with the layer's
 * router, expert and shared-expert tensors, the model's activation, routing
 * and output buffers, hidden 2560 and the layer's FFN width; it adds the
 * result into the residual stream with qg_hc_write; it never reads anything
 * back to the host (no route-id read, unlike qwen/qwen.c:649); the first call
 * for a layer uploads its 512 experts once per matrix and later calls reuse
 * them; the workspace is sized for the batch capacity and allocated once; a
 * layer without an F32 router is refused; an open route profile gets the
 * QROUTE1 record; qwen_close releases the copies. */
#include "qwen.c"
#include <assert.h>

static int n_layer, n_hc, n_read, n_upload, n_alloc, n_free, n_zero;
static struct {
    float *out, *weights_out;
    int *ids_out;
    const float *x, *router;
    const void *gate, *up, *down, *sg, *su, *sd;
    const float *sr;
    int tokens, gt, ut, dt, sgt, sut, sdt, hidden, ffn;
    void *ws;
} last;
static int upload_count[4];
static size_t ws_tokens;

const char *qg_error(int code) { (void)code; return "stub"; }
int qg_read(void *dst, const void *src, size_t bytes) { memcpy(dst, src, bytes); n_read++; return 0; }
int qg_write(void *dst, const void *src, size_t bytes) { memcpy(dst, src, bytes); return 0; }
int qg_sync(void) { return 0; }
int qg_zero(void *dst, size_t bytes) { memset(dst, 0, bytes); n_zero++; return 0; }
void *qg_alloc(size_t bytes) { n_alloc++; return calloc(1, bytes ? bytes : 1); }
void qg_free(void *p) { if (p) n_free++; free(p); }
void *qg_upload_create(size_t bytes) { (void)bytes; return malloc(1); }
void qg_upload_destroy(void *u) { free(u); }
int qg_upload_experts(void *u, void *dst, const void *src, size_t eb, const int *experts, int count) {
    (void)u; assert(!experts && count == 512);
    memcpy(dst, src, eb * (size_t)count);
    upload_count[n_upload++ % 4] = count;
    return 0;
}
int qg_moe_workspace_bytes(int tokens, int hidden, int ffn, size_t *bytes) {
    ws_tokens = (size_t)tokens; *bytes = (size_t)tokens * hidden + ffn; return 0;
}
int qg_moe_layer(float *out, int *ids_out, float *weights_out, const float *x, int tokens, const float *router,
                 const float *bias, const void *gate, int gt, const void *up, int ut, const void *down, int dt,
                 const void *sg, int sgt, const void *su, int sut, const void *sd, int sdt, const float *sr,
                 int hidden, int ffn, void *ws) {
    assert(!bias);
    n_layer++;
    last.out = out; last.ids_out = ids_out; last.weights_out = weights_out; last.x = x; last.tokens = tokens;
    last.router = router; last.gate = gate; last.gt = gt; last.up = up; last.ut = ut; last.down = down; last.dt = dt;
    last.sg = sg; last.sgt = sgt; last.su = su; last.sut = sut; last.sd = sd; last.sdt = sdt; last.sr = sr;
    last.hidden = hidden; last.ffn = ffn; last.ws = ws;
    for (int i = 0; i < tokens * 10; i++) { ids_out[i] = i % 512; weights_out[i] = 0.1f; }
    return 0;
}
int qg_hc_write(float *residual, const float *x, const float *inject, int width, int tokens) {
    (void)residual; (void)inject; assert(x == last.out && width == D && tokens == last.tokens); n_hc++; return 0;
}

int main(void) {
    static qwen_model m;
    enum { FFN = 640 };
    static unsigned char gate_h[512 * 8], up_h[512 * 8], down_h[512 * 8];
    static float router_d[4], sr_d[4], x[17 * D], h[17 * HD], moeout[17 * D], rw[17 * 10], inject[17 * 4];
    static int rid[17 * 10];
    static unsigned char sg_d[8], su_d[8], sd_d[8];
    tensor eg = {.host = gate_h, .bytes = sizeof(gate_h), .type = 12, .dim = {D, FFN, 512, 1}};
    tensor eu = {.host = up_h, .bytes = sizeof(up_h), .type = 12, .dim = {D, FFN, 512, 1}};
    tensor ed = {.host = down_h, .bytes = sizeof(down_h), .type = 20, .dim = {FFN, D, 512, 1}};
    tensor router = {.device = router_d, .type = 0}, sr = {.device = sr_d, .type = 0};
    tensor sg = {.device = sg_d, .type = 12}, su = {.device = su_d, .type = 12}, sd = {.device = sd_d, .type = 20};
    for (int i = 0; i < (int)sizeof(gate_h); i++) { gate_h[i] = (unsigned char)i; up_h[i] = (unsigned char)(i * 3); }
    m.batch_capacity = 17; m.x = x; m.h = h; m.moeout = moeout; m.route_ids = rid; m.route_weights = rw;
    m.inject = inject;
    layer *l = &m.layers[12];
    l->router = &router; l->eg = &eg; l->eu = &eu; l->ed = &ed; l->sg = &sg; l->su = &su; l->sd = &sd; l->sr = &sr;

    assert(moe(&m, l, 17, 0) == 0);
    assert(n_layer == 1 && n_hc == 1 && n_read == 0 && n_upload == 3 && ws_tokens == 17);
    assert(last.out == moeout && last.ids_out == rid && last.weights_out == rw && last.x == x && last.tokens == 17);
    assert(last.router == router_d && last.sr == sr_d && last.sg == sg_d && last.su == su_d && last.sd == sd_d);
    assert(last.gt == 12 && last.ut == 12 && last.dt == 20 && last.sgt == 12 && last.sut == 12 && last.sdt == 20);
    assert(last.hidden == D && last.ffn == FFN && last.ws);
    assert(last.gate != gate_h && !memcmp(last.gate, gate_h, sizeof(gate_h)) && !memcmp(last.up, up_h, sizeof(up_h)));
    const void *resident_gate = last.gate, *ws = last.ws;
    const int allocs = n_alloc;

    assert(moe(&m, l, 5, 0) == 0); /* warm: no upload, no allocation, same copies */
    assert(n_layer == 2 && n_hc == 2 && n_read == 0 && n_upload == 3 && n_alloc == allocs);
    assert(last.gate == resident_gate && last.ws == ws && last.tokens == 5);

    layer *l2 = &m.layers[15]; /* a second layer gets its own copies */
    *l2 = *l;
    assert(moe(&m, l2, 17, 0) == 0 && n_upload == 6 && last.gate != resident_gate);

    tensor mtp_g = eg, mtp_u = eu, mtp_d = ed; /* experts already on the device are used in place */
    mtp_g.device = gate_h; mtp_u.device = up_h; mtp_d.device = down_h;
    layer *ln = &m.layers[NL];
    *ln = *l; ln->eg = &mtp_g; ln->eu = &mtp_u; ln->ed = &mtp_d;
    assert(moe(&m, ln, 3, 1) == 0 && n_upload == 6 && last.gate == gate_h && last.down == down_h);

    char path[] = "/tmp/nebula_moe_stub_routesXXXXXX";
    int fd = mkstemp(path);
    assert(fd >= 0);
    close(fd);
    m.route_profile = fopen(path, "wb");
    assert(m.route_profile && fwrite("QROUTE1\n", 1, 8, m.route_profile) == 8);
    m.target_pos = 40;
    assert(moe(&m, l, 2, 0) == 0 && n_read == 2);
    fclose(m.route_profile);
    m.route_profile = NULL;
    FILE *f = fopen(path, "rb");
    unsigned char blob[8 + 12 + 2 * 2 * 10 * 4];
    assert(fread(blob, 1, sizeof(blob), f) == sizeof(blob) && fgetc(f) == EOF);
    fclose(f);
    unlink(path);
    uint32_t head[3];
    memcpy(head, blob + 8, 12);
    assert(!memcmp(blob, "QROUTE1\n", 8) && head[0] == 12 && head[1] == 40 && head[2] == 2);

    tensor bad = router; /* a non-F32 router is refused */
    bad.type = 1;
    l->router = &bad;
    assert(moe(&m, l, 4, 0) == -1 && strstr(qwen_last_error(), "F32 router"));
    l->router = &router;

    const int frees = n_free;
    nebula_moe_release(&m); /* what qwen_close calls first */
    assert(n_free == frees + 2 * 3 + 1 && nebula_moe_state.model == NULL);
    puts("all-resident MoE drop-in: one qg_moe_layer per layer, no host reads, experts uploaded once, "
         "route profile, release passed.");
    return 0;
}
