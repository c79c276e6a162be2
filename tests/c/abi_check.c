/* Drives libfeml_b200 from plain C11 (no Python, no GPU): the graph builder
 * mirror compiles a plan through a host-memory backend implemented here
 * against fb_backend_vtable (the C image of feml-core's `dyn Backend`,
 * feml-core/src/backend.rs:86-122, as feml-core's own DummyBackend tests do,
 * graph.rs:453-503), tensor IO round-trips through the plan, and the error
 * paths report through feml_b200_last_error. Prints "ok" and exits 0. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "feml_b200.h"

#define CHECK(c)                                                                 \
    do {                                                                         \
        if (!(c)) {                                                              \
            fprintf(stderr, "check failed at line %d: %s (%s)\n", __LINE__, #c, \
                    feml_b200_last_error());                                     \
            return 1;                                                            \
        }                                                                        \
    } while (0)

enum { kMaxBufs = 16 };
typedef struct {
    uint8_t *data[kMaxBufs];
    uint64_t size[kMaxBufs];
    int live;
} host_backend;

static const char *hb_name(void *ctx) {
    (void)ctx;
    return "host";
}
static int hb_create(void *ctx, uint64_t size, int32_t usage, uint32_t *handle) {
    host_backend *b = (host_backend *)ctx;
    (void)usage;
    for (uint32_t h = 1; h < kMaxBufs; h++)
        if (!b->data[h]) {
            b->data[h] = (uint8_t *)calloc(size ? size : 1, 1);
            if (!b->data[h]) return FB_ERR_INVALID;
            b->size[h] = size;
            b->live++;
            *handle = h;
            return FB_OK;
        }
    return FB_ERR_INVALID;
}
static int hb_release(void *ctx, uint32_t h) {
    host_backend *b = (host_backend *)ctx;
    if (h >= kMaxBufs || !b->data[h]) return FB_ERR_INVALID;
    free(b->data[h]);
    b->data[h] = NULL;
    b->live--;
    return FB_OK;
}
static int hb_write(void *ctx, uint32_t h, uint64_t off, const void *src, uint64_t n) {
    host_backend *b = (host_backend *)ctx;
    if (h >= kMaxBufs || !b->data[h] || off > b->size[h] || n > b->size[h] - off) return FB_ERR_INVALID;
    memcpy(b->data[h] + off, src, n);
    return FB_OK;
}
static int hb_read(void *ctx, uint32_t h, uint64_t off, void *dst, uint64_t n) {
    host_backend *b = (host_backend *)ctx;
    if (h >= kMaxBufs || !b->data[h] || off > b->size[h] || n > b->size[h] - off) return FB_ERR_INVALID;
    memcpy(dst, b->data[h] + off, n);
    return FB_OK;
}
static int hb_fill(void *ctx, uint32_t h, uint64_t off, uint8_t v, uint64_t n) {
    host_backend *b = (host_backend *)ctx;
    if (h >= kMaxBufs || !b->data[h] || off > b->size[h] || n > b->size[h] - off) return FB_ERR_INVALID;
    memset(b->data[h] + off, v, n);
    return FB_OK;
}
static int hb_sync(void *ctx) {
    (void)ctx;
    return FB_OK;
}
static int hb_compute(void *ctx, const fb_plan *plan) {
    (void)ctx;
    (void)plan;
    return FB_OK;
}
static int hb_supports(void *ctx, int32_t op, const int32_t *dts, int32_t n) {
    (void)ctx;
    (void)dts;
    (void)n;
    return op == FB_OP_MUL_MAT || op == FB_OP_RMS_NORM;
}

int main(void) {
    CHECK(feml_b200_version() != NULL && strlen(feml_b200_version()) > 0);

    /* layout of a quantized row (Layout::new, layout.rs:32-48) */
    const int64_t qdims[2] = {512, 3};
    uint64_t nb[4];
    CHECK(fb_layout_new(FB_Q4_K, qdims, 2, nb) == FB_OK);
    CHECK(nb[0] == 144 && nb[1] == 2 * 144 && nb[2] == 3 * nb[1]);

    host_backend hb;
    memset(&hb, 0, sizeof hb);
    fb_backend_vtable vt = {&hb, hb_name, hb_create, hb_release, hb_write, hb_read, hb_fill,
                            hb_sync, hb_compute, hb_supports, NULL};

    /* x -> rms_norm -> mul_mat(w Q8_0) */
    fb_graph *g = NULL;
    CHECK(fb_graph_new(&g) == FB_OK);
    const int64_t xd[2] = {256, 2}, wd[2] = {256, 8};
    uint32_t x, w, r, y;
    CHECK(fb_graph_input(g, "x", FB_F32, xd, 2, &x) == FB_OK);
    CHECK(fb_graph_weight(g, "w", FB_Q8_0, wd, 2, &w) == FB_OK);
    CHECK(fb_graph_rms_norm(g, x, 1e-5f, &r) == FB_OK);
    CHECK(fb_graph_mul_mat(g, w, r, &y) == FB_OK);
    CHECK(fb_graph_mark_output(g, y) == FB_OK);
    /* a shape error is reported, not raised */
    uint32_t bad;
    const int64_t bd[2] = {100, 2};
    uint32_t xb;
    CHECK(fb_graph_input(g, "xb", FB_F32, bd, 2, &xb) == FB_OK);
    CHECK(fb_graph_mul_mat(g, w, xb, &bad) == FB_ERR_SHAPE);
    CHECK(strstr(feml_b200_last_error(), "mul_mat") != NULL);

    fb_compiled_plan *cp = NULL;
    CHECK(fb_graph_compile(g, &vt, &cp) == FB_OK);
    const fb_plan *p = fb_plan_get(cp);
    CHECK(p && p->n_nodes == 2 && p->n_buffers == 2 && hb.live == 2);
    CHECK(p->tensors[p->nodes[0]].op == FB_OP_RMS_NORM && p->tensors[p->nodes[1]].op == FB_OP_MUL_MAT);
    for (int64_t i = 0; i < p->n_tensors; i++) CHECK(p->tensors[i].offset % 32 == 0);
    float eps;
    memcpy(&eps, &p->tensors[p->nodes[0]].op_params[0], 4);
    CHECK(eps == 1e-5f);

    /* tensor IO round trip; a wrong size is rejected */
    float xs[512], back[512];
    for (int i = 0; i < 512; i++) xs[i] = (float)i * 0.25f - 7.0f;
    CHECK(fb_plan_write_tensor(cp, &vt, x, xs, sizeof xs) == FB_OK);
    CHECK(fb_plan_read_tensor(cp, &vt, x, back, sizeof back) == FB_OK);
    CHECK(memcmp(xs, back, sizeof xs) == 0);
    CHECK(fb_plan_write_tensor(cp, &vt, x, xs, sizeof xs - 4) != FB_OK);

    CHECK(fb_plan_release(cp, &vt) == FB_OK);
    CHECK(hb.live == 0);
    fb_plan_free(cp);
    fb_graph_free(g);

    /* GGUF: a missing file is an error with a message */
    fb_gguf *gg = NULL;
    CHECK(feml_b200_gguf_open("/nonexistent/model.gguf", &gg) == FB_ERR_INVALID && gg == NULL);
    CHECK(strstr(feml_b200_last_error(), "gguf") != NULL);

    printf("ok\n");
    return 0;
}
