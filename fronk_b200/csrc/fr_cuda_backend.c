/* fr_cuda_backend.c - the fr_backend plugin table of the B200 backend.
 *
 * Registers like backends/user-template.c: probe/load/unload/run/bench/
 * self_test with the contract of src/backend.h:1-5,52-67.  Host side is plain
 * C over the frc_* C ABI; there is no CPU fallback: without an sm_100 device
 * probe and load return FR_UNSUPPORTED.
 *
 * Differences a discrete GPU forces (documented, not hidden):
 *  - load copies the borrowed unit into HBM (set-up time); unload frees it
 *    (backends/ref.c:19-28 borrow instead and read the bytes at every run).
 *    A unit lent from writable memory may change while it is loaded (the
 *    reference's own self-test, src/native.c:121-131, corrupts scales of a
 *    loaded unit and expects run to see them), so for such a block run first
 *    copies the request's layer again (frc_refresh_layer).  Units mapped
 *    read-only, as the node's loader maps them (src/units.c:25-75), are
 *    copied once.
 *  - bench and self_test call the reference's own fr_bench_execute_backend and
 *    fr_native_self_test when the process links them (they are looked up at
 *    call time).  Without them, bench measures and fits the same cost model
 *    itself (frc_costmodel_measure); self_test reports FR_UNSUPPORTED.
 * Build inside the reference tree with -DFR_USE_REFERENCE_HEADERS and
 * -I<reference>/src to compile against src/backend.h itself.
 */
#define _GNU_SOURCE
#ifdef FR_USE_REFERENCE_HEADERS
#include "backend.h"
#include "native.h"
extern const fr_backend fr_cuda, fr_cuda_f32, fr_cuda_avx2;
int fr_cuda_select_device(int device);
int fr_cuda_close(const fr_backend *backend);
int fr_cuda_avx2_workers(unsigned workers);
#else
#include "../../include/fr_backend_abi.h"
#endif
#include "../../include/fronk_b200.h"
#include <dlfcn.h>
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

typedef struct {
    frc_context *ctx;
    int act;
    unsigned char loaded[FR_BLOCKS];
    unsigned char writable[FR_BLOCKS];  /* lent from writable memory: refreshed per run */
    const unsigned char *unit[FR_BLOCKS];
} slot_state;

static slot_state q8_state = {NULL, FRC_ACT_Q8, {0}, {0}, {0}}, f32_state = {NULL, FRC_ACT_F32, {0}, {0}, {0}},
                  avx2_state = {NULL, FRC_ACT_AVX2, {0}, {0}, {0}};
static unsigned avx2_workers = 1; /* fr_cuda_avx2's worker count (frc_set_avx2_workers) */

/* 1 when any page of [p, p + len) is mapped writable (from /proc/self/maps;
 * 1 as well when that cannot be read: refreshing is the safe side). */
static int range_writable(const void *p, size_t len) {
    FILE *f = fopen("/proc/self/maps", "r");
    if (!f) return 1;
    const uintptr_t lo = (uintptr_t)p, hi = lo + len;
    char line[512];
    int w = 0;
    while (!w && fgets(line, sizeof line, f)) {
        unsigned long long a = 0, b = 0;
        char perms[8] = {0};
        if (sscanf(line, "%llx-%llx %7s", &a, &b, perms) != 3) continue;
        if (a < hi && b > lo && perms[1] == 'w') w = 1;
    }
    fclose(f);
    return w;
}
static int device_index = 0;

static slot_state *state_of(const fr_backend *b) {
    return b == &fr_cuda ? &q8_state : b == &fr_cuda_f32 ? &f32_state : b == &fr_cuda_avx2 ? &avx2_state : NULL;
}
static int any_loaded(const slot_state *s) {
    for (unsigned b = 0; b < FR_BLOCKS; ++b) if (s->loaded[b]) return 1;
    return 0;
}
static frc_geometry reference_geometry(void) {
    frc_geometry g = {FR_HIDDEN, FR_LAYERS, FRC_Q4_K, FRC_MXFP4};
    return g;
}

int fr_cuda_select_device(int device) {
    if (device < 0) return FR_INVALID;
    if (q8_state.ctx || f32_state.ctx || avx2_state.ctx) return FR_STATE;
    device_index = device;
    return FR_OK;
}

/* The worker count whose job dealing and summation order fr_cuda_avx2
 * reproduces (fr_avx2 takes it from fr_avx2_configure, backends/avx2.c:732-742). */
int fr_cuda_avx2_workers(unsigned workers) {
    if (workers < 1 || workers > 32) return FR_INVALID;
    avx2_workers = workers;
    return avx2_state.ctx ? frc_set_avx2_workers(avx2_state.ctx, workers) : FR_OK;
}

int fr_cuda_close(const fr_backend *backend) {
    slot_state *s = state_of(backend);
    if (!s) return FR_INVALID;
    if (any_loaded(s)) return FR_STATE;
    if (s->ctx) frc_close(s->ctx);
    s->ctx = NULL;
    return FR_OK;
}

/* FR_UNSUPPORTED without an sm_100 device (a device query, no context is
 * opened); otherwise the reference's own hw_probe fills the host fields when
 * it is linked in, and gpu names the device. */
static int probe(fr_hwinfo *out) {
    if (!out) return FR_INVALID;
    char name[128] = {0};
    uint64_t hbm = 0;
    unsigned sms = 0;
    int rc = frc_probe_device(device_index, name, sizeof name, &hbm, &sms);
    if (rc) return rc == FRC_UNSUPPORTED ? FR_UNSUPPORTED : FR_IO;
    int (*hw_probe)(fr_hwinfo *) = (int (*)(fr_hwinfo *))dlsym(RTLD_DEFAULT, "hw_probe");
    fr_hwinfo h;
    memset(&h, 0, sizeof h);
    if (hw_probe && hw_probe(&h)) return FR_IO;
    snprintf(h.gpu, sizeof h.gpu, "%s (sm_100, %u SMs, %llu MiB HBM)", name, sms, (unsigned long long)(hbm >> 20));
    *out = h;
    return FR_OK;
}

static int load(slot_state *s, int block, const void *data, size_t len) {
    frc_geometry g = reference_geometry();
    if (block < 0 || block >= FR_BLOCKS || !data || len != frc_unit_bytes(&g)) return FR_INVALID;
    if (s->loaded[block]) return FR_STATE;
    if (!s->ctx) {
        int rc = frc_open(device_index, &g, &s->ctx);
        if (rc) return rc;
        if (s->act == FRC_ACT_AVX2 && (rc = frc_set_avx2_workers(s->ctx, avx2_workers))) return rc;
    }
    int rc = frc_load_unit(s->ctx, block, data, len);
    if (!rc) {
        s->loaded[block] = 1;
        s->unit[block] = (const unsigned char *)data;
        s->writable[block] = (unsigned char)range_writable(data, len);
    }
    return rc;
}

static int unload(slot_state *s, int block) {
    if (block < 0 || block >= FR_BLOCKS) return FR_INVALID;
    if (!s->loaded[block]) return FR_STATE;
    s->loaded[block] = 0;
    s->writable[block] = 0;
    s->unit[block] = NULL;
    return frc_unload_unit(s->ctx, block);
}

/* backends/ref.c:41-56, the request checks in the reference's order. */
static int validate(const fr_req *r) {
    if (!r || r->layer >= FR_LAYERS || r->burst < 1 || r->burst > FR_MAX_BURST || fegetround() != FE_TONEAREST)
        return FR_INVALID;
    for (unsigned t = 0; t < r->burst; ++t) {
        for (unsigned e = 0; e < FR_ACTIVE_ROUTED; ++e) {
            if (r->expert[t][e] >= FR_ROUTED_EXPERTS) return FR_INVALID;
            for (unsigned j = 0; j < e; ++j) if (r->expert[t][j] == r->expert[t][e]) return FR_INVALID;
        }
        for (unsigned e = 0; e < FR_ACTIVE_EXPERTS; ++e) {
            if (!isfinite(r->gate[t][e])) return FR_NUMERIC;
            if (r->gate[t][e] < 0) return FR_INVALID;
        }
        for (unsigned j = 0; j < FR_HIDDEN; ++j) if (!isfinite(r->x[t][j])) return FR_NUMERIC;
    }
    return FR_OK;
}

static fr_part scratch; /* bounded static result: run allocates nothing */

static int run(slot_state *s, const fr_req *req, fr_part *out) {
    if (!out) return FR_INVALID;
    int rc = validate(req);
    if (rc) return rc;
    if (!s->ctx || !any_loaded(s)) return FR_STATE;
    const frc_geometry g = reference_geometry();
    const size_t layer_bytes = frc_layer_bytes(&g);
    for (unsigned b = 0; b < FR_BLOCKS; ++b)
        if (s->loaded[b] && s->writable[b]) {
            rc = frc_refresh_layer(s->ctx, (int)b, req->layer, s->unit[b] + (size_t)req->layer * layer_bytes, layer_bytes);
            if (rc) return rc;
        }
    memset(&scratch, 0, sizeof scratch); /* unused tokens stay zero */
    scratch.layer = req->layer;
    scratch.burst = req->burst;
    rc = frc_run(s->ctx, req->layer, req->burst, &req->expert[0][0], &req->gate[0][0], &req->x[0][0],
                 &scratch.y[0][0], s->act);
    if (rc) return rc;
    *out = scratch; /* published only after full success */
    return FR_OK;
}

typedef int (*bench_fn)(const fr_backend *, int, fr_costmodel *);
typedef int (*self_test_fn)(const fr_backend *);

static int bench(const fr_backend *b, int burst_max, fr_costmodel *out) {
    if (!out) return FR_INVALID;
    bench_fn f = (bench_fn)dlsym(RTLD_DEFAULT, "fr_bench_execute_backend");
    if (f) return f(b, burst_max, out);
    /* without the reference's harness: the same measurement and fit over the
     * loaded blocks (frc_costmodel_measure) */
    slot_state *s = state_of(b);
    if (!s || !s->ctx || !any_loaded(s)) return FR_STATE;
    if (burst_max < 2 || burst_max > FR_MAX_BURST || burst_max > FRC_COST_MAX_BURST) return FR_INVALID;
    const frc_geometry g = reference_geometry();
    frc_costmodel m;
    const int rc = frc_costmodel_measure(s->ctx, &g, 0, (unsigned)burst_max, 15, s->act, &m);
    if (rc) return rc;
    memset(out, 0, sizeof *out);
    out->burst_max = m.burst_max;
    out->t0_ns = m.t0_ns;
    out->bw_eff = m.bw_eff;
    for (unsigned i = 0; i < m.burst_max; ++i) {
        out->ns[i] = m.ns[i];
        out->bytes[i] = m.bytes[i];
    }
    return FR_OK;
}

static int self_test(const fr_backend *b, const char *dir) {
    (void)dir;
    slot_state *s = state_of(b);
    if (any_loaded(s)) return FR_STATE;
    self_test_fn f = (self_test_fn)dlsym(RTLD_DEFAULT, "fr_native_self_test");
    return f ? f(b) : FR_UNSUPPORTED;
}

static int q8_load(int b, const void *p, size_t n) { return load(&q8_state, b, p, n); }
static int f32_load(int b, const void *p, size_t n) { return load(&f32_state, b, p, n); }
static int q8_unload(int b) { return unload(&q8_state, b); }
static int f32_unload(int b) { return unload(&f32_state, b); }
static int q8_run(const fr_req *r, fr_part *o) { return run(&q8_state, r, o); }
static int f32_run(const fr_req *r, fr_part *o) { return run(&f32_state, r, o); }
static int q8_bench(int b, fr_costmodel *o) { return bench(&fr_cuda, b, o); }
static int f32_bench(int b, fr_costmodel *o) { return bench(&fr_cuda_f32, b, o); }
static int q8_test(const char *d) { return self_test(&fr_cuda, d); }
static int f32_test(const char *d) { return self_test(&fr_cuda_f32, d); }
static int avx2_load(int b, const void *p, size_t n) { return load(&avx2_state, b, p, n); }
static int avx2_unload(int b) { return unload(&avx2_state, b); }
static int avx2_run(const fr_req *r, fr_part *o) { return run(&avx2_state, r, o); }
static int avx2_bench(int b, fr_costmodel *o) { return bench(&fr_cuda_avx2, b, o); }
static int avx2_test(const char *d) { return self_test(&fr_cuda_avx2, d); }

const fr_backend fr_cuda = {"cuda", probe, q8_load, q8_unload, q8_run, q8_bench, q8_test};
const fr_backend fr_cuda_f32 = {"cuda-f32", probe, f32_load, f32_unload, f32_run, f32_bench, f32_test};
/* The arithmetic of the reference's AVX2 backend (FRC_ACT_AVX2): a drop-in for
 * fr_avx2 whose results equal its own at the same worker count. */
const fr_backend fr_cuda_avx2 = {"cuda-avx2", probe, avx2_load, avx2_unload, avx2_run, avx2_bench, avx2_test};
