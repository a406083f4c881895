/* ref_bench.c - times the reference's own CPU backends on the decode workload.
 *
 * TEST INFRASTRUCTURE ONLY (the CPU baseline of bench.py).  Compiled against
 * the reference's unmodified sources (src/*.c, backends/ref.c, backends/avx2.c)
 * and this project's input generator, it runs the 48-layer decode pass for
 * TOKENS tokens (default 1): layer l takes x_l, the layer's seeded top-10
 * routing and gates per token, calls backend->run (src/backend.h:64) once per
 * burst of up to FR_MAX_BURST tokens, and feeds x_{l+1} = x_l + y_l.  Units are
 * sparse anonymous mappings of FR_NATIVE_BLOCK_BYTES (as src/native.c:66-75
 * does) holding pool slices in every slot the routing touches.
 *
 *   ref_bench BACKEND BLOCKS POOL STEPS WARMUP SEED [TOKENS [ZIPF [LAYERS]]]
 * ZIPF > 0 draws the routing with Zipf(ZIPF) expert popularity
 * (frc_synth_request_zipf); LAYERS (default 48) shortens the pass.
 * prints one JSON line.
 */
#define _GNU_SOURCE
#include "backend.h"
#include "native.h"
#include "avx2.h"
#include "hw.h"
#include "../include/fronk_b200.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <time.h>

static double now(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}
static int cmp(const void *a, const void *b) {
    double x = *(const double *)a, y = *(const double *)b;
    return x < y ? -1 : x > y;
}

int main(int argc, char **argv) {
    if (argc < 7 || argc > 10) {
        fputs("usage: ref_bench BACKEND BLOCKS POOL STEPS WARMUP SEED [TOKENS [ZIPF [LAYERS]]]\n", stderr);
        return 2;
    }
    const fr_backend *backend = fr_backend_find(argv[1]);
    unsigned blocks = (unsigned)atoi(argv[2]), pool_n = (unsigned)atoi(argv[3]);
    unsigned steps = (unsigned)atoi(argv[4]), warm = (unsigned)atoi(argv[5]);
    uint64_t seed = strtoull(argv[6], NULL, 0);
    const unsigned T = argc >= 8 ? (unsigned)atoi(argv[7]) : 1;
    const double zipf = argc >= 9 ? atof(argv[8]) : 0.0;
    const unsigned L = argc >= 10 ? (unsigned)atoi(argv[9]) : FR_LAYERS;
    if (!L || L > FR_LAYERS) return 2;
    if (!backend || !blocks || blocks > FR_BLOCKS || !pool_n || !steps || !T || T > FRC_MAX_PREFILL_TOKENS) return 2;
    const frc_geometry g = {FR_HIDDEN, FR_LAYERS, FRC_Q4_K, FRC_MXFP4};
    if (frc_slice_bytes(&g) != FR_NATIVE_SLICE_BYTES || frc_unit_bytes(&g) != FR_NATIVE_BLOCK_BYTES) {
        fputs("geometry mismatch\n", stderr);
        return 1;
    }
    /* Pool of distinct routed slices (the shared expert is unused: gate 0). */
    unsigned char *pool = malloc((size_t)pool_n * FR_NATIVE_SLICE_BYTES);
    if (!pool) return 1;
    for (unsigned i = 0; i < pool_n; ++i) frc_synth_slice(&g, seed, i, pool + (size_t)i * FR_NATIVE_SLICE_BYTES);
    /* Routing for every step, layer and token; x only for layer 0 of each step. */
    const unsigned passes = warm + steps;
    const size_t rows = (size_t)passes * L * T;
    uint16_t *expert = malloc(sizeof(uint16_t) * rows * FR_ACTIVE_ROUTED);
    float *gate = malloc(sizeof(float) * rows * FR_ACTIVE_EXPERTS);
    float *x0 = malloc(sizeof(float) * passes * T * FR_HIDDEN), *tmp = malloc(sizeof(float) * T * FR_HIDDEN);
    for (unsigned s = 0; s < passes; ++s)
        for (unsigned l = 0; l < L; ++l) {
            uint64_t rs = frc_rand64(seed, 1000003ull * s + l);
            const size_t r = ((size_t)s * L + l) * T;
            float *xo = l ? tmp : x0 + (size_t)s * T * FR_HIDDEN;
            if (zipf > 0)
                frc_synth_request_zipf(FR_HIDDEN, T, rs, zipf, expert + r * FR_ACTIVE_ROUTED,
                                       gate + r * FR_ACTIVE_EXPERTS, xo);
            else
                frc_synth_request(FR_HIDDEN, T, rs, expert + r * FR_ACTIVE_ROUTED, gate + r * FR_ACTIVE_EXPERTS, xo);
        }
    unsigned char *unit[FR_BLOCKS] = {0};
    int rc = 0;
    static unsigned char filled[FR_LAYERS][FR_ROUTED_EXPERTS];
    for (unsigned b = 0; b < blocks && !rc; ++b) {
        unit[b] = mmap(NULL, FR_NATIVE_BLOCK_BYTES, PROT_READ | PROT_WRITE,
                       MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
        if (unit[b] == MAP_FAILED) { unit[b] = NULL; rc = 1; break; }
        memset(filled, 0, sizeof filled);
        for (unsigned s = 0; s < passes; ++s)
            for (unsigned l = 0; l < L; ++l)
                for (unsigned e = 0; e < T * FR_ACTIVE_ROUTED; ++e) {
                    unsigned id = expert[((size_t)s * L + l) * T * FR_ACTIVE_ROUTED + e];
                    if (filled[l][id]) continue;
                    filled[l][id] = 1;
                    unsigned pick = frc_pool_pick(seed, b, l, id, pool_n);
                    memcpy(unit[b] + fr_native_offset(l, id), pool + (size_t)pick * FR_NATIVE_SLICE_BYTES,
                           FR_NATIVE_SLICE_BYTES);
                }
        rc = backend->load((int)b, unit[b], FR_NATIVE_BLOCK_BYTES);
    }
    if (rc) { fprintf(stderr, "load failed %d\n", rc); return 1; }
    static fr_req req;
    static fr_part part;
    req.burst = 1;
#ifdef FR_AVX2_COMPUTE
    if (backend == &fr_avx2) {
        req.layer = 0;
        memcpy(req.expert[0], expert, sizeof req.expert[0]);
        memcpy(req.gate[0], gate, sizeof req.gate[0]);
        memcpy(req.x[0], x0, sizeof req.x[0]);
        rc = fr_avx2_tune(&req, NULL);
        if (rc) { fprintf(stderr, "tune failed %d\n", rc); return 1; }
    }
#endif
    /* Residual stream h: layer input x = h / sqrt(mean(h^2) + 1e-6) (unit-gain
     * pre-norm), then h += y.  Without the norm the SwiGLU chain diverges. */
    double *ns = malloc(sizeof(double) * steps), checksum = 0;
    float *h = malloc(sizeof(float) * T * FR_HIDDEN);
    for (unsigned s = 0; s < passes && !rc; ++s) {
        memcpy(h, x0 + (size_t)s * T * FR_HIDDEN, sizeof(float) * T * FR_HIDDEN);
        double t0 = now();
        for (unsigned l = 0; l < L && !rc; ++l) {
            const size_t r = ((size_t)s * L + l) * T;
            for (unsigned first = 0; first < T && !rc; first += FR_MAX_BURST) {
                const unsigned n = T - first < FR_MAX_BURST ? T - first : FR_MAX_BURST;
                for (unsigned k = 0; k < n; ++k) {
                    const float *ht = h + (size_t)(first + k) * FR_HIDDEN;
                    float ss = 0;
                    for (unsigned j = 0; j < FR_HIDDEN; ++j) ss += ht[j] * ht[j];
                    float g = 1.0f / sqrtf(ss / FR_HIDDEN + 1e-6f);
                    for (unsigned j = 0; j < FR_HIDDEN; ++j) req.x[k][j] = ht[j] * g;
                    memcpy(req.expert[k], expert + (r + first + k) * FR_ACTIVE_ROUTED, sizeof req.expert[0]);
                    memcpy(req.gate[k], gate + (r + first + k) * FR_ACTIVE_EXPERTS, sizeof req.gate[0]);
                }
                req.layer = l;
                req.burst = n;
                rc = backend->run(&req, &part);
                for (unsigned k = 0; k < n && !rc; ++k)
                    for (unsigned j = 0; j < FR_HIDDEN; ++j)
                        h[(size_t)(first + k) * FR_HIDDEN + j] += part.y[k][j];
            }
        }
        double dt = now() - t0;
        if (s >= warm) {
            ns[s - warm] = dt * 1e9;
            for (size_t j = 0; j < (size_t)T * FR_HIDDEN; ++j) checksum += h[j];
        }
    }
    if (rc) { fprintf(stderr, "run failed %d\n", rc); return 1; }
    double total = 0;
    for (unsigned i = 0; i < steps; ++i) total += ns[i];
    qsort(ns, steps, sizeof(double), cmp);
    unsigned workers = 0;
#ifdef FR_AVX2_COMPUTE
    if (backend == &fr_avx2) {
        fr_avx2_sample sample;
        if (!fr_avx2_sample_get(&sample)) workers = sample.workers;
    }
#endif
    fr_hwinfo hw;
    memset(&hw, 0, sizeof hw);
    hw_probe(&hw);
    printf("{\"backend\": \"%s\", \"hidden\": %d, \"blocks\": %u, \"tokens\": %u, \"layers\": %u, \"zipf\": %g, \"steps\": %u, \"warmup\": %u, "
           "\"ns_per_pass_mean\": %.1f, \"ns_per_pass_p50\": %.1f, \"workers\": %u, \"cores\": %u, "
           "\"logical_cores\": %u, \"cpu\": \"%s\", \"checksum\": %.9g}\n",
           backend->name, FR_HIDDEN, blocks, T, L, zipf, steps, warm, total / steps, ns[steps / 2], workers, hw.cores,
           hw.logical_cores, hw.cpu, checksum);
    for (unsigned b = 0; b < blocks; ++b) {
        backend->unload((int)b);
        munmap(unit[b], FR_NATIVE_BLOCK_BYTES);
    }
    return 0;
}
