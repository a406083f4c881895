/* frc_cost.c - the cost model the reference planner weighs a participant
 * with (fr_costmodel, src/backend.h:30-35): t = t0 + 1e9 * bytes / bw_eff,
 * fitted to measured synchronous runs at bursts 1..burst_max.  The fit
 * restates the reference's (src/bench.c:163-191: least squares of the median
 * times over the weight bytes a burst reads, t0 clamped at zero by refitting
 * through the origin); the measurement restates its resident case: distinct
 * seeded routing with the shared expert active, every loaded block, bytes =
 * blocks x (10 x burst x slice + shared slice) (src/bench.c:157-160).
 * Used by the fr_backend table's bench entry when the reference's own
 * harness (fr_bench_execute_backend) is not linked into the process. */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../include/fronk_b200.h"

int frc_costmodel_fit(const double *ns, const uint64_t *bytes, unsigned n, frc_costmodel *out) {
    if (!ns || !bytes || !out || n < 2 || n > FRC_COST_MAX_BURST) return FRC_INVALID;
    double sx = 0, sy = 0, sxx = 0, sxy = 0;
    for (unsigned b = 0; b < n; ++b) {
        const double x = (double)bytes[b], y = ns[b];
        if (!isfinite(y) || y <= 0 || bytes[b] == 0) return FRC_NUMERIC;
        sx += x; sy += y; sxx += x * x; sxy += x * y;
    }
    double slope = (n * sxy - sx * sy) / (n * sxx - sx * sx), t0 = (sy - slope * sx) / n;
    if (!isfinite(slope) || slope <= 0) return FRC_NUMERIC;
    if (t0 < 0) {  /* nonnegative t0: the least-squares line through the origin */
        t0 = 0;
        slope = sxy / sxx;
    }
    memset(out, 0, sizeof *out);
    out->burst_max = n;
    out->t0_ns = t0;
    out->bw_eff = 1e9 / slope;
    for (unsigned b = 0; b < n; ++b) {
        out->ns[b] = ns[b];
        out->bytes[b] = bytes[b];
    }
    return FRC_OK;
}

static double now_ns(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e9 + (double)ts.tv_nsec;
}

static int cmp_double(const void *a, const void *b) {
    const double x = *(const double *)a, y = *(const double *)b;
    return (x > y) - (x < y);
}

int frc_costmodel_measure(frc_context *c, const frc_geometry *g, unsigned layer, unsigned burst_max,
                          unsigned samples, int act, frc_costmodel *out) {
    if (!c || !g || !out || burst_max < 2 || burst_max > FRC_COST_MAX_BURST || samples < 1 || samples > 1000 ||
        g->hidden == 0 || g->hidden > 8192 || (act != FRC_ACT_Q8 && act != FRC_ACT_F32 && act != FRC_ACT_AVX2))
        return FRC_INVALID;
    uint32_t mask = 0;
    int rc = frc_loaded_mask(c, &mask);
    if (rc) return rc;
    if (!mask) return FRC_STATE;
    const unsigned blocks = (unsigned)__builtin_popcount(mask), d = g->hidden;
    uint16_t *e = malloc(sizeof(uint16_t) * FRC_COST_MAX_BURST * FRC_TOPK);
    float *gt = malloc(sizeof(float) * FRC_COST_MAX_BURST * FRC_ACTIVE);
    float *x = malloc(sizeof(float) * FRC_COST_MAX_BURST * d), *y = malloc(sizeof(float) * FRC_COST_MAX_BURST * d);
    double *t = malloc(sizeof(double) * samples);
    double ns[FRC_COST_MAX_BURST];
    uint64_t bytes[FRC_COST_MAX_BURST];
    rc = (e && gt && x && y && t) ? FRC_OK : FRC_IO;
    for (unsigned b = 1; b <= burst_max && rc == FRC_OK; ++b) {
        for (unsigned s = 0; s <= samples && rc == FRC_OK; ++s) {  /* s == 0: untimed warm-up */
            rc = frc_synth_request(d, b, 0x5eedc057ull + 7919ull * (1000ull * b + s), e, gt, x);
            if (rc) break;
            for (unsigned k = 0; k < b; ++k) gt[k * FRC_ACTIVE + FRC_TOPK] = 0.125f;  /* the shared expert runs */
            const double t0 = now_ns();
            rc = frc_run(c, layer, b, e, gt, x, y, act);
            if (s) t[s - 1] = now_ns() - t0;
        }
        if (rc) break;
        qsort(t, samples, sizeof(double), cmp_double);
        ns[b - 1] = samples % 2 ? t[samples / 2] : 0.5 * (t[samples / 2 - 1] + t[samples / 2]);
        bytes[b - 1] = (uint64_t)blocks * ((uint64_t)FRC_TOPK * b * frc_slice_bytes(g) + frc_shared_bytes(g));
    }
    if (rc == FRC_OK) rc = frc_costmodel_fit(ns, bytes, burst_max, out);
    free(e); free(gt); free(x); free(y); free(t);
    return rc;
}
