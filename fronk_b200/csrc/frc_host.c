/* frc_host.c - a decode pass driven from the host through the synchronous
 * host-buffer call, as a host that owns the layer loop drives the backend:
 * for every layer, x = h / sqrt(mean(h^2) + 1e-6) per token (the pre-norm a
 * decoder block applies before its MoE), y = frc_run_flags(layer, x) with
 * host buffers, h += y.  Only the public C ABI is used; every layer pays its
 * own host->device and device->host copies.  With FRC_RUN_PEER every rank of
 * a box runs the same loop on its share of the slices and the kernel sums
 * each layer over the ranks.  bench.py times it as the end-to-end figure. */
#include <math.h>
#include <string.h>

#include "../../include/fronk_b200.h"

enum { kMaxHidden = 8192 };

int frc_host_pass(frc_context *c, unsigned first_layer, unsigned layers, unsigned tokens, const uint16_t *expert,
                  const float *gate, float *h, unsigned hidden, int act) {
    return frc_host_pass_flags(c, first_layer, layers, tokens, expert, gate, h, hidden, act, 0);
}

int frc_host_pass_flags(frc_context *c, unsigned first_layer, unsigned layers, unsigned tokens,
                        const uint16_t *expert, const float *gate, float *h, unsigned hidden, int act,
                        unsigned flags) {
    if (!c || !expert || !gate || !h || !layers || !tokens || tokens > FRC_MAX_TOKENS || hidden == 0 ||
        hidden > kMaxHidden || hidden % 4)
        return FRC_INVALID;
    static float x[FRC_MAX_TOKENS * kMaxHidden], y[FRC_MAX_TOKENS * kMaxHidden];
    for (unsigned l = 0; l < layers; ++l) {
        for (unsigned t = 0; t < tokens; ++t) {
            const float *ht = h + (size_t)t * hidden;
            double ss = 0.0;
            for (unsigned i = 0; i < hidden; ++i) ss += (double)ht[i] * ht[i];
            const float inv = (float)(1.0 / sqrt(ss / hidden + 1e-6));
            for (unsigned i = 0; i < hidden; ++i) x[(size_t)t * hidden + i] = ht[i] * inv;
        }
        const int rc = frc_run_flags(c, first_layer + l, tokens, expert + (size_t)l * tokens * FRC_TOPK,
                                     gate + (size_t)l * tokens * FRC_ACTIVE, x, y, act, flags);
        if (rc) return rc;
        for (size_t i = 0; i < (size_t)tokens * hidden; ++i) h[i] += y[i];
    }
    return FRC_OK;
}
