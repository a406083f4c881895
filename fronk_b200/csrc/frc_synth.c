/* frc_synth.c - geometry of the native unit layout and synthetic inputs.
 *
 * Geometry mirrors src/native.h:9-21 with the hidden size and routed formats
 * as run-time values.  The encoders are this project's own: the reference has
 * no weight quantizer (its units are a byte gather from the GGUF, src/prep.c:1-7),
 * so synthetic ~N(0, 0.02) weights are quantized here into the byte formats
 * the reference decodes (src/native.c:14-30).
 */
#include "../../include/fronk_b200.h"
#include <math.h>
#include <string.h>

/* ------------------------------------------------------------ geometry */

size_t frc_row_bytes(unsigned type, unsigned n) {
    if (!n) return 0;
    if (type == FRC_Q4_K) return n % 256 ? 0 : (size_t)n / 256 * 144;
    if (type == FRC_MXFP4) return n % 32 ? 0 : (size_t)n / 32 * 17;
    if (type == FRC_Q8_0) return n % 32 ? 0 : (size_t)n / 32 * 34;
    return 0;
}

int frc_geometry_check(const frc_geometry *g) {
    if (!g || !g->hidden || g->hidden % 512 || g->hidden > 8192) return FRC_INVALID;
    if (!g->layers || g->layers > FRC_MAX_LAYERS) return FRC_INVALID;
    if (g->gate_type != FRC_Q4_K && g->gate_type != FRC_MXFP4 && g->gate_type != FRC_Q8_0) return FRC_INVALID;
    if (g->down_type != FRC_MXFP4 && g->down_type != FRC_Q8_0) return FRC_INVALID;
    return FRC_OK;
}

size_t frc_slice_bytes(const frc_geometry *g) {
    if (frc_geometry_check(g)) return 0;
    return 2 * FRC_NEURONS * frc_row_bytes(g->gate_type, g->hidden) +
           (size_t)g->hidden * frc_row_bytes(g->down_type, FRC_NEURONS);
}
size_t frc_shared_bytes(const frc_geometry *g) {
    if (frc_geometry_check(g)) return 0;
    return 3 * (size_t)g->hidden * 34;
}
size_t frc_layer_bytes(const frc_geometry *g) {
    if (frc_geometry_check(g)) return 0;
    return FRC_ROUTED_EXPERTS * frc_slice_bytes(g) + frc_shared_bytes(g);
}
uint64_t frc_unit_bytes(const frc_geometry *g) {
    return (uint64_t)frc_layer_bytes(g) * (g ? g->layers : 0);
}
uint64_t frc_slice_offset(const frc_geometry *g, unsigned layer, unsigned expert) {
    if (frc_geometry_check(g) || layer >= g->layers || expert > FRC_SHARED_EXPERT) return 0;
    return (uint64_t)layer * frc_layer_bytes(g) + (uint64_t)expert * frc_slice_bytes(g);
}

/* ------------------------------------------------------------- random */

/* splitmix64 finalizer over a Weyl sequence, indexed directly. */
uint64_t frc_rand64(uint64_t seed, uint64_t index) {
    uint64_t z = seed + 0x9E3779B97F4A7C15ull * (index + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float frc_normal(uint64_t seed, uint64_t index) {
    uint64_t r = frc_rand64(seed, index);
    int32_t s = (int32_t)(r & 0xffff) + (int32_t)(r >> 16 & 0xffff) + (int32_t)(r >> 32 & 0xffff) +
                (int32_t)(r >> 48) - 131070;
    /* Four uniforms on [0, 65535] have variance 4 * (65536^2 - 1) / 12. */
    return (float)s * 2.64289979e-5f;
}

/* ------------------------------------------------------------ encoders */

/* fp32 -> binary16, round to nearest even, saturating to inf. */
static uint16_t to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    uint32_t sign = x >> 16 & 0x8000u, e = x >> 23 & 0xffu, m = x & 0x7fffffu;
    if (e == 255) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0));
    int he = (int)e - 112; /* half biased exponent */
    uint32_t mant, shift;
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he > 0) { mant = m; shift = 13; }
    else {
        if (he < -10) return (uint16_t)sign;
        mant = m | 0x800000u;
        shift = (uint32_t)(14 - he);
    }
    uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) ++q;
    if (he > 0) return (uint16_t)(sign | (((uint32_t)he << 10) + q)); /* a carry bumps the exponent */
    return (uint16_t)(sign | q);
}
static float from_half(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = h >> 10 & 31u, m = h & 1023u;
    if (!e) {
        float f = ldexpf((float)m, -24);
        return sign ? -f : f;
    }
    uint32_t bits = sign | (e == 31 ? 0x7f800000u : (e + 112u) << 23) | m << 13;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}
static int clampi(float v, int lo, int hi) {
    int i = (int)nearbyintf(v);
    return i < lo ? lo : i > hi ? hi : i;
}

/* Q4_K super-block of 256: per 32 an affine range [lo, hi] with lo <= 0,
 * 6-bit scale and min against fp16 super scales, 4-bit levels. */
static void encode_q4k(const float *w, uint8_t *b) {
    float step[8], off[8], smax = 0, mmax = 0;
    for (unsigned g = 0; g < 8; ++g) {
        float lo = 0, hi = 0;
        for (unsigned j = 0; j < 32; ++j) {
            float v = w[32 * g + j];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        step[g] = (hi - lo) / 15.0f;
        off[g] = -lo;
        if (step[g] > smax) smax = step[g];
        if (off[g] > mmax) mmax = off[g];
    }
    uint16_t dh = to_half(smax / 63.0f), mh = to_half(mmax / 63.0f);
    float d = from_half(dh), dm = from_half(mh);
    unsigned sc[8], mi[8];
    for (unsigned g = 0; g < 8; ++g) {
        sc[g] = d > 0 ? (unsigned)clampi(step[g] / d, 0, 63) : 0;
        mi[g] = dm > 0 ? (unsigned)clampi(off[g] / dm, 0, 63) : 0;
    }
    memset(b, 0, 144);
    b[0] = (uint8_t)dh; b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)mh; b[3] = (uint8_t)(mh >> 8);
    for (unsigned g = 0; g < 4; ++g) {
        b[4 + g] = (uint8_t)(sc[g] | (sc[g + 4] >> 4) << 6);
        b[8 + g] = (uint8_t)(mi[g] | (mi[g + 4] >> 4) << 6);
        b[12 + g] = (uint8_t)((sc[g + 4] & 15) | (mi[g + 4] & 15) << 4);
    }
    for (unsigned j = 0; j < 256; ++j) {
        unsigned g = j / 32;
        float s = d * (float)sc[g], m = dm * (float)mi[g];
        unsigned q = s > 0 ? (unsigned)clampi((w[j] + m) / s, 0, 15) : 0;
        b[16 + (g / 2) * 32 + j % 32] |= (uint8_t)(q << (4 * (g % 2)));
    }
}

/* MXFP4 block of 32: E8M0 exponent so the largest magnitude fits 6, E2M1
 * nearest value per weight (lowest index on a tie). */
static void encode_mxfp4(const float *w, uint8_t *b) {
    static const float level[8] = {0, .5f, 1, 1.5f, 2, 3, 4, 6};
    float amax = 0;
    for (unsigned j = 0; j < 32; ++j) if (fabsf(w[j]) > amax) amax = fabsf(w[j]);
    int k = 0;
    if (amax > 0) {
        int ex;
        float f = frexpf(amax / 6.0f, &ex); /* amax/6 = f * 2^ex, f in [0.5, 1) */
        k = f == 0.5f ? ex - 1 : ex;
        if (k < -127) k = -127;
        if (k > 127) k = 127;
    }
    memset(b, 0, 17);
    b[0] = (uint8_t)(k + 127);
    float scale = ldexpf(1.0f, k);
    for (unsigned j = 0; j < 32; ++j) {
        float r = fabsf(w[j]) / scale;
        unsigned best = 0;
        for (unsigned i = 1; i < 8; ++i) if (fabsf(r - level[i]) < fabsf(r - level[best])) best = i;
        unsigned nib = best | (w[j] < 0 ? 8u : 0u);
        b[1 + j % 16] |= (uint8_t)(nib << (j < 16 ? 0 : 4));
    }
}

/* Q8_0 block of 32: fp16 scale amax/127 and int8 levels. */
static void encode_q80(const float *w, uint8_t *b) {
    float amax = 0;
    for (unsigned j = 0; j < 32; ++j) if (fabsf(w[j]) > amax) amax = fabsf(w[j]);
    uint16_t dh = to_half(amax / 127.0f);
    float d = from_half(dh);
    b[0] = (uint8_t)dh; b[1] = (uint8_t)(dh >> 8);
    for (unsigned j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)(d > 0 ? clampi(w[j] / d, -127, 127) : 0);
}

int frc_encode_row(unsigned type, const float *w, unsigned n, uint8_t *out) {
    if (!w || !out || !frc_row_bytes(type, n)) return FRC_INVALID;
    for (unsigned j = 0; j < n; ++j) if (!isfinite(w[j])) return FRC_NUMERIC;
    if (type == FRC_Q4_K) for (unsigned k = 0; k < n / 256; ++k) encode_q4k(w + 256 * k, out + 144 * k);
    else if (type == FRC_MXFP4) for (unsigned k = 0; k < n / 32; ++k) encode_mxfp4(w + 32 * k, out + 17 * k);
    else for (unsigned k = 0; k < n / 32; ++k) encode_q80(w + 32 * k, out + 34 * k);
    return FRC_OK;
}

/* --------------------------------------------------------------- synth */

enum { WEIGHT_STREAM = 20 }; /* element index bits below the slice key */

static int synth_projections(unsigned d, unsigned in, unsigned down, uint64_t seed, uint64_t key, uint8_t *out) {
    float w[8192];
    uint64_t base = key << WEIGHT_STREAM, i = 0;
    size_t row = frc_row_bytes(in, d);
    if (d > 8192 || !row) return FRC_INVALID;
    for (unsigned r = 0; r < 2 * FRC_NEURONS; ++r) { /* gate rows then up rows */
        for (unsigned j = 0; j < d; ++j) w[j] = 0.02f * frc_normal(seed, base + i++);
        frc_encode_row(in, w, d, out + r * row);
    }
    uint8_t *p = out + 2 * FRC_NEURONS * row;
    size_t drow = frc_row_bytes(down, FRC_NEURONS);
    for (unsigned r = 0; r < d; ++r) {  /* down: d rows of 32 neurons */
        for (unsigned j = 0; j < FRC_NEURONS; ++j) w[j] = 0.02f * frc_normal(seed, base + i++);
        frc_encode_row(down, w, FRC_NEURONS, p + r * drow);
    }
    return FRC_OK;
}

int frc_synth_slice(const frc_geometry *g, uint64_t seed, uint64_t key, uint8_t *out) {
    if (frc_geometry_check(g) || !out) return FRC_INVALID;
    return synth_projections(g->hidden, g->gate_type, g->down_type, seed, key, out);
}

int frc_synth_shared(const frc_geometry *g, uint64_t seed, uint64_t key, uint8_t *out) {
    if (frc_geometry_check(g) || !out) return FRC_INVALID;
    return synth_projections(g->hidden, FRC_Q8_0, FRC_Q8_0, seed, key, out);
}

int frc_synth_request(unsigned hidden, unsigned tokens, uint64_t seed, uint16_t *expert, float *gate, float *x) {
    if (!expert || !gate || !x || !hidden || hidden % 32 || !tokens || tokens > FRC_MAX_PREFILL_TOKENS)
        return FRC_INVALID;
    const uint64_t xs = 1ull << 40, rs = 2ull << 40, gs = 3ull << 40;
    for (unsigned t = 0; t < tokens; ++t) {
        for (unsigned j = 0; j < hidden; ++j) x[(size_t)t * hidden + j] = frc_normal(seed, xs + (uint64_t)t * hidden + j);
        uint16_t perm[FRC_ROUTED_EXPERTS];
        for (unsigned i = 0; i < FRC_ROUTED_EXPERTS; ++i) perm[i] = (uint16_t)i;
        for (unsigned i = 0; i < FRC_TOPK; ++i) { /* partial Fisher-Yates */
            unsigned j = i + (unsigned)(frc_rand64(seed, rs + t * 16u + i) % (FRC_ROUTED_EXPERTS - i));
            uint16_t tmp = perm[i]; perm[i] = perm[j]; perm[j] = tmp;
            expert[t * FRC_TOPK + i] = perm[i];
        }
        float z[FRC_TOPK], m = -INFINITY, sum = 0;
        for (unsigned i = 0; i < FRC_TOPK; ++i) {
            z[i] = frc_normal(seed, gs + t * 16u + i);
            if (z[i] > m) m = z[i];
        }
        for (unsigned i = 0; i < FRC_TOPK; ++i) { z[i] = expf(z[i] - m); sum += z[i]; }
        for (unsigned i = 0; i < FRC_TOPK; ++i) gate[t * FRC_ACTIVE + i] = z[i] / sum;
        gate[t * FRC_ACTIVE + FRC_TOPK] = 0;
    }
    return FRC_OK;
}

int frc_synth_request_zipf(unsigned hidden, unsigned tokens, uint64_t seed, double zs, uint16_t *expert,
                           float *gate, float *x) {
    if (!(zs >= 0) || zs > 16) return FRC_INVALID;
    int rc = frc_synth_request(hidden, tokens, seed, expert, gate, x);
    if (rc) return rc;
    /* popularity rank: a seeded permutation of the experts */
    const uint64_t ps = 4ull << 40, us = 5ull << 40;
    unsigned rank[FRC_ROUTED_EXPERTS];
    for (unsigned i = 0; i < FRC_ROUTED_EXPERTS; ++i) rank[i] = i;
    for (unsigned i = FRC_ROUTED_EXPERTS - 1; i > 0; --i) {
        unsigned j = (unsigned)(frc_rand64(seed, ps + i) % (i + 1));
        unsigned tmp = rank[i]; rank[i] = rank[j]; rank[j] = tmp;
    }
    double logw[FRC_ROUTED_EXPERTS];
    for (unsigned e = 0; e < FRC_ROUTED_EXPERTS; ++e) logw[e] = -zs * log((double)rank[e] + 1.0);
    for (unsigned t = 0; t < tokens; ++t) {
        double key[FRC_ROUTED_EXPERTS];
        for (unsigned e = 0; e < FRC_ROUTED_EXPERTS; ++e) {
            const double u = ((double)(frc_rand64(seed, us + (uint64_t)t * FRC_ROUTED_EXPERTS + e) >> 11) + 0.5) *
                             (1.0 / 9007199254740992.0);
            key[e] = logw[e] - log(-log(u));
        }
        for (unsigned i = 0; i < FRC_TOPK; ++i) { /* selection of the ten largest keys, descending */
            unsigned best = 0;
            for (unsigned e = 1; e < FRC_ROUTED_EXPERTS; ++e) if (key[e] > key[best]) best = e;
            expert[t * FRC_TOPK + i] = (uint16_t)best;
            key[best] = -INFINITY;
        }
    }
    return FRC_OK;
}

/* Pool slot choice for benchmark-scale units (shared with the device fill). */
unsigned frc_pool_pick(uint64_t seed, unsigned block, unsigned layer, unsigned expert, unsigned count) {
    if (!count) return 0;
    return (unsigned)(frc_rand64(seed, ((uint64_t)block * FRC_MAX_LAYERS + layer) * 513u + expert) % count);
}
