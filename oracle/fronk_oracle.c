/* fronk_oracle.c - CPU restatement of the reference's expert-slice arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of it.
 * Build with -ffp-contract=off: every fp32 rounding below is deliberate.
 * Each function cites the reference lines it restates (paths inside the
 * fedesnore/fronk tree).
 */
#include "fronk_oracle.h"
#include <fenv.h>
#include <float.h>
#include <stdlib.h>
#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------- scalars */

/* src/q4.c:12-20: exact binary16 decode, subnormals and specials included. */
float or_f16(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    if (!e) {
        float f = ldexpf((float)m, -24);
        return sign ? -f : f;
    }
    uint32_t bits = sign | (e == 31 ? 0x7f800000u : (e + 112u) << 23) | m << 13;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (uint16_t)p[1] << 8); }

/* src/q4.c:37-61, split so the int8 values and scales are visible.  Groups of
 * 64 (a final 32-element group is a short group), scale = max/127,
 * multiplier 127/max (x/max*127 if that overflows), nearest-even, clamp. */
int or_q8_quantize(const float *x, size_t n, int8_t *q, float *scale) {
    if (!x || !q || !scale || !n || n % 32 || fegetround() != FE_TONEAREST) return OR_INVALID;
    for (size_t k = 0; k < n; k += 64) {
        size_t count = n - k < 64 ? n - k : 64;
        float max = 0;
        for (size_t j = 0; j < count; ++j) {
            if (!isfinite(x[k + j])) return OR_NUMERIC;
            if (fabsf(x[k + j]) > max) max = fabsf(x[k + j]);
        }
        float s = max / 127.0f;
        scale[k / 64] = s;
        if (!s) {
            for (size_t j = 0; j < count; ++j) q[k + j] = 0;
            continue;
        }
        float inv = 127.0f / max;
        for (size_t j = 0; j < count; ++j) {
            float v = isfinite(inv) ? x[k + j] * inv : (x[k + j] / max) * 127.0f;
            v = nearbyintf(v);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            q[k + j] = (int8_t)v;
        }
    }
    return OR_OK;
}

/* src/q4.c:37-61 as written: the dequantized value comes from the rounded
 * float, so a negative input that rounds to zero gives -0.0. */
int or_q8_activation(const float *x, float *out, size_t n) {
    if (!x || !out || !n || n % 32 || fegetround() != FE_TONEAREST) return OR_INVALID;
    for (size_t k = 0; k < n; k += 64) {
        size_t count = n - k < 64 ? n - k : 64;
        float max = 0;
        for (size_t j = 0; j < count; ++j) {
            if (!isfinite(x[k + j])) return OR_NUMERIC;
            if (fabsf(x[k + j]) > max) max = fabsf(x[k + j]);
        }
        float s = max / 127.0f;
        if (!s) {
            for (size_t j = 0; j < count; ++j) out[k + j] = 0;
            continue;
        }
        float inv = 127.0f / max;
        for (size_t j = 0; j < count; ++j) {
            float v = isfinite(inv) ? x[k + j] * inv : (x[k + j] / max) * 127.0f;
            v = nearbyintf(v);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            double d = (double)v * s; /* capped: rounded max/127 can overshoot FLT_MAX */
            if (d > FLT_MAX) d = FLT_MAX;
            if (d < -FLT_MAX) d = -FLT_MAX;
            out[k + j] = (float)d;
        }
    }
    return OR_OK;
}

/* src/q4.c:22-35: legacy Q4_0 groups of 32, (nibble - 8) * fp16 scale. */
int or_q4_0_dot(const uint8_t *q, const float *x, size_t n, double *out) {
    if (!q || !x || !out || !n || n % 32) return OR_INVALID;
    double sum = 0;
    for (size_t k = 0; k < n; k += 32, q += 18) {
        float s = or_f16(le16(q));
        if (!isfinite(s)) return OR_NUMERIC;
        for (unsigned j = 0; j < 32; ++j) {
            int v = (j < 16 ? q[2 + j] & 15 : q[2 + j - 16] >> 4) - 8;
            sum += ((double)v * s) * x[k + j];
        }
    }
    if (!isfinite(sum)) return OR_NUMERIC;
    *out = sum;
    return OR_OK;
}

/* E2M1 magnitudes of src/native.c:10 (index = nibble). */
static const float kE2M1[16] = {0, .5f, 1, 1.5f, 2, 3, 4, 6, 0, -.5f, -1, -1.5f, -2, -3, -4, -6};
/* The same values doubled, as integers: the MXFP4 integer dot uses them. */
static const int kE2M1x2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* Q4_K 6-bit scale/min unpacking, src/native.c:17-18. */
static void q4k_scale_min(const uint8_t *s, unsigned g, unsigned *sc, unsigned *mi) {
    if (g < 4) {
        *sc = s[g] & 63;
        *mi = s[g + 4] & 63;
    } else {
        *sc = (s[g + 4] & 15) | ((unsigned)(s[g - 4] >> 6) << 4);
        *mi = (unsigned)(s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
    }
}

/* One decoded weight, the fp32 expressions of src/native.c:14-30.
 * Returns 0 for the reserved MXFP4 exponent 255 (caller reports NUMERIC). */
static int weight(const uint8_t *p, unsigned type, unsigned j, float *w) {
    if (type == OR_Q4_K) {
        const uint8_t *b = p + (size_t)(j / 256) * 144, *s = b + 4;
        unsigned g = j % 256 / 32, sc, mi;
        q4k_scale_min(s, g, &sc, &mi);
        float d = or_f16(le16(b)), m = or_f16(le16(b + 2));
        unsigned q = (b[16 + (g / 2) * 32 + j % 32] >> ((g % 2) * 4)) & 15;
        *w = (d * (float)sc) * (float)q - m * (float)mi;
    } else if (type == OR_MXFP4) {
        const uint8_t *b = p + (size_t)(j / 32) * 17;
        if (b[0] == 255) return 0;
        *w = ldexpf(1.0f, (int)b[0] - 127) * kE2M1[(b[1 + j % 16] >> ((j % 32 / 16) * 4)) & 15];
    } else {
        const uint8_t *b = p + (size_t)(j / 32) * 34;
        *w = or_f16(le16(b)) * (float)(int8_t)b[2 + j % 32];
    }
    return 1;
}

static int type_ok(unsigned type) { return type == OR_Q4_K || type == OR_MXFP4 || type == OR_Q8_0; }

/* src/native.c:7-37. */
int or_native_dot(const uint8_t *p, unsigned type, const float *x, unsigned n, double *out) {
    if (!p || !x || !out || !n || !type_ok(type) || n % (type == OR_Q4_K ? 256 : 32)) return OR_INVALID;
    double sum = 0;
    for (unsigned j = 0; j < n; ++j) {
        float w;
        if (!weight(p, type, j, &w)) return OR_NUMERIC;
        if (!isfinite(w) || !isfinite(x[j])) return OR_NUMERIC;
        sum += (double)w * x[j];
    }
    if (!isfinite(sum)) return OR_NUMERIC;
    *out = sum;
    return OR_OK;
}

int or_decode_row(const uint8_t *p, unsigned type, unsigned n, float *w) {
    if (!p || !w || !n || !type_ok(type) || n % (type == OR_Q4_K ? 256 : 32)) return OR_INVALID;
    int rc = OR_OK;
    for (unsigned j = 0; j < n; ++j) {
        if (!weight(p, type, j, &w[j])) {
            w[j] = NAN;
            rc = OR_NUMERIC;
        } else if (!isfinite(w[j])) {
            rc = OR_NUMERIC;
        }
    }
    return rc;
}

/* --------------------------------------------------------------- geometry */

/* src/native.h:19-21 */
size_t or_row_bytes(unsigned type, unsigned n) {
    if (type == OR_Q4_K) return n % 256 ? 0 : (size_t)n / 256 * 144;
    if (type == OR_MXFP4) return n % 32 ? 0 : (size_t)n / 32 * 17;
    if (type == OR_Q8_0) return n % 32 ? 0 : (size_t)n / 32 * 34;
    if (type == OR_Q4_0) return n % 32 ? 0 : (size_t)n / 32 * 18;
    return 0;
}
/* src/native.h:9-11 with run-time d and formats. */
size_t or_slice_bytes(unsigned d, unsigned gt, unsigned dt) {
    return 2 * OR_NEURONS * or_row_bytes(gt, d) + (size_t)d * or_row_bytes(dt, OR_NEURONS);
}
/* src/native.h:12-13 */
size_t or_shared_bytes(unsigned d) { return 3 * (size_t)d * 34; }
/* src/native.h:14 */
size_t or_layer_bytes(unsigned d, unsigned gt, unsigned dt) {
    return OR_ROUTED * or_slice_bytes(d, gt, dt) + or_shared_bytes(d);
}
/* src/backend.h:44-48: 513 slices of three Q4_0 projections. */
size_t or_legacy_layer_bytes(unsigned d) { return (size_t)(OR_ROUTED + 1) * 3 * OR_NEURONS * or_row_bytes(OR_Q4_0, d); }

/* -------------------------------------------------------------- reference */

/* backends/ref.c:37-40 */
static int narrow(double v, float *out) {
    if (!isfinite(v) || fabs(v) > FLT_MAX) return OR_NUMERIC;
    *out = (float)v;
    return OR_OK;
}

/* backends/ref.c:41-56 (token count bounded by OR_MAX_TOKENS instead of 8). */
static int validate_n(unsigned hidden, unsigned tokens, unsigned max_tokens, const uint16_t *expert,
                      const float *gate, const float *x) {
    if (!expert || !gate || !x || tokens < 1 || tokens > max_tokens || fegetround() != FE_TONEAREST)
        return OR_INVALID;
    for (unsigned t = 0; t < tokens; ++t) {
        const uint16_t *id = expert + (size_t)t * OR_TOPK;
        for (unsigned e = 0; e < OR_TOPK; ++e) {
            if (id[e] >= OR_ROUTED) return OR_INVALID;
            for (unsigned j = 0; j < e; ++j) if (id[j] == id[e]) return OR_INVALID;
        }
        for (unsigned e = 0; e < OR_ACTIVE; ++e) {
            float g = gate[(size_t)t * OR_ACTIVE + e];
            if (!isfinite(g)) return OR_NUMERIC;
            if (g < 0) return OR_INVALID;
        }
        for (unsigned j = 0; j < hidden; ++j) if (!isfinite(x[(size_t)t * hidden + j])) return OR_NUMERIC;
    }
    return OR_OK;
}
static int validate(unsigned hidden, unsigned tokens, const uint16_t *expert, const float *gate, const float *x) {
    return validate_n(hidden, tokens, OR_MAX_TOKENS, expert, gate, x);
}

static int model_ok(const or_model *m) {
    if (!m || !m->hidden || m->hidden % 256) return 0;
    if (!m->legacy && (!type_ok(m->gate_type) || (m->down_type != OR_MXFP4 && m->down_type != OR_Q8_0))) return 0;
    return 1;
}
static int any_loaded(const or_model *m) {
    for (unsigned b = 0; b < OR_BLOCKS; ++b) if (m->layer[b]) return 1;
    return 0;
}

/* backends/ref.c:57-98: token, routed experts in request order, shared expert
 * when its gate is nonzero, ascending blocks, dimension; double sums. */
int or_ref_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
               const float *x, float *y, int q8) {
    if (!model_ok(m) || !y) return OR_INVALID;
    const unsigned d = m->hidden;
    int rc = validate(d, tokens, expert, gate, x);
    if (rc) return rc;
    if (!any_loaded(m)) return OR_STATE;
    static double acc[8192];
    static float xq[8192], result[OR_MAX_TOKENS * 8192];
    if (d > 8192) return OR_INVALID;
    for (unsigned t = 0; t < tokens; ++t) {
        memset(acc, 0, d * sizeof(double));
        const float *xt = x + (size_t)t * d;
        if (q8) {
            rc = or_q8_activation(xt, xq, d);
            if (rc) return rc;
            xt = xq;
        }
        for (unsigned e = 0; e < OR_ACTIVE; ++e) {
            float g = gate[(size_t)t * OR_ACTIVE + e];
            if (e == OR_TOPK && g == 0) continue; /* backends/ref.c:68 */
            unsigned id = e == OR_TOPK ? OR_SHARED : expert[(size_t)t * OR_TOPK + e];
            for (unsigned b = 0; b < OR_BLOCKS; ++b) {
                if (!m->layer[b]) continue;
                unsigned in = id == OR_SHARED ? OR_Q8_0 : m->gate_type;
                unsigned down = id == OR_SHARED ? OR_Q8_0 : m->down_type;
                size_t proj, in_row, down_row;
                const uint8_t *p;
                if (m->legacy) {
                    in = down = OR_Q4_0;
                    in_row = or_row_bytes(OR_Q4_0, d);
                    proj = OR_NEURONS * in_row;
                    down_row = 18;
                    p = m->layer[b] + (size_t)id * 3 * proj;
                } else {
                    in_row = or_row_bytes(in, d);
                    proj = id == OR_SHARED ? (size_t)d * 34 : OR_NEURONS * in_row;
                    down_row = or_row_bytes(down, OR_NEURONS);
                    p = m->layer[b] + (size_t)id * or_slice_bytes(d, m->gate_type, m->down_type);
                }
                float h[OR_NEURONS];
                for (unsigned n = 0; n < OR_NEURONS; ++n) {
                    double ad, ud;
                    float a, u;
                    const uint8_t *gr = p + n * in_row, *ur = p + proj + n * in_row;
                    rc = m->legacy ? or_q4_0_dot(gr, xt, d, &ad) : or_native_dot(gr, in, xt, d, &ad);
                    if (rc) return rc;
                    rc = m->legacy ? or_q4_0_dot(ur, xt, d, &ud) : or_native_dot(ur, in, xt, d, &ud);
                    if (rc) return rc;
                    if (narrow(ad, &a) || narrow(ud, &u)) return OR_NUMERIC;
                    double sig = a >= 0 ? 1 / (1 + exp(-(double)a)) : exp((double)a) / (1 + exp((double)a));
                    if (narrow((double)a * sig * u, &h[n])) return OR_NUMERIC;
                }
                if (q8) {
                    rc = or_q8_activation(h, h, OR_NEURONS);
                    if (rc) return rc;
                }
                for (unsigned r = 0; r < d; ++r) {
                    double dot;
                    const uint8_t *row = p + 2 * proj + r * down_row;
                    rc = m->legacy ? or_q4_0_dot(row, h, OR_NEURONS, &dot) : or_native_dot(row, down, h, OR_NEURONS, &dot);
                    if (rc) return rc;
                    acc[r] += (double)g * dot;
                }
            }
        }
        for (unsigned r = 0; r < d; ++r)
            if (narrow(acc[r], &result[(size_t)t * d + r])) return OR_NUMERIC;
    }
    memcpy(y, result, (size_t)tokens * d * sizeof(float));
    return OR_OK;
}

/* --------------------------------------------- the AVX2 backend's arithmetic */

/* backends/avx2.c:184-203 (quantize8): one fp32 scale per `group` values,
 * amax / 127; the values x * (127 / amax) rounded to nearest even and
 * saturated to int8 (cvtps, packs); when s is not NULL the int16 sum of the
 * rounded values of each 32. */
static void avx2_quantize8(const float *x, unsigned n, unsigned group, int8_t *q, float *d, int16_t *s) {
    for (unsigned i = 0; i < n; i += group) {
        float amax = 0;
        for (unsigned j = 0; j < group; ++j) {
            const float a = fabsf(x[i + j]);
            if (a > amax) amax = a;
        }
        d[i / group] = amax / 127.0f;
        const float inv = amax != 0 ? 127.0f / amax : 0;
        for (unsigned j = 0; j < group; j += 32) {
            int sum = 0;
            for (unsigned k = 0; k < 32; ++k) {
                const int v = (int)nearbyintf(x[i + j + k] * inv);
                sum += v;
                q[i + j + k] = (int8_t)(v > 127 ? 127 : v < -128 ? -128 : v);
            }
            if (s) s[(i + j) / 32] = (int16_t)sum;
        }
    }
}

/* native_sum (backends/avx2.c:178-181): lanes i and i + 4 added, then two
 * horizontal adds. */
static float avx2_hsum8(const float v[8]) {
    const float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    return (a0 + a1) + (a2 + a3);
}

/* One Q4_K row against one token, as q4k_pair (backends/avx2.c:262-319)
 * computes each of its two rows: per super-block eight int32 lanes (lane k:
 * bytes 4k..4k+3 of every 32-byte nibble run, times the group scale), fmadd
 * into eight fp32 lanes with d * xd; the min terms as four int32 lanes
 * (mins of groups 2j, 2j+1 against the activation sums), fmadd with
 * dmin * xd; result native_sum(lanes) - ((m0 + m1) + (m2 + m3)). */
static float avx2_q4k_row(const uint8_t *row, const int8_t *xq, const float *xd, const int16_t *xs, unsigned d) {
    float acc[8] = {0}, mins[4] = {0};
    for (unsigned sb = 0; sb < d / 256; ++sb) {
        const uint8_t *b = row + (size_t)sb * 144;
        const float dd = or_f16(le16(b)), dm = or_f16(le16(b + 2));
        unsigned sc[8], mi[8];
        for (unsigned g = 0; g < 8; ++g) q4k_scale_min(b + 4, g, &sc[g], &mi[g]);
        int32_t is[8] = {0};
        for (unsigned gp = 0; gp < 4; ++gp) {
            const uint8_t *qs = b + 16 + gp * 32;
            const int8_t *xl = xq + sb * 256 + gp * 64, *xh = xl + 32;
            for (unsigned k = 0; k < 8; ++k) {
                int32_t lo = 0, hi = 0;
                for (unsigned i = 0; i < 4; ++i) {
                    lo += (qs[4 * k + i] & 15) * xl[4 * k + i];
                    hi += (qs[4 * k + i] >> 4) * xh[4 * k + i];
                }
                is[k] += (int32_t)sc[2 * gp] * lo + (int32_t)sc[2 * gp + 1] * hi;
            }
        }
        const float dxd = dd * xd[sb], mxd = dm * xd[sb];
        for (unsigned k = 0; k < 8; ++k) acc[k] = fmaf((float)is[k], dxd, acc[k]);
        for (unsigned j = 0; j < 4; ++j) {
            const int32_t mm = (int32_t)mi[2 * j] * xs[sb * 8 + 2 * j] + (int32_t)mi[2 * j + 1] * xs[sb * 8 + 2 * j + 1];
            mins[j] = fmaf((float)mm, mxd, mins[j]);
        }
    }
    return avx2_hsum8(acc) - ((mins[0] + mins[1]) + (mins[2] + mins[3]));
}

/* One Q8_0 row (reference bytes) against one token, the Q8_0 branch of row4
 * (backends/avx2.c:239-247): per 32-block eight int32 lanes of four products,
 * fmadd into eight fp32 lanes with d * xd of the super-block; a nonfinite
 * block scale is NUMERIC. */
static int avx2_q80_row(const uint8_t *row, const int8_t *xq, const float *xd, unsigned d, float *out) {
    float acc[8] = {0};
    for (unsigned blk = 0; blk < d / 32; ++blk) {
        const uint8_t *b = row + (size_t)blk * 34;
        const float sc = or_f16(le16(b));
        if (!isfinite(sc)) return OR_NUMERIC;
        const float s = sc * xd[blk / 8];
        for (unsigned j = 0; j < 8; ++j) {
            int32_t dot = 0;
            for (unsigned i = 0; i < 4; ++i) dot += (int8_t)b[2 + 4 * j + i] * xq[blk * 32 + 4 * j + i];
            acc[j] = fmaf((float)dot, s, acc[j]);
        }
    }
    *out = avx2_hsum8(acc);
    return OR_OK;
}

/* The SiLU product of native_job (backends/avx2.c:427-429), fp32 throughout.
 * libm_expf selects the C library's expf, as the backend calls it; otherwise
 * exp in double rounded once to fp32 (the correctly rounded value but for
 * double-rounding ties), the CUDA path's form. */
static float avx2_swiglu(float v, float u, int libm_expf) {
    const float e = libm_expf ? expf(-v) : (float)exp(-(double)v);
    return v / (1 + e) * u;
}

/* backends/avx2.c:615-715 (run) and :404-458 (native_job) with the default
 * build (no ranked or union mode): x quantized per 256; experts in the
 * order the tokens first name them (routed ranks 0-9, then the shared expert
 * when its gate is nonzero); jobs (block, expert) block-major over the loaded
 * blocks in ascending order, dealt round robin to `workers` workers; each
 * worker accumulates its jobs' down terms with fmadd into its own zeroed
 * output in job order, and y is the fp32 sum of the workers' outputs in
 * worker order.  Gate/up: Q4_K routed rows, Q8_0 shared rows; hidden slice
 * quantized per 32; down: MXFP4 routed, Q8_0 shared.  `order` (norder
 * entries) gives the blocks' load order, the backend's slot order
 * (backends/avx2.c:602-606); NULL: ascending. */
int or_avx2_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                const float *x, float *y, unsigned workers, int libm_expf, const uint8_t *order, unsigned norder) {
    if (!model_ok(m) || m->legacy || m->gate_type != OR_Q4_K || m->down_type != OR_MXFP4 || !y || !workers ||
        workers > 32)
        return OR_INVALID;
    const unsigned d = m->hidden;
    int rc = validate(d, tokens, expert, gate, x);
    if (rc) return rc;
    if (!any_loaded(m)) return OR_STATE;
    if (d > 8192) return OR_INVALID;
    unsigned blocks[OR_BLOCKS], nb = 0;
    if (order) { /* the backend's slots in load order: every loaded block once */
        unsigned seen = 0;
        for (unsigned i = 0; i < norder; ++i) {
            if (order[i] >= OR_BLOCKS || !m->layer[order[i]] || (seen >> order[i] & 1)) return OR_INVALID;
            seen |= 1u << order[i];
            blocks[nb++] = order[i];
        }
        for (unsigned b = 0; b < OR_BLOCKS; ++b) if (m->layer[b] && !(seen >> b & 1)) return OR_INVALID;
    } else {
        for (unsigned b = 0; b < OR_BLOCKS; ++b) if (m->layer[b]) blocks[nb++] = b;
    }
    /* experts in first-named order, per-token gates and token masks */
    enum { MAXE = OR_MAX_TOKENS * OR_ACTIVE };
    unsigned ids[MAXE], mask[MAXE], ne = 0;
    float eg[MAXE][OR_MAX_TOKENS];
    for (unsigned t = 0; t < tokens; ++t)
        for (unsigned j = 0; j < OR_ACTIVE; ++j) {
            const float g = gate[(size_t)t * OR_ACTIVE + j];
            if (j == OR_TOPK && g == 0) continue;
            const unsigned id = j == OR_TOPK ? OR_SHARED : expert[(size_t)t * OR_TOPK + j];
            unsigned e = 0;
            while (e < ne && ids[e] != id) ++e;
            if (e == ne) { ids[ne] = id; mask[ne] = 0; ++ne; }
            mask[e] |= 1u << t;
            eg[e][t] = g;
        }
    int8_t *xq = malloc((size_t)tokens * d);
    float *xd = malloc(sizeof(float) * tokens * (d / 256));
    int16_t *xs = malloc(sizeof(int16_t) * tokens * (d / 32));
    float *out = calloc((size_t)workers * tokens * d, sizeof(float));
    if (!xq || !xd || !xs || !out) { rc = OR_INVALID; goto done; }
    for (unsigned t = 0; t < tokens; ++t)
        avx2_quantize8(x + (size_t)t * d, d, 256, xq + (size_t)t * d, xd + t * (d / 256), xs + t * (d / 32));
    const size_t slice = or_slice_bytes(d, OR_Q4_K, OR_MXFP4), row = or_row_bytes(OR_Q4_K, d);
    const size_t srow = or_row_bytes(OR_Q8_0, d);
    const unsigned jobs = nb * ne;
    for (unsigned w = 0; w < workers; ++w)
        for (unsigned index = w; index < jobs; index += workers) {
            const unsigned e = index % ne, id = ids[e];
            const int shared = id == OR_SHARED;
            const uint8_t *p = m->layer[blocks[index / ne]] + (size_t)id * slice;
            const size_t in_row = shared ? srow : row, proj = OR_NEURONS * in_row;
            float *o = out + (size_t)w * tokens * d;
            for (unsigned t = 0; t < tokens; ++t) {
                if (!(mask[e] >> t & 1)) continue;
                const int8_t *q = xq + (size_t)t * d;
                float h[OR_NEURONS], md;
                int8_t mid[OR_NEURONS];
                for (unsigned n = 0; n < OR_NEURONS; ++n) {
                    float a, u;
                    if (shared) {
                        if (avx2_q80_row(p + n * in_row, q, xd + t * (d / 256), d, &a) ||
                            avx2_q80_row(p + proj + n * in_row, q, xd + t * (d / 256), d, &u)) {
                            rc = OR_NUMERIC;
                            goto done;
                        }
                    } else {
                        a = avx2_q4k_row(p + n * in_row, q, xd + t * (d / 256), xs + t * (d / 32), d);
                        u = avx2_q4k_row(p + proj + n * in_row, q, xd + t * (d / 256), xs + t * (d / 32), d);
                    }
                    h[n] = avx2_swiglu(a, u, libm_expf);
                }
                for (unsigned n = 0; n < OR_NEURONS; ++n)
                    if (!isfinite(h[n])) { rc = OR_NUMERIC; goto done; }
                avx2_quantize8(h, OR_NEURONS, OR_NEURONS, mid, &md, NULL);
                const float c = md * eg[e][t];
                const uint8_t *down = p + 2 * proj;
                for (unsigned r = 0; r < d; ++r) {
                    int32_t sum = 0;
                    float yr;
                    if (shared) {
                        const uint8_t *b = down + (size_t)r * 34;
                        const float sc = or_f16(le16(b));
                        if (!isfinite(sc)) { rc = OR_NUMERIC; goto done; }
                        for (unsigned n = 0; n < OR_NEURONS; ++n) sum += (int8_t)b[2 + n] * mid[n];
                        yr = (float)sum * sc;
                    } else {
                        /* down8_mxfp4 (backends/avx2.c:331-362): the scale
                         * byte e gives 2^(e-127) (e = 0: 2^-127), halved */
                        const uint8_t *b = down + (size_t)r * 17;
                        const uint32_t bits = b[0] ? (uint32_t)b[0] << 23 : 0x00400000u;
                        float rs;
                        memcpy(&rs, &bits, sizeof rs);
                        rs *= .5f;
                        for (unsigned j = 0; j < 16; ++j)
                            sum += kE2M1x2[b[1 + j] & 15] * mid[j] + kE2M1x2[b[1 + j] >> 4] * mid[j + 16];
                        yr = (float)sum * rs;
                    }
                    o[(size_t)t * d + r] = fmaf(yr, c, o[(size_t)t * d + r]);
                }
            }
        }
    for (unsigned t = 0; t < tokens; ++t)
        for (unsigned r = 0; r < d; ++r) {
            float v = 0;
            for (unsigned w = 0; w < workers; ++w) v += out[((size_t)w * tokens + t) * d + r];
            if (!isfinite(v)) { rc = OR_NUMERIC; goto done; }
            out[(size_t)t * d + r] = v;  /* worker 0's row is no longer read */
        }
    memcpy(y, out, (size_t)tokens * d * sizeof(float));
done:
    free(xq); free(xd); free(xs); free(out);
    return rc;
}

/* ------------------------------------------------------ GPU Q8 arithmetic */

/* Integer dot of one 32-weight block against 32 int8 activations. */
static int32_t idot_block(const uint8_t *p, unsigned type, unsigned blk, const int8_t *v) {
    int32_t s = 0;
    if (type == OR_Q4_K) {
        const uint8_t *b = p + (size_t)(blk / 8) * 144;
        unsigned g = blk % 8;
        for (unsigned j = 0; j < 32; ++j) s += (int32_t)((b[16 + (g / 2) * 32 + j] >> ((g % 2) * 4)) & 15) * v[j];
    } else if (type == OR_MXFP4) {
        const uint8_t *b = p + (size_t)blk * 17;
        for (unsigned j = 0; j < 32; ++j) s += kE2M1x2[(b[1 + j % 16] >> ((j / 16) * 4)) & 15] * v[j];
    } else {
        const uint8_t *b = p + (size_t)blk * 34;
        for (unsigned j = 0; j < 32; ++j) s += (int32_t)(int8_t)b[2 + j] * v[j];
    }
    return s;
}

int or_block_idots(const uint8_t *p, unsigned type, unsigned n, const int8_t *v, int32_t *out) {
    if (!p || !v || !out || !n || !type_ok(type) || n % (type == OR_Q4_K ? 256 : 32)) return OR_INVALID;
    for (unsigned b = 0; b < n / 32; ++b) out[b] = idot_block(p, type, b, v + 32 * b);
    return OR_OK;
}

/* Scale of block blk for the integer path: fp16 d (Q8_0) or 2^(e-128)
 * (MXFP4: the E2M1 table is doubled).  0 when the scale is not finite. */
static int block_scale(const uint8_t *p, unsigned type, unsigned blk, float *s) {
    if (type == OR_MXFP4) {
        unsigned e = p[(size_t)blk * 17];
        if (e == 255) return 0;
        *s = ldexpf(1.0f, (int)e - 128);
        return 1;
    }
    *s = or_f16(le16(p + (size_t)blk * 34));
    return isfinite(*s);
}

/* One token's quantized activations as the GPU holds them.  The reference
 * multiplies each weight by the dequantized activation X_j = fl32(v_j * s)
 * (src/q4.c:54-58).  With s = M * 2^E (M the 24-bit significand of the
 * group's scale, E the exponent of its last bit), X_j - v_j * s = r_j * 2^E
 * for an integer r_j with |r_j| <= 64 (the product has at most 31
 * significant bits, so rounding drops at most seven).  Hence every block term
 * of the reference's sum is an exact combination of two integer dots, one
 * against v and one against r. */
typedef struct {
    unsigned d;
    const int8_t *q;     /* [d] v */
    const int8_t *r;     /* [d] rounding residuals of the dequantized values */
    const float *scale;  /* [d/64] s */
    const double *ulp;   /* [d/64] 2^E */
    const int32_t *sum;  /* [d/32] sums of v per 32 */
    const int32_t *rsum; /* [d/32] sums of r per 32 */
} qx;

/* 2^E for a group scale s (E = the exponent of s's last significand bit). */
static double scale_ulp(float s) {
    uint32_t bits;
    memcpy(&bits, &s, sizeof bits);
    int ef = (int)((bits >> 23) & 255u);
    return ldexp(1.0, (ef ? ef : 1) - 150);
}

/* A group scale s as M * 2^E: M its 24-bit significand (no hidden bit for a
 * subnormal), E the exponent of its last bit. */
static void scale_parts(float s, int64_t *M, int *E) {
    uint32_t bits;
    memcpy(&bits, &s, sizeof bits);
    const int ef = (int)((bits >> 23) & 255u);
    *M = ef ? (int64_t)((bits & 0x7fffffu) | 0x800000u) : (int64_t)(bits & 0x7fffffu);
    *E = (ef ? ef : 1) - 150;
}

/* The residuals r_j of one token (see qx), dequantizing exactly as
 * src/q4.c:54-58 does (the FLT_MAX cap included). */
static void q8_residuals(const int8_t *v, const float *scale, unsigned d, int8_t *r) {
    for (unsigned j = 0; j < d; ++j) {
        const float s = scale[j / 64];
        double deq = (double)v[j] * s;
        if (deq > FLT_MAX) deq = FLT_MAX;
        if (deq < -FLT_MAX) deq = -FLT_MAX;
        const float X = (float)deq;
        r[j] = (int8_t)(((double)X - (double)v[j] * s) / scale_ulp(s));
    }
}

/* The gate or up dot of one row as the GPU forms it, which is the reference's
 * sum of w_j * X_j carried out exactly up to double rounding.  Eight lanes
 * share the row; lane L takes the 256-element spans (four x groups of 64: a
 * Q4_K super-block, eight MXFP4 / Q8_0 blocks) q = L, L+8, ...; then a
 * butterfly over the eight lanes (xor 4, 2, 1), in double.
 *   Q4_K super-block (d, dmin; sub-block scales sc, mins mi; w = d*sc*q -
 *   dmin*mi, the reference's fp32 weight when that subtraction is exact):
 *     per group p (sub-blocks k = 2gp, 2gp+1; I_k = sum q*v, R_k = sum q*r,
 *     V_k = sum v, RS_k = sum r):
 *       K1 = sc0*I0 + sc1*I1, K3 = sc0*R0 + sc1*R1,
 *       K2 = mi0*V0 + mi1*V1, K4 = mi0*RS0 + mi1*RS1  (exact integers)
 *       PP = fma(s, K1, PP); PP = fma(2^E, K3, PP)
 *       QQ = fma(s, K2, QQ); QQ = fma(2^E, K4, QQ)
 *     acc = fma(d, PP, acc); acc = fma(-dmin, QQ, acc)
 *   MXFP4 / Q8_0 block b of group p (c = 2^(e-128) with the doubled E2M1
 *   table, or the fp16 scale):
 *       acc = fma(c, fma(s, I_b, 2^E * R_b), acc)   (the inner value is exact)
 * Returns OR_NUMERIC on a nonfinite scale. */
enum { PORT_ROW_LANES = 8 };
static int lane_dot(const uint8_t *row, unsigned type, const qx *x, double *out) {
    double lane[PORT_ROW_LANES];
    const unsigned spans = x->d / 256;
    for (unsigned L = 0; L < PORT_ROW_LANES; ++L) {
        double acc = 0;
        for (unsigned q = L; q < spans; q += PORT_ROW_LANES) {
            if (type == OR_Q4_K) {
                const uint8_t *b = row + (size_t)q * 144;
                const float d = or_f16(le16(b)), dm = or_f16(le16(b + 2));
                if (!isfinite(d) || !isfinite(dm)) return OR_NUMERIC;
                double PP = 0, QQ = 0;
                for (unsigned gp = 0; gp < 4; ++gp) {
                    const unsigned p = 4 * q + gp;
                    const int8_t *v = x->q + 64 * p, *r = x->r + 64 * p;
                    unsigned sc0, mi0, sc1, mi1;
                    q4k_scale_min(b + 4, 2 * gp, &sc0, &mi0);
                    q4k_scale_min(b + 4, 2 * gp + 1, &sc1, &mi1);
                    int32_t i0 = 0, i1 = 0, r0 = 0, r1 = 0;
                    for (unsigned j = 0; j < 32; ++j) {
                        const uint8_t byte = b[16 + 32 * gp + j];
                        i0 += (int32_t)(byte & 15) * v[j];
                        i1 += (int32_t)(byte >> 4) * v[32 + j];
                        r0 += (int32_t)(byte & 15) * r[j];
                        r1 += (int32_t)(byte >> 4) * r[32 + j];
                    }
                    const int32_t K1 = (int32_t)sc0 * i0 + (int32_t)sc1 * i1, K3 = (int32_t)sc0 * r0 + (int32_t)sc1 * r1;
                    const int32_t K2 = (int32_t)mi0 * x->sum[2 * p] + (int32_t)mi1 * x->sum[2 * p + 1];
                    const int32_t K4 = (int32_t)mi0 * x->rsum[2 * p] + (int32_t)mi1 * x->rsum[2 * p + 1];
                    int64_t M;
                    int E;
                    scale_parts(x->scale[p], &M, &E);
                    const double t = x->ulp[p];
                    /* s*K1 + 2^E*K3 = (M*K1 + K3) * 2^E: an exact integer, one fma */
                    PP = fma((double)(M * K1 + K3), t, PP);
                    QQ = fma((double)(M * K2 + K4), t, QQ);
                }
                acc = fma((double)d, PP, acc);
                acc = fma(-(double)dm, QQ, acc);
            } else {
                for (unsigned gp = 0; gp < 4; ++gp) {
                    const unsigned p = 4 * q + gp;
                    const double t = x->ulp[p];
                    for (unsigned k = 0; k < 2; ++k) {
                        const unsigned blk = 2 * p + k;
                        float c;
                        if (!block_scale(row, type, blk, &c)) return OR_NUMERIC;
                        const int32_t I = idot_block(row, type, blk, x->q + 32 * blk);
                        const int32_t R = idot_block(row, type, blk, x->r + 32 * blk);
                        int64_t M;
                        int E;
                        scale_parts(x->scale[p], &M, &E);
                        /* c * (s*I + 2^E*R) = (M*I + R) * (c * 2^E): exact integer
                         * times an exact double, one fma */
                        acc = fma((double)(M * I + R), (double)c * t, acc);
                    }
                }
            }
        }
        lane[L] = acc;
    }
    for (unsigned off = PORT_ROW_LANES / 2; off; off >>= 1) {
        double next[PORT_ROW_LANES];
        for (unsigned L = 0; L < PORT_ROW_LANES; ++L) next[L] = lane[L] + lane[L ^ off];
        memcpy(lane, next, sizeof lane);
    }
    *out = lane[0];
    return OR_OK;
}

/* Down row r of a slice (32 neurons, one block) against int8 hidden values:
 * c = scale * (float)I, exact for MXFP4. */
static int down_term(const uint8_t *down, unsigned type, unsigned r, const int8_t *v, float *c) {
    float s;
    if (!block_scale(down, type, r, &s)) return 0;
    *c = s * (float)idot_block(down, type, r, v);
    return 1;
}

enum { PORT_SPLIT = 4 }; /* down-projection partial sums per row (kernel DN_SPLIT) */

int or_port_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                const float *x, float *y, float *h, size_t h_cap, size_t *h_count) {
    if (!model_ok(m) || m->legacy || !y) return OR_INVALID;
    const unsigned d = m->hidden;
    if (d % 512 || d > 8192) return OR_INVALID;
    int rc = validate(d, tokens, expert, gate, x);
    if (rc) return rc;
    if (!any_loaded(m)) return OR_STATE;

    /* Plan: unique routed experts in first-appearance order (token-major),
     * then the shared expert if any token gives it a nonzero gate. */
    unsigned uid[OR_MAX_TOKENS * OR_TOPK + 1], umask[OR_MAX_TOKENS * OR_TOPK + 1], U = 0;
    float ugate[OR_MAX_TOKENS * OR_TOPK + 1][OR_MAX_TOKENS];
    memset(ugate, 0, sizeof ugate);
    for (unsigned t = 0; t < tokens; ++t)
        for (unsigned e = 0; e < OR_TOPK; ++e) {
            unsigned id = expert[t * OR_TOPK + e], u = 0;
            while (u < U && uid[u] != id) ++u;
            if (u == U) { uid[U] = id; umask[U] = 0; ++U; }
            umask[u] |= 1u << t;
            ugate[u][t] = gate[t * OR_ACTIVE + e];
        }
    unsigned shared_mask = 0;
    for (unsigned t = 0; t < tokens; ++t) if (gate[t * OR_ACTIVE + OR_TOPK] != 0) shared_mask |= 1u << t;
    if (shared_mask) {
        uid[U] = OR_SHARED; umask[U] = shared_mask;
        for (unsigned t = 0; t < tokens; ++t) ugate[U][t] = gate[t * OR_ACTIVE + OR_TOPK];
        ++U;
    }
    unsigned blocks[OR_BLOCKS], S = 0;
    for (unsigned b = 0; b < OR_BLOCKS; ++b) if (m->layer[b]) blocks[S++] = b;

    /* Activations: int8 per 64-group scale, per-32 sums. */
    static int8_t q[OR_MAX_TOKENS][8192], res[OR_MAX_TOKENS][8192];
    static float scale[OR_MAX_TOKENS][128];
    static double ulp[OR_MAX_TOKENS][128];
    static int32_t sums[OR_MAX_TOKENS][256], rsums[OR_MAX_TOKENS][256];
    qx xs[OR_MAX_TOKENS];
    for (unsigned t = 0; t < tokens; ++t) {
        rc = or_q8_quantize(x + (size_t)t * d, d, q[t], scale[t]);
        if (rc) return rc;
        q8_residuals(q[t], scale[t], d, res[t]);
        for (unsigned k = 0; k < d / 64; ++k) ulp[t][k] = scale_ulp(scale[t][k]);
        for (unsigned k = 0; k < d / 32; ++k) {
            int32_t s = 0, sr = 0;
            for (unsigned j = 0; j < 32; ++j) {
                s += q[t][32 * k + j];
                sr += res[t][32 * k + j];
            }
            sums[t][k] = s;
            rsums[t][k] = sr;
        }
        xs[t] = (qx){d, q[t], res[t], scale[t], ulp[t], sums[t], rsums[t]};
    }

    size_t need = (size_t)U * S * tokens * OR_NEURONS;
    if (h_count) *h_count = need;
    if (h && h_cap < need) return OR_INVALID;
    if (h) memset(h, 0, need * sizeof(float));

    /* part[u][t][r]: expert u's down-projection partial for token t. */
    float *part = calloc((size_t)U * tokens * d, sizeof(float));
    if (!part) return OR_INVALID;
    const size_t slice = or_slice_bytes(d, m->gate_type, m->down_type);
    for (unsigned u = 0; u < U; ++u) {
        const int shared = uid[u] == OR_SHARED;
        const unsigned in = shared ? OR_Q8_0 : m->gate_type, down = shared ? OR_Q8_0 : m->down_type;
        const size_t in_row = or_row_bytes(in, d), proj = shared ? (size_t)d * 34 : OR_NEURONS * in_row;
        /* Every referenced block is checked, whatever the gate (src/backend.h:58-59). */
        for (unsigned si = 0; si < S; ++si) {
            const uint8_t *p = m->layer[blocks[si]] + (size_t)uid[u] * slice;
            for (unsigned r = 0; r < d; ++r) {
                float s;
                if (!block_scale(p + 2 * proj, down, r, &s)) { rc = OR_NUMERIC; goto done; }
            }
        }
        for (unsigned t = 0; t < tokens; ++t) {
            if (!(umask[u] >> t & 1)) continue;
            static int8_t hv[OR_BLOCKS][OR_NEURONS];
            float gs[OR_BLOCKS];
            for (unsigned si = 0; si < S; ++si) {
                const uint8_t *p = m->layer[blocks[si]] + (size_t)uid[u] * slice;
                float hs[OR_NEURONS], hsc;
                for (unsigned n = 0; n < OR_NEURONS; ++n) {
                    double ad, ud;
                    float a, uu;
                    rc = lane_dot(p + n * in_row, in, &xs[t], &ad);
                    if (rc) goto done;
                    rc = lane_dot(p + proj + n * in_row, in, &xs[t], &ud);
                    if (rc) goto done;
                    if (narrow(ad, &a) || narrow(ud, &uu)) { rc = OR_NUMERIC; goto done; }
                    double sig = a >= 0 ? 1 / (1 + exp(-(double)a)) : exp((double)a) / (1 + exp((double)a));
                    if (narrow((double)a * sig * uu, &hs[n])) { rc = OR_NUMERIC; goto done; }
                }
                if (h) memcpy(h + (((size_t)u * S + si) * tokens + t) * OR_NEURONS, hs, sizeof hs);
                rc = or_q8_quantize(hs, OR_NEURONS, hv[si], &hsc);
                if (rc) goto done;
                gs[si] = hsc * ugate[u][t];
            }
            for (unsigned r = 0; r < d; ++r) {
                float split[PORT_SPLIT] = {0};
                for (unsigned si = 0; si < S; ++si) {
                    const uint8_t *p = m->layer[blocks[si]] + (size_t)uid[u] * slice;
                    float c;
                    if (!down_term(p + 2 * proj, down, r, hv[si], &c)) { rc = OR_NUMERIC; goto done; }
                    split[si % PORT_SPLIT] = fmaf(c, gs[si], split[si % PORT_SPLIT]);
                }
                float sum = split[0];
                for (unsigned k = 1; k < PORT_SPLIT; ++k) sum = sum + split[k];
                part[((size_t)u * tokens + t) * d + r] = sum;
            }
        }
    }
    /* Each token sums its routed experts in its own request order, then the
     * shared expert, so its result does not depend on the rest of the burst. */
    static float out[OR_MAX_TOKENS * 8192];
    for (unsigned t = 0; t < tokens; ++t)
        for (unsigned r = 0; r < d; ++r) {
            float acc = 0;
            for (unsigned e = 0; e < OR_TOPK; ++e) {
                unsigned u = 0;
                while (uid[u] != expert[t * OR_TOPK + e]) ++u;
                acc = acc + part[((size_t)u * tokens + t) * d + r];
            }
            if (shared_mask >> t & 1) acc = acc + part[((size_t)(U - 1) * tokens + t) * d + r];
            if (!isfinite(acc)) { rc = OR_NUMERIC; goto done; }
            out[(size_t)t * d + r] = acc;
        }
    memcpy(y, out, (size_t)tokens * d * sizeof(float));
done:
    free(part);
    return rc;
}

/* ------------------------------------------------- GPU prefill arithmetic */

/* The batched (prefill) path of the CUDA backend, for bursts of up to
 * OR_MAX_PREFILL tokens with MXFP4 gate/up rows, MXFP4 or Q8_0 down rows and
 * no shared expert (the backend runs other requests through the decode
 * arithmetic, or_port_run, in bursts of 16).  Each token's result depends only
 * on its own row:
 *   x: per-64 Q8 quantization (src/q4.c:37-61), as or_port_run;
 *   gate/up dot of neuron n: the reference's sum of w_j * fl32(v_j * s)
 *     exactly up to double rounding (the tensor cores give the int32 block
 *     dots I_b against the int8 activations v and R_b against their
 *     dequantization residuals r): over the row's 32-weight blocks b in
 *     order, with the group scale s = M * 2^E and the block scale 2^(e-128)
 *     of the doubled E2M1 table, Z = M * I_b + R_b (an exact integer) and
 *     acc = fma((double)Z, 2^(e - 128 + E), acc), narrowed to fp32;
 *   h = SwiGLU in double (backends/ref.c:81-83), Q8 per 32 (hq, hscale);
 *   expert partial row r: over the loaded blocks s in ascending order,
 *     acc = fmaf((float)I_{s,r} * hscale_s, wscale_{s,r}, acc);
 *   y[t][r]: over the token's ten routed experts in request order,
 *     acc = fmaf(gate, partial, acc).
 * Pairs (expert, token) are numbered expert-major, tokens ascending;
 * hq [pair][block][32] and hs [pair][block] receive the hidden values when not
 * NULL (*pairs gets the pair count). */
static int validate_n(unsigned hidden, unsigned tokens, unsigned max_tokens, const uint16_t *expert,
                      const float *gate, const float *x);

int or_prefill_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                   const float *x, float *y, int8_t *hq, float *hs, size_t pair_cap, size_t *pairs) {
    if (!model_ok(m) || m->legacy || !y || (m->gate_type != OR_MXFP4 && m->gate_type != OR_Q4_K) ||
        m->down_type == OR_Q4_K)
        return OR_INVALID;
    const unsigned d = m->hidden, gt = m->gate_type;
    if (d % 512 || d > 8192) return OR_INVALID;
    int rc = validate_n(d, tokens, OR_MAX_PREFILL, expert, gate, x);
    if (rc) return rc;
    if (!any_loaded(m)) return OR_STATE;
    unsigned blocks[OR_BLOCKS], S = 0;
    for (unsigned b = 0; b < OR_BLOCKS; ++b) if (m->layer[b]) blocks[S++] = b;
    const unsigned dt = m->down_type, nb = d / 32;
    const size_t slice = or_slice_bytes(d, gt, dt), in_row = or_row_bytes(gt, d);
    const size_t proj = OR_NEURONS * in_row, down_row = or_row_bytes(dt, OR_NEURONS);
    /* the shared expert's slice (Q8_0 gate/up and down rows, src/native.h:1-3) */
    const size_t sh_row = or_row_bytes(OR_Q8_0, d), sh_proj = (size_t)d * 34;

    /* pairs, expert-major; the shared expert (512) last, for the tokens whose
     * shared gate is not zero */
    const unsigned PMAX = tokens * OR_ACTIVE;
    unsigned *pair_t = malloc(sizeof(unsigned) * PMAX), *pair_e = malloc(sizeof(unsigned) * PMAX);
    unsigned *slot_pair = malloc(sizeof(unsigned) * PMAX);
    int8_t *q = malloc((size_t)tokens * d), *res = malloc((size_t)tokens * d);
    int8_t *hv = malloc((size_t)PMAX * S * OR_NEURONS);
    float *xsc = malloc(sizeof(float) * tokens * (d / 64)), *hsc = malloc(sizeof(float) * PMAX * S);
    float *part = malloc(sizeof(float) * (size_t)PMAX * d), *out = malloc(sizeof(float) * (size_t)tokens * d);
    rc = OR_INVALID;
    if (!pair_t || !pair_e || !slot_pair || !q || !res || !hv || !xsc || !hsc || !part || !out) goto done;
    unsigned P = 0;
    for (unsigned e = 0; e < OR_ROUTED; ++e)
        for (unsigned t = 0; t < tokens; ++t)
            for (unsigned j = 0; j < OR_TOPK; ++j)
                if (expert[(size_t)t * OR_TOPK + j] == e) {
                    pair_t[P] = t; pair_e[P] = e; slot_pair[t * OR_ACTIVE + j] = P; ++P;
                }
    for (unsigned t = 0; t < tokens; ++t) {
        slot_pair[t * OR_ACTIVE + OR_TOPK] = ~0u;
        if (gate[(size_t)t * OR_ACTIVE + OR_TOPK] != 0) {
            pair_t[P] = t; pair_e[P] = OR_SHARED; slot_pair[t * OR_ACTIVE + OR_TOPK] = P; ++P;
        }
    }
    if (pairs) *pairs = P;
    if ((hq || hs) && pair_cap < P) goto done;
    for (unsigned t = 0; t < tokens; ++t) {
        rc = or_q8_quantize(x + (size_t)t * d, d, q + (size_t)t * d, xsc + (size_t)t * (d / 64));
        if (rc) goto done;
        q8_residuals(q + (size_t)t * d, xsc + (size_t)t * (d / 64), d, res + (size_t)t * d);
    }
    /* Every referenced block scale must be finite, whatever the gate. */
    rc = OR_NUMERIC;
    for (unsigned p = 0; p < P; ++p)
        for (unsigned si = 0; si < S; ++si) {
            const uint8_t *sl = m->layer[blocks[si]] + (size_t)pair_e[p] * slice;
            float sc;
            if (pair_e[p] == OR_SHARED) {
                for (unsigned n = 0; n < 2 * OR_NEURONS; ++n)
                    for (unsigned b = 0; b < nb; ++b)
                        if (!block_scale(sl + n * sh_row, OR_Q8_0, b, &sc)) goto done;
                for (unsigned r = 0; r < d; ++r)
                    if (!block_scale(sl + 2 * sh_proj, OR_Q8_0, r, &sc)) goto done;
                continue;
            }
            for (unsigned n = 0; n < 2 * OR_NEURONS; ++n)
                for (unsigned b = 0; b < nb; ++b) {
                    if (gt == OR_MXFP4 && !block_scale(sl + n * in_row, OR_MXFP4, b, &sc)) goto done;
                    if (gt == OR_Q4_K && b % 8 == 0) {  /* d and dmin of each super-block */
                        const uint8_t *sb = sl + n * in_row + (size_t)(b / 8) * 144;
                        if (!isfinite(or_f16(le16(sb))) || !isfinite(or_f16(le16(sb + 2)))) goto done;
                    }
                }
            for (unsigned r = 0; r < d; ++r)
                if (!block_scale(sl + 2 * proj + r * down_row, dt, 0, &sc)) goto done;
        }
    for (unsigned p = 0; p < P; ++p) {
        const unsigned t = pair_t[p];
        const int8_t *qt = q + (size_t)t * d, *rt = res + (size_t)t * d;
        const float *xs = xsc + (size_t)t * (d / 64);
        for (unsigned si = 0; si < S; ++si) {
            const uint8_t *sl = m->layer[blocks[si]] + (size_t)pair_e[p] * slice;
            float h[OR_NEURONS];
            for (unsigned n = 0; n < OR_NEURONS; ++n) {
                float gu[2];
                double gd[2];
                for (unsigned w = 0; w < 2; ++w) {
                    const int sh = pair_e[p] == OR_SHARED;
                    const uint8_t *row = sh ? sl + (w ? sh_proj : 0) + n * sh_row : sl + (w ? proj : 0) + n * in_row;
                    double acc = 0;
                    if (sh) {
                        /* Q8_0 rows of the shared expert: each block's exact
                         * integer Z = M*I + R times the exact double d * 2^E */
                        for (unsigned b = 0; b < nb; ++b) {
                            float db;
                            block_scale(row, OR_Q8_0, b, &db);
                            const int32_t I = idot_block(row, OR_Q8_0, b, qt + 32 * b);
                            const int32_t R = idot_block(row, OR_Q8_0, b, rt + 32 * b);
                            int64_t M;
                            int E;
                            scale_parts(xs[b / 2], &M, &E);
                            acc = fma((double)(M * I + R), (double)db * ldexp(1.0, E), acc);
                        }
                    } else if (gt == OR_Q4_K) {
                        /* Q4_K rows, one 256-weight super-block a chunk, its four
                         * 64-weight x groups in order: with K1 = sc0*I0 + sc1*I1,
                         * K3 = sc0*R0 + sc1*R1 (dots against v and r),
                         * K2 = mi0*V0 + mi1*V1, K4 = mi0*RS0 + mi1*RS1 (the blocks'
                         * sums of v and r) and s = M * 2^E, the group's term of the
                         * reference's sum of w * fl32(v * s) (src/native.c:14-30,
                         * backends/ref.c:74-79) is (M*K1 + K3) * d * 2^E -
                         * (M*K2 + K4) * dmin * 2^E, both products exact. */
                        for (unsigned k = 0; k < d / 256; ++k) {
                            const uint8_t *sb = row + (size_t)k * 144;
                            const double dd = or_f16(le16(sb)), dm = or_f16(le16(sb + 2));
                            for (unsigned gp = 0; gp < 4; ++gp) {
                                const unsigned g = 4 * k + gp;
                                const int8_t *v = qt + 64 * g, *r = rt + 64 * g;
                                unsigned sc0, mi0, sc1, mi1;
                                q4k_scale_min(sb + 4, 2 * gp, &sc0, &mi0);
                                q4k_scale_min(sb + 4, 2 * gp + 1, &sc1, &mi1);
                                int32_t i0 = 0, i1 = 0, r0 = 0, r1 = 0, v0 = 0, v1 = 0, s0 = 0, s1 = 0;
                                for (unsigned j = 0; j < 32; ++j) {
                                    const uint8_t byte = sb[16 + 32 * gp + j];
                                    i0 += (int32_t)(byte & 15) * v[j];
                                    i1 += (int32_t)(byte >> 4) * v[32 + j];
                                    r0 += (int32_t)(byte & 15) * r[j];
                                    r1 += (int32_t)(byte >> 4) * r[32 + j];
                                    v0 += v[j]; v1 += v[32 + j];
                                    s0 += r[j]; s1 += r[32 + j];
                                }
                                const int64_t K1 = (int64_t)sc0 * i0 + (int64_t)sc1 * i1;
                                const int64_t K3 = (int64_t)sc0 * r0 + (int64_t)sc1 * r1;
                                const int64_t K2 = (int64_t)mi0 * v0 + (int64_t)mi1 * v1;
                                const int64_t K4 = (int64_t)mi0 * s0 + (int64_t)mi1 * s1;
                                int64_t M;
                                int E;
                                scale_parts(xs[g], &M, &E);
                                const double P = ldexp(1.0, E);
                                acc = fma((double)(M * K1 + K3), dd * P, acc);
                                acc = fma((double)(M * K2 + K4), -dm * P, acc);
                            }
                        }
                    } else for (unsigned b = 0; b < nb; ++b) {
                        const int e = row[(size_t)b * 17];
                        const int32_t I = idot_block(row, OR_MXFP4, b, qt + 32 * b);
                        const int32_t R = idot_block(row, OR_MXFP4, b, rt + 32 * b);
                        int64_t M;
                        int E;
                        scale_parts(xs[b / 2], &M, &E);
                        const int64_t Z = M * I + R;  /* exact: |Z| < 2^47 */
                        acc = fma((double)Z, ldexp(1.0, e - 128 + E), acc);
                    }
                    gd[w] = acc;
                }
                if (narrow(gd[0], &gu[0]) || narrow(gd[1], &gu[1])) goto done;
                const double a = gu[0];
                const double sig = a >= 0 ? 1 / (1 + exp(-a)) : exp(a) / (1 + exp(a));
                if (narrow(a * sig * gu[1], &h[n])) goto done;
            }
            int8_t *hp = hv + ((size_t)p * S + si) * OR_NEURONS;
            if (or_q8_quantize(h, OR_NEURONS, hp, hsc + (size_t)p * S + si)) goto done;
        }
        const int shp = pair_e[p] == OR_SHARED;
        const unsigned pdt = shp ? OR_Q8_0 : dt;
        const size_t pdrow = shp ? 34 : down_row, pproj = shp ? sh_proj : proj;
        for (unsigned r = 0; r < d; ++r) {
            float acc = 0;
            for (unsigned si = 0; si < S; ++si) {
                const uint8_t *down = m->layer[blocks[si]] + (size_t)pair_e[p] * slice + 2 * pproj;
                float ws;
                block_scale(down + r * pdrow, pdt, 0, &ws);
                const int32_t I = idot_block(down + r * pdrow, pdt, 0, hv + ((size_t)p * S + si) * OR_NEURONS);
                acc = fmaf((float)I * hsc[(size_t)p * S + si], ws, acc);
            }
            part[(size_t)p * d + r] = acc;
        }
    }
    for (unsigned t = 0; t < tokens; ++t)
        for (unsigned r = 0; r < d; ++r) {
            float acc = 0;
            for (unsigned j = 0; j < OR_TOPK; ++j)
                acc = fmaf(gate[(size_t)t * OR_ACTIVE + j], part[(size_t)slot_pair[t * OR_ACTIVE + j] * d + r], acc);
            if (slot_pair[t * OR_ACTIVE + OR_TOPK] != ~0u)  /* then the shared expert */
                acc = fmaf(gate[(size_t)t * OR_ACTIVE + OR_TOPK], part[(size_t)slot_pair[t * OR_ACTIVE + OR_TOPK] * d + r], acc);
            if (!isfinite(acc)) goto done;
            out[(size_t)t * d + r] = acc;
        }
    if (hq) memcpy(hq, hv, (size_t)P * S * OR_NEURONS);
    if (hs) memcpy(hs, hsc, sizeof(float) * P * S);
    memcpy(y, out, sizeof(float) * (size_t)tokens * d);
    rc = OR_OK;
done:
    free(pair_t); free(pair_e); free(slot_pair); free(q); free(res); free(hv); free(xsc); free(hsc); free(part); free(out);
    return rc;
}

/* --------------------------------------------------------------- metrics */

/* src/backend.c:74-92 */
int or_compare(const float *ref, const float *actual, size_t n, double out[3]) {
    if (!ref || !actual || !out || !n) return OR_INVALID;
    double r2 = 0, a2 = 0, d2 = 0, dot = 0, rmax = 0, dmax = 0;
    for (size_t i = 0; i < n; ++i) {
        double r = ref[i], a = actual[i], df = a - r;
        if (!isfinite(r) || !isfinite(a)) return OR_NUMERIC;
        r2 += r * r; a2 += a * a; d2 += df * df; dot += r * a;
        if (fabs(r) > rmax) rmax = fabs(r);
        if (fabs(df) > dmax) dmax = fabs(df);
    }
    if (!r2) {
        out[0] = a2 ? INFINITY : 0; out[1] = a2 ? INFINITY : 0; out[2] = a2 ? 0 : 1;
    } else {
        out[0] = sqrt(d2 / r2); out[1] = dmax / rmax;
        out[2] = a2 ? dot / (sqrt(r2) * sqrt(a2)) : 0;
        if (out[2] > 1) out[2] = 1;
        if (out[2] < -1) out[2] = -1;
    }
    return OR_OK;
}
