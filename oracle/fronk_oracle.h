/* fronk_oracle.h - CPU restatement of the reference's expert-slice arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (fronk_b200/, include/)
 * links, loads or calls this code; only tests/, the smoke check and the CPU
 * baseline leg of bench.py use it, and only as the checker.
 *
 * Two oracles live here:
 *   or_ref_run   - backends/ref.c:57-98 ("ref" and "ref-q8") with the hidden
 *                  size and the routed block formats as run-time values; double
 *                  accumulation, the reference's order.  Pinned bit-for-bit
 *                  against the unmodified reference (compiled from its own
 *                  sources) at d = 2560 and against its golden vectors.
 *   or_port_run  - the arithmetic the CUDA Q8 path performs (same operations,
 *                  same order): integer block dots of the int8 activations
 *                  and of their dequantization residuals, exact block terms
 *                  summed in double (the reference's narrowed gate/up
 *                  values), fp32 down terms; the GPU must reproduce its hidden
 *                  activations bit for bit and its output within 1e-5, and it
 *                  stays within 1e-5 of ref-q8.
 */
#ifndef FRONK_ORACLE_H
#define FRONK_ORACLE_H
#include <stddef.h>
#include <stdint.h>

enum { OR_OK = 0, OR_INVALID = -1, OR_STATE = -2, OR_NUMERIC = -3 };
enum { OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q4_K = 12, OR_MXFP4 = 39 };
enum { OR_BLOCKS = 20, OR_ROUTED = 512, OR_SHARED = 512, OR_TOPK = 10, OR_ACTIVE = 11,
       OR_NEURONS = 32, OR_MAX_TOKENS = 16, OR_MAX_PREFILL = 512 };

/* One layer of every loaded block.  layer[b] points at the first byte of the
 * requested layer inside unit b (NULL: block b not loaded).  Native layout:
 * 512 routed slices [gate 32 rows][up 32 rows][down d rows] then the Q8_0
 * shared slice (src/native.h:1-18).  Legacy layout (legacy = 1): 513 slices of
 * three Q4_0 projections (src/backend.h:38-48). */
typedef struct {
    unsigned hidden, gate_type, down_type, legacy;
    const uint8_t *layer[OR_BLOCKS];
} or_model;

/* src/q4.c:12-20 */
float or_f16(uint16_t bits);
/* src/q4.c:37-61: dequantized Q8 activations, groups of 64. */
int or_q8_activation(const float *x, float *out, size_t n);
/* The same quantization, exposing int8 values and one scale per 64. */
int or_q8_quantize(const float *x, size_t n, int8_t *q, float *scale);
/* src/q4.c:22-35 (legacy Q4_0 dot). */
int or_q4_0_dot(const uint8_t *q, const float *x, size_t n, double *out);
/* src/native.c:7-37. */
int or_native_dot(const uint8_t *p, unsigned type, const float *x, unsigned n, double *out);
/* The weights native.c decodes (same fp32 expression), element by element;
 * returns OR_NUMERIC if any is nonfinite (all n are still written). */
int or_decode_row(const uint8_t *p, unsigned type, unsigned n, float *w);

/* Geometry of the native layout with run-time d (src/native.h:9-21). */
size_t or_row_bytes(unsigned type, unsigned n);
size_t or_slice_bytes(unsigned hidden, unsigned gate_type, unsigned down_type);
size_t or_shared_bytes(unsigned hidden);
size_t or_layer_bytes(unsigned hidden, unsigned gate_type, unsigned down_type);
size_t or_legacy_layer_bytes(unsigned hidden);

/* backends/ref.c:41-98.  expert [T][10], gate [T][11], x [T][d], y [T][d].
 * q8 selects ref-q8.  y is written only on OR_OK. */
int or_ref_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
               const float *x, float *y, int q8);

/* The reference's AVX2 backend (backends/avx2.c, default build) restated
 * portably: int8 activations with one fp32 scale per 256 and int16 sums per
 * 32, its lane-wise fp32 accumulation and horizontal-add order, fp32 SiLU,
 * the hidden slice per 32, jobs dealt round robin to `workers` workers
 * (1-32) and the workers' outputs summed in order.  Native Q4_K / MXFP4
 * layout only.  libm_expf = 1 uses the C library's expf (bit-identical to
 * the compiled backend at the same worker count); 0 uses exp in double
 * rounded to fp32, the CUDA path's form.  order / norder: the blocks in
 * load order (the backend's job order); NULL: ascending.  y is written only
 * on OR_OK. */
int or_avx2_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                const float *x, float *y, unsigned workers, int libm_expf, const uint8_t *order, unsigned norder);

/* The CUDA Q8 path's arithmetic.  y as above.  When h is not NULL it receives
 * the hidden activations in the kernel's item order
 * [unique expert][loaded block][token][32] (zeros for tokens not routed to the
 * expert), at most h_cap floats; *h_count gets the size. */
int or_port_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                const float *x, float *y, float *h, size_t h_cap, size_t *h_count);

/* The CUDA prefill path's arithmetic (bursts of up to OR_MAX_PREFILL tokens,
 * MXFP4 or Q4_K gate/up, MXFP4 or Q8_0 down, the Q8_0 shared expert as
 * expert 512 for tokens with a shared gate): see fronk_oracle.c.
 * hq [pair][loaded block][32] / hs [pair][loaded block] (pairs expert-major,
 * tokens ascending) receive the quantized hidden values when not NULL. */
int or_prefill_run(const or_model *m, unsigned tokens, const uint16_t *expert, const float *gate,
                   const float *x, float *y, int8_t *hq, float *hs, size_t pair_cap, size_t *pairs);

/* Integer dot products of one row of n weights against int8 activations, one
 * per 32-weight block: Q4_K sum(q*v) with the unsigned nibble q (the sub-block
 * scale and min are applied later), MXFP4 sum(2*E2M1*v), Q8_0 sum(q*v). */
int or_block_idots(const uint8_t *p, unsigned type, unsigned n, const int8_t *v, int32_t *out);

/* Per-token conformance metrics of src/backend.c:74-92 in double. */
int or_compare(const float *ref, const float *actual, size_t n, double out[3]);
#endif
