/* fronk_b200.h - C ABI of the B200 expert neuron-slice backend.
 *
 * One call computes one MoE layer for 1..16 tokens: for every token, the gated
 * sum over its ten routed experts (plus the shared expert when its gate is
 * nonzero) of down[:,S] . (SiLU(gate[S,:] . x) * (up[S,:] . x)), over every
 * 32-neuron slice S loaded into this context.  It replaces the compute of the
 * reference's fr_backend.run (src/backend.h:52-67, backends/ref.c:57-98) and
 * takes the hidden size, the routed block formats and the token count as run
 * time values, so the reference geometry (d = 2560) and the benchmark one
 * (d = 2048) share one build.
 *
 * Plain C types only.  Every function returns an FRC_* status (the reference's
 * FR_* values, src/backend.h:17-18); nothing throws across this boundary.
 * A context belongs to one host thread at a time (calls are externally
 * serialized, as src/backend.h:1-2 requires of backends).
 */
#ifndef FRONK_B200_H
#define FRONK_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes, same values as src/backend.h:17-18. */
enum { FRC_OK = 0, FRC_INVALID = -1, FRC_STATE = -2, FRC_NUMERIC = -3,
       FRC_IO = -4, FRC_UNSUPPORTED = -5, FRC_MISMATCH = -6 };

/* Block type ids, same values as src/native.h:8. */
enum { FRC_Q8_0 = 8, FRC_Q4_K = 12, FRC_MXFP4 = 39 };

/* Activation precision of a run.  FRC_ACT_F32 multiplies exactly decoded
 * weights by fp32 activations (the arithmetic of backends/ref.c "ref").
 * FRC_ACT_Q8 first quantizes x per 64 and each 32-neuron hidden slice to int8
 * with the scheme of src/q4.c:37-61 (the "ref-q8" activation format,
 * backends/ref.c:66,85) and takes integer block dot products.
 * FRC_ACT_AVX2 is the arithmetic of the reference's AVX2 backend
 * (backends/avx2.c, default build): x as int8 with one fp32 scale per 256
 * and int16 sums per 32 (quantize8, :184-203), its lane-wise fp32 sums in its
 * order, fp32 SiLU, the hidden slice per 32, and the jobs (block, expert)
 * dealt to frc_set_avx2_workers workers, whose sums are added in worker
 * order.  Its results equal fr_avx2's at that worker count bit for bit, but
 * for the C library's rare last-bit expf roundings (here exp is evaluated in
 * double and rounded once).  frc_run / frc_run_flags (no run flag) only, up
 * to FRC_MAX_TOKENS tokens, on the reference's native layout (Q4_K gate/up,
 * MXFP4 down); FRC_UNSUPPORTED otherwise. */
enum { FRC_ACT_F32 = 0, FRC_ACT_Q8 = 1, FRC_ACT_AVX2 = 2 };

/* Model constants of src/model.h:18-27. */
enum { FRC_MAX_BLOCKS = 20, FRC_ROUTED_EXPERTS = 512, FRC_SHARED_EXPERT = 512,
       FRC_TOPK = 10, FRC_ACTIVE = 11, FRC_NEURONS = 32, FRC_MAX_TOKENS = 16,
       FRC_MAX_LAYERS = 64, FRC_MAX_PREFILL_TOKENS = 512 };

/* Shape of one ownership unit (a "block" of the reference: the same 32
 * neurons of every expert in every layer).  The reference's own layout is
 * {2560, 48, FRC_Q4_K, FRC_MXFP4} (src/native.h:9-18); the shared expert is
 * always Q8_0 for gate, up and down. */
typedef struct {
    uint32_t hidden;     /* d: a multiple of 512, at most 8192 */
    uint32_t layers;     /* 1..FRC_MAX_LAYERS */
    uint32_t gate_type;  /* routed gate and up rows: FRC_Q4_K, FRC_MXFP4 or FRC_Q8_0 */
    uint32_t down_type;  /* routed down rows (32 neurons each): FRC_MXFP4 or FRC_Q8_0 */
} frc_geometry;

/* ---- Geometry (host only; mirrors src/native.h:9-21 with run-time d) ---- */
/* Bytes of one row of n weights of the given type (src/native.h:19-21); 0 if invalid. */
size_t frc_row_bytes(unsigned type, unsigned n);
/* Bytes of one routed 32-neuron slice: 32 gate rows, 32 up rows, d down rows. */
size_t frc_slice_bytes(const frc_geometry *g);
/* Bytes of the shared expert's slice (three Q8_0 projections). */
size_t frc_shared_bytes(const frc_geometry *g);
/* Bytes of one layer: 512 routed slices then the shared slice. */
size_t frc_layer_bytes(const frc_geometry *g);
/* Bytes of one unit (all layers); FR_NATIVE_BLOCK_BYTES for the reference geometry. */
uint64_t frc_unit_bytes(const frc_geometry *g);
/* Offset of (layer, expert) inside a unit (src/native.h:16-18); expert 512 is shared. */
uint64_t frc_slice_offset(const frc_geometry *g, unsigned layer, unsigned expert);
/* FRC_OK when g is a supported geometry. */
int frc_geometry_check(const frc_geometry *g);

/* ---- Context ---- */
typedef struct frc_context frc_context;

/* Device query without a context (nothing is allocated): FRC_OK when device
 * `device` is an sm_100 part; its name (NUL-terminated, at most cap bytes),
 * HBM bytes and SM count when the pointers are not NULL.  The fr_backend
 * probe entry's device check (src/hw.h:19-24). */
int frc_probe_device(int device, char *name, size_t cap, uint64_t *hbm_bytes, unsigned *sms);

/* Opens device `device` for units of geometry g.  Allocates all run-time
 * scratch now; run calls allocate nothing (src/backend.h:5).  FRC_UNSUPPORTED
 * when the device is not an sm_100 part. */
int frc_open(int device, const frc_geometry *g, frc_context **out);
int frc_close(frc_context *c);
/* Copies a whole unit (frc_unit_bytes, reference byte layout, host memory)
 * into HBM, re-laid out for aligned 128-bit access.  This is the set-up copy a
 * discrete GPU needs where the CPU backends borrow the mapping
 * (src/backend.h:55-60).  Occupied block: FRC_STATE; bad index/size: FRC_INVALID. */
int frc_load_unit(frc_context *c, int block, const void *unit, size_t len);
/* Loads only one layer of a unit (frc_layer_bytes from a host buffer).  The
 * block then counts as loaded; layers never loaded are reported by run as
 * FRC_STATE.  Used for sparse correctness fixtures. */
int frc_load_layer(frc_context *c, int block, unsigned layer, const void *layer_bytes, size_t len);
int frc_unload_unit(frc_context *c, int block);
/* Copies one layer of a loaded block again from host memory (frc_layer_bytes
 * of that layer, reference layout), replacing the HBM copy.  For callers that
 * lend the backend a writable unit and may change it after load: the
 * reference's backends read the borrowed bytes at every run
 * (src/backend.h:52-60), a discrete GPU computes from its copy.
 * FRC_STATE when that layer is not loaded. */
int frc_refresh_layer(frc_context *c, int block, unsigned layer, const void *layer_bytes, size_t len);
/* Bit b set when block b is loaded. */
int frc_loaded_mask(const frc_context *c, uint32_t *mask);

/* ---- Units from disk (the reference node's loader, src/units.c:25-75) ----
 * A unit directory holds unit-BB.bin (block BB's weights, frc_unit_bytes in
 * the reference layout) and unit-BB.sha256 (64 lowercase hex digits and a
 * newline).  frc_units_open maps each block of `mask` read-only, checks the
 * digest file, the size and, with verify, the file's SHA-256, and copies the
 * unit into HBM (frc_load_unit); the mapping is released after the copy.
 * On the first failure the blocks this call loaded are unloaded again.
 * Errors: FRC_IO (a file missing, unreadable or of another size),
 * FRC_INVALID (a malformed digest file, bad arguments), FRC_MISMATCH (the
 * SHA-256 differs), FRC_STATE (a block already loaded). */
int frc_units_open(frc_context *c, const char *directory, uint32_t mask, int verify);
/* The same file checks for one block, without a device (unit_bytes 0: any
 * size). */
int frc_unit_verify(const char *directory, unsigned block, uint64_t unit_bytes, int verify);
/* SHA-256 (FIPS 180-4) of len bytes into out[32] (src/sha256.c's role). */
int frc_sha256(const void *data, size_t len, uint8_t out[32]);

/* ---- In-box head plane (the reference head's fan-out and gather of one
 * layer, src/plane.c:252-374, over the GPUs of one box) ----
 * One context per GPU, each holding its share of the blocks (the planner's
 * split).  frc_plane_run rounds x to fp16 once, as the head does for every
 * node and its own slice (src/plane.c:258-262, src/wire.c:46-67), runs the
 * layer on every participant's stream (Q8 activations), and sums the parts
 * that are done by the deadline in participant order; bit i of *missing is
 * set for a participant that missed it, and its part is left out, as the
 * reference head leaves out a late node.  Participant 0 is the head's own
 * slice (its part is added in fp32); the parts of the others, standing for
 * remote nodes, are rounded through fp16 as the reference sends them, and a
 * part with a value that has no finite fp16 form is left out and reported
 * missing, as the node drops such a reply.  A late participant's next call
 * waits (bounded) for its earlier one.  FRC_INVALID: bad arguments or an x
 * value with no finite fp16 form (nothing runs); a participant's device
 * error fails the call with y untouched.  Contexts must share a geometry and
 * outlive the plane; the plane runs on their own streams and scratch, so no
 * other call may use those contexts while a plane call is in flight. */
typedef struct frc_plane frc_plane;
int frc_plane_open(frc_context *const *ctx, unsigned count, frc_plane **out);
int frc_plane_run(frc_plane *p, unsigned layer, unsigned tokens, const uint16_t *expert, const float *gate,
                  const float *x, uint64_t deadline_ns, float *y, uint32_t *missing);
int frc_plane_close(frc_plane *p);
/* The device status (FRC_OK or an error code) of participant i's last part
 * that missed its deadline, read when that participant's next call found it
 * done: such a part was left out of its own call, so its status is kept here
 * instead of failing a later layer. */
int frc_plane_late_status(const frc_plane *p, unsigned participant, int *status);
/* ---- Cost model (fr_costmodel, src/backend.h:30-35) ----
 * t = t0 + 1e9 * bytes / bw_eff for a burst that reads `bytes` of weights,
 * the form the reference planner weighs participants with.  Same fields and
 * meaning as fr_costmodel. */
enum { FRC_COST_MAX_BURST = 8 };
typedef struct {
    unsigned burst_max;
    double t0_ns, bw_eff;                 /* bytes/second */
    double ns[FRC_COST_MAX_BURST];        /* median time of a synchronous run, burst b+1 */
    uint64_t bytes[FRC_COST_MAX_BURST];   /* weight bytes it reads */
} frc_costmodel;
/* The reference's fit (src/bench.c:163-191): least squares of ns over bytes
 * for bursts 1..n (2 <= n <= 8); a negative t0 is clamped to 0 by fitting
 * through the origin.  FRC_NUMERIC for nonpositive or nonfinite times or a
 * nonpositive slope. */
int frc_costmodel_fit(const double *ns, const uint64_t *bytes, unsigned n, frc_costmodel *out);
/* Measures and fits it on this context: `samples` synchronous frc_run calls
 * of layer `layer` at each burst 1..burst_max in activation mode `act` (any
 * of the three; the fallback bench of each plugin table measures its own)
 * (distinct seeded routing, the shared expert active), medians, bytes =
 * loaded blocks x (10 x burst x slice + shared slice) (src/bench.c:157-160).
 * g: the context's geometry.  FRC_STATE when nothing is loaded. */
int frc_costmodel_measure(frc_context *c, const frc_geometry *g, unsigned layer, unsigned burst_max,
                          unsigned samples, int act, frc_costmodel *out);

/* x rounded through fp16 as the head sends it: round to nearest even;
 * FRC_INVALID when a value is not finite or rounds past 65504, or the
 * rounding mode is not to-nearest. */
int frc_round_half(const float *x, size_t n, float *out);

/* Synchronous run from host memory, the semantics of fr_backend.run
 * (src/backend.h:1-5, backends/ref.c:41-98): validates the request (ids < 512
 * and distinct per token, gates finite and >= 0, x finite, FE_TONEAREST),
 * then computes y[tokens][d].  On any error y is left byte-identical.
 *   expert: [tokens][10] routed ids      gate: [tokens][11], shared last
 *   x:      [tokens][d]                  y:    [tokens][d]
 * Errors: FRC_INVALID, FRC_NUMERIC (nonfinite input, a nonfinite scale in any
 * referenced block even with gate 0, fp32 overflow), FRC_STATE (nothing loaded). */
int frc_run(frc_context *c, unsigned layer, unsigned tokens, const uint16_t *expert,
            const float *gate, const float *x, float *y, int act);
/* frc_run with run flags; no counterpart in the reference.  The one flag
 * taken is FRC_RUN_PEER (up to 16 tokens a call): y is the sum over every
 * rank of the in-box reduce group (frc_peer_attach), so each process of a
 * box can drive its share of the slices from host buffers; every rank makes
 * the same sequence of calls. */
int frc_run_flags(frc_context *c, unsigned layer, unsigned tokens, const uint16_t *expert,
                  const float *gate, const float *x, float *y, int act, unsigned flags);

/* Flags of frc_run_device.
 * FRC_RUN_X_BF16: x holds bf16 values ([tokens][d] 16-bit words, the upper
 * half of an fp32 bit pattern), widened exactly to fp32 on the device; the
 * tensor-core burst path only (more than 16 tokens, Q8, MXFP4 or Q4_K
 * gate/up rows, MXFP4 down rows, no other flag); any other call with it is
 * FRC_UNSUPPORTED.
 * FRC_RUN_OVERLAP: the launch may start while the kernel before it on the
 * stream is finishing (programmatic dependent launch): it plans and starts
 * streaming this layer's weights at once and waits for that kernel only
 * before it reads x / x_add or writes anything.  The caller guarantees that
 * the preceding kernel writes neither the weights nor expert / gate (writing
 * x, as a previous layer or an all-reduce does, is fine).
 * FRC_RUN_PEER: y is the sum over every rank of the in-box reduce group
 * (frc_peer_attach) of each rank's partial, added in rank order: identical
 * on every rank.  Every rank must make the same sequence of FRC_RUN_PEER
 * calls (same token counts), one process per GPU. */
enum { FRC_RUN_RMSNORM = 1, FRC_RUN_OVERLAP = 2, FRC_RUN_PEER = 4, FRC_RUN_X_BF16 = 8 };

/* Asynchronous run on device memory, enqueued on `stream` (a cudaStream_t, or
 * NULL for the legacy default stream); nothing is validated on the host and
 * nothing synchronizes, so it can be captured in a CUDA graph.  The kernel
 * forms v = x + x_add (x_add may be NULL) and, when x_out is not NULL, stores
 * v there (a residual stream; x_out must not alias x or x_add).  With
 * FRC_RUN_RMSNORM the layer's input is v / sqrt(mean(v^2) + 1e-6) per token
 * (the pre-norm a decoder block applies before its MoE), otherwise v.
 * Numeric and bounds failures set the context's device status word, read by
 * frc_status. */
int frc_run_device(frc_context *c, unsigned layer, unsigned tokens, const uint16_t *expert,
                   const float *gate, const float *x, const float *x_add, float *x_out,
                   float *y, int act, unsigned flags, void *stream);
/* frc_run_device with the hand-off between the kernel's item phase and its
 * reduce (the down terms and their weights) held in a device array fixed at
 * module load (8 MiB per device) instead of context scratch: the call
 * allocates nothing.  Needs 11 x tokens x slices x (hidden + 1) floats: up
 * to 4 tokens with 20 slices at hidden 2048 (more with fewer slices); a
 * larger call returns FRC_INVALID and launches nothing.  No fp32 copy of the
 * hidden activations is kept (frc_debug_hidden does not see these calls).
 * The array is shared by all contexts and streams of a device: overlapping
 * calls on one device race, callers serialise them.  The first call on a
 * device looks the array up; make it before any stream capture.
 * No counterpart in the reference (backend.h has no device-pointer entry). */
int frc_run_device_fixed(frc_context *c, unsigned layer, unsigned tokens, const uint16_t *expert,
                         const float *gate, const float *x, const float *x_add, float *x_out,
                         float *y, int act, unsigned flags, void *stream);
/* ---- In-box reduce over NVLink peer memory (replaces the per-layer
 * all-reduce of the slice partials; the reference's fanout/plane gather,
 * src/plane.c:110-121, inside one box).  One process per GPU:
 *   1. every rank: frc_peer_export(c, world, handle) - allocates this
 *      context's inbox and writes its IPC handle (FRC_PEER_HANDLE_BYTES);
 *   2. the ranks exchange handles (any host channel);
 *   3. every rank: frc_peer_attach(c, rank, world, handles[world]);
 *   4. run with FRC_RUN_PEER.  A rank whose peers stop answering gets
 *      FRC_IO from frc_status after a bounded wait; the group then detaches
 *      and attaches again.
 * No counterpart in the reference (its gather is TCP/UDP between nodes). */
enum { FRC_PEER_HANDLE_BYTES = 64 };
int frc_peer_export(frc_context *c, unsigned world, void *handle);
int frc_peer_attach(frc_context *c, unsigned rank, unsigned world, const void *handles);
int frc_peer_detach(frc_context *c);

/* A decode pass for `tokens` tokens driven from the host, layer by layer
 * through frc_run (host buffers, one synchronous call per layer): per token
 * x = h / sqrt(mean(h^2) + 1e-6), y = run(layer, x), h += y, for layers
 * first_layer .. first_layer + layers - 1.  expert: [layers][tokens][10],
 * gate: [layers][tokens][11]; h ([tokens][hidden]) is the residual stream,
 * updated in place.  The end-to-end path of a host that owns the layer loop
 * (the reference's head calls fr_backend.run once per layer the same way).
 * Not reentrant (static staging). */
int frc_host_pass(frc_context *c, unsigned first_layer, unsigned layers, unsigned tokens,
                  const uint16_t *expert, const float *gate, float *h, unsigned hidden, int act);
/* frc_host_pass through frc_run_flags (FRC_RUN_PEER: one process per GPU of
 * a box, each holding its share of the slices, every layer summed over the
 * ranks inside the kernel, so every rank's h stays identical). */
int frc_host_pass_flags(frc_context *c, unsigned first_layer, unsigned layers, unsigned tokens,
                        const uint16_t *expert, const float *gate, float *h, unsigned hidden, int act,
                        unsigned flags);
/* Waits for `stream`, returns and clears the device status (FRC_OK,
 * FRC_NUMERIC, FRC_INVALID for an out-of-range id, FRC_IO for a timed-out wait). */
int frc_status(frc_context *c, void *stream);
/* Every bounded wait inside the layer kernel (its TMA ring, grid barrier,
 * split-item exchange and in-box reduce) gives up after `ns` nanoseconds
 * (1 us .. 60 s; 2 s when never set), sets the device status that frc_status
 * / frc_run report as FRC_IO, and the launch ends: y of a frc_run call is left
 * untouched and the next call on the context runs normally.  No counterpart in
 * the reference (its timeouts are the plane's deadline, src/plane.c). */
int frc_set_wait_limit(frc_context *c, uint64_t ns);
/* FRC_ACT_AVX2: the worker count (1-32, default 1) whose job dealing and
 * worker-ordered sum the run reproduces (backends/avx2.c:506-529, :703-708;
 * fr_avx2 picks it with fr_avx2_configure).  Jobs are block-major over the
 * blocks in load order, which becomes ascending after an unload, as the AVX2
 * backend keeps its slots (backends/avx2.c:602-613). */
int frc_set_avx2_workers(frc_context *c, unsigned workers);
/* Event timing of FRC_ACT_AVX2 calls: while enabled, each records CUDA events
 * on the context's stream around its three launches (activation
 * quantization, jobs, reduction); frc_avx2_times writes the last call's three
 * durations in ms.  For measurement. */
int frc_avx2_timing(frc_context *c, int enable);
int frc_avx2_times(frc_context *c, float *ms);
/* Tests and measurements: which kernel may serve one-token FRC_ACT_Q8 calls.
 * 1 (the default): the row-owner kernel (gate/up work dealt to every CTA in
 * chunks of 8 neurons, each CTA then forms its own rows of y from all
 * items' hidden values) when at most two slices are loaded, else the item
 * kernel; 0: always the item kernel that serves larger bursts; 2: the
 * row-owner kernel whenever its staging fits.  Both kernels compute the same
 * values in the same order. */
int frc_debug_layer_variant(frc_context *c, int variant);
/* Tests only: raises the layer kernel's grid-barrier target by `extra`
 * arrivals (0 restores it), so that the barrier's bounded wait runs out. */
int frc_debug_barrier_extra(frc_context *c, unsigned extra);
/* Count of kernels this context has launched since open. */
uint64_t frc_launch_count(const frc_context *c);
const char *frc_strerror(int rc);
/* Text of the last failure on this context (static storage). */
const char *frc_last_error(const frc_context *c);

/* ---- Synthetic inputs (host only) ---- */
/* Counter-based generator: splitmix64 of (seed, index). */
uint64_t frc_rand64(uint64_t seed, uint64_t index);
/* Approximately N(0,1): Irwin-Hall sum of four 16-bit uniforms, scaled to unit
 * variance.  Exact integer-then-one-multiply arithmetic, so every platform
 * gives the same float. */
float frc_normal(uint64_t seed, uint64_t index);
/* Encodes n weights into one row of the given type (reference byte layout):
 * Q4_K super-blocks of 256, MXFP4 blocks of 32, Q8_0 blocks of 32. */
int frc_encode_row(unsigned type, const float *w, unsigned n, uint8_t *out);
/* One routed slice in reference layout, weights ~N(0, 0.02) quantized to the
 * geometry's formats; `key` selects the slice's random stream. */
int frc_synth_slice(const frc_geometry *g, uint64_t seed, uint64_t key, uint8_t *out);
/* The shared expert's slice (Q8_0 x3), weights ~N(0, 0.02). */
int frc_synth_shared(const frc_geometry *g, uint64_t seed, uint64_t key, uint8_t *out);
/* A request of up to FRC_MAX_PREFILL_TOKENS tokens: x ~ N(0,1); 10 of 512
 * experts uniform without replacement; gates softmax(N(0,1)) over the 10;
 * shared gate 0.  Token t's values do not depend on the token count. */
int frc_synth_request(unsigned hidden, unsigned tokens, uint64_t seed,
                      uint16_t *expert, float *gate, float *x);
/* The same with Zipf(s)-skewed expert popularity: expert e has weight
 * (rank(e) + 1)^-s, rank a seeded permutation of the 512 experts, and each
 * token draws 10 without replacement in proportion to the weights (Gumbel
 * top-k), most likely first.  x and gates as frc_synth_request. */
int frc_synth_request_zipf(unsigned hidden, unsigned tokens, uint64_t seed, double s,
                           uint16_t *expert, float *gate, float *x);

/* ---- Benchmark-scale units without host encoding ---- */
/* Uploads `count` routed slices and one shared slice (reference layout) as a
 * device pool. */
int frc_pool_load(frc_context *c, const uint8_t *slices, unsigned count, const uint8_t *shared);
/* Fills every routed slot and the shared slot of (block, layer) from the pool
 * on the device: slot e takes pool slice frc_pool_pick(seed, block, layer, e, count). */
int frc_fill_layer(frc_context *c, int block, unsigned layer, uint64_t seed);
unsigned frc_pool_pick(uint64_t seed, unsigned block, unsigned layer, unsigned expert, unsigned count);

/* ---- Diagnostics used by the parity tests ---- */
/* GPU decode of `rows` rows of n weights (reference layout) to fp32. */
int frc_debug_decode(frc_context *c, unsigned type, const uint8_t *rows, unsigned n,
                     unsigned count, float *out);
/* GPU activation quantization of tokens x d values: int8 values, one fp32
 * scale per 64, and the dequantized fp32 values of src/q4.c:37-61. */
int frc_debug_quantize(frc_context *c, unsigned tokens, const float *x, int8_t *q,
                       float *scale, float *deq);
/* Tensor-core (tcgen05 kind::i8) check: d[128][n] = a[128][k] * b[n][k]^T in
 * int32, row-major host arrays; n a multiple of 16 up to 256, k a multiple of
 * 32 up to 256. */
int frc_debug_umma(frc_context *c, unsigned n, unsigned k, const int8_t *a, const int8_t *b, int32_t *d);
/* Event timing of the prefill path (bursts above FRC_MAX_TOKENS on the
 * tensor cores): while enabled, every prefill call records CUDA events on its
 * stream around its five stages (quantize, group, gate/up MMA, down MMA,
 * combine); frc_prefill_times waits for the last call's final event and
 * writes the five durations in ms.  For measurement; leave it disabled in
 * captured graphs. */
int frc_prefill_timing(frc_context *c, int enable);
int frc_prefill_times(frc_context *c, float *ms);
/* Quantized hidden values of the last prefill burst (more than
 * FRC_MAX_TOKENS tokens on the tensor-core path): hq [pair][loaded block][32]
 * int8 in neuron order and hs [pair][loaded block] fp32 scales, pairs
 * (expert, token) expert-major with tokens ascending.  *pairs receives the
 * pair count; with hq and hs NULL only the count is returned. */
int frc_debug_prefill_hidden(frc_context *c, int8_t *hq, float *hs, size_t cap, size_t *pairs);
/* Hidden activations h of the last frc_run, in item order
 * [unique expert][loaded block][token][32] (zero where the token does not use
 * the expert); *count receives the number of floats. */
int frc_debug_hidden(frc_context *c, float *h, size_t cap, size_t *count);
/* Per-CTA globaltimer stamps of the last layer launch, [cta][16]: entry, plan,
 * norm sums, activations, gate/up done, barrier done, down done, exit, then
 * finer points inside the plan (8-10) and the down phase (11-13).
 * Only libraries built with FRC_PHASES record them (else FRC_UNSUPPORTED);
 * the counterpart of the reference's compile-time FR_PHASES timers. */
int frc_debug_phases(frc_context *c, uint64_t *out, size_t cap, size_t *count);

#ifdef __cplusplus
}
#endif
#endif
