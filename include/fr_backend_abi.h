/* fr_backend_abi.h - the reference's backend plugin contract, restated.
 *
 * These are the types of src/backend.h:20-67 and src/hw.h:19-24 with the
 * same member order, types and sizes, so a table built against this header is
 * the same object as one built against the reference's headers.  A build
 * inside the reference tree compiles fr_cuda_backend.c against the
 * reference's own src/backend.h instead (FR_USE_REFERENCE_HEADERS); this copy
 * exists so the library also builds without the reference sources.
 * FR_HIDDEN defaults to the reference's 2560 (src/model.h:16).
 */
#ifndef FR_BACKEND_ABI_H
#define FR_BACKEND_ABI_H
#include <stddef.h>
#include <stdint.h>

#ifndef FR_HIDDEN
#define FR_HIDDEN 2560
#endif
#define FR_LAYERS 48
#define FR_ROUTED_EXPERTS 512
#define FR_SHARED_EXPERT 512
#define FR_ACTIVE_ROUTED 10
#define FR_ACTIVE_EXPERTS 11
#define FR_BLOCK_NEURONS 32
#define FR_BLOCKS 20
#define FR_MAX_BURST 8

enum { FR_OK = 0, FR_INVALID = -1, FR_STATE = -2, FR_NUMERIC = -3,
       FR_IO = -4, FR_UNSUPPORTED = -5, FR_MISMATCH = -6 };

/* src/hw.h:19-24 */
typedef struct {
    char os[16], arch[16], version[64], cpu[128], gpu[128], name[64];
    unsigned cores, logical_cores, isa, metal, translated;
    uint64_t id, total, available, margin, cap, blocks, metal_limit, frequency, wired_mb;
    uint64_t head_reserve, head_cap, head_blocks, head_fixed;
} fr_hwinfo;

/* src/backend.h:20-35 */
typedef struct {
    unsigned layer, burst;
    uint16_t expert[FR_MAX_BURST][FR_ACTIVE_ROUTED];
    float gate[FR_MAX_BURST][FR_ACTIVE_EXPERTS];
    float x[FR_MAX_BURST][FR_HIDDEN];
} fr_req;
typedef struct {
    unsigned layer, burst;
    float y[FR_MAX_BURST][FR_HIDDEN];
} fr_part;
typedef struct {
    unsigned burst_max;
    double t0_ns, bw_eff;
    double ns[FR_MAX_BURST];
    uint64_t bytes[FR_MAX_BURST];
} fr_costmodel;

/* src/backend.h:52-67 */
typedef struct fr_backend {
    const char *name;
    int (*probe)(fr_hwinfo *out);
    int (*load)(int block, const void *data, size_t len);
    int (*unload)(int block);
    int (*run)(const fr_req *req, fr_part *out);
    int (*bench)(int burst_max, fr_costmodel *out);
    int (*self_test)(const char *vectors_dir);
} fr_backend;

/* The B200 backends.  "cuda": Q8 activations (the production path).
 * "cuda-f32": fp32 activations, the arithmetic of the reference's "ref".
 * "cuda-avx2": the arithmetic of the reference's "avx2" backend
 * (backends/avx2.c), its results at the worker count fr_cuda_avx2_workers
 * sets. */
extern const fr_backend fr_cuda, fr_cuda_f32, fr_cuda_avx2;

/* Device the backends open on first load (default 0); FR_STATE once open. */
int fr_cuda_select_device(int device);
/* Releases the backend's device context; FR_STATE while blocks are loaded. */
int fr_cuda_close(const fr_backend *backend);
/* fr_cuda_avx2: the AVX2 backend worker count (1-32, default 1) whose job
 * dealing and summation order it reproduces. */
int fr_cuda_avx2_workers(unsigned workers);
#endif
