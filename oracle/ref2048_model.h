/* ref2048_model.h - model geometry for building the reference at d = 2048.
 *
 * TEST INFRASTRUCTURE ONLY.  Passed with -include when compiling the
 * unmodified reference sources: it defines src/model.h's include guard and its
 * constants first, so the reference's model.h body is skipped and every
 * FR_HIDDEN-derived layout (fr_req, FR_NATIVE_* sizes) follows d = 2048.  All
 * other constants keep the reference's values (src/model.h:13-35).
 */
#ifndef FR_MODEL_H
#define FR_MODEL_H
#include <stdint.h>
#define FR_MODEL_NAME "Qwen3.8-Flash-Next"
#define FR_LAYERS 48
#define FR_DELTANET_LAYERS 36
#define FR_QSA_LAYERS 12
#define FR_HIDDEN 2048
#define FR_ROUTED_EXPERTS 512
#define FR_SHARED_EXPERTS 1
#define FR_EXPERTS (FR_ROUTED_EXPERTS + FR_SHARED_EXPERTS)
#define FR_SHARED_EXPERT FR_ROUTED_EXPERTS
#define FR_ACTIVE_ROUTED 10
#define FR_ACTIVE_EXPERTS (FR_ACTIVE_ROUTED + FR_SHARED_EXPERTS)
#define FR_INTERMEDIATE 640
#define FR_BLOCK_NEURONS 32
#define FR_BLOCKS (FR_INTERMEDIATE / FR_BLOCK_NEURONS)
#define FR_MAX_BURST 8
#define FR_BENCH_BURST_MAX 4
#define FR_Q4_WEIGHTS 32
#define FR_Q4_BYTES 18
#define FR_EXPERT_PARAMS (UINT64_C(3) * FR_LAYERS * FR_EXPERTS * FR_HIDDEN * FR_INTERMEDIATE)
#define FR_EXPERT_BYTES (FR_EXPERT_PARAMS / FR_Q4_WEIGHTS * FR_Q4_BYTES)
#define FR_WEIGHT_BLOCK_BYTES (FR_EXPERT_BYTES / FR_BLOCKS)
#endif
