// frc.cu - B200 (sm_100a) expert neuron-slice backend: set-up kernels, the
// host runtime and the C ABI (include/fronk_b200.h).  The MoE layer kernel
// itself is in frc_layer.cuh: one cooperative launch per layer, static work
// split, every CTA's weight bytes requested up front through a TMA ring,
// integer block dots, a fixed reduction order and no float atomics (results
// are bitwise repeatable).
#include <chrono>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <fenv.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "../../include/fronk_b200.h"
#include "frc_device.cuh"

using namespace frc;

#include "frc_layer.cuh"
#include "frc_layer_rb.cuh"
#include "frc_umma.cuh"
#include "frc_prefill.cuh"
#include "frc_avx2.cuh"
#include "frc_units.h"

// ===================================================== set-up kernels

// Reference byte layout -> device layout.  Q4_K rows are kept; MXFP4 and
// Q8_0 runs of blocks are split into [scales][payloads] so payloads are
// 16-byte aligned.  One CTA per slice; routed slices first, then `shared`
// trailing shared slices.
struct SliceShape {
  unsigned d, gate_type, down_type;
  unsigned row_bytes, slice_bytes, shared_row, shared_bytes;
};

__device__ void transcode_run(const uint8_t* src, uint8_t* dst, unsigned type, unsigned nblocks) {
  if (type == kQ4K) {
    for (unsigned i = threadIdx.x; i < nblocks * 144 / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    return;
  }
  const unsigned bs = type == kMXFP4 ? 17 : 34, hs = type == kMXFP4 ? 1 : 2, ps = bs - hs;
  for (unsigned i = threadIdx.x; i < nblocks; i += blockDim.x) {
    const uint8_t* b = src + static_cast<size_t>(i) * bs;
    for (unsigned h = 0; h < hs; ++h) dst[i * hs + h] = b[h];
    uint8_t* o = dst + static_cast<size_t>(nblocks) * hs + static_cast<size_t>(i) * ps;
    for (unsigned h = 0; h < ps; ++h) o[h] = b[hs + h];
  }
}

// Hands a call's [status word][y] to the host: launched right behind the
// layer kernel with programmatic stream serialization, it waits for that
// grid to complete (griddepcontrol.wait returns once the prerequisite grid
// has finished and its memory is visible) and stores the words into mapped
// pinned memory, which the host reads after synchronising the stream.  A
// device-to-host copy behind the kernel instead costs ~10 us more per call.
__global__ void __launch_bounds__(512) publish_kernel(const uint4* __restrict__ src, uint4* dst, unsigned n16) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

__global__ void transcode_kernel(const uint8_t* src, uint8_t* dst, unsigned routed, SliceShape s) {
  const unsigned sl = blockIdx.x;
  const bool shared = sl >= routed;
  const size_t off = shared ? static_cast<size_t>(routed) * s.slice_bytes + static_cast<size_t>(sl - routed) * s.shared_bytes
                            : static_cast<size_t>(sl) * s.slice_bytes;
  const uint8_t* in = src + off;
  uint8_t* out = dst + off;
  const unsigned gt = shared ? kQ80 : s.gate_type, dt = shared ? kQ80 : s.down_type;
  const unsigned rowb = shared ? s.shared_row : s.row_bytes;
  const unsigned nb = gt == kQ4K ? s.d / 256 : s.d / 32;
  for (unsigned r = 0; r < 64; ++r) transcode_run(in + r * rowb, out + r * rowb, gt, nb);
  transcode_run(in + 64 * rowb, out + 64 * rowb, dt, s.d);
}

__global__ void rows_transcode_kernel(const uint8_t* src, uint8_t* dst, unsigned type, unsigned n, unsigned rowb) {
  transcode_run(src + static_cast<size_t>(blockIdx.x) * rowb, dst + static_cast<size_t>(blockIdx.x) * rowb, type,
                type == kQ4K ? n / 256 : n / 32);
}

// Pool -> every slot of one layer (uint4 copies; all sizes are multiples of 16).
__global__ void fill_kernel(const uint8_t* pool, unsigned count, uint8_t* layer, size_t slice_bytes,
                            size_t shared_bytes, uint64_t seed, unsigned block, unsigned layer_index) {
  const unsigned e = blockIdx.x;
  const uint8_t* src;
  size_t bytes;
  if (e < 512) {
    const unsigned pick = static_cast<unsigned>(
        rand64(seed, (static_cast<uint64_t>(block) * FRC_MAX_LAYERS + layer_index) * 513u + e) % count);
    src = pool + static_cast<size_t>(pick) * slice_bytes;
    bytes = slice_bytes;
  } else {
    src = pool + static_cast<size_t>(count) * slice_bytes;
    bytes = shared_bytes;
  }
  uint4* dst = reinterpret_cast<uint4*>(layer + static_cast<size_t>(e) * slice_bytes);
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  for (size_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) dst[i] = s4[i];
}

// Diagnostics: exact fp32 decode of device rows; activation quantization.
__global__ void decode_kernel(const uint8_t* rows, unsigned type, unsigned n, unsigned rowb, float* out) {
  const uint8_t* row = rows + static_cast<size_t>(blockIdx.x) * rowb;
  for (unsigned j = threadIdx.x; j < n; j += blockDim.x) out[static_cast<size_t>(blockIdx.x) * n + j] = weight_any(row, type, n, j);
}

__global__ void quantize_kernel(const float* x, unsigned n, int8_t* q, float* scale, float* deq) {
  // one warp per 64-group, two values per lane: the same operations as the layer prologue
  const unsigned g = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (64 * g >= n) return;
  const float2 v = reinterpret_cast<const float2*>(x + 64 * g)[lane];
  float amax = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
  for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = __fdiv_rn(amax, 127.0f);
  const float r0 = q8_round(v.x, amax, s), r1 = q8_round(v.y, amax, s);
  q[64 * g + 2 * lane] = static_cast<int8_t>(static_cast<int>(r0));
  q[64 * g + 2 * lane + 1] = static_cast<int8_t>(static_cast<int>(r1));
  if (lane == 0) scale[g] = s;
  const double lim = 3.4028234663852886e38;
  double d0 = static_cast<double>(r0) * s, d1 = static_cast<double>(r1) * s;
  d0 = fmin(fmax(d0, -lim), lim);
  d1 = fmin(fmax(d1, -lim), lim);
  deq[64 * g + 2 * lane] = __double2float_rn(d0);
  deq[64 * g + 2 * lane + 1] = __double2float_rn(d1);
}

// Tensor-core check: D[128][N] = A[128][K] * B[N][K]^T in int32 through
// tcgen05 (K/32 MMA steps, accumulators in tensor memory, read back with
// tcgen05.ld).  One CTA of 128 threads; K a multiple of 32 up to 256, N a
// multiple of 16 up to 256.
__global__ void __launch_bounds__(128) umma_check_kernel(const int8_t* A, const int8_t* B, int32_t* D, unsigned N,
                                                         unsigned K, unsigned* status) {
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ uint32_t taddr_s;
  uint8_t* As = sm;
  uint8_t* Bs = sm + 128 * K;
  const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, kc = K / 16;
  for (unsigned i = tid; i < 128 * kc; i += 128) {
    const unsigned r = i / kc, c = i % kc;
    *reinterpret_cast<uint4*>(As + umma_off(r, 16 * c, K)) = *reinterpret_cast<const uint4*>(A + r * K + 16 * c);
  }
  for (unsigned i = tid; i < N * kc; i += 128) {
    const unsigned r = i / kc, c = i % kc;
    *reinterpret_cast<uint4*>(Bs + umma_off(r, 16 * c, K)) = *reinterpret_cast<const uint4*>(B + r * K + 16 * c);
  }
  fence_proxy_async();
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  const unsigned ncols = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
  if (warp == 0) {
    tmem_alloc(&taddr_s, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = taddr_s;
  if (tid == 0) {
    const uint32_t a0 = smem_u32(As), b0 = smem_u32(Bs), idesc = umma_idesc_i8(128, N);
    for (unsigned s = 0; s < K / 32; ++s)
      umma_i8(taddr, umma_desc(a0 + 256 * s, 128, 8 * K), umma_desc(b0 + 256 * s, 128, 8 * K), idesc, s > 0);
    umma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0);
  tc_fence_after();
  if (ok) {
    for (unsigned c = 0; c < N; c += 16) {
      uint32_t r[16];
      tmem_ld16(taddr + ((32 * warp) << 16) + c, r);
      tmem_wait_ld();
#pragma unroll
      for (unsigned j = 0; j < 16; ++j) D[(32 * warp + lane) * N + c + j] = static_cast<int32_t>(r[j]);
    }
  } else if (lane == 0) {
    atomicOr(status, kStTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(taddr, ncols);
}

// ========================================================= host runtime

struct frc_context {
  int device = 0, sms = 0;
  frc_geometry g{};
  size_t row_bytes = 0, proj_bytes = 0, slice_bytes = 0, shared_row = 0, shared_proj = 0, shared_bytes = 0, layer_bytes = 0;
  uint8_t* layer_ptr[FRC_MAX_BLOCKS][FRC_MAX_LAYERS] = {};
  uint8_t* staging = nullptr;
  float* hidden = nullptr;
  float* partial = nullptr;
  float* gsv = nullptr;
  unsigned long long* phases = nullptr;
  LayerCtl* ctl = nullptr;
  unsigned* status = nullptr;
  float* xchg = nullptr;    // split items: hidden values [item][32]
  unsigned* xcnt = nullptr; // and the parts that wrote them [item]
  // row-owner kernel: per-item chunk arrivals (zero between launches) and
  // the quantized hidden slices [item][32] + scales [item]
  unsigned* rb_cnt = nullptr;
  uint8_t* rb_hq = nullptr;
  float* rb_hs = nullptr;
  // frc_run staging: one copy in ([x][gate][expert], packed for the call's
  // token count) and one copy out ([status word, 16 B][y]).  h_out is mapped
  // into the device's address space (h_out_dev): calls of up to
  // FRC_MAX_TOKENS tokens have a kernel store [status][y] there instead of a
  // device-to-host copy.
  uint8_t *d_in = nullptr, *d_out = nullptr, *h_in = nullptr, *h_out = nullptr, *h_out_dev = nullptr;
  float *d_y = nullptr, *h_y = nullptr;  // inside d_out / h_out
  unsigned* h_status = nullptr;          // start of h_out

  // FRC_ACT_AVX2: the activation quantization [T][d] int8, [T][d/256] f32,
  // [T][d/32] i16 (kMaxTokens rows each), the worker count whose job
  // dealing it reproduces, and the blocks in load order (the AVX2 backend's
  // job order: appended at load, ascending again after an unload)
  uint8_t* avx2_x = nullptr;
  unsigned avx2_workers = 1;
  uint8_t slot_order[FRC_MAX_BLOCKS] = {};
  unsigned slot_count = 0;

  cudaStream_t stream = nullptr;
  uint8_t* pool = nullptr;
  unsigned pool_count = 0;
  unsigned long long launches = 0;
  bool attr_set[2][3] = {};   // [activation mode][variant: tokens, one token, split items]
  unsigned occ_smem[2][3] = {};
  int occ_val[2][3] = {};
  unsigned last_T = 0, last_S = 0, last_G = 0;
  // in-box reduce: this rank's inbox (IPC-exported), every rank's inbox as
  // mapped here, the per-CTA launch counters
  uint8_t* inbox = nullptr;
  uint8_t* peer[kMaxPeers] = {};
  unsigned rank = 0, world = 0;
  uint16_t last_expert[FRC_MAX_TOKENS * FRC_TOPK] = {};
  float last_gate[FRC_MAX_TOKENS * FRC_ACTIVE] = {};
  // prefill (bursts above FRC_MAX_TOKENS; MXFP4 gate/up and down only):
  // activations, pairs, work lists, hidden values and expert partials
  int8_t* pf_xq = nullptr;
  int8_t* pf_xr = nullptr;
  float* pf_xs = nullptr;
  int2* pf_xme = nullptr;
  uint16_t* pf_pair_token = nullptr;
  unsigned* pf_slot_pair = nullptr;
  unsigned* pf_counts = nullptr;
  uint4* pf_items_gu = nullptr;
  uint4* pf_items_dn = nullptr;
  int8_t* pf_hq = nullptr;
  float* pf_hs = nullptr;
  float* pf_ye = nullptr;
  int2* pf_xvr = nullptr;  // Q4_K gate/up: per token and 32-block {sum v, sum r}
  int8_t* pf_xqn = nullptr;  // v and r in natural order (the shared expert's Q8_0 rows)
  int8_t* pf_xrn = nullptr;
  bool pf_attr = false;
  unsigned last_pf_S = 0;
  // tensor maps of the loaded layer regions (valid while tmap_of matches layer_ptr)
  CUtensorMap tmap[FRC_MAX_BLOCKS][FRC_MAX_LAYERS];
  const uint8_t* tmap_of[FRC_MAX_BLOCKS][FRC_MAX_LAYERS] = {};
  // optional CUDA events around the five prefill stages (frc_prefill_timing)
  cudaEvent_t pf_ev[6] = {};
  // and around the three FRC_ACT_AVX2 launches (frc_avx2_timing)
  cudaEvent_t av_ev[4] = {};
  bool av_timing = false, av_timed = false, av_attr = false;
  int av_stage_per_sm = 0;  // CTAs of the staged AVX2 job kernel an SM holds
  bool pf_timing = false, pf_timed = false;
  // bounded waits of the layer kernel (frc_set_wait_limit) and the test-only
  // grid-barrier offset (frc_debug_barrier_extra)
  unsigned long long wait_ns = kWaitNs;
  unsigned bar_extra = 0;
  // one-token Q8 calls: the row-owner kernel (frc_layer_rb.cuh) unless
  // frc_debug_layer_variant chose the item kernel; its attribute and the
  // occupancy of its last shared-memory size
  int rb = 1;  // 0 item kernel, 1 row-owner up to kRbMaxSlices slices, 2 row-owner whenever it fits
  bool rb_attr = false;
  unsigned rb_occ_smem = 0;
  int rb_occ_val = 0;
  char err[256] = {};
};

// Prefill bounds: pairs of one call, and work items (tiles of 64 tokens of
// each expert: at most pairs / 64 + 512 of them).
constexpr size_t kPfMaxPairs = size_t(FRC_MAX_PREFILL_TOKENS) * FRC_ACTIVE;  // ten routed + the shared expert
constexpr size_t kPfMaxTiles = kPfMaxPairs / kPfTile + FRC_ROUTED_EXPERTS + 1;

static int fail(frc_context* c, int rc, const char* fmt, ...) {
  if (c) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(c->err, sizeof c->err, fmt, ap);
    va_end(ap);
  }
  return rc;
}
#define CK(call)                                                                             \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) return fail(c, FRC_IO, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

static unsigned align_up(unsigned v, unsigned a) { return (v + a - 1) / a * a; }

// Bytes of one token's frc_run input: x, gate, expert ids.
static size_t kInBytesPerToken(unsigned d) { return sizeof(float) * (d + FRC_ACTIVE) + sizeof(uint16_t) * FRC_TOPK; }

// fp32 hidden activations of the largest call: [unique expert][slice][token][32]
constexpr size_t kHiddenBytes = sizeof(float) * kMaxUnique * kMaxBlocks * kMaxTokens * 32;
// items of a one-token call: eleven experts x 20 slices
constexpr unsigned kRbItems = 11 * kMaxBlocks;
// slices loaded up to which one-token calls take the row-owner kernel
constexpr unsigned kRbMaxSlices = 2;

// Dynamic shared memory a CTA may use with two CTAs an SM (228 KB an SM,
// 1 KB reserved a CTA), and with one.
constexpr unsigned kSmemTwoPerSm = (228 * 1024 - 2 * 1024) / 2;
constexpr unsigned kSmemOnePerSm = 227 * 1024;

// Shared memory of one layer CTA within `limit` bytes and the chunking of an
// item into ring slots.  A slot is sized for a gate/up chunk of 16 routed
// neurons (both rows), halved while fewer than four slots fit; the shared
// expert's chunk and the down chunks are cut to the slot.  Returns false
// when two slots of one neuron pair do not fit.
static bool smem_layout(const frc_context* c, unsigned T, unsigned G, int act, unsigned limit, LayerSmem* out) {
  const unsigned d = c->g.hidden, P = d / 64;
  if (T * d / 512 > kActWarps * kMaxRounds) return false;  // activation sums: one a warp-pass of 512 floats
  LayerSmem m{};
  unsigned o = 64 + 256;  // mbarriers, then 64 misc words
  auto take = [&](unsigned bytes) { unsigned at = o; o = align_up(o + bytes, 16); return at; };
  m.ids = take(2 * T * 10);
  m.gates = take(4 * T * 11);
  // plan tables sized for this launch's tokens (one token: eleven experts,
  // no first-appearance table), which leaves the rest to the ring
  const unsigned mu = T * 10 + 1 < kMaxUnique ? T * 10 + 1 : kMaxUnique;
  m.max_unique = mu;
  m.first = T > 1 ? take(4 * 512) : 0;
  m.uid = take(2 * mu);
  m.umask = take(4 * mu);
  m.ugate = take(4 * mu * T);
  m.upre = take(4 * (mu + 1));
  m.rms = take(4 * T);
  m.bases = take(8 * kMaxBlocks);
  m.rpart = take(4 * kActWarps * ((T * d / 16 + kActThreads - 1) / kActThreads));  // [round][warp] sums
  m.tokpair = take(2 * (T * 11));
  if (act == FRC_ACT_Q8) {
    m.xq = take(T * d);
    m.xr = take(T * d);
    m.xp = c->g.gate_type == FRC_MXFP4 ? take(T * d) : 0;
    m.xrp = c->g.gate_type == FRC_MXFP4 ? take(T * d) : 0;
    m.xst = take(16 * T * P);
    m.xvr = take(16 * T * P);
    m.hq = take(32 * T);
  } else {
    m.xf = take(4 * T * d);
    m.hq = take(4 * 32 * T);
  }
  m.gv = take(4 * 32 * T);
  m.uv = take(4 * 32 * T);
  m.hg = take(4 * T);
  m.ylocal = take(4 * T * 4 * ((d / 4 + G - 1) / G));
  o = align_up(o, 128);
  if (o >= limit) return false;
  const unsigned avail = limit - o, rowb = static_cast<unsigned>(c->row_bytes);
  const unsigned srow = static_cast<unsigned>(c->shared_row);
  const unsigned ss_r = c->g.down_type == FRC_Q8_0 ? 2 : 1, pb_r = c->g.down_type == FRC_Q8_0 ? 32 : 16;
  unsigned kn = 16;
  while (kn > 4 && avail / (2 * kn * rowb) < 4) kn /= 2;
  unsigned slot = 2 * kn * rowb;
  // the smallest shared chunk (four neurons) and down chunk (16 rows) must fit too
  slot = slot > 8 * srow ? slot : 8 * srow;
  slot = slot > 16 * 34 ? slot : 16 * 34;
  slot = align_up(slot, 128);
  unsigned K = avail / slot;
  // the reduce stages one token's terms [11][S][rows], weights [11][S] and
  // sums [11][rows] in the ring (rows: 4-row units, S up to 20)
  const unsigned rows4 = 4 * ((d / 4 + G - 1) / G);
  const unsigned staged = 4 * (11 * kMaxBlocks * (rows4 + 1) + 11 * rows4);
  if (K < 2 || K * slot < staged) return false;
  K = K < kMaxSlots ? K : kMaxSlots;
  // At most five copies in flight a CTA (one token: 4-5 slots ran 1 % faster
  // than 6, the extra copies delaying every CTA's first chunks), while five
  // slots still hold the reduce's staging.
  if (K > kRingSlots && kRingSlots * slot >= staged) K = kRingSlots;
  unsigned kns = 16;
  while (kns > 1 && 2 * kns * srow > slot) kns /= 2;
  if (kn < 4 || kns < 4) return false;  // a gate/up chunk holds at least one warp's four neurons
  auto down_rows = [&](unsigned per_row) {
    unsigned dn = slot / per_row / 16 * 16;
    dn = dn < d ? dn : d;
    const unsigned n = (d + dn - 1) / dn;
    return align_up((d + n - 1) / n, 16);
  };
  m.ring = o;
  m.slot_bytes = slot;
  m.slots = K;
  m.kn_r = kn;
  m.kn_s = kns;
  m.dn_r = down_rows(ss_r + pb_r);
  m.dn_s = down_rows(2 + 32);
  m.total = o + K * slot;
  m.mag_ch_r = div_magic(32 / m.kn_r + (d + m.dn_r - 1) / m.dn_r);
  m.mag_ch_s = div_magic(32 / m.kn_s + (d + m.dn_s - 1) / m.dn_s);
  *out = m;
  return true;
}

template <int ACT>
static int launch_layer(frc_context* c, LayerParams& a, cudaStream_t s, bool overlap) {
  const int ai = ACT == FRC_ACT_Q8;
  auto prepare = [&](void (*kern)(LayerParams), int split) -> int {
    if (!c->attr_set[ai][split]) {
      CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
      c->attr_set[ai][split] = true;
    }
    return FRC_OK;
  };
  // CTAs an SM for `bytes` of shared memory (cached: it depends only on the
  // kernel variant and the size)
  auto occupancy = [&](void (*kern)(LayerParams), int split, unsigned bytes, int* per_sm) -> int {
    if (c->occ_smem[ai][split] == bytes) {
      *per_sm = c->occ_val[ai][split];
      return FRC_OK;
    }
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kern, kLayerThreads, bytes));
    c->occ_smem[ai][split] = bytes;
    c->occ_val[ai][split] = *per_sm;
    return FRC_OK;
  };
  // one token: the variant with the token count folded to 1
  const int var = a.T == 1 ? 1 : 0;
  auto kern = var ? moe_layer_kernel<ACT, false, true> : moe_layer_kernel<ACT, false, false>;
  int orc;
  if ((orc = prepare(kern, var))) return orc;
  // Two CTAs an SM when their shared memory fits, else one; all resident
  // (the kernel has a grid barrier).
  unsigned per = 2, G = 2 * static_cast<unsigned>(c->sms);
  int per_sm = 0;
  bool fits = smem_layout(c, a.T, G, ACT, kSmemTwoPerSm, &a.sm);
  // Two CTAs an SM only while each keeps a full ring (eight-neuron gate/up
  // chunks, four slots): with more tokens the activations crowd the ring out
  // and a CTA waits on its own refills (16 tokens ran 35 % faster on one CTA
  // an SM with its larger ring; 4 and 8 tokens ran faster on two).
  if (fits) fits = a.sm.kn_r >= 8 && a.sm.slots >= 4;
  if (fits) {
    if ((orc = occupancy(kern, var, a.sm.total, &per_sm))) return orc;
    fits = per_sm >= 2;
  }
  if (!fits) {
    per = 1;
    G = static_cast<unsigned>(c->sms);
    if (!smem_layout(c, a.T, G, ACT, kSmemOnePerSm, &a.sm))
      return fail(c, FRC_INVALID, "%u tokens need too much shared memory", a.T);
    if ((orc = occupancy(kern, var, a.sm.total, &per_sm))) return orc;
  }
  if (per_sm < static_cast<int>(per)) return fail(c, FRC_INVALID, "layer kernel does not fit an SM (%u bytes)", a.sm.total);
  // One token and few items (slices split over several GPUs): split each
  // item in H parts on H CTAs when all parts fit one round of the grid, so
  // the weight stream and the chain of each CTA shrink with the item.
  a.H = 1;
  a.Hshift = 0;
  if (a.T == 1)
    for (unsigned h = 4, sh = 2; h > 1; h >>= 1, --sh)
      if (h * 11 * a.S <= G && (32 / a.sm.kn_r) % h == 0 && (32 / a.sm.kn_s) % h == 0) {
        a.H = h;
        a.Hshift = sh;
        break;
      }
  if (a.H > 1) {
    auto ks = moe_layer_kernel<ACT, true, true>;
    int ps = 0;
    if ((orc = prepare(ks, 2)) || (orc = occupancy(ks, 2, a.sm.total, &ps))) return orc;
    if (ps >= static_cast<int>(per)) kern = ks;
    else { a.H = 1; a.Hshift = 0; }  // the split variant does not fit as many CTAs
  }
  {
    const unsigned d = a.d, H = a.H;
    a.sm.mag_ch_r = div_magic(32 / a.sm.kn_r / H + (d / H + a.sm.dn_r - 1) / a.sm.dn_r);
    a.sm.mag_ch_s = div_magic(32 / a.sm.kn_s / H + (d / H + a.sm.dn_s - 1) / a.sm.dn_s);
  }
  a.xchg = c->xchg;
  a.xcnt = c->xcnt;
  a.bar_inc = 2 * static_cast<unsigned>(c->sms) / G;  // G is one or two CTAs an SM
  a.wait_ns = c->wait_ns;
  a.bar_extra = c->bar_extra;
  // Co-residency of the grid (checked above) is what the grid barrier needs.
  // A plain launch asks the runtime to check it; an overlapped launch
  // (programmatic stream serialization) gets it as the previous launch's
  // CTAs leave their SMs.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if (overlap) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  } else {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.gridDim = dim3(G);
  c->last_G = G;
  cfg.blockDim = dim3(kLayerThreads);
  cfg.dynamicSmemBytes = a.sm.total;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, kern, a));
  ++c->launches;
  return FRC_OK;
}

// Shared memory of the row-owner kernel within `limit` bytes: plan tables,
// one token's activations, this CTA's down-row staging (every item's rows
// [y0, y0 + R), R at most rows_max), and a ring of gate/up chunks (8 routed
// neurons, 4 shared) that phase B reuses for the hidden values and terms.
static bool smem_layout_rb(const frc_context* c, unsigned G, unsigned S, bool shared, unsigned limit, LayerSmem* out) {
  const unsigned d = c->g.hidden, P = d / 64;
  LayerSmem m{};
  unsigned o = 64 + 256;
  auto take = [&](unsigned bytes) { unsigned at = o; o = align_up(o + bytes, 16); return at; };
  m.uid = take(2 * 11);
  m.ugate = take(4 * 11);
  m.rms = take(4);
  m.rpart = take(4 * kActWarps * ((d / 16 + kActThreads - 1) / kActThreads));
  const bool mx = c->g.gate_type == FRC_MXFP4;
  m.xq = take(d);
  m.xr = take(d);
  m.xp = mx ? take(d) : 0;
  m.xrp = mx ? take(d) : 0;
  m.xst = take(16 * P);
  m.xvr = take(16 * P);
  const unsigned NU = d / 4, RM = 4 * ((NU + G - 1) / G);
  m.rows_max = RM;
  m.ylocal = take(4 * RM);
  const unsigned pb_r = c->g.down_type == FRC_Q8_0 ? 32 : 16;
  m.dnw = (15 + 2 * RM + 15) / 16;  // scale bytes from a 16-byte boundary: at most 15 + 2 x rows
  m.dnb_r = RM * pb_r + 16 * m.dnw;
  m.dnb_s = RM * 32 + 16 * m.dnw;
  m.dnb = take(10 * S * m.dnb_r + (shared ? S * m.dnb_s : 0));
  o = align_up(o, 128);
  if (o >= limit) return false;
  const unsigned rowb = static_cast<unsigned>(c->row_bytes), srow = static_cast<unsigned>(c->shared_row);
  unsigned slot = 2 * 8 * rowb > 2 * 4 * srow ? 2 * 8 * rowb : 2 * 4 * srow;
  slot = align_up(slot, 128);
  unsigned K = (limit - o) / slot;
  K = K < kRingSlots ? K : kRingSlots;
  const unsigned NI = (10 + (shared ? 1 : 0)) * S;
  const unsigned staged = align_up(NI * 32, 16) + 4 * ((NI + 3) & ~3u) + 4 * NI * RM + 4 * ((11 * RM + 3) & ~3u);
  if (K < 2 || K * slot < staged) return false;
  if ((48 * S + G - 1) / G > 16) return false;  // chunks a CTA: the kernel lists the items it completes in 16 words
  m.ring = o;
  m.slot_bytes = slot;
  m.slots = K;
  m.kn_r = 8;
  m.kn_s = 4;
  m.total = o + K * slot;
  *out = m;
  return true;
}

static int launch_layer_rb(frc_context* c, LayerParams& a, cudaStream_t s, bool overlap, bool shared) {
  if (!c->rb_attr) {
    CK(cudaFuncSetAttribute(moe_layer_rb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    c->rb_attr = true;
  }
  auto occupancy = [&](unsigned bytes, int* per_sm) -> int {
    if (c->rb_occ_smem != bytes) {
      CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c->rb_occ_val, moe_layer_rb_kernel, kLayerThreads, bytes));
      c->rb_occ_smem = bytes;
    }
    *per_sm = c->rb_occ_val;
    return FRC_OK;
  };
  // two CTAs an SM when their shared memory fits, else one; all resident
  unsigned G = 2 * static_cast<unsigned>(c->sms);
  int per_sm = 0, orc;
  bool fits = smem_layout_rb(c, G, a.S, shared, kSmemTwoPerSm, &a.sm);
  if (fits) {
    if ((orc = occupancy(a.sm.total, &per_sm))) return orc;
    fits = per_sm >= 2;
  }
  if (!fits) {
    G = static_cast<unsigned>(c->sms);
    if (!smem_layout_rb(c, G, a.S, shared, kSmemOnePerSm, &a.sm))
      return fail(c, FRC_INVALID, "one-token layer does not fit shared memory (%u slices)", a.S);
    if ((orc = occupancy(a.sm.total, &per_sm))) return orc;
    if (per_sm < 1) return fail(c, FRC_INVALID, "layer kernel does not fit an SM (%u bytes)", a.sm.total);
  }
  a.H = 1;
  a.Hshift = 0;
  a.bar_inc = 2 * static_cast<unsigned>(c->sms) / G;
  a.wait_ns = c->wait_ns;
  a.bar_extra = c->bar_extra;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if (overlap) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  } else {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.gridDim = dim3(G);
  c->last_G = G;
  cfg.blockDim = dim3(kLayerThreads);
  cfg.dynamicSmemBytes = a.sm.total;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, moe_layer_rb_kernel, a));
  ++c->launches;
  return FRC_OK;
}

// Device buffers a launch writes and reads back: the down terms and their
// weights (handed from the item phase to the reduce) and the optional fp32
// copy of the hidden activations.
struct RunScratch {
  float* partial;  // [pair][S][d]
  float* gsv;      // [pair][S]
  float* hidden;   // [u*S+s][T][32] or null
};

static int run_long(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                    const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags,
                    cudaStream_t s, const struct RunScratch* scratch, bool chunks);

static int run_device(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                      const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags,
                      cudaStream_t s, const RunScratch* scratch = nullptr, bool chunks = false,
                      unsigned* status = nullptr) {
  if (!c || !expert || !gate || !x || !y) return fail(c, FRC_INVALID, "null argument");
  if (act == FRC_ACT_AVX2) return fail(c, FRC_UNSUPPORTED, "FRC_ACT_AVX2: through frc_run (host buffers) only");
  if (act != FRC_ACT_Q8 && act != FRC_ACT_F32) return fail(c, FRC_INVALID, "unknown activation mode");
  if (T > FRC_MAX_TOKENS) return run_long(c, layer, T, expert, gate, x, x_add, x_out, y, act, flags, s, scratch, chunks);
  if (flags & FRC_RUN_X_BF16)
    return fail(c, FRC_UNSUPPORTED, "bf16 x: only bursts of more than %u tokens", FRC_MAX_TOKENS);
  if (T < 1 || T > FRC_MAX_TOKENS || layer >= c->g.layers) return fail(c, FRC_INVALID, "tokens or layer out of range");
  if (act != FRC_ACT_Q8 && act != FRC_ACT_F32) return fail(c, FRC_INVALID, "unknown activation mode");
  LayerParams a{};
  unsigned S = 0;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b) {
    bool any = false;
    for (unsigned l = 0; l < c->g.layers; ++l) any |= c->layer_ptr[b][l] != nullptr;
    if (!any) continue;
    if (!c->layer_ptr[b][layer]) return fail(c, FRC_STATE, "block %u is loaded but not layer %u", b, layer);
    a.base[S++] = c->layer_ptr[b][layer];
  }
  if (!S) return fail(c, FRC_STATE, "no block loaded");
  a.expert = expert; a.gate = gate; a.x = x; a.x_add = x_add; a.x_out = x_out; a.y = y;
  if (scratch) {
    a.partial = scratch->partial; a.gsv = scratch->gsv; a.hidden = scratch->hidden;
  } else {
    a.partial = c->partial; a.gsv = c->gsv; a.hidden = c->hidden;
  }
  a.ctl = c->ctl; a.status = status ? status : c->status;
  if (flags & FRC_RUN_PEER) {
    if (c->world < 2) return fail(c, FRC_STATE, "FRC_RUN_PEER without frc_peer_attach");
    for (unsigned r = 0; r < c->world; ++r) a.peer[r] = c->peer[r];
    a.rank = c->rank; a.world = c->world;
  } else {
    a.world = 1;
  }
  a.phases = c->phases;
  a.S = S; a.T = T; a.d = c->g.hidden;
  a.mag_S = div_magic(S);
  a.norm = flags & FRC_RUN_RMSNORM ? 1u : 0u;
  a.gate_type = c->g.gate_type; a.down_type = c->g.down_type;
  a.row_bytes = static_cast<unsigned>(c->row_bytes); a.proj_bytes = static_cast<unsigned>(c->proj_bytes);
  a.shared_row = static_cast<unsigned>(c->shared_row); a.shared_proj = static_cast<unsigned>(c->shared_proj);
  a.slice_bytes = static_cast<unsigned>(c->slice_bytes);
  c->last_S = S;
  const bool overlap = (flags & FRC_RUN_OVERLAP) != 0;
  LayerSmem probe;
  // one token over at most kRbMaxSlices slices (an 8-GPU share): the
  // row-owner kernel, 3 % faster there; with more slices its gather of
  // every item's down rows costs more than it saves (measured 1..20 slices)
  if (T == 1 && act == FRC_ACT_Q8 && (c->rb == 2 || (c->rb == 1 && S <= kRbMaxSlices)) &&
      (smem_layout_rb(c, 2 * static_cast<unsigned>(c->sms), S, true, kSmemTwoPerSm, &probe) ||
       smem_layout_rb(c, static_cast<unsigned>(c->sms), S, true, kSmemOnePerSm, &probe))) {
    // the row-owner kernel when its staging fits (all of the benchmark's and
    // the reference's geometries; very wide layers fall back to the item
    // kernel).  Hidden values go through global memory (the fixed-scratch
    // call lends its array, which the down terms do not use); the staging
    // holds the shared expert's rows too, since its gate is on the device.
    a.rb_cnt = c->rb_cnt;
    a.rb_hq = c->rb_hq;
    a.rb_hs = c->rb_hs;
    if (!a.hidden) {
      a.hidden = a.partial;
      a.rb_hq = reinterpret_cast<uint8_t*>(a.partial + 32 * kRbItems);
      a.rb_hs = a.partial + 40 * kRbItems;
    }
    return launch_layer_rb(c, a, s, overlap, true);
  }
  if (act == FRC_ACT_Q8) return launch_layer<FRC_ACT_Q8>(c, a, s, overlap);
  return launch_layer<FRC_ACT_F32>(c, a, s, overlap);
}

// A burst of more than FRC_MAX_TOKENS tokens.  With MXFP4 or Q4_K gate/up
// rows, MXFP4 down rows, Q8 activations and no run flag but FRC_RUN_X_BF16
// it takes the tensor-core prefill path (frc_prefill.cuh; the Q8_0 shared
// expert included); otherwise it runs as bursts of FRC_MAX_TOKENS through
// the layer kernel (`chunks` forces that).
// The layer region of (block, layer) as a 2D byte array of row_bytes-long
// rows (every slice of an MXFP4/MXFP4 layer is a whole number of them), for
// 128-byte x 64-row tiled TMA boxes, 128-byte swizzle.  Encoded once per
// region through the driver's cuTensorMapEncodeTiled.
static PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
static std::mutex g_encode_mu;

static int layer_tmap(frc_context* c, unsigned b, unsigned layer, CUtensorMap* out) {
  const uint8_t* base = c->layer_ptr[b][layer];
  if (c->tmap_of[b][layer] != base) {
    {
      std::lock_guard<std::mutex> lock(g_encode_mu);
      if (!g_encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
          return fail(c, FRC_IO, "cuTensorMapEncodeTiled not available");
        g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
    }
    CUresult r;
    if (c->g.gate_type == FRC_Q4_K) {
      // Q4_K gate/up rows (the reference layout: a slice is not a whole
      // number of rows): bytes of a row x the slice's 64 gate/up rows x the
      // 512 routed slices; a 144 B x 64-row box is one super-block of them
      const cuuint64_t dims[3] = {c->row_bytes, 64, FRC_ROUTED_EXPERTS};
      const cuuint64_t strides[2] = {c->row_bytes, c->slice_bytes};
      const cuuint32_t box[3] = {144, 64, 1}, estr[3] = {1, 1, 1};
      r = g_encode_tiled(&c->tmap[b][layer], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const cuuint64_t dims[2] = {c->row_bytes, c->layer_bytes / c->row_bytes};
      const cuuint64_t strides[1] = {c->row_bytes};
      const cuuint32_t box[2] = {128, 64}, estr[2] = {1, 1};
      r = g_encode_tiled(&c->tmap[b][layer], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return fail(c, FRC_IO, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    c->tmap_of[b][layer] = base;
  }
  *out = c->tmap[b][layer];
  return FRC_OK;
}

static int run_prefill(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                       const float* x, float* y, cudaStream_t s, bool x_bf16) {
  PrefillArgs a{};
  unsigned S = 0;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b) {
    bool any = false;
    for (unsigned l = 0; l < c->g.layers; ++l) any |= c->layer_ptr[b][l] != nullptr;
    if (!any) continue;
    if (!c->layer_ptr[b][layer]) return fail(c, FRC_STATE, "block %u is loaded but not layer %u", b, layer);
    const int rc = layer_tmap(c, b, layer, &a.tmap[S]);
    if (rc) return rc;
    a.base[S++] = c->layer_ptr[b][layer];
  }
  if (!S) return fail(c, FRC_STATE, "no block loaded");
  const unsigned d = c->g.hidden;
  a.x = x; a.expert = expert; a.gate = gate; a.y = y;
  a.T = T; a.d = d; a.S = S;
  a.x_bf16 = x_bf16 ? 1u : 0u;
  a.q4k = c->g.gate_type == FRC_Q4_K ? 1u : 0u;
  a.xvr = a.q4k ? c->pf_xvr : nullptr;
  a.xqn = c->pf_xqn; a.xrn = c->pf_xrn;
  a.shared_row = static_cast<unsigned>(c->shared_row);
  a.shared_proj = static_cast<unsigned>(c->shared_proj);
  a.row_bytes = static_cast<unsigned>(c->row_bytes);
  a.slice_bytes = c->slice_bytes;
  a.slice_rows = static_cast<unsigned>(c->slice_bytes / c->row_bytes);
  a.xq = c->pf_xq; a.xr = c->pf_xr; a.xs = c->pf_xs; a.xme = c->pf_xme;
  a.pair_token = c->pf_pair_token; a.slot_pair = c->pf_slot_pair;
  a.counts = c->pf_counts; a.items_gu = c->pf_items_gu; a.items_dn = c->pf_items_dn;
  a.hq = c->pf_hq; a.hs = c->pf_hs; a.ye = c->pf_ye; a.status = c->status;
  a.phases = c->phases;
  c->last_G = 4 * c->sms;  // frc_debug_phases: [cta][64] stamps
  const unsigned smem = sizeof(PfSmem);
  if (!c->pf_attr) {
    const void* kernels[] = {reinterpret_cast<const void*>(prefill_mma_kernel<kGateUp, false, false>),
                             reinterpret_cast<const void*>(prefill_mma_kernel<kGateUp, true, false>),
                             reinterpret_cast<const void*>(prefill_mma_kernel<kGateUp, false, true>),
                             reinterpret_cast<const void*>(prefill_mma_kernel<kDown, false, false>),
                             reinterpret_cast<const void*>(prefill_mma_kernel<kDown, false, true>)};
    for (const void* k : kernels) CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    // The kernels' setmaxnreg split is sized for 128 registers a thread at
    // launch: with fewer, the epilogue's increase could never be granted.
    for (const void* k : kernels) {
      cudaFuncAttributes fa;
      CK(cudaFuncGetAttributes(&fa, k));
      if (fa.numRegs != 128)
        return fail(c, FRC_UNSUPPORTED, "prefill kernel built with %d registers a thread (its split needs 128)",
                    fa.numRegs);
    }
    c->pf_attr = true;
  }
  const unsigned groups = T * (d / 64);
  const bool timed = c->pf_timing;
  auto mark = [&](unsigned i) { if (timed) cudaEventRecord(c->pf_ev[i], s); };
  mark(0);
  prefill_quantize_kernel<<<(groups + 7) / 8, 256, 0, s>>>(a);
  mark(1);
  prefill_group_kernel<<<1, 1024, 0, s>>>(a);
  mark(2);
  // the shared expert's items (none unless a token has a shared gate: the
  // launch then ends at once), then the routed experts'
  prefill_mma_kernel<kGateUp, false, true><<<c->sms, kPfThreads, smem, s>>>(a);
  if (a.q4k) prefill_mma_kernel<kGateUp, true, false><<<c->sms, kPfThreads, smem, s>>>(a);
  else prefill_mma_kernel<kGateUp, false, false><<<c->sms, kPfThreads, smem, s>>>(a);
  mark(3);
  prefill_mma_kernel<kDown, false, true><<<c->sms, kPfThreads, smem, s>>>(a);
  prefill_mma_kernel<kDown, false, false><<<c->sms, kPfThreads, smem, s>>>(a);
  mark(4);
  prefill_combine_kernel<<<dim3((d / 4 + 255) / 256, T), 256, 0, s>>>(a);
  mark(5);
  c->pf_timed = timed;
  CK(cudaGetLastError());
  c->launches += 7;
  c->last_pf_S = S;
  return FRC_OK;
}

static int run_long(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                    const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags,
                    cudaStream_t s, const RunScratch* scratch, bool chunks) {
  if (T > FRC_MAX_PREFILL_TOKENS || layer >= c->g.layers) return fail(c, FRC_INVALID, "tokens or layer out of range");
  if (!chunks && act == FRC_ACT_Q8 && (flags & ~unsigned(FRC_RUN_X_BF16)) == 0 && !scratch && c->pf_ye)
    return run_prefill(c, layer, T, expert, gate, x, y, s, (flags & FRC_RUN_X_BF16) != 0);
  if (flags & FRC_RUN_X_BF16)
    return fail(c, FRC_UNSUPPORTED, "bf16 x: only bursts on the tensor-core path (MXFP4 or Q4_K gate/up, MXFP4 down, Q8, no other flag)");
  const size_t d = c->g.hidden;
  for (unsigned t0 = 0; t0 < T; t0 += FRC_MAX_TOKENS) {
    const unsigned n = T - t0 < FRC_MAX_TOKENS ? T - t0 : FRC_MAX_TOKENS;
    const int rc = run_device(c, layer, n, expert + t0 * FRC_TOPK, gate + t0 * FRC_ACTIVE, x + t0 * d,
                              x_add ? x_add + t0 * d : nullptr, x_out ? x_out + t0 * d : nullptr, y + t0 * d, act,
                              flags, s, scratch);
    if (rc) return rc;
  }
  return FRC_OK;
}

// After a launch whose bounded wait ran out (every kernel of the context has
// ended: the caller synchronized): the grid barrier's counter is off its
// lattice and the split-item counts may be partial; both restart at zero.
// The in-box reduce epoch is kept (the group detaches and attaches again).
static int reset_after_timeout(frc_context* c, cudaStream_t s) {
  CK(cudaMemsetAsync(c->ctl, 0, offsetof(LayerCtl, peer_epoch), s));
  CK(cudaMemsetAsync(c->xcnt, 0, sizeof(unsigned) * kMaxUnique, s));
  CK(cudaMemsetAsync(c->rb_cnt, 0, sizeof(unsigned) * kRbItems, s));
  CK(cudaStreamSynchronize(s));
  return FRC_OK;
}

static int status_code(unsigned st) {
  if (st & kStTimeout) return FRC_IO;
  if (st & kStInvalid) return FRC_INVALID;
  if (st & kStNumeric) return FRC_NUMERIC;
  return FRC_OK;
}

// ------------------------------------------------ fixed-scratch layer run
// frc_run_device_fixed is frc_run_device with one difference: the buffers a
// launch writes and then reads back (the down terms and their weights, handed
// from the item phase to the reduce) live in the device array below, fixed
// when the module loads, instead of in the buffers frc_open allocated for the
// context, and no fp32 copy of the hidden activations is kept.  The call
// itself allocates nothing, on the first call or later: no cudaMalloc, no
// cudaFree, no allocating library routine.  It is meant for embedders whose
// device memory is carved up once at start-up (a serving process whose own
// pool owns every free byte after warm-up, so a later allocation fails or
// synchronises the device) and that want the footprint of a layer run known
// when the library is linked.
//
// Limit: kFixedScratchBytes.  A run needs 11 T x S x (d + 1) floats for T
// tokens over S loaded slices (every token's ten routed experts plus the
// shared one); with all 20 slices at d = 2048 that is up to 4 tokens a call.
// Larger calls are rejected with FRC_INVALID before anything is launched.
// Nothing in the array has to start at zero: every entry a launch reads was
// written earlier in the same launch.  The array is shared by every context
// and stream of a device, so two overlapping fixed-scratch calls on one device
// (different streams, or different contexts) race on it; callers serialise
// them.  The first call on each device looks the array's address up (with the
// context's device current); it does that set-up and nothing else extra, so
// make it before capturing the call into a CUDA graph.
constexpr size_t kFixedScratchBytes = size_t(8) << 20;
static __device__ __align__(256) float g_fixed_scratch[kFixedScratchBytes / sizeof(float)];
constexpr int kFixedDevices = 64;
static std::mutex g_fixed_mu;
static float* g_fixed_ptr[kFixedDevices];

// Floats of the down terms ([pair][S][d]) of the largest T-token call; the
// weights ([pair][S]) follow them.
static size_t fixed_partial(unsigned S, unsigned T, unsigned d) { return size_t(11) * T * S * d; }
static size_t fixed_need(unsigned S, unsigned T, unsigned d) {
  return sizeof(float) * (fixed_partial(S, T, d) + size_t(11) * T * S);
}

extern "C" {

const char* frc_strerror(int rc) {
  switch (rc) {
    case FRC_OK: return "ok";
    case FRC_INVALID: return "invalid argument or request";
    case FRC_STATE: return "wrong state (nothing loaded, slot occupied or empty)";
    case FRC_NUMERIC: return "nonfinite value, nonfinite scale or fp32 overflow";
    case FRC_IO: return "device or runtime failure";
    case FRC_UNSUPPORTED: return "no usable sm_100 device";
    case FRC_MISMATCH: return "result mismatch";
  }
  return "unknown status";
}

const char* frc_last_error(const frc_context* c) { return c ? c->err : "no context"; }
uint64_t frc_launch_count(const frc_context* c) { return c ? c->launches : 0; }

int frc_probe_device(int device, char* name, size_t cap, uint64_t* hbm_bytes, unsigned* sms) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return FRC_UNSUPPORTED;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return FRC_UNSUPPORTED;
  if (name && cap) {
    strncpy(name, prop.name, cap - 1);
    name[cap - 1] = 0;
  }
  if (hbm_bytes) *hbm_bytes = prop.totalGlobalMem;
  if (sms) *sms = static_cast<unsigned>(prop.multiProcessorCount);
  return FRC_OK;
}

int frc_set_wait_limit(frc_context* c, uint64_t ns) {
  if (!c || ns < 1000 || ns > 60000000000ull) return fail(c, FRC_INVALID, "wait limit must be 1 us .. 60 s");
  c->wait_ns = ns;
  return FRC_OK;
}

int frc_debug_layer_variant(frc_context* c, int variant) {
  if (!c || variant < 0 || variant > 2) return FRC_INVALID;
  c->rb = variant;
  return FRC_OK;
}

int frc_debug_barrier_extra(frc_context* c, unsigned extra) {
  if (!c || extra > 1024) return FRC_INVALID;
  c->bar_extra = extra;
  return FRC_OK;
}

int frc_open(int device, const frc_geometry* g, frc_context** out) {
  frc_context* c = nullptr;
  if (!out || frc_geometry_check(g)) return FRC_INVALID;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return FRC_UNSUPPORTED;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return FRC_UNSUPPORTED;
  c = new frc_context();
  c->device = device;
  c->sms = prop.multiProcessorCount;
  c->g = *g;
  const unsigned d = g->hidden;
  c->row_bytes = frc_row_bytes(g->gate_type, d);
  c->proj_bytes = FRC_NEURONS * c->row_bytes;
  c->slice_bytes = frc_slice_bytes(g);
  c->shared_row = frc_row_bytes(FRC_Q8_0, d);
  c->shared_proj = FRC_NEURONS * c->shared_row;
  c->shared_bytes = frc_shared_bytes(g);
  c->layer_bytes = frc_layer_bytes(g);
  int rc = FRC_OK;
  auto alloc = [&](void** p, size_t bytes) {
    if (rc == FRC_OK && cudaMalloc(p, bytes) != cudaSuccess) rc = fail(c, FRC_IO, "cudaMalloc(%zu) failed", bytes);
  };
  if (cudaSetDevice(device) != cudaSuccess) rc = FRC_IO;
  alloc(reinterpret_cast<void**>(&c->hidden), kHiddenBytes);
  alloc(reinterpret_cast<void**>(&c->partial), sizeof(float) * kMaxPairs * kMaxBlocks * d);
  alloc(reinterpret_cast<void**>(&c->gsv), sizeof(float) * kMaxPairs * kMaxBlocks);
  alloc(reinterpret_cast<void**>(&c->avx2_x), kMaxTokens * (static_cast<size_t>(d) + d / 256 * 4 + d / 32 * 2));
  alloc(reinterpret_cast<void**>(&c->ctl), sizeof(LayerCtl));
  alloc(reinterpret_cast<void**>(&c->xchg), sizeof(float) * kMaxUnique * 32);
  alloc(reinterpret_cast<void**>(&c->xcnt), sizeof(unsigned) * kMaxUnique);
  alloc(reinterpret_cast<void**>(&c->rb_cnt), sizeof(unsigned) * kRbItems);
  alloc(reinterpret_cast<void**>(&c->rb_hq), 32 * kRbItems);
  alloc(reinterpret_cast<void**>(&c->rb_hs), sizeof(float) * kRbItems);
  alloc(reinterpret_cast<void**>(&c->phases), sizeof(unsigned long long) * 16 * 1024);
  const size_t in_bytes = kInBytesPerToken(d) * FRC_MAX_PREFILL_TOKENS,
               out_bytes = 16 + sizeof(float) * FRC_MAX_PREFILL_TOKENS * d;
  // the tensor-core burst path: MXFP4 gate/up (a 2D map of whole rows over
  // the layer region) or Q4_K gate/up (a 3D map: byte, row, slice), MXFP4
  // down rows
  const bool pf_mx = g->gate_type == FRC_MXFP4 && c->slice_bytes % c->row_bytes == 0 &&
                     c->layer_bytes % c->row_bytes == 0;
  const bool pf_q4 = g->gate_type == FRC_Q4_K && d % 256 == 0 && c->slice_bytes % 16 == 0;
  if (g->down_type == FRC_MXFP4 && (pf_mx || pf_q4)) {
    const size_t T = FRC_MAX_PREFILL_TOKENS;
    alloc(reinterpret_cast<void**>(&c->pf_xq), T * d);
    alloc(reinterpret_cast<void**>(&c->pf_xr), T * d);
    alloc(reinterpret_cast<void**>(&c->pf_xs), sizeof(float) * T * (d / 64));
    alloc(reinterpret_cast<void**>(&c->pf_xme), sizeof(int2) * T * (d / 64));
    alloc(reinterpret_cast<void**>(&c->pf_pair_token), sizeof(uint16_t) * kPfMaxPairs);
    alloc(reinterpret_cast<void**>(&c->pf_slot_pair), sizeof(unsigned) * kPfMaxPairs);
    alloc(reinterpret_cast<void**>(&c->pf_counts), sizeof(unsigned) * 8);
    alloc(reinterpret_cast<void**>(&c->pf_items_gu), sizeof(uint4) * kPfMaxTiles * ((FRC_MAX_BLOCKS + 1) / 2));
    alloc(reinterpret_cast<void**>(&c->pf_items_dn), sizeof(uint4) * kPfMaxTiles * (d / 128));
    alloc(reinterpret_cast<void**>(&c->pf_hq), kPfMaxPairs * FRC_MAX_BLOCKS * 32);
    alloc(reinterpret_cast<void**>(&c->pf_hs), sizeof(float) * kPfMaxPairs * FRC_MAX_BLOCKS);
    alloc(reinterpret_cast<void**>(&c->pf_ye), sizeof(float) * kPfMaxPairs * d);
    if (pf_q4) alloc(reinterpret_cast<void**>(&c->pf_xvr), sizeof(int2) * T * (d / 32));
    alloc(reinterpret_cast<void**>(&c->pf_xqn), T * d);
    alloc(reinterpret_cast<void**>(&c->pf_xrn), T * d);
  }
  alloc(reinterpret_cast<void**>(&c->d_in), in_bytes);
  alloc(reinterpret_cast<void**>(&c->d_out), out_bytes);
  if (rc == FRC_OK) {
    c->status = reinterpret_cast<unsigned*>(c->d_out);
    c->d_y = reinterpret_cast<float*>(c->d_out + 16);
    if (cudaMallocHost(reinterpret_cast<void**>(&c->h_in), in_bytes) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void**>(&c->h_out), out_bytes, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_out_dev), c->h_out, 0) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess)
      rc = fail(c, FRC_IO, "pinned buffers or stream");
  }
  if (rc == FRC_OK) {
    c->h_status = reinterpret_cast<unsigned*>(c->h_out);
    c->h_y = reinterpret_cast<float*>(c->h_out + 16);
  }
  if (rc == FRC_OK && (cudaMemset(c->ctl, 0, sizeof(LayerCtl)) != cudaSuccess ||
                       cudaMemset(c->xcnt, 0, sizeof(unsigned) * kMaxUnique) != cudaSuccess ||
                       cudaMemset(c->rb_cnt, 0, sizeof(unsigned) * kRbItems) != cudaSuccess ||
                       cudaMemset(c->status, 0, sizeof(unsigned)) != cudaSuccess ||
                       cudaMemset(c->hidden, 0, kHiddenBytes) != cudaSuccess))
    rc = fail(c, FRC_IO, "cudaMemset");
  if (rc != FRC_OK) {
    frc_close(c);
    return rc;
  }
  *out = c;
  return FRC_OK;
}

int frc_close(frc_context* c) {
  if (!c) return FRC_INVALID;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  frc_peer_detach(c);
  for (auto& b : c->layer_ptr)
    for (auto& p : b) if (p) cudaFree(p);
  cudaFree(c->staging); cudaFree(c->hidden); cudaFree(c->partial); cudaFree(c->gsv); cudaFree(c->phases); cudaFree(c->ctl);
  cudaFree(c->xchg); cudaFree(c->xcnt); cudaFree(c->rb_cnt); cudaFree(c->rb_hq); cudaFree(c->rb_hs);
  cudaFree(c->d_in); cudaFree(c->d_out); cudaFree(c->pool);
  cudaFree(c->pf_xq); cudaFree(c->pf_xr); cudaFree(c->pf_xs); cudaFree(c->pf_xme); cudaFree(c->pf_pair_token); cudaFree(c->pf_slot_pair); cudaFree(c->pf_counts);
  cudaFree(c->pf_items_gu); cudaFree(c->pf_items_dn); cudaFree(c->pf_hq); cudaFree(c->pf_hs); cudaFree(c->pf_ye);
  cudaFree(c->pf_xvr); cudaFree(c->pf_xqn); cudaFree(c->pf_xrn); cudaFree(c->avx2_x);
  cudaFreeHost(c->h_in); cudaFreeHost(c->h_out);
  if (c->stream) cudaStreamDestroy(c->stream);
  for (auto e : c->pf_ev) if (e) cudaEventDestroy(e);
  for (auto e : c->av_ev) if (e) cudaEventDestroy(e);
  delete c;
  return FRC_OK;
}

static SliceShape shape_of(const frc_context* c) {
  SliceShape s{};
  s.d = c->g.hidden; s.gate_type = c->g.gate_type; s.down_type = c->g.down_type;
  s.row_bytes = static_cast<unsigned>(c->row_bytes); s.slice_bytes = static_cast<unsigned>(c->slice_bytes);
  s.shared_row = static_cast<unsigned>(c->shared_row); s.shared_bytes = static_cast<unsigned>(c->shared_bytes);
  return s;
}

// Allocates the region of (block, layer) if it is not there; a block's first
// region appends the block to the load order.
static int ensure_layer(frc_context* c, int block, unsigned layer) {
  if (c->layer_ptr[block][layer]) return FRC_OK;
  bool first = true;
  for (unsigned l = 0; l < FRC_MAX_LAYERS; ++l) first &= c->layer_ptr[block][l] == nullptr;
  CK(cudaMalloc(&c->layer_ptr[block][layer], c->layer_bytes));
  if (first) c->slot_order[c->slot_count++] = static_cast<uint8_t>(block);
  return FRC_OK;
}

int frc_load_layer(frc_context* c, int block, unsigned layer, const void* bytes, size_t len) {
  if (!c || block < 0 || block >= FRC_MAX_BLOCKS || layer >= c->g.layers || !bytes || len != c->layer_bytes)
    return fail(c, FRC_INVALID, "bad load_layer arguments");
  if (c->layer_ptr[block][layer]) return fail(c, FRC_STATE, "layer %u of block %d already loaded", layer, block);
  CK(cudaSetDevice(c->device));
  if (!c->staging) CK(cudaMalloc(&c->staging, c->layer_bytes));
  int rc = ensure_layer(c, block, layer);
  if (rc) return rc;
  CK(cudaMemcpyAsync(c->staging, bytes, c->layer_bytes, cudaMemcpyHostToDevice, c->stream));
  transcode_kernel<<<FRC_ROUTED_EXPERTS + 1, 256, 0, c->stream>>>(c->staging, c->layer_ptr[block][layer], FRC_ROUTED_EXPERTS, shape_of(c));
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  return FRC_OK;
}

int frc_refresh_layer(frc_context* c, int block, unsigned layer, const void* bytes, size_t len) {
  if (!c || block < 0 || block >= FRC_MAX_BLOCKS || layer >= c->g.layers || !bytes || len != c->layer_bytes)
    return fail(c, FRC_INVALID, "bad refresh_layer arguments");
  if (!c->layer_ptr[block][layer]) return fail(c, FRC_STATE, "layer %u of block %d not loaded", layer, block);
  CK(cudaSetDevice(c->device));
  if (!c->staging) CK(cudaMalloc(&c->staging, c->layer_bytes));
  CK(cudaMemcpyAsync(c->staging, bytes, c->layer_bytes, cudaMemcpyHostToDevice, c->stream));
  transcode_kernel<<<FRC_ROUTED_EXPERTS + 1, 256, 0, c->stream>>>(c->staging, c->layer_ptr[block][layer], FRC_ROUTED_EXPERTS, shape_of(c));
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  return FRC_OK;
}

int frc_load_unit(frc_context* c, int block, const void* unit, size_t len) {
  if (!c || block < 0 || block >= FRC_MAX_BLOCKS || !unit || len != frc_unit_bytes(&c->g))
    return fail(c, FRC_INVALID, "bad load_unit arguments");
  for (unsigned l = 0; l < c->g.layers; ++l)
    if (c->layer_ptr[block][l]) return fail(c, FRC_STATE, "block %d already loaded", block);
  for (unsigned l = 0; l < c->g.layers; ++l) {
    int rc = frc_load_layer(c, block, l, static_cast<const uint8_t*>(unit) + static_cast<size_t>(l) * c->layer_bytes, c->layer_bytes);
    if (rc) {
      frc_unload_unit(c, block);
      return rc;
    }
  }
  return FRC_OK;
}

int frc_unload_unit(frc_context* c, int block) {
  if (!c || block < 0 || block >= FRC_MAX_BLOCKS) return fail(c, FRC_INVALID, "bad block");
  bool any = false;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (unsigned l = 0; l < FRC_MAX_LAYERS; ++l)
    if (c->layer_ptr[block][l]) {
      cudaFree(c->layer_ptr[block][l]);
      c->layer_ptr[block][l] = nullptr;
      any = true;
    }
  // the remaining blocks ascending, as the AVX2 backend rebuilds its slots
  // after an unload (backends/avx2.c:607-613)
  c->slot_count = 0;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b)
    for (unsigned l = 0; l < FRC_MAX_LAYERS; ++l)
      if (c->layer_ptr[b][l]) { c->slot_order[c->slot_count++] = static_cast<uint8_t>(b); break; }
  return any ? FRC_OK : fail(c, FRC_STATE, "block %d not loaded", block);
}

// The reference node's unit loader (src/units.c:25-75) over frc_load_unit:
// each block of the mask is mapped and checked (frc_units.c), copied to HBM,
// and unmapped; a failure unloads the blocks this call loaded.
int frc_units_open(frc_context* c, const char* directory, uint32_t mask, int verify) {
  if (!c || !directory || !mask || mask >= (1u << FRC_MAX_BLOCKS)) return fail(c, FRC_INVALID, "bad units_open arguments");
  const uint64_t want = frc_unit_bytes(&c->g);
  uint32_t done = 0;
  int rc = FRC_OK;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS && rc == FRC_OK; ++b) {
    if (!(mask >> b & 1)) continue;
    const void* data = nullptr;
    size_t len = 0;
    char why[512];
    rc = frc_unit_map(directory, b, want, verify, &data, &len, why, sizeof why);
    if (rc) {
      fail(c, rc, "%s", why);
      break;
    }
    rc = frc_load_unit(c, static_cast<int>(b), data, len);
    frc_unit_unmap(data, len);
    if (rc == FRC_OK) done |= 1u << b;
  }
  if (rc)
    for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b)
      if (done >> b & 1) frc_unload_unit(c, static_cast<int>(b));
  return rc;
}

int frc_loaded_mask(const frc_context* c, uint32_t* mask) {
  if (!c || !mask) return FRC_INVALID;
  uint32_t m = 0;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b)
    for (unsigned l = 0; l < c->g.layers; ++l)
      if (c->layer_ptr[b][l]) { m |= 1u << b; break; }
  *mask = m;
  return FRC_OK;
}

// backends/ref.c:41-56, in its order: per token ids, gates, activations.
static int validate(const frc_context* c, unsigned T, const uint16_t* expert, const float* gate, const float* x) {
  if (fegetround() != FE_TONEAREST) return FRC_INVALID;
  const unsigned d = c->g.hidden;
  for (unsigned t = 0; t < T; ++t) {
    const uint16_t* id = expert + t * FRC_TOPK;
    for (unsigned e = 0; e < FRC_TOPK; ++e) {
      if (id[e] >= FRC_ROUTED_EXPERTS) return FRC_INVALID;
      for (unsigned j = 0; j < e; ++j) if (id[j] == id[e]) return FRC_INVALID;
    }
    for (unsigned e = 0; e < FRC_ACTIVE; ++e) {
      const float gv = gate[t * FRC_ACTIVE + e];
      if (!isfinite(gv)) return FRC_NUMERIC;
      if (gv < 0) return FRC_INVALID;
    }
    for (unsigned j = 0; j < d; ++j) if (!isfinite(x[static_cast<size_t>(t) * d + j])) return FRC_NUMERIC;
  }
  return FRC_OK;
}

// The end of a call of up to FRC_MAX_TOKENS tokens whose status word and y
// sit at d_in + st_off: the publish kernel stores [status][y] into the mapped
// h_out, the stream is synchronised, and y is handed over only when the
// status is clean.
static int finish_small(frc_context* c, size_t st_off, size_t xb, float* y) {
  const unsigned n16 = static_cast<unsigned>((16 + xb) / 16);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(std::min(8u, (n16 + 1023) / 1024));  // up to 8 CTAs of 512 threads
  cfg.blockDim = dim3(512);
  cfg.stream = c->stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, publish_kernel, reinterpret_cast<const uint4*>(c->d_in + st_off),
                        reinterpret_cast<uint4*>(c->h_out_dev), n16));
  CK(cudaStreamSynchronize(c->stream));
  const unsigned st = *c->h_status;
  if (st & kStTimeout) {
    const int rrc = reset_after_timeout(c, c->stream);
    if (rrc) return rrc;
  }
  if (status_code(st)) return fail(c, status_code(st), "device status 0x%x", st);
  memcpy(y, c->h_y, xb);  // published only after the whole layer succeeded
  return FRC_OK;
}

// FRC_ACT_AVX2 (frc_avx2.cuh) through host buffers: the experts in the order
// the tokens first name them (routed ranks 0-9, then the shared expert when
// its gate is nonzero: backends/avx2.c:660-672), their token masks and the
// (expert, token) pairs are planned here and travel in the request's copy:
// [x][plan] then the status word and y.
static int run_avx2(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                    const float* x, float* y, unsigned flags) {
  if (flags) return fail(c, FRC_UNSUPPORTED, "FRC_ACT_AVX2 takes no run flags");
  if (T > FRC_MAX_TOKENS) return fail(c, FRC_UNSUPPORTED, "FRC_ACT_AVX2: up to %u tokens a call", FRC_MAX_TOKENS);
  if (c->g.gate_type != FRC_Q4_K || c->g.down_type != FRC_MXFP4)
    return fail(c, FRC_UNSUPPORTED, "FRC_ACT_AVX2: the reference's native layout (Q4_K gate/up, MXFP4 down) only");
  int rc = validate(c, T, expert, gate, x);
  if (rc) return fail(c, rc, "request rejected");
  CK(cudaSetDevice(c->device));
  Avx2Params a{};
  unsigned S = 0;
  for (unsigned i = 0; i < c->slot_count; ++i) {
    const unsigned b = c->slot_order[i];
    if (!c->layer_ptr[b][layer]) return fail(c, FRC_STATE, "block %u is loaded but not layer %u", b, layer);
    a.base[S++] = c->layer_ptr[b][layer];
  }
  if (!S) return fail(c, FRC_STATE, "no block loaded");
  uint16_t ids[kMaxPairs], pbase[kMaxPairs];
  uint32_t mask[kMaxPairs];
  float eg[kMaxPairs][kMaxTokens], pgate[kMaxPairs];
  unsigned E = 0, P = 0;
  for (unsigned t = 0; t < T; ++t)
    for (unsigned j = 0; j < FRC_ACTIVE; ++j) {
      const float g = gate[t * FRC_ACTIVE + j];
      if (j == FRC_TOPK && g == 0) continue;
      const unsigned id = j == FRC_TOPK ? FRC_ROUTED_EXPERTS : expert[t * FRC_TOPK + j];
      unsigned e = 0;
      while (e < E && ids[e] != id) ++e;
      if (e == E) {
        ids[E] = static_cast<uint16_t>(id);
        mask[E++] = 0;
      }
      mask[e] |= 1u << t;
      eg[e][t] = g;
    }
  for (unsigned e = 0; e < E; ++e) {
    pbase[e] = static_cast<uint16_t>(P);
    for (unsigned t = 0; t < T; ++t)
      if (mask[e] >> t & 1u) pgate[P++] = eg[e][t];
  }
  // each token's fmadd chains: its term slots (s * P + pair) in job order,
  // jobs (slot s, expert j) block-major and dealt round robin to W workers
  const unsigned W = c->avx2_workers, jobs = S * E, stride = S * FRC_ACTIVE;
  constexpr unsigned kBound = kAvx2MaxWorkers + 1;
  uint16_t bounds[kMaxTokens * kBound], chain[kMaxTokens * kMaxBlocks * FRC_ACTIVE];
  for (unsigned t = 0; t < T; ++t) {
    unsigned n = 0;
    for (unsigned w = 0; w < W; ++w) {
      bounds[t * kBound + w] = static_cast<uint16_t>(n);
      for (unsigned idx = w; idx < jobs; idx += W) {
        const unsigned s = idx / E, j = idx % E;
        if (mask[j] >> t & 1u)
          chain[t * stride + n++] = static_cast<uint16_t>(s * P + pbase[j] + __builtin_popcount(mask[j] & ((1u << t) - 1u)));
      }
    }
    bounds[t * kBound + W] = static_cast<uint16_t>(n);
  }
  const unsigned d = c->g.hidden;
  const size_t xb = sizeof(float) * T * d, po = (xb + 15) & ~size_t(15);
  const size_t bo = po + 12 * kMaxPairs, co = bo + 2 * kMaxTokens * kBound;
  const size_t st_off = (co + 2 * static_cast<size_t>(T) * stride + 15) & ~size_t(15);
  uint8_t* h = c->h_in;
  memcpy(h, x, xb);
  memcpy(h + po, mask, 4 * E);
  memcpy(h + po + 4 * kMaxPairs, pgate, 4 * P);
  memcpy(h + po + 8 * kMaxPairs, ids, 2 * E);
  memcpy(h + po + 10 * kMaxPairs, pbase, 2 * E);
  memcpy(h + bo, bounds, 2 * static_cast<size_t>(T) * kBound);
  memcpy(h + co, chain, 2 * static_cast<size_t>(T) * stride);
  memset(h + st_off, 0, 16);
  CK(cudaMemcpyAsync(c->d_in, h, st_off + 16, cudaMemcpyHostToDevice, c->stream));
  const uint8_t* dp = c->d_in + po;
  a.x = reinterpret_cast<const float*>(c->d_in);
  a.mask = reinterpret_cast<const uint32_t*>(dp);
  a.pgate = reinterpret_cast<const float*>(dp + 4 * kMaxPairs);
  a.ids = reinterpret_cast<const uint16_t*>(dp + 8 * kMaxPairs);
  a.pbase = reinterpret_cast<const uint16_t*>(dp + 10 * kMaxPairs);
  a.bounds = reinterpret_cast<const uint16_t*>(c->d_in + bo);
  a.chain = reinterpret_cast<const uint16_t*>(c->d_in + co);
  a.chain_stride = stride;
  a.xq = reinterpret_cast<int8_t*>(c->avx2_x);
  a.xd = reinterpret_cast<float*>(c->avx2_x + static_cast<size_t>(kMaxTokens) * d);
  a.xs = reinterpret_cast<int16_t*>(c->avx2_x + static_cast<size_t>(kMaxTokens) * (d + d / 256 * 4));
  a.terms = c->partial;
  a.coef = c->gsv;
  a.status = reinterpret_cast<unsigned*>(c->d_in + st_off);
  a.y = reinterpret_cast<float*>(c->d_in + st_off + 16);
  a.d = d; a.T = T; a.S = S; a.E = E; a.P = P; a.W = W;
  a.row_bytes = static_cast<unsigned>(c->row_bytes); a.proj_bytes = static_cast<unsigned>(c->proj_bytes);
  a.slice_bytes = static_cast<unsigned>(c->slice_bytes);
  a.shared_row = static_cast<unsigned>(c->shared_row); a.shared_proj = static_cast<unsigned>(c->shared_proj);
  const bool timed = c->av_timing;
  auto mark = [&](unsigned i) { if (timed) cudaEventRecord(c->av_ev[i], c->stream); };
  mark(0);
  avx2_quantize_kernel<<<T, 256, 0, c->stream>>>(a);
  mark(1);
  // Staging the routed slices in shared memory holds one or two CTAs on an
  // SM, with no overlap of a CTA's copy and its arithmetic: it pays when all
  // the jobs run in one wave (one token: 22 us against 29 us for the jobs of
  // a decode48 layer) and costs when they do not (16 tokens: 171 against 137).
  bool stage = false;
  if (c->slice_bytes <= kAvx2StageMax) {
    if (!c->av_attr) {
      CK(cudaFuncSetAttribute(avx2_job_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kAvx2StageMax)));
      CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c->av_stage_per_sm, avx2_job_kernel<true>, 256,
                                                       c->slice_bytes));
      c->av_attr = true;
    }
    stage = static_cast<unsigned>(c->av_stage_per_sm) * static_cast<unsigned>(c->sms) >= S * E;
  }
  if (stage) {
    avx2_job_kernel<true><<<S * E, 256, c->slice_bytes, c->stream>>>(a);
  } else {
    avx2_job_kernel<false><<<S * E, 256, 0, c->stream>>>(a);
  }
  mark(2);
  avx2_reduce_kernel<<<T * d / 64, 64, 0, c->stream>>>(a);
  mark(3);
  CK(cudaGetLastError());
  c->av_timed = timed;
  c->launches += 3;
  return finish_small(c, st_off, xb, y);
}

int frc_avx2_timing(frc_context* c, int enable) {
  if (!c) return FRC_INVALID;
  CK(cudaSetDevice(c->device));
  if (enable && !c->av_ev[0])
    for (auto& e : c->av_ev) CK(cudaEventCreate(&e));
  c->av_timing = enable != 0;
  return FRC_OK;
}

int frc_avx2_times(frc_context* c, float* ms) {
  if (!c || !ms || !c->av_timed) return fail(c, FRC_INVALID, "no timed FRC_ACT_AVX2 run");
  CK(cudaSetDevice(c->device));
  CK(cudaEventSynchronize(c->av_ev[3]));
  for (unsigned i = 0; i < 3; ++i) CK(cudaEventElapsedTime(&ms[i], c->av_ev[i], c->av_ev[i + 1]));
  return FRC_OK;
}

int frc_set_avx2_workers(frc_context* c, unsigned workers) {
  if (!c || workers < 1 || workers > kAvx2MaxWorkers) return fail(c, FRC_INVALID, "FRC_ACT_AVX2 workers: 1-32");
  c->avx2_workers = workers;
  return FRC_OK;
}

int frc_run(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate, const float* x,
            float* y, int act) {
  return frc_run_flags(c, layer, tokens, expert, gate, x, y, act, 0);
}

int frc_run_flags(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate,
                  const float* x, float* y, int act, unsigned flags) {
  if (!c || !expert || !gate || !x || !y || tokens < 1 || tokens > FRC_MAX_PREFILL_TOKENS || layer >= c->g.layers ||
      (act != FRC_ACT_Q8 && act != FRC_ACT_F32 && act != FRC_ACT_AVX2))
    return fail(c, FRC_INVALID, "bad run arguments");
  if (flags & ~unsigned(FRC_RUN_PEER)) return fail(c, FRC_INVALID, "frc_run_flags: only FRC_RUN_PEER");
  if (act == FRC_ACT_AVX2) return run_avx2(c, layer, tokens, expert, gate, x, y, flags);
  if ((flags & FRC_RUN_PEER) && tokens > FRC_MAX_TOKENS)
    return fail(c, FRC_UNSUPPORTED, "FRC_RUN_PEER: up to %u tokens a call", FRC_MAX_TOKENS);
  int rc = validate(c, tokens, expert, gate, x);
  if (rc) return fail(c, rc, "request rejected");
  CK(cudaSetDevice(c->device));
  // one copy in: [x][gate][expert] packed for this call's token count
  const size_t xb = sizeof(float) * tokens * c->g.hidden, gb = sizeof(float) * tokens * FRC_ACTIVE;
  const size_t eb = sizeof(uint16_t) * tokens * FRC_TOPK;
  memcpy(c->h_in, x, xb);
  memcpy(c->h_in + xb, gate, gb);
  memcpy(c->h_in + xb + gb, expert, eb);
  if (tokens <= FRC_MAX_TOKENS) {
    // The layer kernel's status word and y follow the request in the same
    // device buffer: the copy in zeroes the status word (no separate memset),
    // and one copy out brings back [status][y].
    const size_t st_off = (xb + gb + eb + 15) & ~size_t(15);
    memset(c->h_in + st_off, 0, 16);
    CK(cudaMemcpyAsync(c->d_in, c->h_in, st_off + 16, cudaMemcpyHostToDevice, c->stream));
    unsigned* d_st = reinterpret_cast<unsigned*>(c->d_in + st_off);
    rc = run_device(c, layer, tokens, reinterpret_cast<const uint16_t*>(c->d_in + xb + gb),
                    reinterpret_cast<const float*>(c->d_in + xb), reinterpret_cast<const float*>(c->d_in), nullptr,
                    nullptr, reinterpret_cast<float*>(c->d_in + st_off + 16), act, flags, c->stream, nullptr, false,
                    d_st);
    if (rc) return rc;
    c->last_T = tokens;
    memcpy(c->last_expert, expert, eb);
    memcpy(c->last_gate, gate, gb);
    return finish_small(c, st_off, xb, y);
  }
  CK(cudaMemcpyAsync(c->d_in, c->h_in, xb + gb + eb, cudaMemcpyHostToDevice, c->stream));
  rc = run_device(c, layer, tokens, reinterpret_cast<const uint16_t*>(c->d_in + xb + gb),
                  reinterpret_cast<const float*>(c->d_in + xb), reinterpret_cast<const float*>(c->d_in), nullptr,
                  nullptr, c->d_y, act, 0, c->stream, nullptr);
  if (rc) return rc;
  if (tokens <= FRC_MAX_TOKENS) {
    c->last_T = tokens;
    memcpy(c->last_expert, expert, eb);
    memcpy(c->last_gate, gate, gb);
  }
  // one copy out: the status word and y
  CK(cudaMemcpyAsync(c->h_out, c->d_out, 16 + xb, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaMemsetAsync(c->status, 0, sizeof(unsigned), c->stream));
  CK(cudaStreamSynchronize(c->stream));
  const unsigned st = *c->h_status;
  if (st & kStTimeout) {
    const int rrc = reset_after_timeout(c, c->stream);
    if (rrc) return rrc;
  }
  if (status_code(st)) return fail(c, status_code(st), "device status 0x%x", st);
  memcpy(y, c->h_y, xb);  // published only after the whole layer succeeded
  return FRC_OK;
}

int frc_run_device(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate,
                   const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags, void* stream) {
  if (!c) return FRC_INVALID;
  if (cudaSetDevice(c->device) != cudaSuccess) return fail(c, FRC_IO, "cudaSetDevice");
  return run_device(c, layer, tokens, expert, gate, x, x_add, x_out, y, act, flags, static_cast<cudaStream_t>(stream));
}

int frc_run_device_fixed(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert,
                         const float* gate, const float* x, const float* x_add, float* x_out, float* y, int act,
                         unsigned flags, void* stream) {
  if (!c) return FRC_INVALID;
  if (c->device < 0 || c->device >= kFixedDevices) return fail(c, FRC_UNSUPPORTED, "device %d has no fixed scratch slot", c->device);
  if (tokens < 1 || tokens > FRC_MAX_TOKENS) return fail(c, FRC_INVALID, "tokens or layer out of range");
  unsigned S = 0;
  for (unsigned b = 0; b < FRC_MAX_BLOCKS; ++b) {
    bool any = false;
    for (unsigned l = 0; l < c->g.layers; ++l) any |= c->layer_ptr[b][l] != nullptr;
    S += any;
  }
  const size_t need = fixed_need(S, tokens, c->g.hidden);
  if (need > kFixedScratchBytes)
    return fail(c, FRC_INVALID, "frc_run_device_fixed: %u tokens over %u slices need %zu bytes of fixed scratch, limit %zu",
                tokens, S, need, kFixedScratchBytes);
  if (cudaSetDevice(c->device) != cudaSuccess) return fail(c, FRC_IO, "cudaSetDevice");
  float* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_fixed_mu);
    if (!g_fixed_ptr[c->device]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_fixed_scratch);
      if (e != cudaSuccess || !p)
        return fail(c, FRC_IO, "cudaGetSymbolAddress(fixed scratch): %s", cudaGetErrorString(e));
      g_fixed_ptr[c->device] = static_cast<float*>(p);
    }
    base = g_fixed_ptr[c->device];
  }
  const RunScratch sc{base, base + fixed_partial(S, tokens, c->g.hidden), nullptr};
  return run_device(c, layer, tokens, expert, gate, x, x_add, x_out, y, act, flags, static_cast<cudaStream_t>(stream),
                    &sc);
}

// ------------------------------------------------------ in-box reduce
// Inbox bytes for `world` ranks: double-buffered slots [2][world][16][d] f32,
// then the flags [world][2 * SMs] u32 (one per source rank and CTA).
// Inbox: [2 epoch parities][world sources][16 tokens][d] entries of 8 bytes
// (the value and the epoch of the launch that wrote it).
static size_t inbox_bytes(const frc_context* c, unsigned world, unsigned) {
  return 2 * static_cast<size_t>(world) * kMaxTokens * c->g.hidden * 2 * sizeof(float);
}

int frc_peer_export(frc_context* c, unsigned world, void* handle) {
  if (!c || !handle || world < 2 || world > kMaxPeers) return fail(c, FRC_INVALID, "world must be 2..%u", kMaxPeers);
  if (c->inbox) return fail(c, FRC_STATE, "inbox already exported");
  CK(cudaSetDevice(c->device));
  const unsigned gmax = 2 * static_cast<unsigned>(c->sms);
  const size_t bytes = inbox_bytes(c, world, gmax);
  CK(cudaMalloc(&c->inbox, bytes));
  CK(cudaMemset(c->inbox, 0, bytes));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, c->inbox));
  static_assert(sizeof(h) == FRC_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof h);
  c->world = world;
  return FRC_OK;
}

int frc_peer_attach(frc_context* c, unsigned rank, unsigned world, const void* handles) {
  if (!c || !handles || rank >= world || world != c->world || !c->inbox)
    return fail(c, FRC_INVALID, "attach needs the exported world, rank < world and every handle");
  CK(cudaSetDevice(c->device));
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (unsigned r = 0; r < world; ++r) {
    if (r == rank) {
      c->peer[r] = c->inbox;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + r * FRC_PEER_HANDLE_BYTES, sizeof h);
    void* p = nullptr;
    CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->peer[r] = static_cast<uint8_t*>(p);
  }
  c->rank = rank;
  // epochs restart with the fresh inbox, the same on every rank
  CK(cudaMemsetAsync(reinterpret_cast<uint8_t*>(c->ctl) + offsetof(LayerCtl, peer_epoch), 0, sizeof(unsigned),
                     c->stream));
  CK(cudaStreamSynchronize(c->stream));
  return FRC_OK;
}

int frc_peer_detach(frc_context* c) {
  if (!c) return FRC_INVALID;
  cudaSetDevice(c->device);
  for (unsigned r = 0; r < kMaxPeers; ++r) {
    if (c->peer[r] && c->peer[r] != c->inbox) cudaIpcCloseMemHandle(c->peer[r]);
    c->peer[r] = nullptr;
  }
  cudaFree(c->inbox);
  c->inbox = nullptr;
  c->world = 0;
  c->rank = 0;
  return FRC_OK;
}

int frc_status(frc_context* c, void* stream) {
  if (!c) return FRC_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemcpyAsync(c->h_status, c->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
  CK(cudaMemsetAsync(c->status, 0, sizeof(unsigned), s));
  CK(cudaStreamSynchronize(s));
  const int rc = status_code(*c->h_status);
  if (*c->h_status & kStTimeout) {
    const int rrc = reset_after_timeout(c, s);
    if (rrc) return rrc;
  }
  if (rc) return fail(c, rc, "device status 0x%x", *c->h_status);
  return FRC_OK;
}

// ------------------------------------------------------ in-box head plane
// The reference head's fan-out and gather of one layer (src/plane.c:252-374)
// over the GPUs of one box, one context each.  x is rounded to fp16 once, as
// the head rounds it for every node and for its own slice
// (src/plane.c:258-262, src/wire.c:46-67); every participant runs the layer
// on its own stream; the parts done by the deadline are summed in
// participant order (the reference adds them in arrival order), and the
// others are reported in the missing mask and left out, as the reference's
// head leaves out a node that missed its deadline.

// fp16 round trip of the reference's wire format: round to nearest even to
// fp16's 11 significant bits (multiples of 2^-24 below 2^-14); a value that
// is not finite or rounds past fp16's largest finite value (65504) fails.
static int half_round(float v, float* out) {
  if (!isfinite(v)) return -1;
  const float a = fabsf(v);
  if (a >= 65520.0f) return -1;  // rounds to infinity
  float q;
  if (a < 0x1p-14f) {
    q = nearbyintf(a * 0x1p24f) * 0x1p-24f;  // subnormal spacing 2^-24 (scalings are exact)
  } else {
    int e;
    frexpf(a, &e);                            // a in [2^(e-1), 2^e)
    const float ulp = ldexpf(1.0f, e - 11);   // 10 fraction bits
    q = nearbyintf(a / ulp) * ulp;
  }
  *out = copysignf(q, v);
  return 0;
}

int frc_round_half(const float* x, size_t n, float* out) {
  if ((!x || !out) && n) return FRC_INVALID;
  if (fegetround() != FE_TONEAREST) return FRC_INVALID;
  for (size_t i = 0; i < n; ++i)
    if (half_round(x[i], &out[i])) return FRC_INVALID;
  return FRC_OK;
}

struct frc_plane {
  unsigned n = 0, d = 0;
  frc_context* ctx[kMaxPeers] = {};
  uint8_t* d_in[kMaxPeers] = {};  // [x 16 x d f32][gate 16 x 11 f32][expert 16 x 10 u16]
  float* d_y[kMaxPeers] = {};
  uint8_t* h_in[kMaxPeers] = {};  // pinned staging of the same layout
  float* h_y[kMaxPeers] = {};     // pinned [16][d]
  cudaEvent_t done[kMaxPeers] = {};
  bool pending[kMaxPeers] = {};   // this participant's last call may still be running
  int late_status[kMaxPeers] = {}; // device status of a part that missed its deadline (read later)
  float* xr = nullptr;            // [16][d] rounded x
};

static size_t plane_in_bytes(unsigned d) {
  return sizeof(float) * kMaxTokens * d + sizeof(float) * kMaxTokens * FRC_ACTIVE + sizeof(uint16_t) * kMaxTokens * FRC_TOPK;
}

int frc_plane_close(frc_plane* p) {
  if (!p) return FRC_INVALID;
  for (unsigned i = 0; i < p->n; ++i) {
    if (!p->ctx[i]) continue;
    cudaSetDevice(p->ctx[i]->device);
    cudaStreamSynchronize(p->ctx[i]->stream);
    if (p->done[i]) cudaEventDestroy(p->done[i]);
    cudaFree(p->d_in[i]);
    cudaFree(p->d_y[i]);
    cudaFreeHost(p->h_in[i]);
    cudaFreeHost(p->h_y[i]);
  }
  free(p->xr);
  delete p;
  return FRC_OK;
}

int frc_plane_open(frc_context* const* ctx, unsigned count, frc_plane** out) {
  if (!ctx || !out || count < 1 || count > kMaxPeers) return FRC_INVALID;
  *out = nullptr;
  for (unsigned i = 0; i < count; ++i)
    if (!ctx[i] || memcmp(&ctx[i]->g, &ctx[0]->g, sizeof(frc_geometry))) return FRC_INVALID;
  frc_plane* p = new frc_plane();
  p->n = count;
  p->d = ctx[0]->g.hidden;
  p->xr = static_cast<float*>(malloc(sizeof(float) * kMaxTokens * p->d));
  int rc = p->xr ? FRC_OK : FRC_IO;
  for (unsigned i = 0; i < count && rc == FRC_OK; ++i) {
    frc_context* c = ctx[i];
    p->ctx[i] = c;
    if (cudaSetDevice(c->device) != cudaSuccess || cudaMalloc(&p->d_in[i], plane_in_bytes(p->d)) != cudaSuccess ||
        cudaMalloc(&p->d_y[i], sizeof(float) * kMaxTokens * p->d) != cudaSuccess ||
        cudaMallocHost(&p->h_in[i], plane_in_bytes(p->d)) != cudaSuccess ||
        cudaMallocHost(&p->h_y[i], sizeof(float) * kMaxTokens * p->d) != cudaSuccess ||
        cudaEventCreateWithFlags(&p->done[i], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(c, FRC_IO, "plane buffers");
  }
  if (rc) {
    frc_plane_close(p);
    return rc;
  }
  *out = p;
  return FRC_OK;
}

int frc_plane_run(frc_plane* p, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate,
                  const float* x, uint64_t deadline_ns, float* y, uint32_t* missing) {
  if (!p || !expert || !gate || !x || !y || !missing || tokens < 1 || tokens > kMaxTokens || !deadline_ns)
    return FRC_INVALID;
  const unsigned d = p->d;
  const size_t xb = sizeof(float) * tokens * d, gb = sizeof(float) * tokens * FRC_ACTIVE;
  const size_t eb = sizeof(uint16_t) * tokens * FRC_TOPK;
  // every participant sees the same rounded activations; nothing is sent
  // when one of them is not representable
  if (frc_round_half(x, static_cast<size_t>(tokens) * d, p->xr)) return FRC_INVALID;
  for (unsigned i = 0; i < p->n; ++i) {
    frc_context* c = p->ctx[i];
    CK(cudaSetDevice(c->device));
    if (p->pending[i]) {  // a late part of an earlier call still owns the staging: wait (bounded)
      const auto t0 = std::chrono::steady_clock::now();
      cudaError_t q;
      while ((q = cudaEventQuery(p->done[i])) == cudaErrorNotReady)
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2))
          return fail(c, FRC_IO, "plane participant %u still busy with an earlier layer", i);
      if (q != cudaSuccess) return fail(c, FRC_IO, "plane participant %u: %s", i, cudaGetErrorString(q));
      p->pending[i] = false;
      // that part was left out of its call; its device status belongs to that
      // call, not to this one: read, clear and keep it (frc_plane_late_status)
      p->late_status[i] = frc_status(c, c->stream);
    }
    memcpy(p->h_in[i], p->xr, xb);
    memcpy(p->h_in[i] + xb, gate, gb);
    memcpy(p->h_in[i] + xb + gb, expert, eb);
    CK(cudaMemcpyAsync(p->d_in[i], p->h_in[i], xb + gb + eb, cudaMemcpyHostToDevice, c->stream));
    const int rc = run_device(c, layer, tokens, reinterpret_cast<const uint16_t*>(p->d_in[i] + xb + gb),
                              reinterpret_cast<const float*>(p->d_in[i] + xb), reinterpret_cast<const float*>(p->d_in[i]),
                              nullptr, nullptr, p->d_y[i], FRC_ACT_Q8, 0, c->stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(p->h_y[i], p->d_y[i], xb, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaEventRecord(p->done[i], c->stream));
    p->pending[i] = true;
  }
  // gather until every part is in or the deadline passes
  uint32_t left = (p->n >= 32 ? 0xffffffffu : (1u << p->n) - 1);
  const auto start = std::chrono::steady_clock::now();
  const auto limit = std::chrono::nanoseconds(deadline_ns);
  for (;;) {
    for (unsigned i = 0; i < p->n; ++i) {
      if (!(left >> i & 1)) continue;
      const cudaError_t q = cudaEventQuery(p->done[i]);
      if (q == cudaSuccess) {
        left &= ~(1u << i);
        p->pending[i] = false;
      } else if (q != cudaErrorNotReady) {
        return fail(p->ctx[i], FRC_IO, "plane participant %u: %s", i, cudaGetErrorString(q));
      }
    }
    if (!left || std::chrono::steady_clock::now() - start >= limit) break;
  }
  // a part that arrived with a device error fails the call (y untouched)
  for (unsigned i = 0; i < p->n; ++i)
    if (!(left >> i & 1)) {
      const int rc = frc_status(p->ctx[i], p->ctx[i]->stream);
      if (rc) return rc;
    }
  // Participant 0 is the head's own slice (fp32, as the head adds its local
  // part).  Every other participant stands for a remote node, whose part the
  // reference sends as fp16 (src/plane.c:181, src/wire.c:46-67): rounded to
  // nearest even here, and a part with a value that has no finite fp16 form
  // is left out and reported missing, as the node drops such a reply.
  const size_t n = static_cast<size_t>(tokens) * d;
  for (unsigned i = 1; i < p->n; ++i)
    if (!(left >> i & 1) && frc_round_half(p->h_y[i], n, p->h_y[i])) left |= 1u << i;
  for (size_t k = 0; k < n; ++k) {
    float s = 0.0f;
    for (unsigned i = 0; i < p->n; ++i)
      if (!(left >> i & 1)) s += p->h_y[i][k];
    y[k] = s;
  }
  *missing = left;
  return FRC_OK;
}

int frc_plane_late_status(const frc_plane* p, unsigned participant, int* status) {
  if (!p || !status || participant >= p->n) return FRC_INVALID;
  *status = p->late_status[participant];
  return FRC_OK;
}

int frc_pool_load(frc_context* c, const uint8_t* slices, unsigned count, const uint8_t* shared) {
  if (!c || !slices || !shared || !count) return fail(c, FRC_INVALID, "bad pool");
  CK(cudaSetDevice(c->device));
  const size_t bytes = count * c->slice_bytes + c->shared_bytes;
  uint8_t* tmp = nullptr;
  if (c->pool) CK(cudaFree(c->pool));
  c->pool = nullptr;
  CK(cudaMalloc(&c->pool, bytes));
  CK(cudaMalloc(&tmp, bytes));
  CK(cudaMemcpy(tmp, slices, count * c->slice_bytes, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(tmp + count * c->slice_bytes, shared, c->shared_bytes, cudaMemcpyHostToDevice));
  transcode_kernel<<<count + 1, 256, 0, c->stream>>>(tmp, c->pool, count, shape_of(c));
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaFree(tmp));
  c->pool_count = count;
  return FRC_OK;
}

int frc_fill_layer(frc_context* c, int block, unsigned layer, uint64_t seed) {
  if (!c || block < 0 || block >= FRC_MAX_BLOCKS || layer >= c->g.layers) return fail(c, FRC_INVALID, "bad fill");
  if (!c->pool) return fail(c, FRC_STATE, "no pool loaded");
  CK(cudaSetDevice(c->device));
  int rc = ensure_layer(c, block, layer);
  if (rc) return rc;
  fill_kernel<<<FRC_ROUTED_EXPERTS + 1, 256, 0, c->stream>>>(c->pool, c->pool_count, c->layer_ptr[block][layer],
                                                             c->slice_bytes, c->shared_bytes, seed, block, layer);
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  return FRC_OK;
}

int frc_debug_decode(frc_context* c, unsigned type, const uint8_t* rows, unsigned n, unsigned count, float* out) {
  const size_t rowb = frc_row_bytes(type, n);
  if (!c || !rows || !out || !count || !rowb) return fail(c, FRC_INVALID, "bad decode");
  CK(cudaSetDevice(c->device));
  uint8_t *src = nullptr, *dst = nullptr;
  float* o = nullptr;
  CK(cudaMalloc(&src, count * rowb));
  CK(cudaMalloc(&dst, count * rowb));
  CK(cudaMalloc(&o, sizeof(float) * count * n));
  CK(cudaMemcpy(src, rows, count * rowb, cudaMemcpyHostToDevice));
  rows_transcode_kernel<<<count, 256, 0, c->stream>>>(src, dst, type, n, static_cast<unsigned>(rowb));
  decode_kernel<<<count, 256, 0, c->stream>>>(dst, type, n, static_cast<unsigned>(rowb), o);
  CK(cudaGetLastError());
  c->launches += 2;
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaMemcpy(out, o, sizeof(float) * count * n, cudaMemcpyDeviceToHost));
  cudaFree(src); cudaFree(dst); cudaFree(o);
  return FRC_OK;
}

int frc_debug_quantize(frc_context* c, unsigned tokens, const float* x, int8_t* q, float* scale, float* deq) {
  if (!c || !x || !q || !scale || !deq || !tokens) return fail(c, FRC_INVALID, "bad quantize");
  CK(cudaSetDevice(c->device));
  const unsigned n = tokens * c->g.hidden;
  float *dx = nullptr, *ds = nullptr, *dd = nullptr;
  int8_t* dq = nullptr;
  CK(cudaMalloc(&dx, sizeof(float) * n));
  CK(cudaMalloc(&dq, n));
  CK(cudaMalloc(&ds, sizeof(float) * n / 64));
  CK(cudaMalloc(&dd, sizeof(float) * n));
  CK(cudaMemcpy(dx, x, sizeof(float) * n, cudaMemcpyHostToDevice));
  const unsigned groups = n / 64;
  quantize_kernel<<<(groups + 7) / 8, 256, 0, c->stream>>>(dx, n, dq, ds, dd);
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  CK(cudaMemcpy(q, dq, n, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(scale, ds, sizeof(float) * n / 64, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(deq, dd, sizeof(float) * n, cudaMemcpyDeviceToHost));
  cudaFree(dx); cudaFree(dq); cudaFree(ds); cudaFree(dd);
  return FRC_OK;
}

int frc_debug_umma(frc_context* c, unsigned n, unsigned k, const int8_t* a, const int8_t* b, int32_t* d) {
  if (!c || !a || !b || !d || !n || n > 256 || n % 16 || !k || k > 256 || k % 32)
    return fail(c, FRC_INVALID, "bad umma check shape");
  CK(cudaSetDevice(c->device));
  int8_t *da = nullptr, *db = nullptr;
  int32_t* dd = nullptr;
  CK(cudaMalloc(&da, 128 * k));
  CK(cudaMalloc(&db, n * k));
  CK(cudaMalloc(&dd, sizeof(int32_t) * 128 * n));
  CK(cudaMemcpy(da, a, 128 * k, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(db, b, n * k, cudaMemcpyHostToDevice));
  CK(cudaMemsetAsync(c->status, 0, sizeof(unsigned), c->stream));
  const unsigned smem = (128 + n) * k;
  CK(cudaFuncSetAttribute(umma_check_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  umma_check_kernel<<<1, 128, smem, c->stream>>>(da, db, dd, n, k, c->status);
  CK(cudaGetLastError());
  ++c->launches;
  CK(cudaStreamSynchronize(c->stream));
  unsigned st = 0;
  CK(cudaMemcpy(&st, c->status, sizeof st, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(d, dd, sizeof(int32_t) * 128 * n, cudaMemcpyDeviceToHost));
  cudaFree(da); cudaFree(db); cudaFree(dd);
  return st ? fail(c, FRC_IO, "umma check timed out") : FRC_OK;
}

int frc_prefill_timing(frc_context* c, int enable) {
  if (!c) return FRC_INVALID;
  CK(cudaSetDevice(c->device));
  if (enable && !c->pf_ev[0])
    for (auto& e : c->pf_ev) CK(cudaEventCreate(&e));
  c->pf_timing = enable != 0;
  return FRC_OK;
}

int frc_prefill_times(frc_context* c, float* ms) {
  if (!c || !ms || !c->pf_timed) return fail(c, FRC_INVALID, "no timed prefill run");
  CK(cudaSetDevice(c->device));
  CK(cudaEventSynchronize(c->pf_ev[5]));
  for (unsigned i = 0; i < 5; ++i) CK(cudaEventElapsedTime(&ms[i], c->pf_ev[i], c->pf_ev[i + 1]));
  return FRC_OK;
}

int frc_debug_prefill_hidden(frc_context* c, int8_t* hq, float* hs, size_t cap, size_t* pairs) {
  if (!c || !pairs || !c->pf_counts || !c->last_pf_S) return fail(c, FRC_INVALID, "no prefill run to report");
  CK(cudaSetDevice(c->device));
  CK(cudaStreamSynchronize(c->stream));
  unsigned cnt[4] = {0, 0, 0, 0};
  CK(cudaMemcpy(cnt, c->pf_counts, sizeof cnt, cudaMemcpyDeviceToHost));
  const unsigned P = cnt[0], routed = cnt[3];  // the shared expert's pairs follow the routed ones
  *pairs = P;
  if (!hq && !hs) return FRC_OK;
  if (cap < P) return fail(c, FRC_INVALID, "capacity %zu below %u pairs", cap, P);
  const size_t S = c->last_pf_S, n = static_cast<size_t>(P) * S * 32;
  if (hq) {
    int8_t* tmp = static_cast<int8_t*>(malloc(n));
    if (!tmp) return fail(c, FRC_IO, "host buffer");
    const cudaError_t e = cudaMemcpy(tmp, c->pf_hq, n, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess)  // device order: prmt order within each 32-block (routed), natural (shared)
      for (size_t blk = 0; blk < n / 32; ++blk)
        for (unsigned k = 0; k < 32; ++k) hq[32 * blk + k] = tmp[32 * blk + (blk / S < routed ? prmt_pos(k) : k)];
    free(tmp);
    if (e != cudaSuccess) return fail(c, FRC_IO, "%s", cudaGetErrorString(e));
  }
  if (hs) CK(cudaMemcpy(hs, c->pf_hs, sizeof(float) * P * S, cudaMemcpyDeviceToHost));
  return FRC_OK;
}

int frc_debug_hidden(frc_context* c, float* h, size_t cap, size_t* count) {
  if (!c || !count || !c->last_T) return fail(c, FRC_INVALID, "no run to report");
  const unsigned T = c->last_T, S = c->last_S;
  unsigned uid[kMaxUnique], umask[kMaxUnique], U = 0;
  for (unsigned t = 0; t < T; ++t)
    for (unsigned e = 0; e < FRC_TOPK; ++e) {
      const unsigned id = c->last_expert[t * FRC_TOPK + e];
      unsigned u = 0;
      while (u < U && uid[u] != id) ++u;
      if (u == U) { uid[U] = id; umask[U++] = 0; }
      umask[u] |= 1u << t;
    }
  unsigned sm = 0;
  for (unsigned t = 0; t < T; ++t) if (c->last_gate[t * FRC_ACTIVE + FRC_TOPK] != 0) sm |= 1u << t;
  if (sm) { uid[U] = FRC_SHARED_EXPERT; umask[U++] = sm; }
  const size_t need = static_cast<size_t>(U) * S * T * 32;
  *count = need;
  if (!h) return FRC_OK;
  if (cap < need) return fail(c, FRC_INVALID, "buffer too small");
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpy(h, c->hidden, need * sizeof(float), cudaMemcpyDeviceToHost));
  for (unsigned u = 0; u < U; ++u)
    for (unsigned si = 0; si < S; ++si)
      for (unsigned t = 0; t < T; ++t)
        if (!(umask[u] >> t & 1)) memset(h + ((static_cast<size_t>(u) * S + si) * T + t) * 32, 0, 32 * sizeof(float));
  return FRC_OK;
}

int frc_debug_phases(frc_context* c, uint64_t* out, size_t cap, size_t* count) {
  if (!c || !count) return FRC_INVALID;
  *count = 16 * static_cast<size_t>(c->last_G ? c->last_G : c->sms);
#ifndef FRC_PHASES
  return fail(c, FRC_UNSUPPORTED, "built without FRC_PHASES");
#else
  if (!out) return FRC_OK;
  if (cap < *count) return fail(c, FRC_INVALID, "buffer too small");
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpy(out, c->phases, *count * sizeof(uint64_t), cudaMemcpyDeviceToHost));
  return FRC_OK;
#endif
}

}  // extern "C"
