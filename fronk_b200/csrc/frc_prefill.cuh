// frc_prefill.cuh - the batched (prefill) path: bursts of up to 512 tokens
// with MXFP4 or Q4_K gate/up rows and MXFP4 down rows on the 5th-generation
// tensor cores, the Q8_0 shared expert included.
//
// One layer call is seven launches on one stream:
//   1. prefill_quantize_kernel: x (fp32 or bf16) -> int8 v per 64 (the ref-q8
//      scheme of src/q4.c:37-61), each 32-block stored in the nibble order of
//      an MXFP4 block (prmt order) and in natural order, one fp32 scale s per
//      64 and, for the exact block terms, the residuals r = (fl32(v * s) -
//      v * s) / 2^E of the dequantized values (s = M * 2^E, |r| <= 64), and
//      (Q4_K rows) each block's sums of v and r;
//   2. prefill_group_kernel (one CTA): validation, the (expert, token) pairs
//      expert-major with tokens ascending (a bitmap per expert, ranks by
//      popcount), the shared expert as expert 512 for the tokens whose
//      shared gate is not zero, and the work lists, its items first, then
//      the routed experts' biggest first;
//   3. prefill_mma_kernel<kGateUp, Q4, SH> (SH = the shared expert's items,
//      then the routed ones): item = (expert, pair of loaded blocks, up to
//      64 of its tokens).  A = the 128 gate/up rows of the two slices as int8
//      (doubled E2M1 values, Q4_K nibbles, or the shared expert's Q8_0
//      values), B = the tokens' v (rows [0, npad)) and r (rows [npad,
//      2 npad)), D = int32 in tensor memory, one tcgen05.mma kind::i8 per
//      32-weight block (the dots I with v and R with r); the epilogue forms
//      each block's (or Q4_K x group's) exact term from M * I + R and the
//      scales, sums the terms in double, narrows the sum to fp32, then
//      SwiGLU (double) and Q8 per 32 give hq / hscale per (pair, block);
//   4. prefill_mma_kernel<kDown, false, SH>: item = (expert, 128 output rows,
//      tokens); A = MXFP4 (or the shared expert's Q8_0) down rows, B = hq,
//      one MMA per loaded block;
//   5. prefill_combine_kernel: y[t] = sum over the token's routed experts in
//      request order, then its shared expert, of gate * partial, fmaf in fp32.
// The arithmetic is restated step for step by the oracle's or_prefill_run.
//
// Inside an MMA kernel (one CTA per SM, 448 threads) warps have roles:
//   warps 0-3 convert: raw MXFP4 payload (staged by TMA bulk copies) ->
//     int8 A tiles in the K-major no-swizzle layout of frc_umma.cuh, and
//     gather the B rows, row scales and column scales with cp.async;
//   warps 4-11 are the epilogue, two warpgroups splitting the tile's token
//     columns (TMEM lanes 0-127 = A rows);
//   warp 12 issues the bulk copies; warp 13 owns tensor memory and issues
//   the MMAs (one thread).
// Rings: 3 raw stages, 2 A/B stages (freed by the MMAs' commit), 4 scale
// stages (freed by the epilogue), and all 512 tensor-memory columns as two
// groups of accumulator buffers (gate/up: two MMA steps of 128 columns,
// down: four of 64), so that the epilogue takes one barrier and several
// independent TMEM reads per group.
// Every wait gives up after 2 s (kStTimeout) so a fault cannot hang the GPU.
#pragma once
#include <cuda.h>

namespace frc {

constexpr unsigned kPfTile = 64;        // tokens per item
constexpr unsigned kPfRaw = 3;          // raw payload stages
constexpr unsigned kPfAB = 2;           // A/B operand stages (released by the MMA's commit)
constexpr unsigned kPfSc = 4;           // scale stages (released by the epilogue)
// raw stage: gate/up MXFP4 128 rows x 128 B (two 128-byte swizzled boxes),
// gate/up Q4_K 128 rows x 144 B (one super-block a row, two unswizzled
// boxes), down 8 blocks x 128 rows x 16 B
constexpr unsigned kPfRawBytes = 18432;
constexpr unsigned kPfQ4Box = 64 * 144;  // one slice's Q4_K box
constexpr unsigned kPfA = 128 * 256;    // A stage: 128 rows x K 256
// B stage: 128 rows x K 256.  Gate/up: rows [0, npad) the tile's tokens'
// int8 activations v, rows [npad, 2 npad) their dequantization residuals r
// (npad = tokens rounded up to 16, MMA N 2 npad); down: rows [0, npad) the
// pairs' quantized hidden values (MMA N npad).
constexpr unsigned kPfB = 2 * kPfTile * 256;
constexpr unsigned kPfCols = 512;       // tensor memory columns: two groups of accumulator buffers
// Accumulator groups: group g takes columns [256 g, 256 g + 256) as GS
// buffers of BW columns, one MMA step each.  Gate/up: BW = 2 npad (the v
// then the r results), GS = 128 / npad (a whole 8-step chunk for tiles of
// up to 16 tokens, so that the epilogue reads many steps at once); down:
// BW = 64, GS = 4.
template <unsigned MODE>
__device__ __forceinline__ unsigned pf_bw(unsigned npad) { return MODE == 0 ? 2 * npad : 64u; }
template <unsigned MODE>
__device__ __forceinline__ unsigned pf_gs(unsigned npad) { return MODE == 0 ? 128 / npad : 4u; }
constexpr unsigned kPfThreads = 448;     // 14 warps
enum : unsigned { kGateUp = 0, kDown = 1 };

struct PrefillArgs {
  const float* x;          // [T][d] fp32, or bf16 words when x_bf16
  const uint16_t* expert;  // [T][10]
  const float* gate;       // [T][11]
  float* y;                // [T][d]
  unsigned T, d, S;        // tokens, hidden size, loaded blocks
  unsigned x_bf16;         // x holds bf16 values (widened exactly)
  unsigned q4k;            // gate/up rows are Q4_K (the reference's unit layout), else MXFP4
  unsigned row_bytes;      // MXFP4 gate/up row: d/32 scales + d/2 payload
  unsigned long long slice_bytes;
  unsigned slice_rows;     // slice_bytes / row_bytes
  const uint8_t* base[kMaxBlocks];  // this layer of each loaded block, ascending
  // the same layer regions as 2D byte arrays of row_bytes-long rows, for
  // tiled TMA loads of 128-byte x 64-row boxes with the 128-byte swizzle
  CUtensorMap tmap[kMaxBlocks];
  // scratch
  int8_t* xq;              // [T][d], prmt order per 32-block
  int8_t* xr;              // [T][d], the residuals of the dequantized values, same order
  float* xs;               // [T][d/64]
  int2* xme;               // [T][d/64] {M, E << 20}: xs = M * 2^E
  int2* xvr;               // [T][d/32] {V, RS}: the block's sums of v and of r (Q4_K mins)
  int8_t* xqn;             // [T][d] v in natural order (the shared expert's Q8_0 rows)
  int8_t* xrn;             // [T][d] r in natural order
  unsigned shared_row, shared_proj;  // the shared slice's Q8_0 gate/up row and 32 rows, bytes
  uint16_t* pair_token;    // [P]
  unsigned* slot_pair;     // [T][11]: each routed slot's pair, then the shared expert's (or ~0)
  unsigned* counts;        // [0] pairs, [1] gate/up items, [2] down items, [3] routed pairs,
                           // [4] / [5] the shared expert's gate/up / down items
  uint4* items_gu;         // {expert, first pair, tokens, block pair}
  uint4* items_dn;         // {expert, first pair, tokens, row tile}
  int8_t* hq;              // [P][S][32], prmt order per block
  float* hs;               // [P][S]
  float* ye;               // [P][d]
  unsigned* status;
  unsigned long long* phases;  // FRC_PHASES builds: [cta][64] globaltimer stamps
};

// FRC_PHASES builds: per CTA, the clock64 cycles that one thread of each role
// spends in its waits and in its work, summed over the launch, in
// a.phases[cta][64]: converters (thread 0) 0 raw landed, 1 conversion,
// 2 free stages, 3 gathers issued, 4 own copies landed; producer (thread 384)
// 8 free raw stage, 9 copies issued; MMA (thread 416) 12 operands staged,
// 13 free accumulators, 14 MMAs issued; epilogue warpgroups (threads 128,
// 256) 16/24 scales staged, 17/25 accumulators ready, 18/26 block terms,
// 19/27 item tail; 40 the CTA's cycles from entry to exit.
#ifdef FRC_PHASES
__device__ __forceinline__ long long pf_now() { return clock64(); }
struct PfClock {
  long long t;
  long long ph[5];
  __device__ PfClock() : t(pf_now()), ph{0, 0, 0, 0, 0} {}
  __device__ void lap(unsigned k) {
    const long long n = pf_now();
    ph[k] += n - t;
    t = n;
  }
  __device__ void store(unsigned long long* out, unsigned base, bool who) const {
    if (out && who)
      for (unsigned k = 0; k < 5; ++k) out[blockIdx.x * 64 + base + k] = static_cast<unsigned long long>(ph[k]);
  }
};
#define PF_PH(x) x
#else
#define PF_PH(x)
#endif

// ------------------------------------------------------------- helpers

__device__ __forceinline__ bool pf_wait(uint64_t* bar, unsigned parity, volatile unsigned* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 1000000)) {
    if (*abort) return false;
    if (globaltimer() - start > kWaitNs) {
      *abort = 1;
      return false;
    }
  }
  return true;
}
// The same decision for a whole warp (lane 0 waits): warp-collective
// instructions after it (tcgen05.ld, __syncwarp) need every lane.
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, unsigned parity, volatile unsigned* abort) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = pf_wait(bar, parity, abort);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void conv_sync() { asm volatile("bar.sync 3, 128;" ::: "memory"); }
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Named barrier of one epilogue warpgroup (ids 1 and 2).
__device__ __forceinline__ void epi_sync(unsigned wg) { asm volatile("bar.sync %0, 128;" ::"r"(wg + 1) : "memory"); }
// Tiled 2D TMA load (no multicast): box at byte column x, row y of the map.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Q8Group::q with the group's scale and multiplier given (the same values):
// the nearest-even rounding through 1.5 * 2^23 (|v| <= 127 here) and the
// clamp in integers, no float-to-int conversion.
__device__ __forceinline__ int q8_fast(float x, float amax, float scale, float inv) {
  if (scale == 0.0f) return 0;
  float v;
  if (isfinite(inv)) v = __fmul_rn(x, inv);
  else v = __fmul_rn(__fdiv_rn(x, amax), 127.0f);
  const int r = __float_as_int(__fadd_rn(v, 12582912.0f)) - 0x4B400000;
  return max(-127, min(127, r));
}

// SwiGLU of backends/ref.c:81-83 without branches: with e = exp(-|a|) the
// stable sigmoid is 1/(1+e) for a >= 0 and e/(1+e) for a < 0, the same
// double operations as swiglu() in frc_device.cuh.  `fail` on a nonfinite
// or fp32-overflowing result.
__device__ __forceinline__ float swiglu_nb(float a, float u, bool& fail) {
  const double ad = a;
  const double e = exp(-fabs(ad));
  const double sig = (a >= 0 ? 1.0 : e) / (1.0 + e);
  const double v = ad * sig * static_cast<double>(u);
  fail = !(fabs(v) <= 3.4028234663852886e38);
  return __double2float_rn(v);
}

// 16 payload bytes of one MXFP4 block (byte j: element j low nibble, element
// j+16 high nibble) -> 32 int8 doubled E2M1 values in prmt order: for word m,
// bytes (j, j+16, j+1, j+17) then (j+2, j+18, j+3, j+19), j = 4m.
__device__ __forceinline__ void mxfp4_to_i8(uint4 q, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  uint32_t o[8];
#pragma unroll
  for (unsigned m = 0; m < 4; ++m) {
#pragma unroll
    for (unsigned h = 0; h < 2; ++h) {
      const uint32_t sel = h ? w[m] >> 16 : w[m];
      const uint32_t pos = prmt(kE2M1Lo, kE2M1Hi, sel), neg = prmt(kE2M1Lo, kE2M1Hi, sel ^ 0x8888u);
      // byte-wise pos - neg (one of them is 0, both <= 12): with a bias of
      // 0x80 a byte no borrow crosses a byte; one three-input add
      o[2 * m + h] = ((pos + 0x80808080u) - neg) ^ 0x80808080u;
    }
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

// One Q4_K super-block of an A row (144 bytes: fp16 d, fp16 dmin, 12 bytes
// of 6-bit scales and mins, 128 bytes of nibbles; src/native.c:14-19) ->
// 256 int8 q in the B rows' prmt order per 32-block, its eight scales and
// mins, and {d, dmin}.  Sub-block 2g is the low nibbles of bytes 32g..32g+31,
// 2g+1 their high nibbles (element i of a sub-block in byte i).
__device__ __forceinline__ void q4k_row_to_i8(const uint8_t* rowp, uint8_t* A, unsigned m, uint8_t* sm, float2& dd) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(rowp);
  dd = make_float2(h2f(hdr.x & 0xffffu), h2f(hdr.x >> 16));
  const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};  // scale bytes s[0..11]
  auto sb = [&](unsigned i) { return (sw[i >> 2] >> (8 * (i & 3))) & 255u; };
  uint32_t scv[2] = {0, 0}, miv[2] = {0, 0};
#pragma unroll
  for (unsigned g = 0; g < 8; ++g) {
    const unsigned sc = g < 4 ? sb(g) & 63 : (sb(g + 4) & 15) | ((sb(g - 4) >> 6) << 4);
    const unsigned mi = g < 4 ? sb(g + 4) & 63 : (sb(g + 4) >> 4) | ((sb(g) >> 6) << 4);
    scv[g >> 2] |= sc << (8 * (g & 3));
    miv[g >> 2] |= mi << (8 * (g & 3));
  }
  *reinterpret_cast<uint4*>(sm) = make_uint4(scv[0], scv[1], miv[0], miv[1]);
#pragma unroll
  for (unsigned gp = 0; gp < 4; ++gp) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(rowp + 16 + 32 * gp);
    const uint4 w1 = *reinterpret_cast<const uint4*>(rowp + 32 + 32 * gp);
    const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
      // elements (j, j+16, j+1, j+17) and (j+2, j+18, j+3, j+19), j = 4k
      const uint32_t o0 = prmt(W[k], W[k + 4], 0x5140u), o1 = prmt(W[k], W[k + 4], 0x7362u);
      lo[2 * k] = o0 & 0x0f0f0f0fu;
      lo[2 * k + 1] = o1 & 0x0f0f0f0fu;
      hi[2 * k] = (o0 >> 4) & 0x0f0f0f0fu;
      hi[2 * k + 1] = (o1 >> 4) & 0x0f0f0f0fu;
    }
    *reinterpret_cast<uint4*>(A + umma_off(m, 64 * gp, 256)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(A + umma_off(m, 64 * gp + 16, 256)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    *reinterpret_cast<uint4*>(A + umma_off(m, 64 * gp + 32, 256)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(A + umma_off(m, 64 * gp + 48, 256)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  }
}

// --------------------------------------------------------- 1. quantize

// One warp per 64-group, two values per lane; the operations of
// quantize_kernel, the int8 values written in prmt order.
__global__ void prefill_quantize_kernel(PrefillArgs a) {
  const unsigned g = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  const unsigned groups = a.T * (a.d / 64);
  if (g >= groups) return;
  float2 v;
  if (a.x_bf16) {  // two bf16 words: the upper halves of two fp32 patterns
    const uint32_t w = reinterpret_cast<const uint32_t*>(a.x)[32 * static_cast<size_t>(g) + lane];
    v = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    v = reinterpret_cast<const float2*>(a.x + 64 * static_cast<size_t>(g))[lane];
  }
  const bool bad = !isfinite(v.x) || !isfinite(v.y);
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0) atomicOr(a.status, kStNumeric);
    return;
  }
  float amax = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
  for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const Q8Group q(amax);
  int8_t* out = a.xq + 64 * static_cast<size_t>(g);
  int8_t* rout = a.xr + 64 * static_cast<size_t>(g);
  const unsigned n0 = 2 * lane, blk = n0 >> 5, n = n0 & 31;
  const int q0 = q.q(v.x), q1 = q.q(v.y);
  out[32 * blk + prmt_pos(n)] = static_cast<int8_t>(q0);
  out[32 * blk + prmt_pos(n + 1)] = static_cast<int8_t>(q1);
  // the residuals X - v * s = r * 2^E of the reference's dequantized values
  // X = fl32(v * s) (src/q4.c:54-58, the FLT_MAX cap included), as in the
  // decode kernel's activation pass
  const unsigned ef = scale_ef(q.scale), shr = 150 - ef;
  const float f1 = __uint_as_float((127 + (shr >> 1)) << 23), f2 = __uint_as_float((127 + shr - (shr >> 1)) << 23);
  auto resid = [&](int qv) {
    const float vf = i2f(qv);
    float X = __fmul_rn(vf, q.scale);
    if (fabsf(X) > 3.40282347e38f) X = copysignf(3.40282347e38f, vf);
    return f2i_small(__fmul_rn(__fmul_rn(__fmaf_rn(-vf, q.scale, X), f1), f2));
  };
  const int r0 = resid(q0), r1 = resid(q1);
  rout[32 * blk + prmt_pos(n)] = static_cast<int8_t>(r0);
  rout[32 * blk + prmt_pos(n + 1)] = static_cast<int8_t>(r1);
  // natural order too, for the shared expert's rows (copied to the operand
  // tiles as they are)
  reinterpret_cast<char2*>(a.xqn + 64 * static_cast<size_t>(g))[lane] =
      make_char2(static_cast<char>(q0), static_cast<char>(q1));
  reinterpret_cast<char2*>(a.xrn + 64 * static_cast<size_t>(g))[lane] =
      make_char2(static_cast<char>(r0), static_cast<char>(r1));
  if (a.xvr) {  // Q4_K rows: each 32-block's sums of v and of r (lanes 0-15, 16-31)
    int sv = q0 + q1, sr = r0 + r1;
#pragma unroll
    for (unsigned o = 8; o; o >>= 1) {
      sv += __shfl_xor_sync(0xffffffffu, sv, o);
      sr += __shfl_xor_sync(0xffffffffu, sr, o);
    }
    if ((lane & 15) == 0) a.xvr[2 * static_cast<size_t>(g) + blk] = make_int2(sv, sr);
  }
  if (lane == 0) {
    a.xs[g] = q.scale;
    const unsigned sb = __float_as_uint(q.scale);
    // {M, E << 20} (E shifted into a double's exponent field)
    a.xme[g] = make_int2(static_cast<int>((sb >> 23 & 255u) ? (sb & 0x7fffffu) | 0x800000u : sb & 0x7fffffu),
                         static_cast<int>((ef - 150u) << 20));
  }
}

// ------------------------------------------------------------ 2. group

// Exclusive prefix sum of v over threads 0..511 of a 1024-thread CTA (the
// others pass 0); *total receives the sum.  Every thread must call it.
__device__ __forceinline__ unsigned scan512(unsigned v, unsigned* ws, unsigned& total) {
  const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned x = v;
#pragma unroll
  for (unsigned o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31 && w < 16) ws[w] = x;
  __syncthreads();
  if (w == 0) {
    unsigned t = lane < 16 ? ws[lane] : 0u;
#pragma unroll
    for (unsigned o = 1; o < 16; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < 16) ws[lane] = t;
  }
  __syncthreads();
  const unsigned excl = x - v + (w > 0 && w < 16 ? ws[w - 1] : 0u);
  total = ws[15];
  __syncthreads();
  return excl;
}

// Single CTA of 1024 threads.  Validation (ids < 512 and distinct per token,
// gates finite and >= 0, shared gate 0), pairs, work lists.
__global__ void __launch_bounds__(1024) prefill_group_kernel(PrefillArgs a) {
  __shared__ uint32_t bits[512][16];  // token bitmap per expert (T <= 512)
  __shared__ uint32_t shbits[16];     // tokens whose shared-expert gate is not zero
  __shared__ unsigned cnt[512], rank_of[512], ibase_gu[513], ibase_dn[513], poff[513];
  __shared__ unsigned by_rank[512], scan_ws[16], nsh_s;
  const unsigned tid = threadIdx.x, T = a.T, words = (T + 31) / 32;
  for (unsigned i = tid; i < 512 * 16; i += blockDim.x) (&bits[0][0])[i] = 0;
  if (tid < 16) shbits[tid] = 0;
  __syncthreads();
  unsigned st = 0;
  for (unsigned i = tid; i < T * 10; i += blockDim.x) {
    const unsigned t = i / 10, e = a.expert[i];
    if (e >= 512) { st |= kStInvalid; continue; }
    const uint32_t bit = 1u << (t & 31);
    if (atomicOr(&bits[e][t >> 5], bit) & bit) st |= kStInvalid;  // the same expert twice in one token
  }
  for (unsigned i = tid; i < T * 11; i += blockDim.x) {
    const float g = a.gate[i];
    if (!isfinite(g)) st |= kStNumeric;
    else if (g < 0.0f) st |= kStInvalid;
    else if (i % 11 == 10 && g != 0.0f) atomicOr(&shbits[(i / 11) >> 5], 1u << ((i / 11) & 31));
  }
  if (st) atomicOr(a.status, st);
  __syncthreads();
  if (tid == 0) {
    unsigned n = 0;
    for (unsigned w = 0; w < words; ++w) n += __popc(shbits[w]);
    nsh_s = n;
  }
  for (unsigned e = tid; e < 512; e += blockDim.x) {
    unsigned c = 0;
    for (unsigned w = 0; w < words; ++w) c += __popc(bits[e][w]);
    cnt[e] = c;
  }
  __syncthreads();
  // rank experts by token count descending, ties by id
  for (unsigned e = tid; e < 512; e += blockDim.x) {
    const unsigned c = cnt[e];
    unsigned r = 0;
    for (unsigned f = 0; f < 512; ++f) r += cnt[f] > c || (cnt[f] == c && f < e);
    rank_of[e] = r;
    by_rank[r] = e;
  }
  __syncthreads();
  // The shared expert (id 512, Q8_0 rows) takes the pairs after the routed
  // ones (tokens ascending) and the first items of both work lists (it is
  // the biggest expert of a burst that uses it).
  const unsigned npairs = (a.S + 1) / 2, nrt = a.d / 128;
  const unsigned nsh = nsh_s, tiles_sh = (nsh + kPfTile - 1) / kPfTile;
  {
    // pair offsets in expert order, item offsets in rank order: block scans
    unsigned tp, tgu, tdn;
    const unsigned ep = scan512(tid < 512 ? cnt[tid] : 0u, scan_ws, tp);
    const unsigned tiles = tid < 512 ? (cnt[by_rank[tid]] + kPfTile - 1) / kPfTile : 0u;
    const unsigned eg = scan512(tiles * npairs, scan_ws, tgu);
    const unsigned ed = scan512(tiles * nrt, scan_ws, tdn);
    if (tid < 512) {
      poff[tid] = ep;
      ibase_gu[tid] = eg + tiles_sh * npairs;
      ibase_dn[tid] = ed + tiles_sh * nrt;
    }
    if (tid == 0) {
      poff[512] = tp;
      a.counts[0] = tp + nsh;
      a.counts[1] = tgu + tiles_sh * npairs;
      a.counts[2] = tdn + tiles_sh * nrt;
      a.counts[3] = tp;  // routed pairs
      a.counts[4] = tiles_sh * npairs;  // the shared expert's gate/up items (first in the list)
      a.counts[5] = tiles_sh * nrt;     // its down items
    }
  }
  __syncthreads();
  for (unsigned i = tid; i < T * 10; i += blockDim.x) {
    const unsigned t = i / 10, e = a.expert[i];
    if (e >= 512) { a.slot_pair[t * 11 + i % 10] = 0xffffffffu; continue; }
    unsigned r = __popc(bits[e][t >> 5] & ((1u << (t & 31)) - 1));
    for (unsigned w = 0; w < (t >> 5); ++w) r += __popc(bits[e][w]);
    const unsigned p = poff[e] + r;
    a.pair_token[p] = static_cast<uint16_t>(t);
    a.slot_pair[t * 11 + i % 10] = p;
  }
  for (unsigned t = tid; t < T; t += blockDim.x) {
    unsigned p = 0xffffffffu;
    if (shbits[t >> 5] >> (t & 31) & 1u) {
      unsigned r = __popc(shbits[t >> 5] & ((1u << (t & 31)) - 1));
      for (unsigned w = 0; w < (t >> 5); ++w) r += __popc(shbits[w]);
      p = poff[512] + r;
      a.pair_token[p] = static_cast<uint16_t>(t);
    }
    a.slot_pair[t * 11 + 10] = p;
  }
  for (unsigned e = tid; e < 513; e += blockDim.x) {
    const bool sh = e == 512;
    const unsigned c = sh ? nsh : cnt[e], tiles = (c + kPfTile - 1) / kPfTile;
    const unsigned bgu = sh ? 0u : ibase_gu[rank_of[e]], bdn = sh ? 0u : ibase_dn[rank_of[e]];
    for (unsigned k = 0; k < tiles; ++k) {
      const unsigned n = min(kPfTile, c - k * kPfTile), p0 = poff[e] + k * kPfTile;
      for (unsigned q = 0; q < npairs; ++q) a.items_gu[bgu + k * npairs + q] = make_uint4(e, p0, n, q);
      for (unsigned q = 0; q < nrt; ++q) a.items_dn[bdn + k * nrt + q] = make_uint4(e, p0, n, q);
    }
  }
}

// ---------------------------------------------------------- 3/4. MMA

struct PfScales;
template <unsigned MODE>
__device__ __forceinline__ void pf_apply16(const PfScales& sc, unsigned st, unsigned m, unsigned col,
                                           const uint32_t (&v)[16], float* acc, bool live, bool& bad,
                                           bool q8 = false);

// One chunk's scales, in a ring of their own: the epilogue holds a chunk's
// scales long after the MMAs have released its operand stage.
struct PfScales {
  union {
    float col[8][kPfTile];  // down: per block of the chunk, per pair (hidden scale)
    int2 me[4][kPfTile];    // gate/up: per x group of the chunk, per token {M, E << 20}
  };
  int2 vr[8][kPfTile];      // gate/up Q4_K: per block of the chunk, per token {V, RS}
  union {
    uint8_t row[8 * 128];   // E8M0 per A row and block (gate/up MXFP4 [row][8], down [block][128])
    struct {
      uint8_t sm[128][16];  // gate/up Q4_K: per A row, the super-block's 6-bit scales then mins
      float2 dd[128];       // gate/up Q4_K: per A row {d, dmin}
    } q4;
    uint16_t hg[128][8];    // gate/up, shared expert (Q8_0): per A row, the chunk's fp16 block scales
    uint16_t hd[8][128];    // down, shared expert (Q8_0): per block of the chunk, per A row, fp16 scale
  };
};

struct PfSmem {
  uint8_t raw[kPfRaw][kPfRawBytes];
  uint8_t A[kPfAB][kPfA];
  uint8_t B[kPfAB][kPfB];
  PfScales sc[kPfSc];
  float amax[4][kPfTile];         // gate/up epilogue: per-warp amax per token
  unsigned tok[2][kPfTile];       // converters: token ids of the last two items requested
  uint64_t raw_full[kPfRaw], raw_empty[kPfRaw];
  uint64_t ab_full[kPfAB], ab_empty[kPfAB], sc_full[kPfSc], sc_empty[kPfSc];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t taddr;
  unsigned abort;
};

// Packed fp32 pairs (sm_100 f32x2 ops: one instruction, two IEEE results
// with the same rounding as the scalar operations).
__device__ __forceinline__ void add2(float& x, float& y, float bx, float by) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(x), "+f"(y) : "f"(bx), "f"(by));
}
__device__ __forceinline__ void mul2(float& x, float& y, float bx, float by) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(x), "+f"(y) : "f"(bx), "f"(by));
}
// (cx, cy) = fma(a, b, (cx, cy)) pairwise
__device__ __forceinline__ void fma2(float ax, float ay, float bx, float by, float& cx, float& cy) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%0, %1};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(cx), "+f"(cy) : "f"(ax), "f"(ay), "f"(bx), "f"(by));
}

// One MMA step's int32 results for 16 token columns (starting at `col`) of
// A row m: acc[j] = fmaf(float(I) * colscale, rowscale, acc[j]), the row's
// block scale 2^(e-128) (E8M0 e; 255 is nonfinite).  float(I) is exact
// (|I| < 2^22): the bits of I + 1.5 * 2^23 less that constant.
template <unsigned MODE>
__device__ __forceinline__ void pf_apply16(const PfScales& sc, unsigned st, unsigned m, unsigned col,
                                           const uint32_t (&v)[16], float* acc, bool live, bool& bad, bool q8) {
  float ws;
  if (q8) {  // the shared expert's Q8_0 down row: its fp16 scale
    ws = h2f(sc.hd[st][m]);
    bad |= live && !isfinite(ws);
  } else {
    const unsigned e8 = sc.row[MODE == kGateUp ? 8 * m + st : 128 * st + m];
    bad |= live && e8 == 255;
    ws = pow2_m128(e8);
  }
  const float4* cs = reinterpret_cast<const float4*>(sc.col[st] + col);
#pragma unroll
  for (unsigned q4 = 0; q4 < 4; ++q4) {
    const float4 cv = cs[q4];
    const unsigned j = 4 * q4;
    float f0 = __int_as_float(static_cast<int>(v[j]) + 0x4B400000), f1 = __int_as_float(static_cast<int>(v[j + 1]) + 0x4B400000);
    float f2 = __int_as_float(static_cast<int>(v[j + 2]) + 0x4B400000), f3 = __int_as_float(static_cast<int>(v[j + 3]) + 0x4B400000);
    add2(f0, f1, -12582912.0f, -12582912.0f);
    add2(f2, f3, -12582912.0f, -12582912.0f);
    mul2(f0, f1, cv.x, cv.y);
    mul2(f2, f3, cv.z, cv.w);
    fma2(f0, f1, ws, ws, acc[j], acc[j + 1]);
    fma2(f2, f3, ws, ws, acc[j + 2], acc[j + 3]);
  }
}

template <unsigned MODE>
__device__ __forceinline__ unsigned pf_chunks(const PrefillArgs& a) {
  return MODE == kGateUp ? a.d / 256 : (a.S + 7) / 8;
}
template <unsigned MODE>
__device__ __forceinline__ unsigned pf_steps(const PrefillArgs& a, unsigned k) {
  return MODE == kGateUp ? 8u : min(8u, a.S - 8 * k);
}
// Loaded-block index and HBM row (within the slice) of A row m of a gate/up
// item: warp m/32 holds 16 neurons of one block, lanes 0-15 gate, 16-31 up.
__device__ __forceinline__ void gu_row(unsigned m, unsigned pair, unsigned& blk, unsigned& hrow) {
  const unsigned w = m >> 5, l = m & 31;
  blk = 2 * pair + (w >> 1);
  hrow = (l >> 4) * 32 + 16 * (w & 1) + (l & 15);
}

// One accumulator group's exact gate/up block terms for this thread's row m
// and its warpgroup's live units q < nq (columns 8q .. 8q + 3 from tg, which
// carries the warpgroup's offset 4 wg): steps g0 .. g0 + n - 1 of the chunk
// (n even: the group size divides the chunk's eight steps), two steps (one x
// group: one {M, E} per token) x two units at a time, eight 4-column TMEM
// reads and one wait.  With the token's group scale s = M * 2^E and the
// row's block scale 2^(e - 128), Z = M * I + R is an exact integer
// (|Z| < 2^47) and the sum takes fma(Z, 2^(e - 128 + E), acc) in double,
// blocks in order.
__device__ __forceinline__ void gu_terms(double (&accd)[32], const PfScales& sc, uint32_t tg, unsigned bw,
                                         unsigned npad, unsigned wg, unsigned m, unsigned g0, unsigned n, unsigned nq,
                                         bool live, bool& bad) {
  if (nq == 1) {
    // one unit (tiles of up to 8 tokens; n is 8 or 4): four steps a read
    for (unsigned j0 = 0; j0 < n; j0 += 4) {
      const unsigned st = g0 + j0;  // a multiple of 4: x groups st / 2 and st / 2 + 1
      uint32_t vi[16], vr[16];      // [step][4 columns]
#pragma unroll
      for (unsigned js = 0; js < 4; ++js) {
        const uint32_t t = tg + (j0 + js) * bw;
        tmem_ld4(t, vi + 4 * js);
        tmem_ld4(t + npad, vr + 4 * js);
      }
      const unsigned e4 = *reinterpret_cast<const uint32_t*>(sc.row + 8 * m + st);
      bad |= live && __vcmpeq4(e4, 0xffffffffu) != 0;
      tmem_wait_ld();
#pragma unroll
      for (unsigned h = 0; h < 2; ++h) {
        const int4* mev = reinterpret_cast<const int4*>(sc.me[(st >> 1) + h]) + 2 * wg;
        const int4 xa = mev[0], xb = mev[1];
        const int M[4] = {xa.x, xa.z, xb.x, xb.z}, Eh[4] = {xa.y, xa.w, xb.y, xb.w};
        const int wb0 = static_cast<int>(((e4 >> (16 * h)) & 255u) + (1023 - 128)) << 20;
        const int wb1 = static_cast<int>(((e4 >> (16 * h + 8)) & 255u) + (1023 - 128)) << 20;
#pragma unroll
        for (unsigned jj = 0; jj < 4; ++jj) {
          const long long z0 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * h + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * h + jj]));
          const long long z1 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * h + 4 + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * h + 4 + jj]));
          double acc = accd[jj];
          acc = fma(__longlong_as_double(z0) - 6755399441055744.0, __hiloint2double(wb0 + Eh[jj], 0), acc);
          acc = fma(__longlong_as_double(z1) - 6755399441055744.0, __hiloint2double(wb1 + Eh[jj], 0), acc);
          accd[jj] = acc;
        }
      }
    }
    return;
  }
  for (unsigned j0 = 0; j0 < n; j0 += 2) {
    const unsigned st = g0 + j0;  // even
    const unsigned e2 = *reinterpret_cast<const uint16_t*>(sc.row + 8 * m + st);
    const unsigned e0 = e2 & 255u, e1 = e2 >> 8;
    bad |= live && (e0 == 255 || e1 == 255);
    // high words of 2^(e - 128 + E): (e - 128 + 1023) << 20 plus the token's
    // E << 20 (stored shifted)
    const int wb0 = static_cast<int>(e0 + (1023 - 128)) << 20, wb1 = static_cast<int>(e1 + (1023 - 128)) << 20;
    const int4* mev = reinterpret_cast<const int4*>(sc.me[st >> 1]) + 2 * wg;  // unit q: mev[4q], mev[4q + 1]
#pragma unroll
    for (unsigned q0 = 0; q0 < 8; q0 += 2) {
      if (q0 >= nq) break;  // warp-uniform
      uint32_t vi[16], vr[16];  // [unit of the pair][step][4 columns]
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb)
        if (q0 + qb < nq) {
          const uint32_t t = tg + j0 * bw + 8 * (q0 + qb);
          tmem_ld4(t, vi + 8 * qb);                 // I: the v rows' results
          tmem_ld4(t + bw, vi + 8 * qb + 4);
          tmem_ld4(t + npad, vr + 8 * qb);          // R: the r rows' results
          tmem_ld4(t + bw + npad, vr + 8 * qb + 4);
        }
      tmem_wait_ld();
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb) {
        const unsigned q = q0 + qb;
        if (q >= nq) continue;
        const int4 xa = mev[4 * q], xb = mev[4 * q + 1];  // {M, E << 20} of columns 0-1, 2-3
        const int M[4] = {xa.x, xa.z, xb.x, xb.z}, Eh[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
        for (unsigned jj = 0; jj < 4; ++jj) {
          // Z + 1.5 * 2^52 as the bits of a double
          const long long z0 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * qb + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * qb + jj]));
          const long long z1 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * qb + 4 + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * qb + 4 + jj]));
          double acc = accd[4 * q + jj];
          acc = fma(__longlong_as_double(z0) - 6755399441055744.0, __hiloint2double(wb0 + Eh[jj], 0), acc);
          acc = fma(__longlong_as_double(z1) - 6755399441055744.0, __hiloint2double(wb1 + Eh[jj], 0), acc);
          accd[4 * q + jj] = acc;
        }
      }
    }
  }
}

// The Q4_K form of gu_terms: one accumulator group's steps (n even) in x
// groups of two blocks (st, st + 1), two units at a time.  With the row's
// sub-block scales sc and mins mi, the tokens' block sums V, RS of v and r,
// K1 = sc0 I0 + sc1 I1, K3 = sc0 R0 + sc1 R1, K2 = mi0 V0 + mi1 V1,
// K4 = mi0 RS0 + mi1 RS1, the group's term of the reference's sum of
// w * fl32(v * s) is (M K1 + K3) d 2^E - (M K2 + K4) dmin 2^E: two exact
// integers (|M K1 + K3| < 2^47) times exact doubles, added in that order.
__device__ __forceinline__ void gu_terms_q4k(double (&accd)[32], const PfScales& sc, uint32_t tg, unsigned bw,
                                             unsigned npad, unsigned wg, unsigned m, unsigned g0, unsigned n,
                                             unsigned nq, const float2 dd) {
  const double dmul = dd.x, mmul = -static_cast<double>(dd.y);
  for (unsigned j0 = 0; j0 < n; j0 += 2) {
    const unsigned st = g0 + j0;  // even
    const unsigned scp = *reinterpret_cast<const uint16_t*>(&sc.q4.sm[m][st]);
    const unsigned mip = *reinterpret_cast<const uint16_t*>(&sc.q4.sm[m][8 + st]);
    const int sc0 = scp & 255u, sc1 = scp >> 8, mi0 = mip & 255u, mi1 = mip >> 8;
    const int4* mev = reinterpret_cast<const int4*>(sc.me[st >> 1]) + 2 * wg;  // unit q: mev[4q], mev[4q + 1]
    const int2* vr0 = sc.vr[st] + 4 * wg;
    const int2* vr1 = sc.vr[st + 1] + 4 * wg;
#pragma unroll
    for (unsigned q0 = 0; q0 < 8; q0 += 2) {
      if (q0 >= nq) break;  // warp-uniform
      uint32_t vi[16], vr[16];  // [unit of the pair][step][4 columns]
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb)
        if (q0 + qb < nq) {
          const uint32_t t = tg + j0 * bw + 8 * (q0 + qb);
          tmem_ld4(t, vi + 8 * qb);
          tmem_ld4(t + bw, vi + 8 * qb + 4);
          tmem_ld4(t + npad, vr + 8 * qb);
          tmem_ld4(t + bw + npad, vr + 8 * qb + 4);
        }
      tmem_wait_ld();
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb) {
        const unsigned q = q0 + qb;
        if (q >= nq) continue;
        const int4 xa = mev[4 * q], xb = mev[4 * q + 1];  // {M, E << 20} of columns 0-1, 2-3
        const int M[4] = {xa.x, xa.z, xb.x, xb.z}, Eh[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
        for (unsigned jj = 0; jj < 4; ++jj) {
          const int2 s0 = vr0[8 * q + jj], s1 = vr1[8 * q + jj];
          const int K1 = sc0 * static_cast<int>(vi[8 * qb + jj]) + sc1 * static_cast<int>(vi[8 * qb + 4 + jj]);
          const int K3 = sc0 * static_cast<int>(vr[8 * qb + jj]) + sc1 * static_cast<int>(vr[8 * qb + 4 + jj]);
          const int K2 = mi0 * s0.x + mi1 * s1.x, K4 = mi0 * s0.y + mi1 * s1.y;
          // Z + 1.5 * 2^52 as the bits of a double
          const long long z1 = static_cast<long long>(M[jj]) * K1 + (0x4338000000000000LL + K3);
          const long long z2 = static_cast<long long>(M[jj]) * K2 + (0x4338000000000000LL + K4);
          const double P = __hiloint2double(Eh[jj] + (1023 << 20), 0);  // 2^E
          double acc = accd[4 * q + jj];
          acc = fma(__longlong_as_double(z1) - 6755399441055744.0, dmul * P, acc);
          acc = fma(__longlong_as_double(z2) - 6755399441055744.0, mmul * P, acc);
          accd[4 * q + jj] = acc;
        }
      }
    }
  }
}

// The shared expert's form of gu_terms (Q8_0 rows, operands in natural
// order): each block's exact Z = M I + R times the exact double d_b 2^E (d_b
// the block's fp16 scale), blocks in order; two steps x two units a read.
__device__ __forceinline__ void gu_terms_q8(double (&accd)[32], const PfScales& sc, uint32_t tg, unsigned bw,
                                            unsigned npad, unsigned wg, unsigned m, unsigned g0, unsigned n,
                                            unsigned nq, bool live, bool& bad) {
  for (unsigned j0 = 0; j0 < n; j0 += 2) {
    const unsigned st = g0 + j0;  // even
    const uint32_t hp = *reinterpret_cast<const uint32_t*>(&sc.hg[m][st]);
    const float f0 = h2f(hp & 0xffffu), f1 = h2f(hp >> 16);
    bad |= live && !(isfinite(f0) && isfinite(f1));
    const double d0 = f0, d1 = f1;
    const int4* mev = reinterpret_cast<const int4*>(sc.me[st >> 1]) + 2 * wg;
#pragma unroll
    for (unsigned q0 = 0; q0 < 8; q0 += 2) {
      if (q0 >= nq) break;  // warp-uniform
      uint32_t vi[16], vr[16];
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb)
        if (q0 + qb < nq) {
          const uint32_t t = tg + j0 * bw + 8 * (q0 + qb);
          tmem_ld4(t, vi + 8 * qb);
          tmem_ld4(t + bw, vi + 8 * qb + 4);
          tmem_ld4(t + npad, vr + 8 * qb);
          tmem_ld4(t + bw + npad, vr + 8 * qb + 4);
        }
      tmem_wait_ld();
#pragma unroll
      for (unsigned qb = 0; qb < 2; ++qb) {
        const unsigned q = q0 + qb;
        if (q >= nq) continue;
        const int4 xa = mev[4 * q], xb = mev[4 * q + 1];
        const int M[4] = {xa.x, xa.z, xb.x, xb.z}, Eh[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
        for (unsigned jj = 0; jj < 4; ++jj) {
          const long long z0 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * qb + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * qb + jj]));
          const long long z1 = static_cast<long long>(M[jj]) * static_cast<int>(vi[8 * qb + 4 + jj]) +
                               (0x4338000000000000LL + static_cast<int>(vr[8 * qb + 4 + jj]));
          const double P = __hiloint2double(Eh[jj] + (1023 << 20), 0);  // 2^E
          double acc = accd[4 * q + jj];
          acc = fma(__longlong_as_double(z0) - 6755399441055744.0, d0 * P, acc);
          acc = fma(__longlong_as_double(z1) - 6755399441055744.0, d1 * P, acc);
          accd[4 * q + jj] = acc;
        }
      }
    }
  }
}

// Register split (setmaxnreg): launched at 128 a thread (448 x 128 =
// 57,344; each SM sub-partition holds four of the 14 warps at most, 16,384
// registers), the converter warpgroup gives up 32 a thread (96) and the two
// epilogue warpgroups take them (144); warps 12-13 keep 128:
// 128 x 96 + 256 x 144 + 64 x 128 = 57,344.
// Q4 (gate/up only): Q4_K gate/up rows, else MXFP4.  SH: the launch over the
// shared expert's items (the first counts[4] / counts[5] of the work lists,
// Q8_0 rows), else over the routed experts' items; the two are separate
// instantiations so that neither carries the other's code and registers.
template <unsigned MODE, bool Q4, bool SH>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_mma_kernel(const __grid_constant__ PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PfSmem& s = *reinterpret_cast<PfSmem*>(smem_raw);
  const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned nall = a.counts[MODE == kGateUp ? 1 : 2], nsh = a.counts[MODE == kGateUp ? 4 : 5];
  const unsigned nitems = SH ? nsh : nall - nsh;
  const uint4* items = (MODE == kGateUp ? a.items_gu : a.items_dn) + (SH ? 0 : nsh);
  const unsigned nk = pf_chunks<MODE>(a), d = a.d, nb = d / 32;
  volatile unsigned* abort = &s.abort;

  if (tid == 0) {
    for (unsigned i = 0; i < kPfRaw; ++i) { mbar_init(&s.raw_full[i], 1); mbar_init(&s.raw_empty[i], 128); }
    for (unsigned i = 0; i < kPfAB; ++i) { mbar_init(&s.ab_full[i], 128); mbar_init(&s.ab_empty[i], 1); }
    for (unsigned i = 0; i < kPfSc; ++i) { mbar_init(&s.sc_full[i], 128); mbar_init(&s.sc_empty[i], 8); }
    for (unsigned i = 0; i < 2; ++i) { mbar_init(&s.acc_full[i], 1); mbar_init(&s.acc_empty[i], 8); }
    s.abort = 0;
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(&s.taddr, kPfCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.taddr;
  PF_PH(const long long t_entry = pf_now(); PfClock clk;)

  if (warp == 12) {
    // ------------------------------------------------ producer: bulk copies
    unsigned c = 0;
    for (unsigned it = blockIdx.x; it < nitems && !*abort; it += gridDim.x) {
      const uint4 item = items[it];
      for (unsigned k = 0; k < nk; ++k, ++c) {
        const unsigned st = c % kPfRaw;
        PF_PH(clk.lap(1);)
        if (!pf_wait_warp(&s.raw_empty[st], ((c / kPfRaw) & 1) ^ 1, abort)) break;
        PF_PH(clk.lap(0);)
        uint8_t* dst = s.raw[st];
        if (SH) {
          // the shared expert's rows reach the operand tiles by cp.async
          // from the converters: the stage completes with no bytes
          if (lane == 0) mbar_expect_tx(&s.raw_full[st], 0);
          __syncwarp();
        } else if (MODE == kGateUp && Q4) {
          // one 144 B x 64-row box per slice: super-block k of its 32 gate and
          // 32 up rows (3D map: byte, row of the slice, slice), unswizzled
          const unsigned nsl = 2 * item.w + 1 < a.S ? 2 : 1;
          if (lane == 0) {
            mbar_expect_tx(&s.raw_full[st], nsl * kPfQ4Box);
            for (unsigned sl = 0; sl < nsl; ++sl)
              tma_load_3d(dst + kPfQ4Box * sl, &a.tmap[2 * item.w + sl], static_cast<int>(144 * k), 0,
                          static_cast<int>(item.x), &s.raw_full[st]);
          }
          __syncwarp();
        } else if (MODE == kGateUp) {
          // one 128 B x 64-row box per slice: bytes [nb + 128k, +128) of its
          // 32 gate and 32 up rows, stored 128-byte swizzled
          const unsigned nsl = 2 * item.w + 1 < a.S ? 2 : 1;
          if (lane == 0) {
            mbar_expect_tx(&s.raw_full[st], nsl * 64 * 128);
            for (unsigned sl = 0; sl < nsl; ++sl)
              tma_load_2d(dst + 8192 * sl, &a.tmap[2 * item.w + sl], static_cast<int>(nb + 128 * k),
                          static_cast<int>(item.x * a.slice_rows), &s.raw_full[st]);
          }
          __syncwarp();
        } else {
          const unsigned steps = pf_steps<MODE>(a, k);
          if (lane == 0) mbar_expect_tx(&s.raw_full[st], steps * 2048);
          __syncwarp();
          if (lane < steps) {
            const unsigned blk = 8 * k + lane;
            const uint8_t* down = a.base[blk] + item.x * a.slice_bytes + 64ull * a.row_bytes;
            bulk_g2s(dst + 2048 * lane, down + d + static_cast<size_t>(item.w) * 128 * 16, 2048, &s.raw_full[st]);
          }
        }
      }
    }
    // every issued copy must have landed before the CTA exits
    for (unsigned i = 0; i < kPfRaw && c > i; ++i) {
      const unsigned last = c - 1 - i;  // the most recent uses of each stage
      if (lane == 0) pf_wait(&s.raw_full[last % kPfRaw], (last / kPfRaw) & 1, abort);
    }
    __syncwarp();
    PF_PH(clk.store(a.phases, 8, MODE == kGateUp && lane == 0);)
  } else if (warp == 13) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      unsigned c = 0, r = 0;
      for (unsigned it = blockIdx.x; it < nitems && !*abort; it += gridDim.x) {
        const uint4 item = items[it];
        const unsigned npad = (item.z + 15) & ~15u;
        // gate/up: N = 2 npad (B rows [0, npad) v, [npad, 2 npad) r)
        const uint32_t idesc = umma_idesc_i8(128, MODE == kGateUp ? 2 * npad : npad);
        for (unsigned k = 0; k < nk && !*abort; ++k, ++c) {
          const unsigned ab = c % kPfAB;
          PF_PH(clk.lap(2);)
          if (!pf_wait(&s.ab_full[ab], (c / kPfAB) & 1, abort)) break;
          PF_PH(clk.lap(0);)
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.A[ab]), b0 = smem_u32(s.B[ab]);
          const unsigned steps = pf_steps<MODE>(a, k);
          const unsigned GS = pf_gs<MODE>(npad), BW = pf_bw<MODE>(npad);
          for (unsigned g0 = 0; g0 < steps; g0 += GS, ++r) {  // groups of up to GS steps
            const unsigned grp = r & 1, n = min(GS, steps - g0);
            PF_PH(clk.lap(2);)
            if (!pf_wait(&s.acc_empty[grp], ((r >> 1) & 1) ^ 1, abort)) break;
            PF_PH(clk.lap(1);)
            tc_fence_after();
            for (unsigned j = 0; j < n; ++j) {
              const unsigned st = g0 + j;
              umma_i8(tmem + 256 * grp + j * BW, umma_desc(a0 + 256 * st, 128, 8 * 256),
                      umma_desc(b0 + 256 * st, 128, 8 * 256), idesc, false);
            }
            umma_commit(&s.acc_full[grp]);
          }
          umma_commit(&s.ab_empty[ab]);
        }
      }
      // the last commit's arrive must land before the CTA exits
      if (c) pf_wait(&s.ab_empty[(c - 1) % kPfAB], ((c - 1) / kPfAB) & 1, abort);
      PF_PH(clk.store(a.phases, 12, MODE == kGateUp);)
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------ converters
    asm volatile("setmaxnreg.dec.sync.aligned.u32 96;" ::: "memory");
    // Software-pipelined: the B rows and scales of chunk c + 1 are requested
    // (cp.async) before chunk c's weights are converted, so the gather's L2
    // latency overlaps the conversion.  No abort test on the loops: all
    // converter threads must reach every conv_sync; after an abort each wait
    // fails at once.
    const unsigned m = tid;  // A row
    // the chunk stream being requested
    unsigned ic = 0, iit = blockIdx.x, ik = 0, iitem = 0;
    uint4 inext = iit < nitems ? items[iit] : make_uint4(0, 0, 0, 0);
    auto issue = [&]() -> bool {
      if (iit >= nitems) return false;
      const uint4 item = inext;
      const unsigned k = ik, ab = ic % kPfAB, sq = ic % kPfSc, steps = pf_steps<MODE>(a, k), tb = iitem & 1;
      PF_PH(clk.lap(4);)
      if (k == 0) {  // the item's token ids, read once (no dependent global loads per chunk)
        conv_sync();
        if (MODE == kGateUp && tid < item.z) s.tok[tb][tid] = a.pair_token[item.y + tid];
        conv_sync();
      }
      PF_PH(clk.lap(3);)
      const bool ok = pf_wait(&s.ab_empty[ab], ((ic / kPfAB) & 1) ^ 1, abort) &&
                      pf_wait(&s.sc_empty[sq], ((ic / kPfSc) & 1) ^ 1, abort);
      PF_PH(clk.lap(2);)
      if (ok) {
        // B rows: the tile's tokens (gate/up: x of token j in row j and its
        // residuals in row npad + j; down: hq of the pair)
        const unsigned npad = (item.z + 15) & ~15u;
        for (unsigned i = tid; i < item.z * (MODE == kGateUp ? 32u : 16u); i += 128) {
          const unsigned j = (i >> 4) % item.z, half = (i >> 4) / item.z, piece = i & 15;
          if (MODE == kDown && piece >= 2 * steps) continue;
          const int8_t* xsrc = SH ? (half ? a.xrn : a.xqn) : (half ? a.xr : a.xq);
          const int8_t* src = MODE == kGateUp
                                  ? xsrc + static_cast<size_t>(s.tok[tb][j]) * d + 256 * k + 16 * piece
                                  : a.hq + (static_cast<size_t>(item.y + j) * a.S + 8 * k) * 32 + 16 * piece;
          cp_async16(s.B[ab] + umma_off(j + half * npad, 16 * piece, 256), src);
        }
        // scales of the chunk's blocks
        if (MODE == kGateUp) {
          unsigned blk, hrow;
          gu_row(m, item.w, blk, hrow);
          if (SH) {
            // the shared expert's Q8_0 row (transcoded: [d/32 fp16 scales][d
            // int8]): chunk k's eight scales and its 256 values, in natural
            // order, straight into the operand tile
            if (blk < a.S) {
              const uint8_t* row = a.base[blk] + 512ull * a.slice_bytes + static_cast<size_t>(hrow) * a.shared_row;
              cp_async16(s.sc[sq].hg[m], row + 16 * k);
              const uint8_t* qs = row + 2 * (d / 32) + 256 * k;
#pragma unroll
              for (unsigned i = 0; i < 16; ++i) cp_async16(s.A[ab] + umma_off(m, 16 * i, 256), qs + 16 * i);
            }
          } else if (!Q4 && blk < a.S) {  // (Q4_K row scales come with the payload)
            const uint8_t* row = a.base[blk] + item.x * a.slice_bytes + static_cast<size_t>(hrow) * a.row_bytes;
            cp_async8(s.sc[sq].row + 8 * m, row + 8 * k);  // gate/up: [row][8 blocks]
          }
          for (unsigned i = tid; i < item.z * 4; i += 128) {
            const unsigned j = i >> 2, g = i & 3;  // x group g of the chunk (blocks 2g, 2g + 1)
            cp_async8(&s.sc[sq].me[g][j], a.xme + static_cast<size_t>(s.tok[tb][j]) * (d / 64) + 4 * k + g);
          }
          if (Q4 && !SH)
            for (unsigned i = tid; i < item.z * 8; i += 128) {
              const unsigned j = i >> 3, b = i & 7;  // block b of the chunk
              cp_async8(&s.sc[sq].vr[b][j], a.xvr + static_cast<size_t>(s.tok[tb][j]) * (d / 32) + 8 * k + b);
            }
        } else if (SH) {
          // the shared expert's Q8_0 down rows 128 w + m of each loaded slice
          // (transcoded: [d fp16 scales][d x 32 int8]): 32 values into the
          // operand tile, and the 128 rows' scales
          for (unsigned b = 0; b < steps; ++b) {
            const uint8_t* down = a.base[8 * k + b] + 512ull * a.slice_bytes + 2ull * a.shared_proj;
            const uint8_t* qs = down + 2 * d + 32 * (static_cast<size_t>(item.w) * 128 + m);
            cp_async16(s.A[ab] + umma_off(m, 32 * b, 256), qs);
            cp_async16(s.A[ab] + umma_off(m, 32 * b + 16, 256), qs + 16);
          }
          for (unsigned i = tid; i < steps * 16; i += 128) {
            const unsigned b = i >> 4, piece = i & 15;
            const uint8_t* down = a.base[8 * k + b] + 512ull * a.slice_bytes + 2ull * a.shared_proj;
            cp_async16(&s.sc[sq].hd[b][8 * piece], down + 2 * (item.w * 128 + 8 * piece));
          }
          for (unsigned i = tid; i < item.z * steps; i += 128) {
            const unsigned j = i / steps, b = i % steps;
            cp_async4(&s.sc[sq].col[b][j], a.hs + static_cast<size_t>(item.y + j) * a.S + 8 * k + b);
          }
        } else {
          for (unsigned i = tid; i < steps * 8; i += 128) {
            const unsigned b = i >> 3, piece = i & 7;
            const uint8_t* down = a.base[8 * k + b] + item.x * a.slice_bytes + 64ull * a.row_bytes;
            cp_async16(s.sc[sq].row + 128 * b + 16 * piece, down + item.w * 128 + 16 * piece);
          }
          for (unsigned i = tid; i < item.z * steps; i += 128) {
            const unsigned j = i / steps, b = i % steps;
            cp_async4(&s.sc[sq].col[b][j], a.hs + static_cast<size_t>(item.y + j) * a.S + 8 * k + b);
          }
        }
      }
      cp_async_commit();  // one group per chunk, empty after a failed wait
      PF_PH(clk.lap(3);)
      ++ic;
      if (++ik == nk) {
        ik = 0;
        ++iitem;
        iit += gridDim.x;
        if (iit < nitems) inext = items[iit];
      }
      return true;
    };
    issue();
    unsigned c = 0;
    for (unsigned it = blockIdx.x; it < nitems; it += gridDim.x) {
      const uint4 item = items[it];
      unsigned blk = 0, hrow = 0;
      if (MODE == kGateUp) gu_row(m, item.w, blk, hrow);
      const bool row_live = MODE != kGateUp || blk < a.S;
      for (unsigned k = 0; k < nk; ++k, ++c) {
        const unsigned st = c % kPfRaw, ab = c % kPfAB, steps = pf_steps<MODE>(a, k);
        const bool more = issue();  // chunk c + 1
        // A: raw payload -> int8
        const bool landed = pf_wait(&s.raw_full[st], (c / kPfRaw) & 1, abort);
        PF_PH(clk.lap(0);)
        uint8_t* A = s.A[ab];
        if (SH) {
          // shared expert: the operand tile arrives by cp.async
        } else if (landed && MODE == kGateUp && Q4) {
          if (row_live) {
            PfScales& scw = s.sc[c % kPfSc];
            q4k_row_to_i8(s.raw[st] + 144 * (64 * (m >> 6) + hrow), A, m, scw.q4.sm[m], scw.q4.dd[m]);
          }
        } else if (landed && MODE == kGateUp) {
          if (row_live) {
            const unsigned R = 64 * (m >> 6) + hrow;  // row of the staged boxes
#pragma unroll
            for (unsigned b = 0; b < 8; ++b) {
              uint4 lo, hi;
              // 128-byte swizzle: 16-byte chunk b of row R sits at chunk b ^ (R % 8)
              mxfp4_to_i8(*reinterpret_cast<const uint4*>(s.raw[st] + 128 * R + 16 * (b ^ (R & 7))), lo, hi);
              *reinterpret_cast<uint4*>(A + umma_off(m, 32 * b, 256)) = lo;
              *reinterpret_cast<uint4*>(A + umma_off(m, 32 * b + 16, 256)) = hi;
            }
          }
        } else if (landed) {
          for (unsigned b = 0; b < steps; ++b) {
            uint4 lo, hi;
            mxfp4_to_i8(*reinterpret_cast<const uint4*>(s.raw[st] + 2048 * b + 16 * m), lo, hi);
            *reinterpret_cast<uint4*>(A + umma_off(m, 32 * b, 256)) = lo;
            *reinterpret_cast<uint4*>(A + umma_off(m, 32 * b + 16, 256)) = hi;
          }
        }
        mbar_arrive(&s.raw_empty[st]);
        PF_PH(clk.lap(1);)
        if (more) cp_async_wait_group1(); else cp_async_wait_all();  // chunk c's copies
        fence_proxy_async();
        mbar_arrive(&s.ab_full[ab]);
        mbar_arrive(&s.sc_full[c % kPfSc]);
      }
    }
    cp_async_wait_all();  // no copy may land after the CTA exits
    PF_PH(clk.lap(4); clk.store(a.phases, 0, MODE == kGateUp && tid == 0);)
  } else {
    // ------------------------------------------------ epilogue (warps 4-11)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 144;" ::: "memory");
    // Two warpgroups split the tile's token columns: down, warps 4-7 take
    // columns 0-31 and warps 8-11 columns 32-63; gate/up, the columns go in
    // units of four, alternately (warpgroup wg: units 2q + wg, columns
    // 8q + 4wg .. +3, accumulators 4q .. 4q + 3), so that both work on the
    // small tiles.  Warp w reads TMEM lanes 32 (w % 4) .. +31 (A rows).
    const unsigned wg = (warp - 4) >> 2, ew = warp & 3, m = 32 * ew + lane, col0 = 32 * wg;
    const uint32_t lane_base = tmem + ((32 * ew) << 16);
    unsigned c = 0, r = 0;
    bool bad = false;
    // No abort test in these loops: the warps of a warpgroup must take the
    // same number of epi_sync barriers; after an abort every wait fails at once.
    for (unsigned it = blockIdx.x; it < nitems; it += gridDim.x) {
      const uint4 item = items[it];
      const unsigned ntok = item.z, npad = (ntok + 15) & ~15u;
      constexpr bool shi = SH;  // the shared expert (Q8_0 rows)
      // gate/up: the units of columns 8q + 4wq .. +3 go to this warpgroup,
      // wq alternating with the CTA's items (one-unit tiles to both); its
      // live units are q < nq (8q + 4wq < ntok)
      const unsigned wq = wg ^ (((it - blockIdx.x) / gridDim.x) & 1u);
      const unsigned nq = ntok > 4 * wq ? (ntok - 4 * wq + 7) / 8 : 0u;
      float acc[32];
      double accd[32];  // gate/up: the exact block terms' double sums
#pragma unroll
      for (unsigned j = 0; j < 32; ++j) {
        acc[j] = 0.0f;
        accd[j] = 0.0;
      }
      bool live = true;
      if (MODE == kGateUp) {
        unsigned blk, hrow;
        gu_row(m, item.w, blk, hrow);
        live = blk < a.S;
      }
      for (unsigned k = 0; k < nk; ++k, ++c) {
        const unsigned sq = c % kPfSc, steps = pf_steps<MODE>(a, k);
        const PfScales& sc = s.sc[sq];
        // the converters' scales of this chunk (the stage cannot move on
        // before this warp releases sc_empty below)
        PF_PH(clk.lap(2);)
        pf_wait_warp(&s.sc_full[sq], (c / kPfSc) & 1, abort);
        PF_PH(clk.lap(0);)
        if (MODE == kGateUp) {
          // exact block terms (the reference's sum of w * fl32(v * s)), gu_terms
          const unsigned GS = pf_gs<MODE>(npad), BW = pf_bw<MODE>(npad);
          float2 dd = make_float2(0.0f, 0.0f);
          if (Q4 && !shi) {  // the super-block's d and dmin of this row: finite, or NUMERIC
            dd = sc.q4.dd[m];
            bad |= live && !(isfinite(dd.x) && isfinite(dd.y));
          }
          for (unsigned g0 = 0; g0 < steps; g0 += GS, ++r) {
            const unsigned grp = r & 1, n = min(GS, steps - g0);
            PF_PH(clk.lap(2);)
            if (!pf_wait_warp(&s.acc_full[grp], (r >> 1) & 1, abort)) continue;
            PF_PH(clk.lap(1);)
            tc_fence_after();
            const uint32_t tg = lane_base + 256 * grp + 4 * wq;
            if (shi) {
              if (nq) gu_terms_q8(accd, sc, tg, BW, npad, wq, m, g0, n, nq, live, bad);
            } else if (Q4) {
              if (nq) gu_terms_q4k(accd, sc, tg, BW, npad, wq, m, g0, n, nq, dd);
            } else if (nq) {
              gu_terms(accd, sc, tg, BW, npad, wq, m, g0, n, nq, live, bad);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.acc_empty[grp]);
          }
        } else {
          for (unsigned g0 = 0; g0 < steps; g0 += 4, ++r) {
            const unsigned grp = r & 1, n = min(4u, steps - g0);
            if (!pf_wait_warp(&s.acc_full[grp], (r >> 1) & 1, abort)) continue;
            tc_fence_after();
            const uint32_t tg = lane_base + 4 * grp * kPfTile + col0;
            // one register buffer of four 16-column reads: with at most 16 live
            // columns here the group's steps are read at once, with 32 two
            // steps at a time
            uint32_t v[4][16];
            if (col0 + 16 < ntok) {  // 32 live columns: two steps at a time
  #pragma unroll
              for (unsigned jb = 0; jb < 4; jb += 2) {
                if (jb < n) {
  #pragma unroll
                  for (unsigned i = 0; i < 4; ++i)
                    if (jb + (i >> 1) < n) tmem_ld16(tg + (jb + (i >> 1)) * kPfTile + 16 * (i & 1), v[i]);
                  tmem_wait_ld();
  #pragma unroll
                  for (unsigned i = 0; i < 4; ++i)
                    if (jb + (i >> 1) < n)
                      pf_apply16<MODE>(sc, g0 + jb + (i >> 1), m, col0 + 16 * (i & 1), v[i], acc + 16 * (i & 1), live,
                                       bad, shi);
                }
              }
            } else if (col0 < ntok) {  // at most 16 live columns: the group's steps at once
  #pragma unroll
              for (unsigned i = 0; i < 4; ++i)
                if (i < n) tmem_ld16(tg + i * kPfTile, v[i]);
              tmem_wait_ld();
  #pragma unroll
              for (unsigned i = 0; i < 4; ++i)
                if (i < n) pf_apply16<MODE>(sc, g0 + i, m, col0, v[i], acc, live, bad, shi);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.acc_empty[grp]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.sc_empty[sq]);
      }
      PF_PH(clk.lap(2);)
      const bool ok = !*abort;
      if (MODE == kGateUp) {
        // narrowed to fp32 as the reference narrows its double sums
        // (backends/ref.c:37-40): a nonfinite or overflowing sum is NUMERIC
#pragma unroll
        for (unsigned j = 0; j < 32; ++j) {
          if (j / 4 >= nq) continue;
          const bool fits = fabs(accd[j]) <= 3.4028234663852886e38;
          bad |= !fits && live && 8 * (j / 4) + 4 * wq + j % 4 < ntok;
          acc[j] = __double2float_rn(fits ? accd[j] : 0.0);
        }
      }
      if (MODE == kDown) {
        if (!ok) continue;
        float* out = a.ye + (static_cast<size_t>(item.y) + col0) * d + 128 * item.w + m;
#pragma unroll
        for (unsigned g = 0; g < 2; ++g)
          if (col0 + 16 * g < ntok) {
#pragma unroll
            for (unsigned jj = 0; jj < 16; ++jj)
              if (col0 + 16 * g + jj < ntok) out[static_cast<size_t>(16 * g + jj) * d] = acc[16 * g + jj];
          }
      } else {
        // SwiGLU: lane l < 16 holds gate row n, lane l + 16 up row n.  Pair i
        // (accumulators 2i, 2i + 1, unit i / 2) is two adjacent tokens: lane
        // l takes the even one, lane l + 16 the odd one,
        // token(i) = 8 (i / 2) + 4 wq + 2 (i % 2) + odd; pairs whose even
        // token is past the tile are skipped (warp-uniform).
        const bool up = lane >= 16;
        const unsigned odd = up ? 1u : 0u;
        auto token = [&](unsigned i) { return 8 * (i / 2) + 4 * wq + 2 * (i % 2) + odd; };
        auto live_pair = [&](unsigned i) { return i / 2 < nq && 8 * (i / 2) + 4 * wq + 2 * (i % 2) < ntok; };
        float h[16];
#pragma unroll
        for (unsigned i = 0; i < 16; ++i) {
          if (!live_pair(i)) continue;
          const float other = __shfl_xor_sync(0xffffffffu, up ? acc[2 * i] : acc[2 * i + 1], 16);
          const float gv = up ? other : acc[2 * i], uv = up ? acc[2 * i + 1] : other;
          bool fail = false;
          h[i] = swiglu_nb(gv, uv, fail);
          bad |= fail && live && token(i) < ntok;
        }
        // amax per token over the block's 32 neurons (16 here, 16 in the partner warp)
#pragma unroll
        for (unsigned i = 0; i < 16; ++i) {
          if (!live_pair(i)) continue;
          float am = fabsf(h[i]);
#pragma unroll
          for (unsigned o = 8; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
          if ((lane & 15) == 0) s.amax[ew][token(i)] = am;
        }
        epi_sync(wg);
        const unsigned blk = 2 * item.w + (ew >> 1), n = 16 * (ew & 1) + (lane & 15);
        if (live && ok) {
          // prmt order for the routed experts' MXFP4 down rows, natural order
          // for the shared expert's Q8_0 ones
          int8_t* hq = a.hq + static_cast<size_t>(item.y) * a.S * 32 + blk * 32 + (shi ? n : prmt_pos(n));
#pragma unroll
          for (unsigned i0 = 0; i0 < 16; i0 += 8) {
            if (!live_pair(i0)) continue;
            // the group's two divisions once per token: lane (lane & 16) + i'
            // of each half computes them for its half's pair i = i0 + i'
            const unsigned tl = token(i0 + (lane & 7));
            const float am_l = fmaxf(s.amax[ew][tl], s.amax[ew ^ 1][tl]);
            const float sc_l = __fdiv_rn(am_l, 127.0f);
            const float inv_l = sc_l != 0.0f ? __fdiv_rn(127.0f, am_l) : 0.0f;
#pragma unroll
            for (unsigned i = i0; i < i0 + 8; ++i) {
              if (!live_pair(i)) continue;
              const unsigned src = (lane & 16) | (i - i0), t = token(i);
              const float am = __shfl_sync(0xffffffffu, am_l, src), sc = __shfl_sync(0xffffffffu, sc_l, src);
              const float inv = __shfl_sync(0xffffffffu, inv_l, src);
              if (t < ntok) {
                hq[static_cast<size_t>(t) * a.S * 32] = static_cast<int8_t>(q8_fast(h[i], am, sc, inv));
                if ((ew & 1) == 0 && (lane & 15) == 0) a.hs[static_cast<size_t>(item.y + t) * a.S + blk] = sc;
              }
            }
          }
        }
        epi_sync(wg);
      }
      PF_PH(clk.lap(3);)
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
    PF_PH(clk.store(a.phases, 16 + 8 * wg, MODE == kGateUp && lane == 0 && ew == 0);)
  }
  if (tid == 0 && *abort) atomicOr(a.status, kStTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 13) tmem_dealloc(tmem, kPfCols);
  PF_PH(if (MODE == kGateUp && tid == 0 && a.phases) a.phases[blockIdx.x * 64 + 40] = pf_now() - t_entry;)
}

// ---------------------------------------------------------- 5. combine

// y[t][r] = fmaf over the token's ten experts in request order of
// gate * partial; one thread per (t, r).
__global__ void prefill_combine_kernel(PrefillArgs a) {
  const unsigned t = blockIdx.y, r = 4 * (blockIdx.x * blockDim.x + threadIdx.x);  // four rows a thread
  if (r >= a.d) return;
  const unsigned P = a.counts[0];
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  // the ten routed experts in request order, then the shared expert
#pragma unroll
  for (unsigned j = 0; j < 11; ++j) {
    const unsigned p = a.slot_pair[t * 11 + j];
    if (j == 10 && p == 0xffffffffu) break;  // no shared expert for this token
    if (p >= P) {  // an id the group kernel rejected (status already set)
      acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      break;
    }
    const float g = a.gate[t * 11 + j];
    const float4 v = *reinterpret_cast<const float4*>(a.ye + static_cast<size_t>(p) * a.d + r);
    acc.x = __fmaf_rn(g, v.x, acc.x);
    acc.y = __fmaf_rn(g, v.y, acc.y);
    acc.z = __fmaf_rn(g, v.z, acc.z);
    acc.w = __fmaf_rn(g, v.w, acc.w);
  }
  if (!isfinite(acc.x) || !isfinite(acc.y) || !isfinite(acc.z) || !isfinite(acc.w)) atomicOr(a.status, kStNumeric);
  *reinterpret_cast<float4*>(a.y + static_cast<size_t>(t) * a.d + r) = acc;
}

}  // namespace frc
