// frc_avx2.cuh - FRC_ACT_AVX2: the arithmetic of the reference's AVX2 backend
// (backends/avx2.c, default build) on the GPU, so that a caller switching
// from fr_avx2 gets its results: bit for bit at the same worker count but
// for the C library's rare last-bit expf roundings (the SiLU here rounds
// exp in double once to fp32).
//
//   x        int8 per 256 with one fp32 scale (amax / 127) and int16 sums of
//            each 32 (quantize8, backends/avx2.c:184-203)
//   gate/up  Q4_K routed rows as q4k_pair (:262-319): eight int32 lanes per
//            super-block (lane k: bytes 4k..4k+3 of each 32-byte nibble run,
//            times the 6-bit group scale), fmadd into eight fp32 lanes with
//            d * xd; the min terms in four int32 lanes (mins of groups 2j,
//            2j+1 against the activation sums), fmadd with dmin * xd; lanes
//            added as its horizontal adds do.  Q8_0 shared rows as row4
//            (:239-247): per 32-block eight lanes of four products, fmadd
//            with d * xd.
//   hidden   v / (1 + exp(-v)) * u in fp32, int8 per 32 (:427-437)
//   down     MXFP4 routed rows as down8_mxfp4 (:331-362), Q8_0 shared rows
//            as down8 (:364-392): exact integer row sums times the row scale;
//            each job's terms and md * gate are kept apart
//   sum      jobs (block, expert) block-major, experts in first-named order,
//            dealt round robin to W workers; each worker's fmadd chain over
//            its jobs from zero, the workers' sums added in order (:506-529,
//            :703-708)
//
// Three launches: the activation quantization (one CTA a token), one CTA a
// job (256 threads = 32 neurons x 8 lanes, the lanes of the AVX2 registers),
// and the reduction (one thread an output value).  The job's weight rows are
// the device layout of the context: Q4_K rows in the reference's bytes,
// MXFP4 and Q8_0 runs as [scales][payloads].
#pragma once
#include "frc_device.cuh"

constexpr unsigned kAvx2MaxWorkers = 32;

struct Avx2Params {
  const uint8_t* base[kMaxBlocks];  // the layer region of each loaded block, in job order
  const float* x;                   // [T][d]
  const uint32_t* mask;             // [E] tokens of each expert
  const float* pgate;               // [P] gate of each (expert, token) pair, expert-major, tokens ascending
  const uint16_t* ids;              // [E] expert ids (512: the shared expert)
  const uint16_t* pbase;            // [E] first pair of each expert
  int8_t* xq;                       // [T][d]
  float* xd;                        // [T][d / 256]
  int16_t* xs;                      // [T][d / 32]
  float* terms;                     // [S][P][d] down terms of each job and token
  float* coef;                      // [S][P] md * gate
  float* y;                         // [T][d]
  const uint16_t* chain;            // [T][chain_stride] per token: its term slots (s * P + pair) in job order, worker by worker
  const uint16_t* bounds;           // [T][kAvx2MaxWorkers + 1] where each worker's part of the chain starts
  unsigned* status;
  unsigned d, T, S, E, P, W, chain_stride;
  unsigned row_bytes, proj_bytes, slice_bytes, shared_row, shared_proj;
};

__device__ __forceinline__ uint32_t av_ld32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ float av_half(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// Four MXFP4 nibbles (low 4 bits of each byte) to the int8 values 2 * E2M1.
__device__ __forceinline__ uint32_t av_e2m1x2(uint32_t nib) {
  const uint32_t sel = (nib & 7u) | ((nib >> 4) & 0x70u) | ((nib >> 8) & 0x700u) | ((nib >> 12) & 0x7000u);
  const uint32_t pos = __byte_perm(0x03020100u, 0x0C080604u, sel);  // 0 1 2 3 4 6 8 12
  const uint32_t neg = __byte_perm(0xFDFEFF00u, 0xF4F8FAFCu, sel);  // 0 -1 -2 -3 -4 -6 -8 -12
  const uint32_t m = ((nib >> 3) & 0x01010101u) * 0xFFu;
  return (pos & ~m) | (neg & m);
}

// x per 256: one warp a group, eight values a lane.
__global__ void __launch_bounds__(256) avx2_quantize_kernel(Avx2Params a) {
  const unsigned t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, d = a.d;
  const float* x = a.x + static_cast<size_t>(t) * d;
  for (unsigned g = warp; g < d / 256; g += 8) {
    const unsigned o = g * 256 + lane * 8;
    const float4 v0 = *reinterpret_cast<const float4*>(x + o), v1 = *reinterpret_cast<const float4*>(x + o + 4);
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float m = 0.f;
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
    for (unsigned off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) a.xd[t * (d / 256) + g] = __fdiv_rn(m, 127.f);
    const float inv = m != 0.f ? __fdiv_rn(127.f, m) : 0.f;
    int sum = 0;
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) {
      int q = __float2int_rn(__fmul_rn(v[i], inv));
      sum += q;
      q = min(127, max(-128, q));
      w[i / 4] |= (static_cast<uint32_t>(q) & 0xffu) << (8 * (i % 4));
    }
    *reinterpret_cast<uint2*>(a.xq + static_cast<size_t>(t) * d + o) = make_uint2(w[0], w[1]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) a.xs[t * (d / 32) + (o >> 5)] = static_cast<int16_t>(sum);
  }
}

// native_sum of the eight lanes held by lanes k = 0..7 of a group of eight
// threads; valid in lane 0 of the group.
__device__ __forceinline__ float av_hsum8(float v) {
  const float a = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
  const float b = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 1, 8));
  return __fadd_rn(b, __shfl_down_sync(0xffffffffu, b, 2, 8));
}

constexpr unsigned kAvx2StageMax = 220u * 1024u;  // routed slices up to this size are staged in shared memory
constexpr unsigned kAvx2Chunk = 32768u;           // bytes a bulk copy of the staging moves

// One job: 32 neurons of expert ids[j] in block slot s, for every token of
// the expert.  Thread = neuron (tid / 8) x lane (tid % 8).  STAGE: a routed
// job first brings its whole slice (gate rows, up rows, down rows: one
// contiguous run of slice_bytes, dynamic shared memory of that size) into
// shared memory with bulk copies on one mbarrier, then reads only shared
// memory; the shared expert's slice, which is larger, is read from global
// memory.  The wait for the copies is bounded: on a timeout the CTA records
// it, waits once more (bounded) for its own copies, and returns.
template <bool STAGE>
__global__ void __launch_bounds__(256) avx2_job_kernel(Avx2Params a) {
  extern __shared__ __align__(128) uint8_t av_slice[];
  __shared__ float sh_h[32];
  __shared__ __align__(16) int8_t sh_mid[32];
  __shared__ uint64_t av_bar;
  __shared__ int av_ok;
  const unsigned tid = threadIdx.x, n = tid >> 3, k = tid & 7, lane = tid & 31;
  const unsigned s = blockIdx.x / a.E, j = blockIdx.x % a.E, d = a.d, id = a.ids[j];
  const bool shared = id >= FRC_ROUTED_EXPERTS;
  const uint8_t* p = a.base[s] + static_cast<size_t>(id) * a.slice_bytes;
  if (STAGE && !shared) {
    if (tid == 0) {
      mbar_init(&av_bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      mbar_expect_tx(&av_bar, a.slice_bytes);
      for (unsigned o = 0; o < a.slice_bytes; o += kAvx2Chunk)
        bulk_g2s(av_slice + o, p + o, min(kAvx2Chunk, a.slice_bytes - o), &av_bar);
      const bool ok = mbar_wait(&av_bar, 0);
      if (!ok) {
        atomicOr(a.status, kStTimeout);
        mbar_wait(&av_bar, 0);  // its own copies end before the CTA does
      }
      av_ok = ok;
    }
    __syncthreads();
    if (!av_ok) return;
    p = av_slice;
  }
  const unsigned in_row = shared ? a.shared_row : a.row_bytes, proj = shared ? a.shared_proj : a.proj_bytes;
  const uint8_t* grow = p + static_cast<size_t>(n) * in_row;
  const uint8_t* urow = grow + proj;
  const uint8_t* down = p + 2 * static_cast<size_t>(proj);
  const uint32_t mask = a.mask[j];
  unsigned pair = a.pbase[j];
  for (unsigned t = 0; t < a.T; ++t) {
    if (!(mask >> t & 1u)) continue;
    const int8_t* xq = a.xq + static_cast<size_t>(t) * d;
    const float* xd = a.xd + t * (d / 256);
    float og, ou;
    if (!shared) {
      const int16_t* xs = a.xs + t * (d / 32);
      float accg = 0.f, accu = 0.f, mins = 0.f;
#pragma unroll 4
      for (unsigned sb = 0; sb < d / 256; ++sb) {
        const uint8_t* gb = grow + sb * 144;
        const uint8_t* ub = urow + sb * 144;
        const uint32_t gh = av_ld32(gb), uh = av_ld32(ub);
        const uint32_t g0 = av_ld32(gb + 4), g1 = av_ld32(gb + 8), g2 = av_ld32(gb + 12);
        const uint32_t u0 = av_ld32(ub + 4), u1 = av_ld32(ub + 8), u2 = av_ld32(ub + 12);
        // 6-bit scales of groups 0-3 / 4-7 and mins of groups 0-3 / 4-7, one byte each
        const uint32_t gs[2] = {g0 & 0x3f3f3f3fu, (g2 & 0x0f0f0f0fu) | (((g0 >> 6) & 0x03030303u) << 4)};
        const uint32_t us[2] = {u0 & 0x3f3f3f3fu, (u2 & 0x0f0f0f0fu) | (((u0 >> 6) & 0x03030303u) << 4)};
        const uint32_t gm[2] = {g1 & 0x3f3f3f3fu, ((g2 >> 4) & 0x0f0f0f0fu) | (((g1 >> 6) & 0x03030303u) << 4)};
        const uint32_t um[2] = {u1 & 0x3f3f3f3fu, ((u2 >> 4) & 0x0f0f0f0fu) | (((u1 >> 6) & 0x03030303u) << 4)};
        int isg = 0, isu = 0;
#pragma unroll
        for (unsigned gp = 0; gp < 4; ++gp) {
          const uint32_t gq = av_ld32(gb + 16 + gp * 32 + 4 * k), uq = av_ld32(ub + 16 + gp * 32 + 4 * k);
          const int xl = static_cast<int>(av_ld32(xq + sb * 256 + gp * 64 + 4 * k));
          const int xh = static_cast<int>(av_ld32(xq + sb * 256 + gp * 64 + 32 + 4 * k));
          const unsigned sh = 16 * (gp & 1);
          const int gsl = (gs[gp >> 1] >> sh) & 0xff, gsh = (gs[gp >> 1] >> (sh + 8)) & 0xff;
          const int usl = (us[gp >> 1] >> sh) & 0xff, ush = (us[gp >> 1] >> (sh + 8)) & 0xff;
          isg += gsl * __dp4a(static_cast<int>(gq & 0x0f0f0f0fu), xl, 0) +
                 gsh * __dp4a(static_cast<int>((gq >> 4) & 0x0f0f0f0fu), xh, 0);
          isu += usl * __dp4a(static_cast<int>(uq & 0x0f0f0f0fu), xl, 0) +
                 ush * __dp4a(static_cast<int>((uq >> 4) & 0x0f0f0f0fu), xh, 0);
        }
        const float xds = xd[sb];
        accg = __fmaf_rn(__int2float_rn(isg), __fmul_rn(av_half(gh), xds), accg);
        accu = __fmaf_rn(__int2float_rn(isu), __fmul_rn(av_half(uh), xds), accu);
        // lanes 0-3: the gate row's min lanes, lanes 4-7: the up row's
        const unsigned mj = k & 3;
        const uint32_t mw = k < 4 ? (mj >> 1 ? gm[1] : gm[0]) : (mj >> 1 ? um[1] : um[0]);
        const unsigned msh = 16 * (mj & 1);
        const int mm = static_cast<int>((mw >> msh) & 0xff) * xs[sb * 8 + 2 * mj] +
                       static_cast<int>((mw >> (msh + 8)) & 0xff) * xs[sb * 8 + 2 * mj + 1];
        mins = __fmaf_rn(__int2float_rn(mm), __fmul_rn(av_half((k < 4 ? gh : uh) >> 16), xds), mins);
      }
      const float tg = av_hsum8(accg), tu = av_hsum8(accu);
      const float mb = __fadd_rn(mins, __shfl_down_sync(0xffffffffu, mins, 1, 8));
      const float mt = __fadd_rn(mb, __shfl_down_sync(0xffffffffu, mb, 2, 8));
      const float mtu = __shfl_sync(0xffffffffu, mt, (lane & ~7u) + 4);
      og = __fsub_rn(tg, mt);
      ou = __fsub_rn(tu, mtu);
    } else {
      const unsigned nb = d / 32;
      float accg = 0.f, accu = 0.f;
      bool bad = false;
      for (unsigned blk = 0; blk < nb; ++blk) {
        const float sg = __half2float(reinterpret_cast<const __half*>(grow)[blk]);
        const float su = __half2float(reinterpret_cast<const __half*>(urow)[blk]);
        bad |= !isfinite(sg) || !isfinite(su);
        const int xw = static_cast<int>(av_ld32(xq + blk * 32 + 4 * k));
        const int dg = __dp4a(static_cast<int>(av_ld32(grow + 2 * nb + blk * 32 + 4 * k)), xw, 0);
        const int du = __dp4a(static_cast<int>(av_ld32(urow + 2 * nb + blk * 32 + 4 * k)), xw, 0);
        const float xds = xd[blk / 8];
        accg = __fmaf_rn(__int2float_rn(dg), __fmul_rn(sg, xds), accg);
        accu = __fmaf_rn(__int2float_rn(du), __fmul_rn(su, xds), accu);
      }
      if (bad && k == 0) atomicOr(a.status, kStNumeric);
      og = av_hsum8(accg);
      ou = av_hsum8(accu);
    }
    if (k == 0) {
      const float e = __double2float_rn(exp(-static_cast<double>(og)));
      const float h = __fmul_rn(__fdiv_rn(og, __fadd_rn(1.f, e)), ou);
      if (!isfinite(h)) atomicOr(a.status, kStNumeric);
      sh_h[n] = h;
    }
    __syncthreads();
    if (tid < 32) {
      const float h = sh_h[tid];
      float m = fabsf(h);
#pragma unroll
      for (unsigned off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float inv = m != 0.f ? __fdiv_rn(127.f, m) : 0.f;
      sh_mid[tid] = static_cast<int8_t>(min(127, max(-128, __float2int_rn(__fmul_rn(h, inv)))));
      if (tid == 0) {
        a.coef[s * a.P + pair] = __fmul_rn(__fdiv_rn(m, 127.f), a.pgate[pair]);
      }
    }
    __syncthreads();
    const uint4 ma = *reinterpret_cast<const uint4*>(sh_mid), mb = *reinterpret_cast<const uint4*>(sh_mid + 16);
    const int mid[8] = {static_cast<int>(ma.x), static_cast<int>(ma.y), static_cast<int>(ma.z), static_cast<int>(ma.w),
                        static_cast<int>(mb.x), static_cast<int>(mb.y), static_cast<int>(mb.z), static_cast<int>(mb.w)};
    float* out = a.terms + (static_cast<size_t>(s) * a.P + pair) * d;
    if (!shared) {
      for (unsigned r = tid; r < d; r += 256) {
        const uint32_t e8 = down[r];
        const uint4 q = *reinterpret_cast<const uint4*>(down + d + 16 * static_cast<size_t>(r));
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        int sum = 0;
#pragma unroll
        for (unsigned w = 0; w < 4; ++w) {
          sum = __dp4a(static_cast<int>(av_e2m1x2(qw[w] & 0x0f0f0f0fu)), mid[w], sum);
          sum = __dp4a(static_cast<int>(av_e2m1x2((qw[w] >> 4) & 0x0f0f0f0fu)), mid[4 + w], sum);
        }
        const float rs = __fmul_rn(__uint_as_float(e8 ? e8 << 23 : 0x00400000u), 0.5f);
        out[r] = __fmul_rn(__int2float_rn(sum), rs);
      }
    } else {
      bool bad = false;
      for (unsigned r = tid; r < d; r += 256) {
        const float sc = __half2float(reinterpret_cast<const __half*>(down)[r]);
        bad |= !isfinite(sc);
        const uint4* q = reinterpret_cast<const uint4*>(down + 2 * static_cast<size_t>(d) + 32 * static_cast<size_t>(r));
        const uint4 q0 = q[0], q1 = q[1];
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        int sum = 0;
#pragma unroll
        for (unsigned w = 0; w < 8; ++w) sum = __dp4a(static_cast<int>(qw[w]), mid[w], sum);
        out[r] = __fmul_rn(__int2float_rn(sum), sc);
      }
      if (bad) atomicOr(a.status, kStNumeric);
    }
    ++pair;
    __syncthreads();  // sh_h / sh_mid are rewritten for the next token
  }
}

// y[t][r]: the workers' fmadd chains over their jobs, added in worker order.
// The chains come from the plan (each token's term slots in job order,
// worker by worker).  A CTA covers 64 values of one token (d is a multiple
// of 64): it first stages the token's slots and their md * gate factors in
// shared memory, then each thread issues its term loads 32 at a time and
// applies the fmadds in order.
__global__ void __launch_bounds__(64) avx2_reduce_kernel(Avx2Params a) {
  constexpr unsigned kBatch = 32, kMaxChain = kMaxBlocks * FRC_ACTIVE;
  __shared__ uint16_t sq[kMaxChain];
  __shared__ float sc[kMaxChain];
  __shared__ uint16_t sb[kAvx2MaxWorkers + 1];
  const unsigned i = blockIdx.x * 64 + threadIdx.x;  // every CTA lies within one token
  const unsigned t = blockIdx.x * 64 / a.d, r = i % a.d;
  const uint16_t* bound = a.bounds + t * (kAvx2MaxWorkers + 1);
  const unsigned n = bound[a.W];
  for (unsigned e = threadIdx.x; e < n; e += 64) {
    const unsigned q = a.chain[t * a.chain_stride + e];
    sq[e] = static_cast<uint16_t>(q);
    sc[e] = a.coef[q];
  }
  for (unsigned w = threadIdx.x; w <= a.W; w += 64) sb[w] = bound[w];
  __syncthreads();
  float value = 0.f;
  for (unsigned w = 0; w < a.W; ++w) {
    float o = 0.f;
    unsigned e = sb[w];
    const unsigned end = sb[w + 1];
    for (; e + kBatch <= end; e += kBatch) {
      float tv[kBatch];
#pragma unroll
      for (unsigned k = 0; k < kBatch; ++k) tv[k] = a.terms[static_cast<size_t>(sq[e + k]) * a.d + r];
#pragma unroll
      for (unsigned k = 0; k < kBatch; ++k) o = __fmaf_rn(tv[k], sc[e + k], o);
    }
    for (; e < end; ++e) o = __fmaf_rn(a.terms[static_cast<size_t>(sq[e]) * a.d + r], sc[e], o);
    value = __fadd_rn(value, o);
  }
  if (!isfinite(value)) atomicOr(a.status, kStNumeric);
  a.y[i] = value;
}
