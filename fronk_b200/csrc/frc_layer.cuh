// frc_layer.cuh - the MoE layer kernel (sm_100a): one cooperative launch per
// layer of 256-thread CTAs, two per SM when their shared memory fits (one
// otherwise), item-major work.
//
// An item is (unique expert u, loaded slice s): 32 neurons, their gate and up
// rows and their columns of the down projection, all in one region of the
// slice (src/q4.c layout, transcoded to device form at load).  Items are
// dealt to CTAs in snake order, the shared expert's items (twice the bytes)
// first, so each CTA streams whole items and keeps the hidden activations on
// chip.
//
//   prologue - routing and x are loaded at once and the plan (unique
//     experts, token masks, (expert, token) pairs) is built by warps 4-7;
//     warp 4 starts the TMA ring (cp.async.bulk, one mbarrier a slot) on the
//     CTA's first chunks; warps 0-3 form the layer input and quantize it
//     meanwhile.
//   items - per item: gate/up chunks (a warp per four neurons, eight lanes a
//     neuron, which also form its SwiGLU in double), the Q8 quantization of
//     the hidden slice (one group of 32) in shared memory, then the down chunk(s), a thread per
//     row: c = scale * int_dot goes to the partial buffer [pair][slice][row].  The last warp to finish with a
//     ring slot refills it, so loads stream with no producer warp.
//   grid barrier (bounded wait).
//   reduce - CTA k owns 4-row units [d/4*k/G, d/4*(k+1)/G) of every token: per (token,
//     row, routing slot) four slice-interleaved fmaf chains of c * gs,
//     combined ((p0+p1)+p2)+p3; then the token's routed experts in its own
//     routing order, then the shared expert.
//
// Arithmetic order (restated by the oracle's or_port_run): eight lanes a
// gate/up row, lane l taking the 256-element spans l, l+8, ... (groups in
// order); butterfly over the eight; the reduce above.  Results
// are bitwise repeatable and a token's output does not depend on the rest of
// the burst.
#pragma once
#include "frc_device.cuh"

namespace frc {

constexpr unsigned kLayerThreads = 256;        // two CTAs an SM when their shared memory fits
constexpr unsigned kLayerWarps = kLayerThreads / 32;
constexpr unsigned kActThreads = 128;          // warps 0-3 form the layer input
constexpr unsigned kActWarps = kActThreads / 32;
constexpr unsigned kPlanWarps = 4;             // warps 4-7 build the plan
constexpr unsigned kPlanThreads = 32 * kPlanWarps;
constexpr unsigned kFirstPlanWarp = kLayerWarps - kPlanWarps;
constexpr unsigned kMaxSlots = 8;              // TMA ring: barriers and counters reserved
constexpr unsigned kRingSlots = 5;             // TMA ring: slots a launch uses at most
constexpr unsigned kMaxRounds = 256;           // warp-passes of the activation sums per warp (512 floats each)
constexpr unsigned kMaxPeers = 8;              // GPUs of one in-box reduce

struct LayerCtl {
  unsigned long long arrived;   // grid barrier arrivals, all launches (never wraps)
  unsigned abort;               // set by a CTA whose bounded wait ran out
  unsigned pad0;
  // In-box reduce launches completed on this context.  Every CTA of a
  // FRC_RUN_PEER launch reads it once it may read memory (after the
  // programmatic-launch wait) and before it arrives at the grid barrier;
  // CTA 0 stores the launch's epoch (read + 1) once the barrier has released,
  // so one launch carries one epoch whatever its grid size.  A timeout reset
  // keeps it; frc_peer_attach zeroes it on every rank.
  unsigned peer_epoch;
  unsigned pad;
};

// Byte offsets of one CTA's dynamic shared memory, and the chunking of an
// item into ring slots (computed on the host).
struct LayerSmem {
  unsigned ids, gates, first, uid, umask, ugate, upre, rms, bases, rpart, tokpair;
  // activations: v and r in natural order (xq, xr) and prmt order (xp, xrp;
  // MXFP4 gate/up only), {s, 2^E} per 64-group (xst), {V, RS} per 32-block
  // (xvr); fp32 activations (xf, the F32 mode)
  unsigned xq, xr, xp, xrp, xst, xvr, xf, gv, uv, hq, hg, ylocal, ring, total;
  unsigned slot_bytes, slots;
  unsigned kn_r, kn_s;  // neurons per gate/up chunk: routed, shared items (powers of two)
  unsigned dn_r, dn_s;  // rows per down chunk: routed, shared items (multiples of 16)
  unsigned mag_ch_r, mag_ch_s;  // div_magic of the chunks per routed / shared item
  unsigned max_unique;          // entries of the plan's per-expert tables (10 x tokens + 1)
  // row-owner kernel (frc_layer_rb.cuh): down-row staging [item] of dnb_r
  // (routed) / dnb_s (shared) bytes, rows_max rows a CTA at most, dnw
  // 16-byte pieces of scales window an item
  unsigned dnb, dnb_r, dnb_s, rows_max, dnw;
};

struct LayerParams {
  const uint8_t* base[kMaxBlocks];
  const uint16_t* expert;
  const float* gate;
  const float* x;
  const float* x_add;
  float* x_out;
  float* y;
  float* hidden;     // [u*S+s][T][32] fp32 copy of the hidden activations, or null
  float* partial;    // [pair][S][d] down terms c
  float* gsv;        // [pair][S] hidden scale x routing weight
  LayerCtl* ctl;
  unsigned* status;
  unsigned long long* phases;  // FRC_PHASES builds: [cta][16] globaltimer stamps
  // In-box reduce over peer memory (world > 1): every rank's inbox as mapped
  // here (peer[rank] is this rank's own) and this rank.  Inbox:
  // [2][world][16][d] 8-byte entries {value, epoch}; the epoch is
  // ctl->peer_epoch + 1.
  uint8_t* peer[kMaxPeers];
  unsigned rank, world;
  // Grid barrier arrivals a CTA adds: (2 x SMs) / grid, so that every launch
  // adds the same total whatever its grid (one or two CTAs an SM).
  unsigned bar_inc;
  // Every bounded wait of the launch gives up after wait_ns (the context's
  // limit, 2 s unless set).  bar_extra > 0 (tests only) raises the grid
  // barrier's target by that many arrivals, so its wait runs out.
  unsigned bar_extra;
  unsigned long long wait_ns;
  // Items split in H parts (1, 2 or 4; one token, one round of parts): part
  // h takes neurons [32h/H, 32(h+1)/H) of the slice and down rows
  // [dh/H, d(h+1)/H); the parts' hidden values meet in xchg [item][32]
  // (xcnt[item] counts the parts that wrote, reset after the grid barrier).
  unsigned H, Hshift;
  float* xchg;
  unsigned* xcnt;
  // row-owner kernel: per-item arrival counts of the gate/up chunks (zero
  // between launches), and the items' quantized hidden slices
  unsigned* rb_cnt;
  uint8_t* rb_hq;   // [item][32] int8 (prmt order for MXFP4 down rows)
  float* rb_hs;     // [item] hidden scale
  LayerSmem sm;
  unsigned S, T, d, norm;
  unsigned mag_S;  // div_magic(S)
  unsigned gate_type, down_type;
  unsigned row_bytes, proj_bytes, shared_row, shared_proj, slice_bytes;
};

// Programmatic dependent launch: the next launch on the stream may start its
// CTAs (as SMs free up) once every CTA of this one has signalled; a launch
// waits for its predecessor's completion and memory before it reads x or
// writes anything the predecessor reads.  Both are no-ops without the launch
// attribute.
__device__ __forceinline__ void pdl_signal() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Barrier among the activation warps (0-3) only.
__device__ __forceinline__ void act_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Barrier among the plan warps (4-7) only.
__device__ __forceinline__ void plan_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Bounded barrier over the co-resident grid, one round trip: every CTA adds
// `inc` to a counter that only grows and waits for the next multiple of the
// launch's total (grid x inc, the same for every launch, so launches of one
// and of two CTAs an SM may follow each other in any order).  A timed-out
// launch leaves the counter off that lattice; frc_status zeroes it before
// anything runs again.
__device__ __forceinline__ bool grid_sync(LayerCtl* ctl, unsigned* flag_smem, unsigned inc, uint64_t limit,
                                          unsigned extra) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long span = static_cast<unsigned long long>(gridDim.x) * inc;
    const unsigned long long old = atomicAdd(&ctl->arrived, static_cast<unsigned long long>(inc));
    const unsigned long long target = (old / span + 1) * span + extra;
    bool ok = true;
    const uint64_t start = globaltimer();
    unsigned spins = 0;
    while (ld_acquire64(&ctl->arrived) < target) {
      if ((++spins & 255) == 0 && (globaltimer() - start > limit || ld_acquire(&ctl->abort))) {
        ok = false;
        break;
      }
    }
    *flag_smem = ok;
  }
  __syncthreads();
  return *flag_smem != 0;
}

// Compile-time phase stamps (the reference's FR_PHASES counterpart,
// backends/avx2.c:38-42): 0 entry, 8 prologue loads, 10 plan, 1 first copies
// issued, 2 norm sums, 3 activations, 15/12 first/second chunk landed, 9
// first item's gate/up, 13 its hidden slice, 14 its down chunk landed, 6 its
// down done, 4 items done, 5 grid barrier, 11 reduce chains, 7 exit.
#ifdef FRC_PHASES
#define PHASE_AT(k, th) \
  do { if (threadIdx.x == (th) && a.phases) a.phases[blockIdx.x * 16 + (k)] = globaltimer(); } while (0)
#else
#define PHASE_AT(k, th) do { } while (0)
#endif
#define PHASE(k) PHASE_AT(k, 0)

// One lane's gate and up sums over its 256-weight spans q = l8, l8+8, ...
// (Q8 activations, groups in order), in double and exact up to double
// rounding (see the row terms in frc_device.cuh).  Q4_K spans are
// super-blocks: per group p the integer combinations K1 = sc0*I0 + sc1*I1,
// K3 = sc0*R0 + sc1*R1, K2 = mi0*V0 + mi1*V1, K4 = mi0*RS0 + mi1*RS1 give
// the exact integers M*K1 + K3 and M*K2 + K4 (s = M 2^E), which enter
// PP += (M*K1 + K3) 2^E and QQ += (M*K2 + K4) 2^E (one fma each), and the
// span adds d*PP - dmin*QQ.  One instantiation per weight type, so the code a launch
// runs is one contiguous block.
template <unsigned TYPE>
__device__ __forceinline__ void gu_sums(const uint8_t* gr, const uint8_t* ur, const XAct& xa, unsigned l8,
                                        unsigned nspan, unsigned nb, bool& bad, double& ag, double& au) {
  for (unsigned q = l8; q < nspan; q += 8) {
    if (TYPE == kQ4K) {
      const uint8_t* bg = gr + q * 144;
      const uint8_t* bu = ur + q * 144;
      const Q4KHead hg(*reinterpret_cast<const uint4*>(bg)), hu(*reinterpret_cast<const uint4*>(bu));
      bad |= !hg.ok() || !hu.ok();
      double pg = 0.0, qg = 0.0, pu = 0.0, qu = 0.0;
#pragma unroll
      for (unsigned gp = 0; gp < 4; ++gp) {
        const unsigned p = 4 * q + gp, half = gp >> 1, sh = 16 * (gp & 1);
        uint32_t xlo[8], rlo[8], xhi[8], rhi[8];
        load_x8(xa.v, p, 0, nspan, xlo);
        load_x8(xa.r, p, 0, nspan, rlo);
        load_x8(xa.v, p, 2, nspan, xhi);
        load_x8(xa.r, p, 2, nspan, rhi);
        const double2 st = xa.st[p];
        const int4 vr = xa.vr[p];
        const long long M = __double2loint(st.y);  // s = M 2^E, st.x = 2^E
        // the exact integer M K + K' as a double (|.| < 2^51: magic 1.5 * 2^52)
        auto zd = [&](int K, int Kr) {
          return __longlong_as_double(M * K + (0x4338000000000000LL + Kr)) - 6755399441055744.0;
        };
        int i0, i1, r0, r1;
        q4k_idots(bg + 16 + 32 * gp, xlo, rlo, xhi, rhi, i0, i1, r0, r1);
        {
          const int sc0 = (hg.sc[half] >> sh) & 0xff, sc1 = (hg.sc[half] >> (sh + 8)) & 0xff;
          const int mi0 = (hg.mi[half] >> sh) & 0xff, mi1 = (hg.mi[half] >> (sh + 8)) & 0xff;
          pg = fma(zd(sc0 * i0 + sc1 * i1, sc0 * r0 + sc1 * r1), st.x, pg);
          qg = fma(zd(mi0 * vr.x + mi1 * vr.z, mi0 * vr.y + mi1 * vr.w), st.x, qg);
        }
        q4k_idots(bu + 16 + 32 * gp, xlo, rlo, xhi, rhi, i0, i1, r0, r1);
        {
          const int sc0 = (hu.sc[half] >> sh) & 0xff, sc1 = (hu.sc[half] >> (sh + 8)) & 0xff;
          const int mi0 = (hu.mi[half] >> sh) & 0xff, mi1 = (hu.mi[half] >> (sh + 8)) & 0xff;
          pu = fma(zd(sc0 * i0 + sc1 * i1, sc0 * r0 + sc1 * r1), st.x, pu);
          qu = fma(zd(mi0 * vr.x + mi1 * vr.z, mi0 * vr.y + mi1 * vr.w), st.x, qu);
        }
      }
      ag = fma(static_cast<double>(hg.d), pg, ag);
      ag = fma(-static_cast<double>(hg.m), qg, ag);
      au = fma(static_cast<double>(hu.d), pu, au);
      au = fma(-static_cast<double>(hu.m), qu, au);
    } else {
#pragma unroll
      for (unsigned gp = 0; gp < 4; ++gp) {
        const unsigned p = 4 * q + gp;
        uint32_t xw[16], rw[16];
        uint32_t(&x0)[8] = *reinterpret_cast<uint32_t(*)[8]>(xw);
        uint32_t(&x1)[8] = *reinterpret_cast<uint32_t(*)[8]>(xw + 8);
        uint32_t(&r0)[8] = *reinterpret_cast<uint32_t(*)[8]>(rw);
        uint32_t(&r1)[8] = *reinterpret_cast<uint32_t(*)[8]>(rw + 8);
        load_x8(xa.v, p, 0, nspan, x0);
        load_x8(xa.v, p, 2, nspan, x1);
        load_x8(xa.r, p, 0, nspan, r0);
        load_x8(xa.r, p, 2, nspan, r1);
        const double2 st = xa.st[p];
        if (TYPE == kMXFP4) {
          ag = group_mxfp4(ag, gr, nb, p, xw, rw, st, bad);
          au = group_mxfp4(au, ur, nb, p, xw, rw, st, bad);
        } else {
          ag = group_q80(ag, gr, nb, p, xw, rw, st, bad);
          au = group_q80(au, ur, nb, p, xw, rw, st, bad);
        }
      }
    }
  }
}

// The reference's narrowing of a double sum to fp32 (backends/ref.c:37-40).
__device__ __forceinline__ bool narrow(double v, float* out) {
  if (!isfinite(v) || fabs(v) > 3.4028234663852886e38) return false;
  *out = __double2float_rn(v);
  return true;
}

// Down term c of row rr of a staged down chunk ([nr scales][nr payloads]),
// hidden slice kk: scale x int_dot (Q8 hidden) or the fp32 dot.  One
// instantiation per weight type.
template <unsigned DT, int ACT>
__device__ __forceinline__ float down_term(const uint8_t* slot, unsigned nr, unsigned rr, const uint8_t* s_hq,
                                           unsigned kk, bool& bad) {
  if (DT == kMXFP4) {
    const unsigned e = slot[rr];
    bad |= e == 255;
    const uint4 w = *reinterpret_cast<const uint4*>(slot + nr + 16 * rr);
    if (ACT == FRC_ACT_Q8) {
      const uint4 h0 = reinterpret_cast<const uint4*>(s_hq)[2 * kk];
      const uint4 h1 = reinterpret_cast<const uint4*>(s_hq)[2 * kk + 1];
      const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      return __fmul_rn(pow2_m128(e), i2f(idot_mxfp4_16(w, hw)));
    }
    const float* hv = reinterpret_cast<const float*>(s_hq) + kk * 32;
    const float sc = __uint_as_float(e ? e << 23 : 0x00400000u);
    const uint8_t* qb = slot + nr + 16 * rr;
    float dot = 0.0f;
    for (unsigned nn = 0; nn < 32; ++nn)
      dot = __fmaf_rn(__fmul_rn(sc, e2m1((qb[nn & 15] >> (nn >> 4 ? 4 : 0)) & 15)), hv[nn], dot);
    return dot;
  }
  const float sw = h2f(slot[2 * rr] | slot[2 * rr + 1] << 8);
  bad |= !isfinite(sw);
  if (ACT == FRC_ACT_Q8) {
    const uint4* wv = reinterpret_cast<const uint4*>(slot + 2 * nr + 32 * rr);
    const uint4 w0 = wv[0], w1 = wv[1];
    const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const uint4 h0 = reinterpret_cast<const uint4*>(s_hq)[2 * kk];
    const uint4 h1 = reinterpret_cast<const uint4*>(s_hq)[2 * kk + 1];
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    int iv = 0;
#pragma unroll
    for (unsigned m = 0; m < 8; ++m) iv = __dp4a(static_cast<int>(ww[m]), static_cast<int>(hw[m]), iv);
    return __fmul_rn(sw, i2f(iv));
  }
  const float* hv = reinterpret_cast<const float*>(s_hq) + kk * 32;
  const int8_t* qb = reinterpret_cast<const int8_t*>(slot + 2 * nr + 32 * rr);
  float dot = 0.0f;
  for (unsigned nn = 0; nn < 32; ++nn) dot = __fmaf_rn(__fmul_rn(sw, static_cast<float>(qb[nn])), hv[nn], dot);
  return dot;
}

// One token: this thread's rows tid + j x kLayerThreads (j < 4) of a down chunk.
template <unsigned DT, int ACT>
__device__ __forceinline__ void down_terms4(const uint8_t* slot, unsigned nr, const uint8_t* s_hq, bool& bad,
                                            float& h0, float& h1, float& h2, float& h3) {
  const unsigned tid = threadIdx.x;
  h0 = tid < nr ? down_term<DT, ACT>(slot, nr, tid, s_hq, 0, bad) : 0.0f;
  h1 = tid + kLayerThreads < nr ? down_term<DT, ACT>(slot, nr, tid + kLayerThreads, s_hq, 0, bad) : 0.0f;
  h2 = tid + 2 * kLayerThreads < nr ? down_term<DT, ACT>(slot, nr, tid + 2 * kLayerThreads, s_hq, 0, bad) : 0.0f;
  h3 = tid + 3 * kLayerThreads < nr ? down_term<DT, ACT>(slot, nr, tid + 3 * kLayerThreads, s_hq, 0, bad) : 0.0f;
}

// Warps 0-3: the layer input.  Reads x (+ x_add; stores the sum to x_out
// from CTA 0), applies the optional RMS pre-norm, and quantizes per 64
// (src/q4.c:37-61) into the activation layout of LayerSmem: v and the
// dequantization residuals r (natural and, for MXFP4 rows, prmt order),
// {s, 2^E} per group and {V, RS} per 32-block; fp32 x in the F32 mode.
// Needs only x, so it runs while the plan warps build the plan and start
// the weight copies.
template <int ACT>
__device__ __forceinline__ void layer_input(const LayerParams& a, uint8_t* smem, unsigned T, unsigned tid,
                                            unsigned lane, unsigned warp, unsigned cta) {
  float* s_rms = reinterpret_cast<float*>(smem + a.sm.rms);
  float* s_rpart = reinterpret_cast<float*>(smem + a.sm.rpart);  // [round][warp] sums of squares
  const unsigned d = a.d, P = d / 64;
  (void)P;
  pdl_wait();
  // A unit is a quarter of a 64-element x group: 16 floats, one thread.
  // Four consecutive lanes hold a group, so its max and sums take two
  // shuffles, and a thread's 16 int8 values are one 16-byte store.
  const unsigned units = T * d / 16, upt = d / 16;  // units in all, per token
  const unsigned upt_magic = 0xffffffffu / upt + 1;  // unit / upt by multiply-high (exact: unit < 2^16)
  auto load_unit = [&](unsigned u, float (&v)[16]) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x) + 4 * u;
    const float4* xa4 = a.x_add ? reinterpret_cast<const float4*>(a.x_add) + 4 * u : nullptr;
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
      float4 w = x4[k];
      if (xa4) {
        const float4 z = xa4[k];
        w.x = __fadd_rn(w.x, z.x); w.y = __fadd_rn(w.y, z.y); w.z = __fadd_rn(w.z, z.z); w.w = __fadd_rn(w.w, z.w);
      }
      v[4 * k] = w.x; v[4 * k + 1] = w.y; v[4 * k + 2] = w.z; v[4 * k + 3] = w.w;
    }
  };
  float v0[16];  // the first unit stays in registers from the sums to the quantization
  if (tid < units) load_unit(tid, v0);
  bool bad = false;
  if (a.norm) {
    // sums of squares per (pass, warp): a warp-pass covers 512 floats, all in one token
    for (unsigned u0 = 0; u0 < units; u0 += kActThreads) {
      const unsigned u = u0 + tid;
      float ss = 0.0f;
      if (u < units) {
        float v[16];
        if (u0 == 0) {
#pragma unroll
          for (unsigned k = 0; k < 16; ++k) v[k] = v0[k];
        } else {
          load_unit(u, v);
        }
#pragma unroll
        for (unsigned k = 0; k < 16; ++k) ss = __fmaf_rn(v[k], v[k], ss);
      }
#pragma unroll
      for (unsigned o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) s_rpart[u0 / 32 + warp] = ss;
    }
    act_sync();
    PHASE(2);
    // token t: warp-passes [t * d/512, (t+1) * d/512); warp w takes tokens
    // w, w+4, ...; lane L adds passes L, L+32, ...; butterfly
    for (unsigned t = warp; t < T; t += kActWarps) {
      const unsigned per = d / 512;
      float tot = 0.0f;
      for (unsigned b = lane; b < per; b += 32) tot = __fadd_rn(tot, s_rpart[t * per + b]);
#pragma unroll
      for (unsigned o = 16; o; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
      if (lane == 0) s_rms[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(d)), 1e-6f)));
    }
    act_sync();
  }
  for (unsigned u0 = 0; u0 < units; u0 += kActThreads) {
    const unsigned u = u0 + tid;
    if (u >= units) break;  // warp-uniform: units is a multiple of 32
    float v[16];
    if (u0 == 0) {
#pragma unroll
      for (unsigned k = 0; k < 16; ++k) v[k] = v0[k];
    } else {
      load_unit(u, v);
    }
    const unsigned t = __umulhi(u, upt_magic), j16 = u - t * upt, p = j16 >> 2, qd = j16 & 3;
#pragma unroll
    for (unsigned k = 0; k < 16; ++k) bad |= !isfinite(v[k]);
    if (a.x_out && cta == 0) {
      float4* xo = reinterpret_cast<float4*>(a.x_out) + 4 * u;
#pragma unroll
      for (unsigned k = 0; k < 4; ++k) xo[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
    if (a.norm) {
      const float g = s_rms[t];
#pragma unroll
      for (unsigned k = 0; k < 16; ++k) v[k] = __fmul_rn(v[k], g);
    }
    if (ACT == FRC_ACT_F32) {
      float4* xf = reinterpret_cast<float4*>(smem + a.sm.xf) + 4 * u;
#pragma unroll
      for (unsigned k = 0; k < 4; ++k) xf[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      continue;
    }
    float amax = 0.0f;
#pragma unroll
    for (unsigned k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const Q8Group qg(amax);
    int qv[16], rv[16], sum = 0, rsum = 0;
    if (__builtin_expect(qg.mul_ok(), 1)) {
#pragma unroll
      for (unsigned k = 0; k < 16; ++k) {
        qv[k] = qg.qm(v[k]);
        sum += qv[k];
      }
    } else {
#pragma unroll
      for (unsigned k = 0; k < 16; ++k) {
        qv[k] = qg.q(v[k]);
        sum += qv[k];
      }
    }
    // Residuals of the reference's dequantized values (src/q4.c:54-58):
    // X = fl32(v * s), capped at FLT_MAX; X - v*s = r * 2^E exactly, E =
    // ef - 150.  The fma gives X - v*s exactly; two power-of-two scalings
    // (each representable) take it to r.
    const unsigned ef = scale_ef(qg.scale), shr = 150 - ef;
    const float f1 = __uint_as_float((127 + (shr >> 1)) << 23), f2 = __uint_as_float((127 + shr - (shr >> 1)) << 23);
#pragma unroll
    for (unsigned k = 0; k < 16; ++k) {
      const float vf = i2f(qv[k]);
      float X = __fmul_rn(vf, qg.scale);
      if (fabsf(X) > 3.40282347e38f) X = copysignf(3.40282347e38f, vf);
      rv[k] = f2i_small(__fmul_rn(__fmul_rn(__fmaf_rn(-vf, qg.scale, X), f1), f2));
      rsum += rv[k];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // quarters 0+1 and 2+3: the two 32-element halves
    rsum += __shfl_xor_sync(0xffffffffu, rsum, 1);
    uint32_t w[4], wr[4];
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
      w[k] = (qv[4 * k] & 0xff) | (qv[4 * k + 1] & 0xff) << 8 | (qv[4 * k + 2] & 0xff) << 16 |
             static_cast<uint32_t>(qv[4 * k + 3] & 0xff) << 24;
      wr[k] = (rv[4 * k] & 0xff) | (rv[4 * k + 1] & 0xff) << 8 | (rv[4 * k + 2] & 0xff) << 16 |
              static_cast<uint32_t>(rv[4 * k + 3] & 0xff) << 24;
    }
    const unsigned slot16 = 16 * xslot(p, qd, d / 256);
    *reinterpret_cast<uint4*>(smem + a.sm.xq + t * d + slot16) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(smem + a.sm.xr + t * d + slot16) = make_uint4(wr[0], wr[1], wr[2], wr[3]);
    if (qd == 0)
      reinterpret_cast<double2*>(smem + a.sm.xst)[t * P + p] =  // {2^E, M}: scale = M 2^E
          make_double2(pow2d(static_cast<int>(ef) - 150),
                       __hiloint2double(0, static_cast<int>((__float_as_uint(qg.scale) >> 23 & 255u)
                                                                ? (__float_as_uint(qg.scale) & 0x7fffffu) | 0x800000u
                                                                : __float_as_uint(qg.scale) & 0x7fffffu)));
    if ((qd & 1) == 0)
      reinterpret_cast<int2*>(smem + a.sm.xvr)[2 * (t * P + p) + (qd >> 1)] = make_int2(sum, rsum);
    if (a.sm.xp) {
      uint8_t* xp = smem + a.sm.xp + t * d;
      uint8_t* xrp = smem + a.sm.xrp + t * d;
#pragma unroll
      for (unsigned k = 0; k < 16; ++k) {
        const unsigned e = 16 * qd + k, wi = (e / 32) * 32 + prmt_pos(e % 32);
        const unsigned at = 16 * xslot(p, wi / 16, d / 256) + wi % 16;
        xp[at] = static_cast<uint8_t>(qv[k] & 0xff);
        xrp[at] = static_cast<uint8_t>(rv[k] & 0xff);
      }
    }
  }
  if (bad) atomicOr(a.status, kStNumeric);
}

// ONE: a one-token launch, the token count folded to 1 at compile time (its
// loops over tokens and the multi-token plan drop out).  SPLIT implies ONE.
// SPLIT: items may be split in a.H parts (one token); without it H is 1 at
// compile time and the split's bookkeeping folds away.
template <int ACT, bool SPLIT, bool ONE>
__global__ void __launch_bounds__(kLayerThreads, 2) moe_layer_kernel(const LayerParams a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);                // kMaxSlots mbarriers
  unsigned* misc = reinterpret_cast<unsigned*>(smem + 64);           // 64 words
  unsigned* s_cnt = misc + 40;                                       // ring slot: readers done with its chunk
  unsigned* s_iss = misc + 48;                                       // ring slot: chunks issued into it
  uint16_t* s_ids = reinterpret_cast<uint16_t*>(smem + a.sm.ids);
  float* s_g = reinterpret_cast<float*>(smem + a.sm.gates);
  int* s_first = reinterpret_cast<int*>(smem + a.sm.first);
  uint16_t* s_uid = reinterpret_cast<uint16_t*>(smem + a.sm.uid);
  unsigned* s_umask = reinterpret_cast<unsigned*>(smem + a.sm.umask);
  float* s_ugate = reinterpret_cast<float*>(smem + a.sm.ugate);
  unsigned* s_upre = reinterpret_cast<unsigned*>(smem + a.sm.upre);  // first pair of each expert
  uint16_t* s_tokpair = reinterpret_cast<uint16_t*>(smem + a.sm.tokpair);  // [token][11] -> pair
  float* s_gv = reinterpret_cast<float*>(smem + a.sm.gv);            // [neuron][k] hidden values
  uint8_t* s_hq = smem + a.sm.hq;                                    // [k][32] int8, or [k][32] f32
  float* s_ylocal = reinterpret_cast<float*>(smem + a.sm.ylocal);    // [t][rows]: this GPU's partial (peer reduce)
  uint8_t* ring = smem + a.sm.ring;
  const unsigned SLOT = a.sm.slot_bytes, K = a.sm.slots;

  const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned T = (ONE || SPLIT) ? 1u : a.T, S = a.S, d = a.d, P = d / 64, G = gridDim.x, cta = blockIdx.x;

  PHASE(0);
  pdl_signal();
  // -------------------------------------------------- this CTA's items
  // Global item order: the shared expert's S items, then routed (u, s)
  // expert-major.  Round r deals items r*G .. r*G+G-1, alternating direction.
  // UR (routed unique experts) and SH (slices of the shared expert, 0 when
  // no token uses it) come from the plan; setup() derives this CTA's list.
  unsigned UR = 0, SH = 0, U = 0, NI = 0, n_my = 0, nsh = 0, n_ch = 0;
  auto item_at = [&](unsigned r) { return r * G + ((r & 1) ? G - 1 - cta : cta); };
  const Div by_S(S, a.mag_S);
  const unsigned H = SPLIT ? a.H : 1u, Hs = SPLIT ? a.Hshift : 0u;
  // part j -> item (u, s) and part h; the item's index ji in item order
  auto item_us = [&](unsigned j, unsigned& u, unsigned& s, unsigned& h, unsigned& ji) {
    ji = j >> Hs;
    h = j & (H - 1);
    if (ji < SH) { u = UR; s = ji; }
    else { u = by_S.q(ji - SH); s = ji - SH - u * S; }
  };
  const unsigned kn_r = a.sm.kn_r, kn_s = a.sm.kn_s, dn_r = a.sm.dn_r, dn_s = a.sm.dn_s;
  const unsigned ngu_r = 32 / kn_r / H, ngu_s = 32 / kn_s / H;  // gate/up chunks a part
  const unsigned dpart = d / H;                                  // down rows a part
  const unsigned ndn_r = (dpart + dn_r - 1) / dn_r, ndn_s = (dpart + dn_s - 1) / dn_s;
  const unsigned ch_r = ngu_r + ndn_r, ch_s = ngu_s + ndn_s;
  const Div by_ch_r(ch_r, a.sm.mag_ch_r), by_ch_s(ch_s, a.sm.mag_ch_s);
  const unsigned ss_r = a.down_type == kQ80 ? 2 : 1, pb_r = a.down_type == kQ80 ? 32 : 16;
  auto setup = [&]() {
    UR = misc[4];
    U = UR + (misc[5] ? 1 : 0);
    SH = misc[5] ? S : 0;
    NI = U * S * H;
    n_my = 0;
    while (item_at(n_my) < NI) ++n_my;
    nsh = 0;
    while (nsh < n_my && item_at(nsh) < SH * H) ++nsh;
    n_ch = nsh * ch_s + (n_my - nsh) * ch_r;
  };

  // chunk c of this CTA -> (item round r, chunk k within the item)
  auto chunk_at = [&](unsigned c, unsigned& r, unsigned& k) {
    if (c < nsh * ch_s) { r = by_ch_s.q(c); k = c - r * ch_s; }
    else { const unsigned cr = c - nsh * ch_s, rr = by_ch_r.q(cr); r = nsh + rr; k = cr - rr * ch_r; }
  };
  // Gate/up chunk k: gate rows k*kn.. then up rows k*kn.. (two copies).
  // Down chunk: rows [r0, r0+nr): their scales, then their payloads.
  auto issue = [&](unsigned c) {
    unsigned r, k, u, s, h, ji;
    chunk_at(c, r, k);
    item_us(item_at(r), u, s, h, ji);
    const bool sh = u >= UR;
    const unsigned rowb = sh ? a.shared_row : a.row_bytes, proj = sh ? a.shared_proj : a.proj_bytes;
    const unsigned kn = sh ? kn_s : kn_r, ngu = sh ? ngu_s : ngu_r, dn = sh ? dn_s : dn_r;
    const unsigned ss = sh ? 2 : ss_r, pb = sh ? 32 : pb_r;
    const uint8_t* src = a.base[s] + static_cast<size_t>(s_uid[u]) * a.slice_bytes;
    const unsigned slot = c % K;
    uint8_t* dst = ring + slot * SLOT;
    reinterpret_cast<volatile unsigned*>(s_iss)[slot] = s_iss[slot] + 1;
    if (k < ngu) {
      const unsigned bytes = kn * rowb, kg = h * ngu + k;  // chunk of the slice's neurons
      mbar_expect_tx(&full[slot], 2 * bytes);
      bulk_g2s(dst, src + kg * bytes, bytes, &full[slot]);
      bulk_g2s(dst + bytes, src + proj + kg * bytes, bytes, &full[slot]);
    } else {
      const unsigned r0 = h * dpart + (k - ngu) * dn, nr = min(dn, (h + 1) * dpart - r0);
      const uint8_t* down = src + 2 * proj;
      mbar_expect_tx(&full[slot], nr * (ss + pb));
      bulk_g2s(dst, down + r0 * ss, nr * ss, &full[slot]);
      bulk_g2s(dst + nr * ss, down + d * ss + r0 * pb, nr * pb, &full[slot]);
    }
  };

  if (warp >= kFirstPlanWarp) {
    // ------------------------------------------------- warps 4-7: plan
    const unsigned ptid = tid - 32 * kFirstPlanWarp, pw = warp - kFirstPlanWarp;
    if (ptid < kMaxSlots) {
      s_cnt[ptid] = 0;
      s_iss[ptid] = 0;
    }
    if (ptid == 0) {  // the ring's barriers, while the routing loads are in flight
      for (unsigned k = 0; k < K; ++k) mbar_init(&full[k], 1);
      fence_mbar_init();
    }
    if (T == 1) {
      // one token: its ten experts in request order are the unique experts,
      // each with one (expert, token) pair
      if (pw == 0) {
        unsigned id = 0;
        float gv = 0.0f;
        if (lane < 10) {
          id = a.expert[lane];
          gv = a.gate[lane];
          if (id >= 512) {
            atomicOr(a.status, kStInvalid);
            id = 0;  // keeps every address in range; the launch reports INVALID
          }
        }
        const float sg = a.gate[10];
        if (lane < 10) {
          s_uid[lane] = static_cast<uint16_t>(id);
          s_umask[lane] = 1;
          s_ugate[lane] = gv;
        }
        if (lane == 10 && sg != 0.0f) {
          s_uid[10] = 512;
          s_umask[10] = 1;
          s_ugate[10] = sg;
        }
        if (lane < 12) s_upre[lane] = lane;
        if (lane < 11) s_tokpair[lane] = static_cast<uint16_t>(lane < 10 ? lane : (sg != 0.0f ? 10u : 0xffffu));
        if (lane == 0) {
          misc[4] = 10;
          misc[5] = sg != 0.0f ? 1u : 0u;
        }
        PHASE_AT(8, kPlanThreads);
      }
    } else {
      for (unsigned i = ptid; i < T * 10; i += kPlanThreads) s_ids[i] = a.expert[i];
      for (unsigned i = ptid; i < T * 11; i += kPlanThreads) s_g[i] = a.gate[i];
      for (unsigned i = ptid; i < 512; i += kPlanThreads) s_first[i] = 0x7fffffff;
      for (unsigned i = ptid; i < a.sm.max_unique; i += kPlanThreads) s_umask[i] = 0;
      for (unsigned i = ptid; i < a.sm.max_unique * T; i += kPlanThreads) s_ugate[i] = 0.0f;
      plan_sync();
      PHASE_AT(8, kPlanThreads);
      bool invalid = false;
      for (unsigned i = ptid; i < T * 10; i += kPlanThreads) {
        const unsigned id = s_ids[i];
        if (id < 512) atomicMin(&s_first[id], static_cast<int>(i));
        else invalid = true;
      }
      if (invalid) atomicOr(a.status, kStInvalid);
      plan_sync();
      // unique experts in first-appearance order: rank = earlier first
      // appearances; up to 160 entries, 128 at a time
      unsigned total = 0;
      for (unsigned base = 0; base < T * 10; base += kPlanThreads) {
        const unsigned i = base + ptid;
        const unsigned id = i < T * 10 ? s_ids[i] : 0xffffu;
        const bool first = id < 512 && s_first[id] == static_cast<int>(i);
        const unsigned ballot = __ballot_sync(0xffffffffu, first);
        if (lane == 0) misc[16 + pw] = __popc(ballot);
        plan_sync();
        unsigned off = total, all = 0;
        for (unsigned w = 0; w < kPlanWarps; ++w) {
          if (w < pw) off += misc[16 + w];
          all += misc[16 + w];
        }
        plan_sync();  // every first-appearance test of this round is done; misc is free
        if (first) {
          const unsigned rank = off + __popc(ballot & ((1u << lane) - 1));
          s_uid[rank] = static_cast<uint16_t>(id);
          s_first[id] = -1 - static_cast<int>(rank);
        }
        total += all;
      }
      if (ptid == 0) misc[4] = total;  // routed experts
      plan_sync();
      for (unsigned k = ptid; k < T * 10; k += kPlanThreads) {
        const unsigned id = s_ids[k];
        if (id >= 512) continue;
        const unsigned u = static_cast<unsigned>(-1 - s_first[id]), t = k / 10;
        atomicOr(&s_umask[u], 1u << t);
        s_ugate[u * T + t] = s_g[t * 11 + k % 10];
      }
      plan_sync();
      const unsigned ur = misc[4];
      unsigned shared_mask = 0;
      for (unsigned t = 0; t < T; ++t)
        if (s_g[t * 11 + 10] != 0.0f) shared_mask |= 1u << t;
      const unsigned nu = ur + (shared_mask ? 1 : 0);
      if (ptid == 0) {
        misc[5] = shared_mask;
        if (shared_mask) {
          s_uid[ur] = 512;
          s_umask[ur] = shared_mask;
        }
      }
      if (shared_mask)
        for (unsigned t = ptid; t < T; t += kPlanThreads) s_ugate[ur * T + t] = s_g[t * 11 + 10];
      plan_sync();
      if (pw == 0) {  // pair offsets: exclusive scan of the token counts, 6 experts a lane
        unsigned cnt[6], tot = 0;
    #pragma unroll
        for (unsigned k = 0; k < 6; ++k) {
          const unsigned u = lane * 6 + k;
          cnt[k] = u < nu ? __popc(s_umask[u]) : 0;
          tot += cnt[k];
        }
        unsigned inc = tot;
    #pragma unroll
        for (unsigned o = 1; o < 32; o <<= 1) {
          const unsigned v = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += v;
        }
        unsigned run = inc - tot;
    #pragma unroll
        for (unsigned k = 0; k < 6; ++k) {
          const unsigned u = lane * 6 + k;
          if (u <= nu) s_upre[u] = run;
          run += cnt[k];
        }
      }
      plan_sync();
      for (unsigned k = ptid; k < T * 11; k += kPlanThreads) {  // (token, routing slot) -> pair
        const unsigned t = k / 11, e = k % 11;
        unsigned pair = 0xffff;
        if (e < 10) {
          const unsigned id = s_ids[t * 10 + e];
          if (id < 512) {
            const unsigned u = static_cast<unsigned>(-1 - s_first[id]);
            pair = s_upre[u] + __popc(s_umask[u] & ((1u << t) - 1));
          }
        } else if (shared_mask >> t & 1) {
          pair = s_upre[ur] + __popc(shared_mask & ((1u << t) - 1));
        }
        s_tokpair[k] = static_cast<uint16_t>(pair);
      }
    }
    plan_sync();
    PHASE_AT(10, kPlanThreads);
    if (pw == 0) {  // the first K chunks, while the activations are still being formed
      setup();
      if (lane < K && lane < n_ch) issue(lane);
      PHASE_AT(1, kPlanThreads);
    }
    pdl_wait();
  }
  if (warp < kActWarps) layer_input<ACT>(a, smem, T, tid, lane, warp, cta);
  __syncthreads();
  setup();
  if (a.world > 1 && tid == 0) misc[6] = *reinterpret_cast<volatile unsigned*>(&a.ctl->peer_epoch) + 1;
  PHASE(3);

  // --------------------------------------------------------------- items
  // Only the warps that read ring chunk c wait for it: a gate/up chunk's
  // kn/4 warps, every warp for a down chunk.  A reader done with it counts
  // itself out of the slot; the last of the `readers` (fence.cta orders
  // their shared-memory reads first) clears the count and refills the slot
  // with chunk c+K.  Nothing else touches the count until that chunk lands
  // (the refill's arrive on the slot's barrier releases the clearing store).
  // A warp whose wait ran out stops counting, so nothing is issued into a
  // slot that a copy may still be writing.
  bool timed_out = false, aborted = false;  // warp-uniform, block-uniform
  auto release = [&](unsigned c, unsigned readers) {
    __syncwarp();
    if (lane == 0 && !timed_out) {
      __threadfence_block();
      const unsigned slot = c % K;
      if (atomicAdd(&s_cnt[slot], 1u) == readers - 1) {
        s_cnt[slot] = 0;
        if (c + K < n_ch) {
          __threadfence_block();
          fence_proxy_async();
          issue(c + K);
        }
      }
    }
  };
  // A reader waits for chunk c only once it is issued into its slot (the
  // slot's previous chunk c-K consumed): then the slot's barrier is at chunk
  // c's phase or past it, and the phase parity names chunk c unambiguously.
  auto wait_chunk = [&](unsigned c) {
    if (!timed_out) {
      const unsigned slot = c % K, j = c / K;
      bool ok = true;
      if (reinterpret_cast<volatile unsigned*>(s_iss)[slot] <= j) {
        const uint64_t start = globaltimer();
        while (reinterpret_cast<volatile unsigned*>(s_iss)[slot] <= j)
          if (globaltimer() - start > a.wait_ns) {
            ok = false;
            break;
          }
      }
      ok = ok && mbar_wait(&full[slot], j & 1, a.wait_ns);
      timed_out = __any_sync(0xffffffffu, !ok);
    }
    return !timed_out;
  };
  unsigned c = 0;
  bool bad = false;
  for (unsigned r = 0; r < n_my && !aborted; ++r) {
    unsigned u, s, h, ji;
    item_us(item_at(r), u, s, h, ji);
    const bool sh = u >= UR;
    const unsigned type = sh ? kQ80 : a.gate_type, dtype = sh ? kQ80 : a.down_type;
    const unsigned rowb = sh ? a.shared_row : a.row_bytes, nb = d / 32;
    const unsigned kn = sh ? kn_s : kn_r, ngu = sh ? ngu_s : ngu_r, dn = sh ? dn_s : dn_r, ndn = sh ? ndn_s : ndn_r;
    const unsigned mask = (ONE || SPLIT) ? 1u : s_umask[u], nt = (ONE || SPLIT) ? 1u : __popc(mask), gp0 = s_upre[u];
    // gate/up: warp w takes neurons 4 (w % (kn/4)) .. +3 of chunk w / (kn/4),
    // eight lanes a neuron.  Lane l8 takes the 256-element spans q = l8,
    // l8+8, ... of both the gate and the up row (they share the x loads),
    // groups in order; butterfly over the eight lanes; lane l8 == 0 then
    // forms the neuron's SwiGLU (double, backends/ref.c:81-83).
    const unsigned quads = kn / 4, my_chunk = warp / quads, l8 = lane & 7, nspan = d / 256;
    for (unsigned k = 0; k < ngu; ++k, ++c) {
      if (k != my_chunk) continue;
      if (wait_chunk(c)) {
        if (c == 0) PHASE(15);
        if (c == 1) PHASE(12);
        const uint8_t* slot = ring + (c % K) * SLOT;
        const unsigned nl = 4 * (warp % quads) + (lane >> 3);  // neuron within the chunk
        const uint8_t* gr = slot + nl * rowb;
        const uint8_t* ur = slot + (kn + nl) * rowb;
        const unsigned n = (h * ngu + k) * kn + nl;
        unsigned mm = mask;
        for (unsigned kk = 0; kk < nt; ++kk) {
          const unsigned t = __ffs(mm) - 1;
          mm &= mm - 1;
          float ag = 0.0f, au = 0.0f;
          bool nar = true;
          if (ACT == FRC_ACT_Q8) {
            const bool mx = type == kMXFP4;
            const XAct xa{smem + (mx ? a.sm.xp : a.sm.xq) + t * d, smem + (mx ? a.sm.xrp : a.sm.xr) + t * d,
                          reinterpret_cast<const double2*>(smem + a.sm.xst) + t * P,
                          reinterpret_cast<const int4*>(smem + a.sm.xvr) + t * P};
            double dg = 0.0, du = 0.0;
            if (type == kQ4K) gu_sums<kQ4K>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
            else if (mx) gu_sums<kMXFP4>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
            else gu_sums<kQ80>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
#pragma unroll
            for (unsigned o = 4; o; o >>= 1) {
              dg = __dadd_rn(dg, __shfl_xor_sync(0xffffffffu, dg, o));
              du = __dadd_rn(du, __shfl_xor_sync(0xffffffffu, du, o));
            }
            nar = narrow(dg, &ag) && narrow(du, &au);
          } else {
            const float* xf = reinterpret_cast<const float*>(smem + a.sm.xf) + t * d;
            for (unsigned q = l8; q < nspan; q += 8)
              for (unsigned e = 256 * q; e < 256 * q + 256; ++e) {
                const float wg = weight_any(gr, type, d, e), wu = weight_any(ur, type, d, e);
                bad |= !isfinite(wg) || !isfinite(wu);
                ag = __fmaf_rn(wg, xf[e], ag);
                au = __fmaf_rn(wu, xf[e], au);
              }
#pragma unroll
            for (unsigned o = 4; o; o >>= 1) {
              ag = __fadd_rn(ag, __shfl_xor_sync(0xffffffffu, ag, o));
              au = __fadd_rn(au, __shfl_xor_sync(0xffffffffu, au, o));
            }
          }
          if (l8 == 0) {
            float h = 0.0f;
            if (!nar || !isfinite(ag) || !isfinite(au) || !swiglu(ag, au, &h)) {
              bad = true;
              h = 0.0f;
            }
            s_gv[n * T + kk] = h;
          }
        }
      }
      release(c, quads);
    }
    if (r == 0) PHASE(9);
    if (__syncthreads_or(timed_out)) { aborted = true; break; }
    if (SPLIT && H > 1) {
      // one token: this part's hidden values go to the item's exchange row;
      // wait (bounded) until all H parts wrote theirs, then take the others
      const unsigned nn = 32 / H, n0 = h * nn;
      if (tid < nn) a.xchg[ji * 32 + n0 + tid] = s_gv[n0 + tid];
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        atomicAdd(&a.xcnt[ji], 1u);
        bool ok = spin_geq(&a.xcnt[ji], H, &a.ctl->abort, a.wait_ns);
        misc[8] = ok ? 1u : 0u;
      }
      __syncthreads();
      if (!misc[8]) { timed_out = true; aborted = true; break; }
      if (tid < 32 && (tid < n0 || tid >= n0 + nn)) s_gv[tid] = __ldcg(a.xchg + ji * 32 + tid);
      __syncthreads();
    }
    // the hidden slice's Q8 quantization (src/q4.c:37-61, one group of 32)
    for (unsigned kk = warp; kk < nt; kk += kLayerWarps) {
      unsigned mm = mask;
      for (unsigned z = 0; z < kk; ++z) mm &= mm - 1;
      const unsigned t = __ffs(mm) - 1;
      const float h = s_gv[lane * T + kk];
      if (a.hidden) a.hidden[((static_cast<size_t>(u) * S + s) * T + t) * 32 + lane] = h;
      float gs;
      if (ACT == FRC_ACT_Q8) {
        float amax = fabsf(h);
#pragma unroll
        for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const Q8Group qg(amax);
        const int qh = __builtin_expect(qg.mul_ok(), 1) ? qg.qm(h) : qg.q(h);
        s_hq[kk * 32 + (dtype == kMXFP4 ? prmt_pos(lane) : lane)] = static_cast<uint8_t>(qh & 0xff);
        gs = __fmul_rn(qg.scale, s_ugate[u * T + t]);
      } else {
        reinterpret_cast<float*>(s_hq)[kk * 32 + lane] = h;
        gs = s_ugate[u * T + t];
      }
      if (lane == 0) a.gsv[(gp0 + kk) * S + s] = gs;
    }
    __syncthreads();
    if (r == 0) PHASE(13);
    // down: rows of chunk k, one a thread; c = scale * int_dot (or the fp32 dot)
    for (unsigned k = 0; k < ndn; ++k, ++c) {
      const unsigned r0 = h * dpart + k * dn, nr = min(dn, (h + 1) * dpart - r0);
      float* out = a.partial + (static_cast<size_t>(gp0) * S + s) * d + r0;
      if (wait_chunk(c)) {
        if (r == 0 && k == 0) PHASE(14);
        const uint8_t* slot = ring + (c % K) * SLOT;
        if (nt == 1 && nr <= 4 * kLayerThreads) {
          // one token, at most four rows a thread: hold the terms in registers,
          // hand the slot back, then store (the release need not wait for them)
          float h0, h1, h2, h3;
          if (dtype == kMXFP4) down_terms4<kMXFP4, ACT>(slot, nr, s_hq, bad, h0, h1, h2, h3);
          else down_terms4<kQ80, ACT>(slot, nr, s_hq, bad, h0, h1, h2, h3);
          release(c, kLayerWarps);
          if (tid < nr) out[tid] = h0;
          if (tid + kLayerThreads < nr) out[tid + kLayerThreads] = h1;
          if (tid + 2 * kLayerThreads < nr) out[tid + 2 * kLayerThreads] = h2;
          if (tid + 3 * kLayerThreads < nr) out[tid + 3 * kLayerThreads] = h3;
          continue;
        }
        if (dtype == kMXFP4) {
          for (unsigned rr = tid; rr < nr; rr += kLayerThreads)
            for (unsigned kk = 0; kk < nt; ++kk)
              out[static_cast<size_t>(kk) * S * d + rr] = down_term<kMXFP4, ACT>(slot, nr, rr, s_hq, kk, bad);
        } else {
          for (unsigned rr = tid; rr < nr; rr += kLayerThreads)
            for (unsigned kk = 0; kk < nt; ++kk)
              out[static_cast<size_t>(kk) * S * d + rr] = down_term<kQ80, ACT>(slot, nr, rr, s_hq, kk, bad);
        }
      }
      release(c, kLayerWarps);
    }
    if (r == 0) PHASE(6);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
  if (__syncthreads_or(timed_out)) aborted = true;
  PHASE(4);

  // -------------------------------------------------------- grid barrier
  if (aborted) {
    if (tid == 0) {
      atomicOr(a.status, kStTimeout);
      atomicExch(&a.ctl->abort, 1u);
    }
  } else if (!grid_sync(a.ctl, misc + 3, a.bar_inc, a.wait_ns, a.bar_extra)) {
    aborted = true;
    if (tid == 0) atomicOr(a.status, kStTimeout);
  } else if (a.world > 1 && cta == 0 && tid == 0) {
    a.ctl->peer_epoch = misc[6];  // every CTA read the previous value before it arrived
  }
  PHASE(5);
  // every part has passed its exchange: the item's first part clears the count
  if (SPLIT && H > 1 && !aborted && tid == 0)
    for (unsigned r = 0; r < n_my; ++r) {
      unsigned u, s, h, ji;
      item_us(item_at(r), u, s, h, ji);
      if (h == 0) a.xcnt[ji] = 0;
    }

  // --------------------------------------------- in-box reduce over NVLink
  // This CTA's rows of every token (this GPU's partial, s_ylocal) go to the
  // same rows of every rank's inbox, each value in one 8-byte store together
  // with this launch's epoch (peer memory over NVLink; no multicast, no
  // fence: value and epoch land together).  The receiving thread polls its
  // own inbox until every rank's entry carries the epoch (bounded wait) and
  // sums the ranks in rank order, so y is identical on every rank.  Slots
  // alternate by epoch parity: a rank writes a slot again only two launches
  // later, after every rank has read it.
  auto peer_reduce = [&](unsigned y0, unsigned R) -> bool {
    const unsigned W = a.world;
    const size_t slot_entries = static_cast<size_t>(kMaxTokens) * d;  // one source's [16][d] entries of 8 bytes
    const unsigned e = misc[6], par = e & 1;  // this launch's epoch (set before the grid barrier)
    const Div by_tr(T * R), by_r2(R);
    for (unsigned q = tid; q < W * T * R; q += kLayerThreads) {
      const unsigned dst = by_tr.q(q), rem = q - dst * T * R, t = by_r2.q(rem), rr = rem - t * R;
      if (dst == a.rank) continue;  // this rank's own share is read from shared memory
      uint2* slot = reinterpret_cast<uint2*>(a.peer[dst]) + (static_cast<size_t>(par) * W + a.rank) * slot_entries +
                    static_cast<size_t>(t) * d + y0 + rr;
      // one aligned 64-bit access: value (low word) and epoch (high word) are seen together
      const unsigned long long word =
          static_cast<unsigned long long>(__float_as_uint(s_ylocal[t * R + rr])) | static_cast<unsigned long long>(e) << 32;
      asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(word) : "memory");
    }
    const uint2* inbox = reinterpret_cast<const uint2*>(a.peer[a.rank]) + static_cast<size_t>(par) * W * slot_entries;
    bool bad_y = false, ok = true;
    const uint64_t start = globaltimer();
    for (unsigned q = tid; q < T * R && ok; q += kLayerThreads) {
      const unsigned t = by_r2.q(q), rr = q - t * R;
      float yv = 0.0f;
      for (unsigned src = 0; src < W; ++src) {
        float v;
        if (src == a.rank) {
          v = s_ylocal[t * R + rr];
        } else {
          const uint2* ent = inbox + static_cast<size_t>(src) * slot_entries + static_cast<size_t>(t) * d + y0 + rr;
          unsigned long long word;
          unsigned spins = 0;
          for (;;) {
            asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(word) : "l"(ent) : "memory");
            if (static_cast<unsigned>(word >> 32) == e) break;
            if ((++spins & 63) == 0 && globaltimer() - start > a.wait_ns) {
              ok = false;
              break;
            }
          }
          v = __uint_as_float(static_cast<unsigned>(word));
        }
        yv = __fadd_rn(yv, v);
      }
      bad_y |= !isfinite(yv);
      a.y[static_cast<size_t>(t) * d + y0 + rr] = yv;
    }
    if (!__syncthreads_and(ok)) {
      if (tid == 0) atomicOr(a.status, kStTimeout);
      return false;
    }
    if (bad_y) atomicOr(a.status, kStNumeric);
    return true;
  };

  // ------------------------------------------------------------- reduce
  // CTA k owns 4-row units [d/4*k/G, d/4*(k+1)/G): its rows of every
  // (pair, slice) term vector arrive by 16-byte cp.async into the idle ring,
  // the weights gs by plain loads, then the chains run from shared memory.
  const unsigned NU = d / 4, u0r = NU * cta / G, nu = NU * (cta + 1) / G - u0r;
  const unsigned y0 = 4 * u0r, R = 4 * nu;
  if (!aborted && R) {
    const unsigned per_tok = 11 * S * (R + 1) + 11 * R;  // floats staged per token
    const unsigned tb = max(1u, min(T, (K * SLOT) / (4 * per_tok)));  // the host checks that one token fits
    float* st = reinterpret_cast<float*>(ring);
    bool nf = false;
    for (unsigned t0 = 0; t0 < T; t0 += tb) {
      const unsigned tn = min(tb, T - t0);
      float* terms = st;                        // [tl][e][s][R]
      float* gsr = st + tn * 11 * S * R;        // [tl][e][s]
      float* part = gsr + tn * 11 * S;          // [tl][e][R]
      const Div by_nu(nu), by_s(S), by_r(R);
      for (unsigned q = tid; q < tn * 11 * S * nu; q += kLayerThreads) {
        const unsigned rest = by_nu.q(q), un = q - rest * nu, te = by_s.q(rest), s = rest - te * S;  // te = tl*11 + e
        const unsigned pair = s_tokpair[t0 * 11 + te];
        if (pair != 0xffff)
          cp_async16(terms + (te * S + s) * R + 4 * un,
                     a.partial + (static_cast<size_t>(pair) * S + s) * d + y0 + 4 * un);
      }
      cp_async_commit();
      for (unsigned q = tid; q < tn * 11 * S; q += kLayerThreads) {
        const unsigned te = by_s.q(q), s = q - te * S;
        const unsigned pair = s_tokpair[t0 * 11 + te];
        gsr[q] = pair != 0xffff ? __ldcg(a.gsv + pair * S + s) : 0.0f;
      }
      cp_async_wait_all();
      __syncthreads();
      if (t0 == 0) PHASE(11);
      for (unsigned q = tid; q < tn * 11 * R; q += kLayerThreads) {
        const unsigned te = by_r.q(q), rr = q - te * R;
        const float* tv = terms + te * S * R + rr;
        const float* gv = gsr + te * S;
        // chain j takes slices s = j mod 4 in ascending order
        float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
        unsigned s = 0;
        for (; s + 4 <= S; s += 4) {
          p0 = __fmaf_rn(tv[s * R], gv[s], p0);
          p1 = __fmaf_rn(tv[(s + 1) * R], gv[s + 1], p1);
          p2 = __fmaf_rn(tv[(s + 2) * R], gv[s + 2], p2);
          p3 = __fmaf_rn(tv[(s + 3) * R], gv[s + 3], p3);
        }
        if (s < S) p0 = __fmaf_rn(tv[s * R], gv[s], p0);
        if (s + 1 < S) p1 = __fmaf_rn(tv[(s + 1) * R], gv[s + 1], p1);
        if (s + 2 < S) p2 = __fmaf_rn(tv[(s + 2) * R], gv[s + 2], p2);
        part[q] = __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3);
      }
      __syncthreads();
      for (unsigned q = tid; q < tn * R; q += kLayerThreads) {
        const unsigned tl = by_r.q(q), rr = q - tl * R, t = t0 + tl;
        float yv = 0.0f;
        for (unsigned e = 0; e <= 10; ++e)
          if (s_tokpair[t * 11 + e] != 0xffff) yv = __fadd_rn(yv, part[(tl * 11 + e) * R + rr]);
        nf |= !isfinite(yv);
        if (a.world > 1) s_ylocal[t * R + rr] = yv;
        else a.y[static_cast<size_t>(t) * d + y0 + rr] = yv;
      }
      __syncthreads();
    }
    if (a.world > 1 && !peer_reduce(y0, R)) aborted = true;
    if (nf) atomicOr(a.status, kStNumeric);
  }
  PHASE(7);
  // Nothing may still be writing this CTA's shared memory when it leaves.
  // After an abort, wait (bounded) for the last copy issued into each slot
  // (its s_iss-th phase).
  if (aborted && tid == 0)
    for (unsigned i = 0; i < K; ++i)
      if (s_iss[i]) mbar_wait(&full[i], (s_iss[i] - 1) & 1);
}

}  // namespace frc
