// frc_layer.cuh - the MoE layer kernel (sm_100a): one cooperative launch per
// layer, one 512-thread CTA per SM, a static work split, and every byte of a
// CTA's weights requested in the first microseconds.
//
//   prologue - routing and x are loaded at once; the plan (unique experts,
//     token masks) is built in parallel.  Warp 0 starts the TMA ring for the
//     CTA's gate/up rows; warps 8-15 issue the 16-byte cp.async loads of its
//     down rows; warps 0-7 quantize x meanwhile.
//   phase 1 - gate/up.  Items (unique expert u, loaded slice s) are laid out
//     item-major as 32 neurons each; CTA c owns neurons [N*c/G, N*(c+1)/G),
//     in chunks of up to 16 neurons (one warp each).  Hidden values go to HBM.
//   grid barrier (bounded wait).
//   phase 2 - down.  CTA c owns output rows [d*c/G, d*(c+1)/G) of every
//     token: it quantizes the hidden slices it needs (src/q4.c:37-61 scheme,
//     one group of 32), forms its rows of every expert's down projection and
//     writes its rows of y (no partial sums leave the CTA).
//
// Arithmetic order (restated by the oracle's or_port_run): gate/up lanes take
// x groups p = lane, lane+32, ...; butterfly sum; per (expert, token, row) four
// slice-interleaved fmaf chains combined ((p0+p1)+p2)+p3; per token its experts
// in its own routing order, then the shared expert.
#pragma once
#include "frc_device.cuh"

namespace frc {

constexpr unsigned kLayerThreads = 512;
constexpr unsigned kLayerWarps = kLayerThreads / 32;
constexpr unsigned kActThreads = 256;          // warps 0-7: activations; 8-15: down-row loads
constexpr unsigned kSlots = 4;                 // TMA ring depth (phase 1)
constexpr unsigned kGuChunk = 16;              // neurons per gate/up chunk (one per warp)
constexpr unsigned kMaxItems = kMaxUnique * kMaxBlocks;
constexpr unsigned kXRegs = 4;                 // float4 activations a thread keeps in registers
constexpr unsigned kMaxRounds = 64;            // 256-float4 rounds of the activation pass

struct LayerCtl {
  unsigned bar_count, bar_gen;  // generation barrier: count returns to 0, gen only grows
  unsigned abort;               // set by a CTA whose bounded wait ran out
  unsigned pad;
};

struct LayerSmem {
  unsigned ids, gates, first, uid, umask, ugate, upre, rms, bases, rpart, pairs, tokpair;
  unsigned xq, xp, xs, xv, xf, split, ring, p2, total;
  unsigned slot_bytes, p2_bytes, chunk;
};

struct LayerParams {
  const uint8_t* base[kMaxBlocks];
  const uint16_t* expert;
  const float* gate;
  const float* x;
  const float* x_add;
  float* x_out;
  float* y;
  float* hidden;     // [item][T][32] fp32
  LayerCtl* ctl;
  unsigned* status;
  unsigned long long* phases;  // FRC_PHASES builds: [cta][16] globaltimer stamps
  LayerSmem sm;
  unsigned S, T, d, norm, rmax;
  unsigned gate_type, down_type;
  unsigned row_bytes, proj_bytes, shared_row, shared_proj, slice_bytes;
};

__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Barrier among the activation warps (0-7) only.
__device__ __forceinline__ void act_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Bounded generation barrier over the co-resident grid.
__device__ __forceinline__ bool grid_sync(LayerCtl* ctl, unsigned* flag_smem) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned gen = ld_acquire(&ctl->bar_gen);
    bool ok = true;
    if (atomicAdd(&ctl->bar_count, 1u) == gridDim.x - 1) {
      atomicExch(&ctl->bar_count, 0u);
      __threadfence();
      st_release(&ctl->bar_gen, gen + 1);
    } else {
      const uint64_t start = globaltimer();
      unsigned spins = 0;
      while (ld_acquire(&ctl->bar_gen) == gen) {
        if ((++spins & 255) == 0 && (globaltimer() - start > kWaitNs || ld_acquire(&ctl->abort))) {
          ok = false;
          break;
        }
      }
    }
    *flag_smem = ok;
  }
  __syncthreads();
  return *flag_smem != 0;
}

// Compile-time phase stamps (the reference's FR_PHASES counterpart,
// backends/avx2.c:38-42): entry, plan, loads issued, activations, phase 1,
// barrier, phase 2, exit.
#ifdef FRC_PHASES
#define PHASE_AT(k, th) \
  do { if (threadIdx.x == (th) && a.phases) a.phases[blockIdx.x * 16 + (k)] = globaltimer(); } while (0)
#else
#define PHASE_AT(k, th) do { } while (0)
#endif
#define PHASE(k) PHASE_AT(k, 0)

template <int ACT>
__global__ void __launch_bounds__(kLayerThreads, 1) moe_layer_kernel(const LayerParams a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);                 // kSlots mbarriers
  unsigned* misc = reinterpret_cast<unsigned*>(smem + 64);           // 64 words
  uint16_t* s_ids = reinterpret_cast<uint16_t*>(smem + a.sm.ids);
  float* s_g = reinterpret_cast<float*>(smem + a.sm.gates);
  int* s_first = reinterpret_cast<int*>(smem + a.sm.first);
  uint16_t* s_uid = reinterpret_cast<uint16_t*>(smem + a.sm.uid);
  unsigned* s_umask = reinterpret_cast<unsigned*>(smem + a.sm.umask);
  float* s_ugate = reinterpret_cast<float*>(smem + a.sm.ugate);
  unsigned* s_upre = reinterpret_cast<unsigned*>(smem + a.sm.upre);  // first pair of each expert
  float* s_rms = reinterpret_cast<float*>(smem + a.sm.rms);
  const uint8_t** s_base = reinterpret_cast<const uint8_t**>(smem + a.sm.bases);
  float* s_rpart = reinterpret_cast<float*>(smem + a.sm.rpart);      // [round][warp] sums of squares
  uint16_t* s_pair = reinterpret_cast<uint16_t*>(smem + a.sm.pairs);   // pair -> expert << 5 | token
  uint16_t* s_tokpair = reinterpret_cast<uint16_t*>(smem + a.sm.tokpair);  // [token][11] -> pair
  uint8_t* ring = smem + a.sm.ring;
  uint8_t* p2 = smem + a.sm.p2;
  float* split = reinterpret_cast<float*>(smem + a.sm.split);      // [pair][row][4]
  const unsigned SLOT = a.sm.slot_bytes;

  const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned T = a.T, S = a.S, d = a.d, P = d / 64, G = gridDim.x, cta = blockIdx.x;
  const unsigned per_token = d / 4, nvec = T * per_token, rounds = (nvec + kActThreads - 1) / kActThreads;
  const bool xregs = rounds <= kXRegs;

  PHASE(0);
  // ------------------------------------------------ loads that need nothing
  float4 xv4[kXRegs];
  if (tid < kActThreads && xregs) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const float4* xa4 = reinterpret_cast<const float4*>(a.x_add);
#pragma unroll
    for (unsigned r = 0; r < kXRegs; ++r) {
      const unsigned f = r * kActThreads + tid;
      xv4[r] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (r < rounds && f < nvec) {
        xv4[r] = x4[f];
        if (xa4) {
          const float4 w = xa4[f];
          xv4[r].x = __fadd_rn(xv4[r].x, w.x); xv4[r].y = __fadd_rn(xv4[r].y, w.y);
          xv4[r].z = __fadd_rn(xv4[r].z, w.z); xv4[r].w = __fadd_rn(xv4[r].w, w.w);
        }
      }
    }
  }
  if (tid == 0) {
    for (unsigned i = 0; i < kSlots; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  for (unsigned i = tid; i < T * 10; i += kLayerThreads) s_ids[i] = a.expert[i];
  for (unsigned i = tid; i < T * 11; i += kLayerThreads) s_g[i] = a.gate[i];
  for (unsigned i = tid; i < S; i += kLayerThreads) s_base[i] = a.base[i];
  for (unsigned i = tid; i < 512; i += kLayerThreads) s_first[i] = 0x7fffffff;
  for (unsigned i = tid; i < kMaxUnique; i += kLayerThreads) s_umask[i] = 0;
  for (unsigned i = tid; i < kMaxUnique * T; i += kLayerThreads) s_ugate[i] = 0.0f;
  __syncthreads();
  PHASE(8);

  // ---------------------------------------------------------------- plan
  if (T == 1) {
    // one token: its ten experts in request order are the unique experts
    if (tid < 10) {
      unsigned id = s_ids[tid];
      if (id >= 512) {
        atomicOr(a.status, kStInvalid);
        id = 0;  // keeps every address in range; the launch reports INVALID
      }
      s_uid[tid] = static_cast<uint16_t>(id);
      s_umask[tid] = 1;
      s_ugate[tid] = s_g[tid];
    }
    if (tid == 0) misc[4] = 10;
  } else {
  {
    bool invalid = false;
    for (unsigned i = tid; i < T * 10; i += kLayerThreads) {
      const unsigned id = s_ids[i];
      if (id < 512) atomicMin(&s_first[id], static_cast<int>(i));
      else invalid = true;
    }
    if (invalid) atomicOr(a.status, kStInvalid);
  }
  __syncthreads();
  {
    const unsigned i = tid;  // T*10 <= 160 < kLayerThreads
    const bool first = i < T * 10 && s_ids[i] < 512 && s_first[s_ids[i]] == static_cast<int>(i);
    const unsigned ballot = __ballot_sync(0xffffffffu, first);
    if (lane == 0) misc[16 + warp] = __popc(ballot);
    __syncthreads();
    unsigned off = 0;
    for (unsigned w = 0; w < warp; ++w) off += misc[16 + w];
    const unsigned rank = off + __popc(ballot & ((1u << lane) - 1));
    if (tid == kLayerThreads - 1) misc[4] = off + __popc(ballot);  // routed experts
    if (first) s_uid[rank] = s_ids[i];
    __syncthreads();
    if (first) s_first[s_ids[i]] = -1 - static_cast<int>(rank);
    __syncthreads();
  }
  for (unsigned i = tid; i < T * 10; i += kLayerThreads) {
    const unsigned id = s_ids[i];
    if (id >= 512) continue;
    const unsigned u = static_cast<unsigned>(-1 - s_first[id]), t = i / 10;
    atomicOr(&s_umask[u], 1u << t);
    s_ugate[u * T + t] = s_g[t * 11 + i % 10];
  }
  }
  __syncthreads();
  const unsigned UR = misc[4];  // routed experts
  unsigned shared_mask = 0;
  for (unsigned t = 0; t < T; ++t)
    if (s_g[t * 11 + 10] != 0.0f) shared_mask |= 1u << t;
  const unsigned U = UR + (shared_mask ? 1 : 0);
  if (shared_mask) {
    if (tid == 0) {
      s_uid[UR] = 512;
      s_umask[UR] = shared_mask;
    }
    for (unsigned t = tid; t < T; t += kLayerThreads) s_ugate[UR * T + t] = s_g[t * 11 + 10];
  }
  __syncthreads();
  if (warp == 0) {  // pair offsets: exclusive scan of the token counts, 6 experts a lane
    unsigned cnt[6], tot = 0;
#pragma unroll
    for (unsigned k = 0; k < 6; ++k) {
      const unsigned u = lane * 6 + k;
      cnt[k] = u < U ? __popc(s_umask[u]) : 0;
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
      if (u <= U) s_upre[u] = run;
      run += cnt[k];
    }
  }
  __syncthreads();
  for (unsigned u = tid; u < U; u += kLayerThreads) {  // pair -> (expert, token) and (token, slot) -> pair
    unsigned mm = s_umask[u], k = s_upre[u];
    while (mm) {
      const unsigned t = __ffs(mm) - 1;
      mm &= mm - 1;
      s_pair[k++] = static_cast<uint16_t>(u << 5 | t);
    }
  }
  for (unsigned i = tid; i < T * 11; i += kLayerThreads) {
    const unsigned t = i / 11, e = i % 11;
    unsigned pair = 0xffff;
    if (e < 10) {
      const unsigned id = s_ids[t * 10 + e];
      if (id < 512) {
        const unsigned u = T == 1 ? e : static_cast<unsigned>(-1 - s_first[id]);
        pair = s_upre[u] + __popc(s_umask[u] & ((1u << t) - 1));
      }
    } else if (shared_mask >> t & 1) {
      pair = s_upre[UR] + __popc(shared_mask & ((1u << t) - 1));
    }
    s_tokpair[i] = static_cast<uint16_t>(pair);
  }
  __syncthreads();

  PHASE(10);
  // -------------------------------------------------- this CTA's work
  const unsigned NR = UR * S * 32, N1 = U * S * 32;
  const unsigned n_begin = N1 * cta / G, n_end = N1 * (cta + 1) / G;  // N1*G < 2^32
  const unsigned r0 = d * cta / G, r1 = d * (cta + 1) / G;
  const unsigned R = r1 - r0;
  // gate/up chunks: a grid of cr neurons over routed items, cs over shared ones
  // (both divide 32, so no chunk crosses an item)
  const unsigned cr = a.sm.chunk;
  unsigned cs = kGuChunk;
  while (cs > 2 && 2 * cs * a.shared_row > SLOT) cs >>= 1;
  const unsigned m0 = n_begin / cr, m1 = n_begin < NR ? (min(n_end, NR) + cr - 1) / cr : m0;
  const unsigned n_rch = m1 - m0;
  const unsigned s_lo = n_end > NR ? (max(n_begin, NR) - NR) / cs : 0;
  const unsigned n_sch = n_end > NR ? (n_end - NR + cs - 1) / cs - s_lo : 0;
  const unsigned n_gu = n_rch + n_sch;
  auto chunk = [&](unsigned jj, unsigned& lo, unsigned& hi) {
    if (jj < n_rch) {
      lo = max(n_begin, (m0 + jj) * cr);
      hi = min(min(n_end, NR), (m0 + jj + 1) * cr);
    } else {
      const unsigned k = s_lo + jj - n_rch;
      lo = max(n_begin, NR + k * cs);
      hi = min(n_end, NR + (k + 1) * cs);
    }
  };
  // One item's piece of the down projection for rows [r0, r1): the scale
  // bytes widened to 16-byte boundaries, then the rows' payloads.
  const unsigned mx_lo = r0 & ~15u, mx_hi = (r1 + 15) & ~15u;            // MXFP4: 1 scale byte a row
  const unsigned q8_lo = (2 * r0) & ~15u, q8_hi = (2 * r1 + 15) & ~15u;  // Q8_0: 2 bytes a row
  const unsigned piece_mx = (mx_hi - mx_lo) + 16 * R, piece_q8 = (q8_hi - q8_lo) + 32 * R;
  const unsigned piece_r = a.down_type == kQ80 ? piece_q8 : piece_mx;
  // phase-2 batches: every expert at once when it fits, else k at a time
  const unsigned ent_bytes = ACT == FRC_ACT_Q8 ? 36 : 132;  // staged hidden slice + its scale
  const unsigned all_bytes = S * (UR * piece_r + (U - UR) * piece_q8) + S * s_upre[U] * ent_bytes;
  const unsigned per_batch =
      all_bytes <= a.sm.p2_bytes ? U : max(1u, a.sm.p2_bytes / (S * piece_q8 + S * T * ent_bytes));
  const unsigned n_batch = R ? (U + per_batch - 1) / per_batch : 0;
  // offset of item (u, s) in the batch that starts at expert u0
  auto piece_off = [&](unsigned u0, unsigned u, unsigned s) {
    const unsigned ur = min(u, UR) > u0 ? min(u, UR) - u0 : 0;
    return ur * S * piece_r + s * (u >= UR ? piece_q8 : piece_r);
  };
  auto batch_pieces = [&](unsigned u0, unsigned u1) {
    const unsigned ur = min(u1, UR) > u0 ? min(u1, UR) - u0 : 0;
    return S * (ur * piece_r + (u1 > UR ? piece_q8 : 0));
  };

  // ------------------------------------------------ phase-1 producer (TMA)
  auto issue = [&](unsigned jj) {  // one lane per chunk
    unsigned lo, hi;
    chunk(jj, lo, hi);
    const unsigned item = lo / 32, u = item / S, si = item % S, cnt = hi - lo;
    const bool shared = u >= UR;
    const unsigned rowb = shared ? a.shared_row : a.row_bytes, proj = shared ? a.shared_proj : a.proj_bytes;
    const uint8_t* src = s_base[si] + static_cast<size_t>(s_uid[u]) * a.slice_bytes + (lo % 32) * rowb;
    const unsigned slot = jj % kSlots;
    uint8_t* dst = ring + slot * SLOT;
    mbar_expect_tx(&bar[slot], 2 * cnt * rowb);
    bulk_g2s(dst, src, cnt * rowb, &bar[slot]);
    bulk_g2s(dst + cnt * rowb, src + proj, cnt * rowb, &bar[slot]);
  };
  if (warp == 0 && lane < kSlots && lane < n_gu) issue(lane);

  // --------------------------------------- phase-2 loads: one warp per item
  auto issue_batch = [&](unsigned bi, unsigned w0, unsigned nw) {
    const unsigned u0 = bi * per_batch, u1 = min(U, u0 + per_batch);
    for (unsigned it = w0; it < (u1 - u0) * S; it += nw) {
      const unsigned u = u0 + it / S, s = it % S;
      const bool q8 = u >= UR || a.down_type == kQ80;
      const unsigned proj = u >= UR ? a.shared_proj : a.proj_bytes;
      const uint8_t* down = s_base[s] + static_cast<size_t>(s_uid[u]) * a.slice_bytes + 2 * proj;
      const unsigned lo = q8 ? q8_lo : mx_lo, hi = q8 ? q8_hi : mx_hi, pb = q8 ? 32 : 16;
      const unsigned ce = (hi - lo) / 16, cpe = ce + pb * R / 16;
      uint8_t* dst = p2 + piece_off(u0, u, s);
      for (unsigned k = lane; k < cpe; k += 32)
        cp_async16(dst + 16 * k, k < ce ? down + lo + 16 * k : down + (q8 ? 2 : 1) * d + pb * r0 + 16 * (k - ce));
    }
    cp_async_commit();
  };
  PHASE(1);

  if (warp >= kActThreads / 32) {
    // ---------------------------------------- warps 8-15: down-row loads
    if (n_batch) issue_batch(0, warp - kActThreads / 32, kLayerWarps - kActThreads / 32);
    PHASE_AT(11, kActThreads);
  } else {
    // --------------------------------------------- warps 0-7: activations
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const float4* xa4 = reinterpret_cast<const float4*>(a.x_add);
    auto load4 = [&](unsigned f, unsigned r) {
      float4 v = xv4[0];
      if (xregs) {
#pragma unroll
        for (unsigned q = 0; q < kXRegs; ++q) if (q == r) v = xv4[q];
        return v;
      }
      v = x4[f];
      if (xa4) {
        const float4 w = xa4[f];
        v.x = __fadd_rn(v.x, w.x); v.y = __fadd_rn(v.y, w.y); v.z = __fadd_rn(v.z, w.z); v.w = __fadd_rn(v.w, w.w);
      }
      return v;
    };
    bool bad = false;
    if (a.norm) {
      // sums of squares per (round, warp); every warp-round lies in one token
      for (unsigned r = 0; r < rounds; ++r) {
        const unsigned f = r * kActThreads + tid;
        float ss = 0.0f;
        if (f < nvec) {
          const float4 v = load4(f, r);
          ss = __fmaf_rn(v.x, v.x, ss); ss = __fmaf_rn(v.y, v.y, ss);
          ss = __fmaf_rn(v.z, v.z, ss); ss = __fmaf_rn(v.w, v.w, ss);
        }
#pragma unroll
        for (unsigned o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if (lane == 0) s_rpart[r * 8 + warp] = ss;
      }
      act_sync();
      PHASE(2);
      for (unsigned t = tid; t < T; t += kActThreads) {
        float tot = 0.0f;
        for (unsigned r = 0; r < rounds; ++r)
          for (unsigned w = 0; w < 8; ++w) {
            const unsigned f = r * kActThreads + w * 32;
            if (f < nvec && f / per_token == t) tot = __fadd_rn(tot, s_rpart[r * 8 + w]);
          }
        s_rms[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(d)), 1e-6f)));
      }
      act_sync();
    }
    for (unsigned r = 0; r < rounds; ++r) {
      const unsigned f = r * kActThreads + tid;
      if (f >= nvec) continue;  // warp-uniform: nvec is a multiple of 128
      float4 v = load4(f, r);
      const unsigned t = f / per_token, j = f % per_token;
      bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
      if (a.x_out && cta == 0) reinterpret_cast<float4*>(a.x_out)[f] = v;
      if (a.norm) {
        const float g = s_rms[t];
        v.x = __fmul_rn(v.x, g); v.y = __fmul_rn(v.y, g); v.z = __fmul_rn(v.z, g); v.w = __fmul_rn(v.w, g);
      }
      if (ACT == FRC_ACT_F32) {
        reinterpret_cast<float4*>(smem + a.sm.xf)[f] = v;
        continue;
      }
      float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
      for (unsigned o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const Q8Group qg(amax);
      const float scale = qg.scale;
      const int q0 = qg.q(v.x), q1 = qg.q(v.y), q2 = qg.q(v.z), q3 = qg.q(v.w);
      int sum = q0 + q1 + q2 + q3;
#pragma unroll
      for (unsigned o = 4; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const unsigned p = j / 16, wq = j % 16;
      uint8_t* xt = smem + a.sm.xq + t * d;
      const uint32_t word = (q0 & 0xff) | (q1 & 0xff) << 8 | (q2 & 0xff) << 16 | static_cast<uint32_t>(q3 & 0xff) << 24;
      *reinterpret_cast<uint32_t*>(xt + 16 * xslot(p, wq / 4) + 4 * (wq % 4)) = word;
      if ((lane & 15) == 0) reinterpret_cast<float*>(smem + a.sm.xs)[t * P + p] = scale;
      if ((lane & 7) == 0)
        reinterpret_cast<float*>(smem + a.sm.xv)[t * 2 * P + 2 * p + ((lane >> 3) & 1)] = static_cast<float>(sum);
      if (a.sm.xp) {
        uint8_t* xp = smem + a.sm.xp + t * d;
        const int qv[4] = {q0, q1, q2, q3};
#pragma unroll
        for (unsigned i = 0; i < 4; ++i) {
          const unsigned e = 4 * j + i, wi = (e % 64) / 32 * 32 + prmt_pos(e % 32);
          xp[16 * xslot(p, wi / 16) + wi % 16] = static_cast<uint8_t>(qv[i] & 0xff);
        }
      }
    }
    if (bad) atomicOr(a.status, kStNumeric);
    PHASE(14);
  }
  __syncthreads();
  PHASE(3);

  // ------------------------------------------------------------- phase 1
  bool aborted = false;
  unsigned j = 0;
  for (; j < n_gu; ++j) {
    const bool ok = mbar_wait(&bar[j % kSlots], (j / kSlots) & 1);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        atomicOr(a.status, kStTimeout);
        atomicExch(&a.ctl->abort, 1u);
      }
      aborted = true;
      break;
    }
    if (j == 0) PHASE(15);
    unsigned lo, hi;
    chunk(j, lo, hi);
    const uint8_t* slot = ring + (j % kSlots) * SLOT;
    const unsigned item = lo / 32, u = item / S, nl = lo % 32, cnt = hi - lo;
    const bool shared = u >= UR;
    const unsigned type = shared ? kQ80 : a.gate_type;
    const unsigned rowb = shared ? a.shared_row : a.row_bytes, nb = d / 32;
    bool bad = false;
    if (warp < cnt) {
      const unsigned n = nl + warp;
      const uint8_t* grow = slot + warp * rowb;
      const uint8_t* urow = slot + (cnt + warp) * rowb;
      unsigned mm = s_umask[u];
      while (mm) {
        const unsigned t = __ffs(mm) - 1;
        mm &= mm - 1;
        float ag = 0.0f, au = 0.0f;
        if (ACT == FRC_ACT_Q8) {
          const uint8_t* xq = smem + (type == kMXFP4 ? a.sm.xp : a.sm.xq) + t * d;
          const float* xs = reinterpret_cast<const float*>(smem + a.sm.xs) + t * P;
          const float* xv = reinterpret_cast<const float*>(smem + a.sm.xv) + t * 2 * P;
          for (unsigned p = lane; p < P; p += 32) {
            uint32_t xw[16];
            load_x16(xq, p, xw);
            float tg, tu;
            if (type == kQ4K) {
              const float v0 = xv[2 * p], v1 = xv[2 * p + 1];
              tg = term_q4k(grow, p, xw, v0, v1, bad);
              tu = term_q4k(urow, p, xw, v0, v1, bad);
            } else if (type == kMXFP4) {
              tg = term_mxfp4(grow, nb, p, xw, bad);
              tu = term_mxfp4(urow, nb, p, xw, bad);
            } else {
              tg = term_q80(grow, nb, p, xw, bad);
              tu = term_q80(urow, nb, p, xw, bad);
            }
            ag = __fmaf_rn(xs[p], tg, ag);
            au = __fmaf_rn(xs[p], tu, au);
          }
        } else {
          const float* xf = reinterpret_cast<const float*>(smem + a.sm.xf) + t * d;
          for (unsigned p = lane; p < P; p += 32)
            for (unsigned jj = 0; jj < 64; ++jj) {
              const unsigned e = 64 * p + jj;
              const float wg = weight_any(grow, type, d, e), wu = weight_any(urow, type, d, e);
              bad |= !isfinite(wg) || !isfinite(wu);
              ag = __fmaf_rn(wg, xf[e], ag);
              au = __fmaf_rn(wu, xf[e], au);
            }
        }
#pragma unroll
        for (unsigned o = 16; o; o >>= 1) {
          ag = __fadd_rn(ag, __shfl_xor_sync(0xffffffffu, ag, o));
          au = __fadd_rn(au, __shfl_xor_sync(0xffffffffu, au, o));
        }
        if (lane == 0) {
          float h = 0.0f;
          if (!isfinite(ag) || !isfinite(au) || !swiglu(ag, au, &h)) bad = true;
          a.hidden[(static_cast<size_t>(item) * T + t) * 32 + n] = h;
        }
      }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
    if (j == 0) PHASE(9);
    __syncthreads();
    if (warp == 0 && lane == 0 && j + kSlots < n_gu) {
      fence_proxy_async();
      issue(j + kSlots);
    }
  }

  // -------------------------------------------------------- grid barrier
  PHASE(4);
  if (!aborted && !grid_sync(a.ctl, misc + 3)) {
    aborted = true;
    if (tid == 0) atomicOr(a.status, kStTimeout);
  }
  PHASE(5);

  // ------------------------------------------------------------- phase 2
  for (unsigned bi = 0; bi < n_batch && !aborted; ++bi) {
    const unsigned u0 = bi * per_batch, u1 = min(U, u0 + per_batch);
    if (bi) issue_batch(bi, warp, kLayerWarps);
    // quantize the hidden slices of this batch: entry (pair, s), pair = token k of expert u
    const unsigned pair0 = s_upre[u0], npair = s_upre[u1] - pair0, E = S * npair;
    uint8_t* hqs = p2 + batch_pieces(u0, u1);
    float* gss = reinterpret_cast<float*>(hqs + (ACT == FRC_ACT_Q8 ? 32 : 128) * E);
    constexpr unsigned kEnt = 16;  // entries a warp keeps in flight
    for (unsigned e0 = warp; e0 < E; e0 += kLayerWarps * kEnt) {
      float hv[kEnt];
#pragma unroll
      for (unsigned z = 0; z < kEnt; ++z) {
        const unsigned ent = e0 + z * kLayerWarps;
        hv[z] = 0.0f;
        if (ent < E) {
          const unsigned pu = s_pair[pair0 + ent / S], s = ent % S;
          hv[z] = __ldcg(&a.hidden[((static_cast<size_t>(pu >> 5) * S + s) * T + (pu & 31)) * 32 + lane]);
        }
      }
#pragma unroll
      for (unsigned z = 0; z < kEnt; ++z) {
        const unsigned ent = e0 + z * kLayerWarps;
        if (ent >= E) break;
        const unsigned pu = s_pair[pair0 + ent / S], u = pu >> 5, t = pu & 31;
        if (ACT == FRC_ACT_Q8) {
          float amax = fabsf(hv[z]);
#pragma unroll
          for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
          const Q8Group qg(amax);
          const int v = qg.q(hv[z]);
          const bool mxd = u < UR && a.down_type == kMXFP4;
          hqs[ent * 32 + (mxd ? prmt_pos(lane) : lane)] = static_cast<uint8_t>(v & 0xff);
          if (lane == 0) gss[ent] = __fmul_rn(qg.scale, s_ugate[u * T + t]);
        } else {
          reinterpret_cast<float*>(hqs)[ent * 32 + lane] = hv[z];  // fp32 mode keeps the hidden values
          if (lane == 0) gss[ent] = s_ugate[u * T + t];
        }
      }
    }
    cp_async_wait_all();
    PHASE(12);
    __syncthreads();
    PHASE(13);
    const unsigned tasks = npair * R * kDnSplit;
    bool bad = false;
    for (unsigned task = tid; task < tasks; task += kLayerThreads) {
      const unsigned q = task % kDnSplit, rr = (task / kDnSplit) % R, pair = pair0 + task / (kDnSplit * R);
      const unsigned u = s_pair[pair] >> 5;
      const bool q8 = u >= UR || a.down_type == kQ80;
      const unsigned pb = u >= UR ? piece_q8 : piece_r, lo = q8 ? q8_lo : mx_lo, hi = q8 ? q8_hi : mx_hi;
      const uint8_t* ubase = p2 + piece_off(u0, u, 0);
      const unsigned r = r0 + rr;
      float acc = 0.0f;
      for (unsigned s = q; s < S; s += kDnSplit) {
        const uint8_t* pc = ubase + s * pb;
        const unsigned ent = (pair - pair0) * S + s;
        const float g = gss[ent];
        float cterm;
        if (ACT == FRC_ACT_Q8) {
          const uint4 h0 = reinterpret_cast<const uint4*>(hqs)[2 * ent];
          const uint4 h1 = reinterpret_cast<const uint4*>(hqs)[2 * ent + 1];
          const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
          if (!q8) {
            const unsigned e = pc[r - lo];
            bad |= e == 255;
            const uint4 w = *reinterpret_cast<const uint4*>(pc + (hi - lo) + 16 * rr);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            int ip = 0, in = 0;
#pragma unroll
            for (unsigned m = 0; m < 4; ++m) {
              ip = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, ww[m])), static_cast<int>(hw[2 * m]), ip);
              in = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, ww[m] ^ 0x8888u)), static_cast<int>(hw[2 * m]), in);
              ip = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, ww[m] >> 16)), static_cast<int>(hw[2 * m + 1]), ip);
              in = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, (ww[m] >> 16) ^ 0x8888u)),
                          static_cast<int>(hw[2 * m + 1]), in);
            }
            cterm = __fmul_rn(pow2_m128(e), i2f(ip - in));
          } else {
            const float sw = h2f(pc[2 * r - lo] | pc[2 * r - lo + 1] << 8);
            bad |= !isfinite(sw);
            const uint4* wv = reinterpret_cast<const uint4*>(pc + (hi - lo) + 32 * rr);
            const uint4 w0 = wv[0], w1 = wv[1];
            const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            int iv = 0;
#pragma unroll
            for (unsigned m = 0; m < 8; ++m) iv = __dp4a(static_cast<int>(ww[m]), static_cast<int>(hw[m]), iv);
            cterm = __fmul_rn(sw, i2f(iv));
          }
        } else {
          const float* hvf = reinterpret_cast<const float*>(hqs) + ent * 32;
          float dot = 0.0f;
          if (!q8) {
            const unsigned e = pc[r - lo];
            bad |= e == 255;
            const float sc = __uint_as_float(e ? e << 23 : 0x00400000u);
            const uint8_t* qb = pc + (hi - lo) + 16 * rr;
            for (unsigned nn = 0; nn < 32; ++nn)
              dot = __fmaf_rn(__fmul_rn(sc, e2m1((qb[nn & 15] >> (nn >> 4 ? 4 : 0)) & 15)), hvf[nn], dot);
          } else {
            const float sw = h2f(pc[2 * r - lo] | pc[2 * r - lo + 1] << 8);
            bad |= !isfinite(sw);
            const int8_t* qb = reinterpret_cast<const int8_t*>(pc + (hi - lo) + 32 * rr);
            for (unsigned nn = 0; nn < 32; ++nn) dot = __fmaf_rn(__fmul_rn(sw, static_cast<float>(qb[nn])), hvf[nn], dot);
          }
          cterm = dot;
        }
        acc = __fmaf_rn(cterm, g, acc);
      }
      split[(pair * R + rr) * kDnSplit + q] = acc;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
    __syncthreads();  // p2 is rewritten by the next batch
  }
  PHASE(6);
  // every token's rows: its experts in its routing order, then the shared expert
  if (!aborted && R) {
    bool nf = false;
    for (unsigned idx = tid; idx < T * R; idx += kLayerThreads) {
      const unsigned t = idx / R, rr = idx % R;
      float yv = 0.0f;
      for (unsigned e = 0; e <= 10; ++e) {
        const unsigned pair = s_tokpair[t * 11 + e];
        if (pair == 0xffff) continue;
        const float* sp = split + (pair * R + rr) * kDnSplit;
        float part = sp[0];
        for (unsigned z = 1; z < kDnSplit; ++z) part = __fadd_rn(part, sp[z]);
        yv = __fadd_rn(yv, part);
      }
      nf |= !isfinite(yv);
      a.y[static_cast<size_t>(t) * d + r0 + rr] = yv;
    }
    if (nf) atomicOr(a.status, kStNumeric);
  }
  PHASE(7);
  // nothing may still be writing this CTA's shared memory when it leaves
  cp_async_wait_all();
  if (aborted)
    for (unsigned jj = j; jj < n_gu && jj < j + kSlots; ++jj) mbar_wait(&bar[jj % kSlots], (jj / kSlots) & 1);
}

}  // namespace frc
