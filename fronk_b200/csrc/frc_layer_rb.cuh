// frc_layer_rb.cuh - the one-token MoE layer kernel with row-owner down
// projections (sm_100a).  One launch per layer; every CTA of the grid works
// in both of its phases.
//
//   phase A - gate/up.  The layer's gate/up work is cut into chunks of kn
//     neurons of one item (an item is a unique expert u and a loaded slice
//     s: 8 neurons routed, 4 for the shared expert's longer Q8_0 rows), dealt
//     to all CTAs in snake order, the shared expert's chunks first.  A chunk
//     is one ring copy (its gate rows, then its up rows); kn/4 warps compute
//     its neurons exactly as moe_layer_kernel does (exact block terms in
//     double, SwiGLU in double) and store the fp32 hidden values to global
//     memory, [u*S + s][32].  Meanwhile the plan warps prefetch, by 16-byte
//     cp.async, the down rows this CTA owns (4-row units [y0, y0 + R)) of
//     every item, with their scales.
//   grid barrier (bounded wait).
//   phase B - each CTA reads every item's 32 hidden values, quantizes them
//     (Q8 per 32, src/q4.c:37-61), forms its rows' down terms c = scale *
//     int_dot and sums them in moe_layer_kernel's reduce order: per routing
//     slot four slice-interleaved fmaf chains of c * gs, combined
//     ((p0+p1)+p2)+p3, then the slots in request order, then the shared
//     expert.  The values and their order are those of moe_layer_kernel
//     (restated by the oracle's or_port_run); only who computes what moves.
//
// Against moe_layer_kernel at one token: 800 chunks over 296 CTAs instead of
// 200 items (a third of the grid idle), and the down terms never leave the
// chip (the item kernel writes and re-reads 1.6 MB of them a layer).
#pragma once
#include "frc_layer.cuh"

namespace frc {

__global__ void __launch_bounds__(kLayerThreads, 2) moe_layer_rb_kernel(const LayerParams a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);                // kMaxSlots mbarriers
  unsigned* misc = reinterpret_cast<unsigned*>(smem + 64);           // 64 words
  unsigned* s_cnt = misc + 40;                                       // ring slot: readers done with its chunk
  unsigned* s_iss = misc + 48;                                       // ring slot: chunks issued into it
  uint64_t* dnbar = reinterpret_cast<uint64_t*>(misc + 56);           // the down-row copies (phase B)
  uint16_t* s_uid = reinterpret_cast<uint16_t*>(smem + a.sm.uid);
  float* s_ugate = reinterpret_cast<float*>(smem + a.sm.ugate);
  float* s_ylocal = reinterpret_cast<float*>(smem + a.sm.ylocal);    // [rows]: this GPU's partial (peer reduce)
  uint8_t* ring = smem + a.sm.ring;
  uint8_t* dnb = smem + a.sm.dnb;                                    // this CTA's down rows of every item
  const unsigned SLOT = a.sm.slot_bytes, K = a.sm.slots;

  const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned S = a.S, d = a.d, G = gridDim.x, cta = blockIdx.x;

  PHASE(0);
  pdl_signal();
  // rows of y this CTA owns: 4-row units [NU*cta/G, NU*(cta+1)/G)
  const unsigned NU = d / 4, u0r = NU * cta / G, nu = NU * (cta + 1) / G - u0r;
  const unsigned y0 = 4 * u0r, R = 4 * nu, RM = a.sm.rows_max;

  // ------------------------------------------------------- chunk space
  // Global chunk order: the shared expert's S items x cps chunks (when a
  // token uses it), then routed items (u, s) u-major x cpr chunks.  Round r
  // deals chunks r*G .. r*G+G-1, alternating direction.
  const Div by_S(S, a.mag_S);
  const unsigned kn_r = a.sm.kn_r, kn_s = a.sm.kn_s;
  const unsigned lr = 31 - __clz(32 / kn_r), ls = 31 - __clz(32 / kn_s);  // log2 chunks per item
  unsigned UR = 10, SH = 0, U = 10, NC = 0, n_my = 0;
  auto chunk_at = [&](unsigned r) { return r * G + ((r & 1) ? G - 1 - cta : cta); };
  auto decode = [&](unsigned g, unsigned& u, unsigned& s, unsigned& k) {
    if (g < (SH << ls)) {
      u = UR;
      s = g >> ls;
      k = g & ((1u << ls) - 1);
    } else {
      const unsigned h = g - (SH << ls), it = h >> lr;
      k = h & ((1u << lr) - 1);
      u = by_S.q(it);
      s = it - u * S;
    }
  };
  auto setup = [&]() {
    SH = misc[5] ? S : 0;
    U = UR + (misc[5] ? 1 : 0);
    NC = (SH << ls) + ((UR * S) << lr);
    n_my = 0;
    while (chunk_at(n_my) < NC) ++n_my;
  };
  // chunk j of this CTA into ring slot j % K: its gate rows, then its up rows
  auto issue = [&](unsigned j) {
    unsigned u, s, k;
    decode(chunk_at(j), u, s, k);
    const bool sh = u >= UR;
    const unsigned rowb = sh ? a.shared_row : a.row_bytes, proj = sh ? a.shared_proj : a.proj_bytes;
    const unsigned kn = sh ? kn_s : kn_r, bytes = kn * rowb;
    const uint8_t* src = a.base[s] + static_cast<size_t>(s_uid[u]) * a.slice_bytes;
    const unsigned slot = j % K;
    uint8_t* dst = ring + slot * SLOT;
    reinterpret_cast<volatile unsigned*>(s_iss)[slot] = s_iss[slot] + 1;
    mbar_expect_tx(&full[slot], 2 * bytes);
    bulk_g2s(dst, src + k * bytes, bytes, &full[slot]);
    bulk_g2s(dst + bytes, src + proj + k * bytes, bytes, &full[slot]);
  };
  // down-row staging of item i = u*S + s: payload [RM][pb] then a window of
  // a.sm.dnw 16-byte pieces of the scales, from the 16-byte boundary at or
  // below row y0's scale, that covers rows [y0, y0 + R)
  const unsigned dt_r = a.down_type, ss_r = dt_r == kQ80 ? 2 : 1, pb_r = dt_r == kQ80 ? 32 : 16;
  auto dn_at = [&](unsigned u, unsigned s) -> uint8_t* {
    return dnb + (u < UR ? (u * S + s) * a.sm.dnb_r : UR * S * a.sm.dnb_r + s * a.sm.dnb_s);
  };

  if (warp >= kFirstPlanWarp) {
    // ------------------------------------------------- warps 4-7: plan
    const unsigned ptid = tid - 32 * kFirstPlanWarp, pw = warp - kFirstPlanWarp;
    if (ptid < kMaxSlots) {
      s_cnt[ptid] = 0;
      s_iss[ptid] = 0;
    }
    if (ptid == 0) {
      for (unsigned k = 0; k < K; ++k) mbar_init(&full[k], 1);
      mbar_init(dnbar, 1);
      fence_mbar_init();
      misc[7] = 0;
    }
    if (pw == 0) {
      // one token: its ten experts in request order are the unique experts
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
        s_ugate[lane] = gv;
      }
      if (lane == 10) {
        s_uid[10] = 512;
        s_ugate[10] = sg;
      }
      if (lane == 0) misc[5] = sg != 0.0f ? 1u : 0u;
      PHASE_AT(8, kPlanThreads);
    }
    plan_sync();
    PHASE_AT(10, kPlanThreads);
    setup();
    if (pw == 0) {  // the first K chunks, while the activations are being formed
      if (lane < K && lane < n_my) issue(lane);
      PHASE_AT(1, kPlanThreads);
    }
    pdl_wait();
  }
  if (warp < kActWarps) layer_input<FRC_ACT_Q8>(a, smem, 1, tid, lane, warp, cta);
  __syncthreads();
  setup();
  if (a.world > 1 && tid == 0) misc[6] = *reinterpret_cast<volatile unsigned*>(&a.ctl->peer_epoch) + 1;
  PHASE(3);
  // This CTA's down rows [y0, y0 + R) of every item for phase B: two bulk
  // copies an item (its rows' payload, and a 16-byte-aligned window of their
  // scales), issued by warps 0-3 once the activations are formed, so that
  // they queue behind the gate/up chunks and do not delay the loads of x.
  if (R && warp < kActWarps) {
    const unsigned plr = R * pb_r, pls = R * 32, win = 16 * a.sm.dnw;  // bytes: routed, shared payload; window
    if (tid == 0) mbar_expect_tx(dnbar, UR * S * (plr + win) + SH * (pls + win));
    act_sync();
    for (unsigned q = tid; q < 2 * (UR + (SH ? 1u : 0u)) * S; q += kActThreads) {
      const unsigned it = q >> 1, u = by_S.q(it), s = it - u * S;
      const bool sh = u >= UR;
      const unsigned ss = sh ? 2 : ss_r, pb = sh ? 32 : pb_r;
      const uint8_t* down = a.base[s] + static_cast<size_t>(s_uid[u]) * a.slice_bytes +
                            2 * static_cast<size_t>(sh ? a.shared_proj : a.proj_bytes);
      uint8_t* dst = dn_at(u, s);
      if ((q & 1) == 0) bulk_g2s(dst, down + static_cast<size_t>(d) * ss + y0 * pb, R * pb, dnbar);
      else bulk_g2s(dst + RM * pb, down + ((ss * y0) & ~15u), win, dnbar);
    }
  }
  PHASE(14);

  // ---------------------------------------------------------- phase A
  // Ring protocol of moe_layer_kernel: only a chunk's kn/4 readers wait for
  // it; the last to hand it back refills the slot with chunk j + K.
  bool timed_out = false, aborted = false;
  auto release = [&](unsigned j, unsigned readers) {
    __syncwarp();
    if (lane == 0 && !timed_out) {
      __threadfence_block();
      const unsigned slot = j % K;
      if (atomicAdd(&s_cnt[slot], 1u) == readers - 1) {
        s_cnt[slot] = 0;
        if (j + K < n_my) {
          __threadfence_block();
          fence_proxy_async();
          issue(j + K);
        }
      }
    }
  };
  auto wait_chunk = [&](unsigned j) {
    if (!timed_out) {
      const unsigned slot = j % K, jj = j / K;
      bool ok = true;
      if (reinterpret_cast<volatile unsigned*>(s_iss)[slot] <= jj) {
        const uint64_t start = globaltimer();
        while (reinterpret_cast<volatile unsigned*>(s_iss)[slot] <= jj)
          if (globaltimer() - start > a.wait_ns) {
            ok = false;
            break;
          }
      }
      ok = ok && mbar_wait(&full[slot], jj & 1, a.wait_ns);
      timed_out = __any_sync(0xffffffffu, !ok);
    }
    return !timed_out;
  };
  bool bad = false;
  const unsigned nspan = d / 256, nb = d / 32, l8 = lane & 7;
  // Chunks are taken four at a time: chunk j0 + (warp / 2) by warps 2(j%4) and
  // 2(j%4)+1 (a shared chunk, four neurons, by the first of them only).
  for (unsigned j0 = 0; j0 < n_my; j0 += 4) {
    const unsigned j = j0 + (warp >> 1), half = warp & 1;
    if (j < n_my) {
      unsigned u, s, k;
      decode(chunk_at(j), u, s, k);
      const bool sh = u >= UR;
      const unsigned kn = sh ? kn_s : kn_r, quads = kn / 4;
      if (half < quads) {
        if (wait_chunk(j)) {
          if (j == 0) PHASE(15);
          const unsigned type = sh ? kQ80 : a.gate_type, rowb = sh ? a.shared_row : a.row_bytes;
          const uint8_t* slot = ring + (j % K) * SLOT;
          const unsigned nl = 4 * half + (lane >> 3);  // neuron within the chunk
          const uint8_t* gr = slot + nl * rowb;
          const uint8_t* ur = slot + (kn + nl) * rowb;
          const bool mx = type == kMXFP4;
          const XAct xa{smem + (mx ? a.sm.xp : a.sm.xq), smem + (mx ? a.sm.xrp : a.sm.xr),
                        reinterpret_cast<const double2*>(smem + a.sm.xst), reinterpret_cast<const int4*>(smem + a.sm.xvr)};
          double dg = 0.0, du = 0.0;
          if (type == kQ4K) gu_sums<kQ4K>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
          else if (mx) gu_sums<kMXFP4>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
          else gu_sums<kQ80>(gr, ur, xa, l8, nspan, nb, bad, dg, du);
#pragma unroll
          for (unsigned o = 4; o; o >>= 1) {
            dg = __dadd_rn(dg, __shfl_xor_sync(0xffffffffu, dg, o));
            du = __dadd_rn(du, __shfl_xor_sync(0xffffffffu, du, o));
          }
          float ag = 0.0f, au = 0.0f, h = 0.0f;
          if (!narrow(dg, &ag) || !narrow(du, &au) || !swiglu(ag, au, &h)) {
            bad = true;
            h = 0.0f;
          }
          if (l8 == 0) a.hidden[(u * S + s) * 32 + k * kn + nl] = h;
        }
        release(j, quads);
      }
    }
  }
  if (n_my) PHASE(9);
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
  bad = false;
  if (__syncthreads_or(timed_out)) aborted = true;
  // An item's hidden slice is quantized (Q8 per 32, src/q4.c:37-61) by the
  // CTA that stores its last chunk: each CTA counts its chunks into the
  // items' arrival counters; the one that completes a count reads the 32
  // values back (L2) and writes the int8 slice and its scale, then clears
  // the counter for the next launch.
  unsigned* s_list = misc + 24;  // items this CTA completes (at most 16 chunks a CTA: checked on the host)
  if (!aborted && tid < n_my) {  // one thread a chunk, so the atomics overlap
    unsigned u, s, k;
    decode(chunk_at(tid), u, s, k);
    const unsigned item = u * S + s, per = u >= UR ? (1u << ls) : (1u << lr);
    __threadfence();
    if (atomicAdd(&a.rb_cnt[item], 1u) == per - 1) {
      a.rb_cnt[item] = 0;
      __threadfence();
      s_list[atomicAdd(&misc[7], 1u)] = item;
    }
  }
  __syncthreads();
  for (unsigned q = warp; q < misc[7]; q += kLayerWarps) {
    const unsigned item = s_list[q], u = by_S.q(item);
    const float h = __ldcg(a.hidden + item * 32 + lane);
    float amax = fabsf(h);
#pragma unroll
    for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const Q8Group qg(amax);
    const int qh = __builtin_expect(qg.mul_ok(), 1) ? qg.qm(h) : qg.q(h);
    const unsigned dtype = u >= UR ? kQ80 : dt_r;
    a.rb_hq[item * 32 + (dtype == kMXFP4 ? prmt_pos(lane) : lane)] = static_cast<uint8_t>(qh & 0xff);
    if (lane == 0) a.rb_hs[item] = qg.scale;
  }
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

  // ------------------------------------------------------------ phase B
  bool dn_landed = false;  // the down-row copies are in (or none were issued)
  if (!aborted && R) {
    if (tid == 0) misc[9] = mbar_wait(dnbar, 0, a.wait_ns) ? 1u : 0u;  // this CTA's down rows
    __syncthreads();
    dn_landed = misc[9] != 0;
    if (!dn_landed) {
      aborted = true;
      if (tid == 0) atomicOr(a.status, kStTimeout);
    }
  }
  if (!aborted && R) {
    const unsigned NI = U * S;
    uint8_t* s_hq = ring;                                                   // [item][32] int8
    float* s_gs = reinterpret_cast<float*>(ring + ((NI * 32 + 15) & ~15u));  // [item] hidden scale x gate
    float* s_terms = s_gs + ((NI + 3) & ~3u);                               // [item][R] down terms
    float* s_part = s_terms + NI * R;                                       // [slot][R]
    // B0: every item's quantized slice and scale (36 B an item); each CTA
    // starts at another item so the grid does not read one line at a time
    {
      const unsigned n16 = NI * 2, off = (cta * 7u) % n16;
      for (unsigned q = tid; q < n16; q += kLayerThreads) {
        const unsigned qq = q + off < n16 ? q + off : q + off - n16;
        cp_async16(s_hq + 16 * qq, a.rb_hq + 16 * qq);
      }
      cp_async_commit();
      for (unsigned i = tid; i < NI; i += kLayerThreads) s_gs[i] = __ldcg(a.rb_hs + i);
      cp_async_wait_all();
    }
    __syncthreads();
    for (unsigned i = tid; i < NI; i += kLayerThreads) s_gs[i] = __fmul_rn(s_gs[i], s_ugate[by_S.q(i)]);
    __syncthreads();
    PHASE(11);
    // B2: down terms of this CTA's rows, c = scale x int_dot (exact for MXFP4)
    const Div by_R(R);
    for (unsigned q = tid; q < NI * R; q += kLayerThreads) {
      const unsigned i = by_R.q(q), rr = q - i * R, u = by_S.q(i), s = i - u * S;
      const bool sh = u >= UR;
      const unsigned dtype = sh ? kQ80 : dt_r, ss = sh ? 2 : ss_r, pb = sh ? 32 : pb_r;
      const uint8_t* st = dn_at(u, s);
      const uint8_t* win = st + RM * pb - ((ss * y0) & ~15u);  // win[ss * row] is row's scale
      const uint4 h0 = reinterpret_cast<const uint4*>(s_hq)[2 * i], h1 = reinterpret_cast<const uint4*>(s_hq)[2 * i + 1];
      const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      float c;
      if (dtype == kMXFP4) {
        const unsigned e = win[y0 + rr];
        bad |= e == 255;
        c = __fmul_rn(pow2_m128(e), i2f(idot_mxfp4_16(*reinterpret_cast<const uint4*>(st + 16 * rr), hw)));
      } else {
        const unsigned r2 = 2 * (y0 + rr);
        const float sw = h2f(win[r2] | win[r2 + 1] << 8);
        bad |= !isfinite(sw);
        const uint4 w0 = reinterpret_cast<const uint4*>(st + 32 * rr)[0], w1 = reinterpret_cast<const uint4*>(st + 32 * rr)[1];
        const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        int iv = 0;
#pragma unroll
        for (unsigned m = 0; m < 8; ++m) iv = __dp4a(static_cast<int>(ww[m]), static_cast<int>(hw[m]), iv);
        c = __fmul_rn(sw, i2f(iv));
      }
      s_terms[q] = c;
    }
    if (__syncthreads_or(bad) && tid == 0) atomicOr(a.status, kStNumeric);
    PHASE(12);
    // B3: per routing slot (the unique expert of the same index), four
    // slice-interleaved chains in ascending slice order
    for (unsigned q = tid; q < U * R; q += kLayerThreads) {
      const unsigned u = by_R.q(q), rr = q - u * R;
      const float* tv = s_terms + u * S * R + rr;
      const float* gv = s_gs + u * S;
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
      s_part[q] = __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3);
    }
    __syncthreads();
    bool nf = false;
    for (unsigned rr = tid; rr < R; rr += kLayerThreads) {
      float yv = 0.0f;
      for (unsigned u = 0; u < U; ++u) yv = __fadd_rn(yv, s_part[u * R + rr]);  // request order, then shared
      nf |= !isfinite(yv);
      if (a.world > 1) s_ylocal[rr] = yv;
      else a.y[y0 + rr] = yv;
    }
    if (nf) atomicOr(a.status, kStNumeric);
    PHASE(13);
    if (a.world > 1) {
      __syncthreads();
      // in-box reduce over NVLink: moe_layer_kernel's exchange (one token)
      const unsigned W = a.world;
      const size_t slot_entries = static_cast<size_t>(kMaxTokens) * d;
      const unsigned e = misc[6], par = e & 1;
      for (unsigned q = tid; q < W * R; q += kLayerThreads) {
        const unsigned dst = q / R, rr = q - dst * R;
        if (dst == a.rank) continue;
        uint2* slot = reinterpret_cast<uint2*>(a.peer[dst]) + (static_cast<size_t>(par) * W + a.rank) * slot_entries + y0 + rr;
        const unsigned long long word =
            static_cast<unsigned long long>(__float_as_uint(s_ylocal[rr])) | static_cast<unsigned long long>(e) << 32;
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(word) : "memory");
      }
      const uint2* inbox = reinterpret_cast<const uint2*>(a.peer[a.rank]) + static_cast<size_t>(par) * W * slot_entries;
      bool ok = true, bad_y = false;
      const uint64_t start = globaltimer();
      for (unsigned rr = tid; rr < R && ok; rr += kLayerThreads) {
        float yv = 0.0f;
        for (unsigned src = 0; src < W; ++src) {
          float v;
          if (src == a.rank) {
            v = s_ylocal[rr];
          } else {
            const uint2* ent = inbox + static_cast<size_t>(src) * slot_entries + y0 + rr;
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
        a.y[y0 + rr] = yv;
      }
      if (!__syncthreads_and(ok)) {
        aborted = true;
        if (tid == 0) atomicOr(a.status, kStTimeout);
      }
      if (bad_y) atomicOr(a.status, kStNumeric);
    }
  }
  PHASE(7);
  // Nothing may still be writing this CTA's shared memory when it leaves:
  // after an abort, wait (bounded) for the last chunk issued into each slot.
  if (aborted && tid == 0) {
    for (unsigned i = 0; i < K; ++i)
      if (s_iss[i]) mbar_wait(&full[i], (s_iss[i] - 1) & 1);
    if (R && !dn_landed) mbar_wait(dnbar, 0);
  }
}

}  // namespace frc
