// frc.cu - B200 (sm_100a) expert neuron-slice kernels and the C ABI around them.
//
// One launch computes one MoE layer (the work of fr_backend.run,
// backends/ref.c:57-98) as a queue of units drawn by every CTA:
//   gate/up unit (item, 8 neurons): 8 gate + 8 up rows of one (expert, slice)
//     item, TMA-staged in shared memory, integer block dots against the
//     token's int8 activations, SwiGLU -> hidden[item][token][neuron];
//   down unit (expert, 64 rows): waits until all gate/up units of the expert
//     are done, quantizes the expert's hidden slices, forms the 64 down rows of
//     every slice and writes the expert's partial; the last down unit of a row
//     chunk sums all experts' partials in a fixed order into y.
// Gate/up units come first in the queue, so a waiting down unit never blocks
// the work it waits for; the queue makes the launch deadlock free for any
// grid size.  No float atomics: results are bitwise repeatable.
#include <cuda_runtime.h>
#include <fenv.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/fronk_b200.h"
#include "frc_device.cuh"

using namespace frc;

// ============================================================ layer kernel

struct Plan {  // per-CTA view of the layer's unique experts
  unsigned U, nGU, nDN, total, nch;
};

template <int ACT, int MAXT>
__global__ void __launch_bounds__(kThreads) layer_kernel(const LayerArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  unsigned* misc = reinterpret_cast<unsigned*>(smem + 16);  // [0..1] next, [2] last, [3] reset, [4] U
  uint16_t* s_ids = reinterpret_cast<uint16_t*>(smem + a.sm.ids);
  float* s_g = reinterpret_cast<float*>(smem + a.sm.gates);
  int* s_first = reinterpret_cast<int*>(smem + a.sm.first);
  uint16_t* s_uid = reinterpret_cast<uint16_t*>(smem + a.sm.uid);
  unsigned* s_umask = reinterpret_cast<unsigned*>(smem + a.sm.umask);
  float* s_ugate = reinterpret_cast<float*>(smem + a.sm.ugate);
  uint8_t* stage0 = smem + a.sm.stage;

  const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned T = a.T, S = a.S, d = a.d, P = d / 64;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  // ---- plan: unique experts in first-appearance order, then the shared one
  for (unsigned i = tid; i < T * 10; i += kThreads) s_ids[i] = a.expert[i];
  for (unsigned i = tid; i < T * 11; i += kThreads) s_g[i] = a.gate[i];
  for (unsigned i = tid; i < 512; i += kThreads) s_first[i] = 0x7fffffff;
  for (unsigned i = tid; i < kMaxUnique; i += kThreads) s_umask[i] = 0;
  for (unsigned i = tid; i < kMaxUnique * T; i += kThreads) s_ugate[i] = 0.0f;
  __syncthreads();
  bool invalid = false;
  for (unsigned i = tid; i < T * 10; i += kThreads) {
    const unsigned id = s_ids[i];
    if (id < 512) atomicMin(&s_first[id], static_cast<int>(i));
    else invalid = true;
  }
  if (invalid) atomicOr(a.status, kStInvalid);
  __syncthreads();
  {
    // rank of each first occurrence; T*10 <= 160 < kThreads
    const unsigned i = tid;
    const bool first = i < T * 10 && s_ids[i] < 512 && s_first[s_ids[i]] == static_cast<int>(i);
    const unsigned ballot = __ballot_sync(0xffffffffu, first);
    unsigned* wcount = misc + 8;  // 8 words
    if (lane == 0) wcount[warp] = __popc(ballot);
    __syncthreads();
    unsigned off = 0;
    for (unsigned w = 0; w < warp; ++w) off += wcount[w];
    const unsigned rank = off + __popc(ballot & ((1u << lane) - 1));
    if (tid == kThreads - 1) misc[4] = off + __popc(ballot);  // routed unique count
    __syncthreads();
    if (first) {
      s_uid[rank] = s_ids[i];
      s_first[s_ids[i]] = -1 - static_cast<int>(rank);  // id -> rank
    }
    __syncthreads();
  }
  unsigned U = misc[4];
  for (unsigned i = tid; i < T * 10; i += kThreads) {
    const unsigned id = s_ids[i];
    if (id >= 512) continue;
    const unsigned u = static_cast<unsigned>(-1 - s_first[id]), t = i / 10;
    atomicOr(&s_umask[u], 1u << t);
    s_ugate[u * T + t] = s_g[t * 11 + i % 10];
  }
  __syncthreads();
  {
    unsigned shared_mask = 0;
    for (unsigned t = 0; t < T; ++t)
      if (s_g[t * 11 + 10] != 0.0f) shared_mask |= 1u << t;
    if (shared_mask) {
      if (tid == 0) {
        s_uid[U] = 512;
        s_umask[U] = shared_mask;
      }
      for (unsigned t = tid; t < T; t += kThreads) s_ugate[U * T + t] = s_g[t * 11 + 10];
      ++U;
    }
  }
  Plan pl;
  pl.U = U;
  pl.nch = d / kDnRows;
  pl.nGU = U * S * kGuUnits;
  pl.nDN = U * pl.nch;
  pl.total = pl.nGU + pl.nDN;
  __syncthreads();

  // ---- stage issue: bulk copies of one unit's bytes into a stage buffer
  auto issue = [&](unsigned k, unsigned st) {
    uint8_t* dst = stage0 + st * a.sm.stage_bytes;
    if (k < pl.nGU) {
      const unsigned item = k / kGuUnits, ng = k % kGuUnits, u = item / S, si = item % S;
      const bool shared = s_uid[u] == 512;
      const unsigned rowb = shared ? a.shared_row : a.row_bytes, proj = shared ? a.shared_proj : a.proj_bytes;
      const uint8_t* src = a.base[si] + static_cast<size_t>(s_uid[u]) * a.slice_bytes + ng * kGuNeurons * rowb;
      const unsigned bytes = kGuNeurons * rowb;
      mbar_expect_tx(&bar[st], 2 * bytes);
      bulk_g2s(dst, src, bytes, &bar[st]);
      bulk_g2s(dst + bytes, src + proj, bytes, &bar[st]);
    } else {
      const unsigned j = k - pl.nGU, u = j / pl.nch, c = j % pl.nch;
      const bool shared = s_uid[u] == 512;
      const unsigned proj = shared ? a.shared_proj : a.proj_bytes;
      const bool mx = !shared && a.down_type == kMXFP4;
      const unsigned hb = mx ? 1 : 2, pb = mx ? 16 : 32;  // scale / payload bytes per row
      const unsigned ib = kDnRows * (hb + pb);
      mbar_expect_tx(&bar[st], S * ib);
      for (unsigned si = 0; si < S; ++si) {
        const uint8_t* down = a.base[si] + static_cast<size_t>(s_uid[u]) * a.slice_bytes + 2 * proj;
        bulk_g2s(dst + si * ib, down + c * kDnRows * hb, kDnRows * hb, &bar[st]);
        bulk_g2s(dst + si * ib + kDnRows * hb, down + d * hb + c * kDnRows * pb, kDnRows * pb, &bar[st]);
      }
    }
  };

  if (tid == 0) {
    const unsigned k0 = atomicAdd(&a.ctl->next, 1u);
    misc[0] = k0;
    if (k0 < pl.total) issue(k0, 0);
  }
  __syncthreads();
  unsigned k = misc[0];

  // ---- activations (CTAs that hold work; CTA 0 always, it owns x_out)
  if (k < pl.total || blockIdx.x == 0) {
    const unsigned per_token = d / 4, nvec = T * per_token;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const float4* xa4 = reinterpret_cast<const float4*>(a.x_add);
    float* s_rms = reinterpret_cast<float*>(smem + a.sm.rms);
    bool bad = false;
    if (a.norm) {
      // per-token 1/rms of v = x + x_add: thread partials, warp tree, warps in order
      float* wsum = reinterpret_cast<float*>(misc + 16);  // 8 floats
      for (unsigned t = 0; t < T; ++t) {
        float ss = 0.0f;
        for (unsigned f = t * per_token + tid; f < (t + 1) * per_token; f += kThreads) {
          float4 v = x4[f];
          if (xa4) {
            const float4 w = xa4[f];
            v.x = __fadd_rn(v.x, w.x); v.y = __fadd_rn(v.y, w.y); v.z = __fadd_rn(v.z, w.z); v.w = __fadd_rn(v.w, w.w);
          }
          ss = __fmaf_rn(v.x, v.x, ss); ss = __fmaf_rn(v.y, v.y, ss);
          ss = __fmaf_rn(v.z, v.z, ss); ss = __fmaf_rn(v.w, v.w, ss);
        }
#pragma unroll
        for (unsigned o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if (lane == 0) wsum[warp] = ss;
        __syncthreads();
        if (tid == 0) {
          float tot = 0.0f;
          for (unsigned w = 0; w < kWarps; ++w) tot = __fadd_rn(tot, wsum[w]);
          s_rms[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(d)), 1e-6f)));
        }
        __syncthreads();
      }
    }
    for (unsigned base = 0; base < nvec; base += kThreads * 4) {
      float4 v[4];
#pragma unroll
      for (unsigned r = 0; r < 4; ++r) {
        const unsigned f = base + r * kThreads + tid;
        if (f < nvec) {
          v[r] = x4[f];
          if (xa4) {
            const float4 w = xa4[f];
            v[r].x = __fadd_rn(v[r].x, w.x); v[r].y = __fadd_rn(v[r].y, w.y);
            v[r].z = __fadd_rn(v[r].z, w.z); v[r].w = __fadd_rn(v[r].w, w.w);
          }
        }
      }
#pragma unroll
      for (unsigned r = 0; r < 4; ++r) {
        const unsigned f = base + r * kThreads + tid;
        if (f >= nvec) continue;  // warp-uniform: nvec is a multiple of 128
        const unsigned t = f / per_token, j = f % per_token;  // element 4j of token t
        bad |= !isfinite(v[r].x) || !isfinite(v[r].y) || !isfinite(v[r].z) || !isfinite(v[r].w);
        if (a.x_out && blockIdx.x == 0) reinterpret_cast<float4*>(a.x_out)[f] = v[r];
        if (a.norm) {
          const float g = s_rms[t];
          v[r].x = __fmul_rn(v[r].x, g); v[r].y = __fmul_rn(v[r].y, g);
          v[r].z = __fmul_rn(v[r].z, g); v[r].w = __fmul_rn(v[r].w, g);
        }
        if (ACT == FRC_ACT_F32) {
          reinterpret_cast<float4*>(smem + a.sm.xf)[f] = v[r];
          continue;
        }
        // group of 64 = 16 consecutive float4 = one half-warp
        float amax = fmaxf(fmaxf(fabsf(v[r].x), fabsf(v[r].y)), fmaxf(fabsf(v[r].z), fabsf(v[r].w)));
#pragma unroll
        for (unsigned o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float scale = __fdiv_rn(amax, 127.0f);
        const int q0 = q8_value(v[r].x, amax, scale), q1 = q8_value(v[r].y, amax, scale);
        const int q2 = q8_value(v[r].z, amax, scale), q3 = q8_value(v[r].w, amax, scale);
        int sum = q0 + q1 + q2 + q3;
#pragma unroll
        for (unsigned o = 4; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const unsigned p = j / 16, wq = j % 16;
        uint8_t* xt = smem + a.sm.xq + t * d;
        const uint32_t word = (q0 & 0xff) | (q1 & 0xff) << 8 | (q2 & 0xff) << 16 | static_cast<uint32_t>(q3 & 0xff) << 24;
        *reinterpret_cast<uint32_t*>(xt + 16 * xslot(p, wq / 4) + 4 * (wq % 4)) = word;
        if ((lane & 15) == 0) reinterpret_cast<float*>(smem + a.sm.xs)[t * P + p] = scale;
        if ((lane & 7) == 0) reinterpret_cast<float*>(smem + a.sm.xv)[t * 2 * P + 2 * p + ((lane >> 3) & 1)] = static_cast<float>(sum);
        if (a.sm.xp) {  // prmt order inside each 32-weight block
          uint8_t* xp = smem + a.sm.xp + t * d;
          const int qv[4] = {q0, q1, q2, q3};
#pragma unroll
          for (unsigned i = 0; i < 4; ++i) {
            const unsigned e = 4 * j + i, wi = (e % 64) / 32 * 32 + prmt_pos(e % 32);  // byte index in group
            xp[16 * xslot(p, wi / 16) + wi % 16] = static_cast<uint8_t>(qv[i] & 0xff);
          }
        }
      }
    }
    if (bad) atomicOr(a.status, kStNumeric);
  }
  __syncthreads();

  // ---- unit loop, double buffered
  unsigned ph0 = 0, ph1 = 0, st = 0, iter = 0;
  bool inflight[2] = {k < pl.total, false};  // a copy issued into the stage and not yet waited for
  while (k < pl.total) {
    if (tid == 0) {
      const unsigned k2 = ld_acquire(&a.ctl->abort) ? 0xffffffffu : atomicAdd(&a.ctl->next, 1u);
      misc[(iter + 1) & 1] = k2;
      if (k2 < pl.total) {
        fence_proxy_async();
        issue(k2, st ^ 1);
      }
    }
    __syncthreads();
    inflight[st ^ 1] = misc[(iter + 1) & 1] < pl.total;
    const bool ok = mbar_wait(&bar[st], st ? ph1 : ph0);
    if (ok) {  // on a timeout the copy may still land: keep the parity, drain before leaving
      if (st) ph1 ^= 1; else ph0 ^= 1;
      inflight[st] = false;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        atomicOr(a.status, kStTimeout);
        atomicExch(&a.ctl->abort, 1u);
      }
      break;
    }
    uint8_t* stage = stage0 + st * a.sm.stage_bytes;

    if (k < pl.nGU) {
      // ---------------------------------------------------- gate/up unit
      const unsigned item = k / kGuUnits, ng = k % kGuUnits, u = item / S, si = item % S;
      const bool shared = s_uid[u] == 512;
      const unsigned type = shared ? kQ80 : a.gate_type;
      const unsigned rowb = shared ? a.shared_row : a.row_bytes, nb = d / 32;
      const uint8_t* grow = stage + warp * rowb;
      const uint8_t* urow = stage + (kGuNeurons + warp) * rowb;
      const unsigned n = ng * kGuNeurons + warp;
      unsigned mask = s_umask[u];
      bool bad = false;
      while (mask) {
        const unsigned t = __ffs(mask) - 1;
        mask &= mask - 1;
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
              const unsigned j = 64 * p + jj;
              const float wg = weight_any(grow, type, d, j), wu = weight_any(urow, type, d, j);
              bad |= !isfinite(wg) || !isfinite(wu);
              ag = __fmaf_rn(wg, xf[j], ag);
              au = __fmaf_rn(wu, xf[j], au);
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
          a.hidden[((static_cast<size_t>(u) * S + si) * T + t) * 32 + n] = h;
        }
      }
      if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
      __threadfence();
      __syncthreads();
      if (tid == 0) atomicAdd(&a.ctl->gu_done[u], 1u);
    } else {
      // ------------------------------------------------------- down unit
      const unsigned j = k - pl.nGU, u = j / pl.nch, c = j % pl.nch;
      const bool shared = s_uid[u] == 512;
      const unsigned down = shared ? kQ80 : a.down_type;
      const unsigned mask = s_umask[u], cnt = __popc(mask);
      bool waited = true;
      if (tid == 0 && !spin_geq(&a.ctl->gu_done[u], S * kGuUnits, &a.ctl->abort)) {
        waited = false;
        atomicOr(a.status, kStTimeout);
        atomicExch(&a.ctl->abort, 1u);
      }
      if (__syncthreads_or(!waited)) break;
      // hidden slices of this expert -> int8 (Q8) or fp32 (F32), [si][k][32]
      for (unsigned idx = warp; idx < S * cnt; idx += kWarps) {
        const unsigned si = idx / cnt, kk = idx % cnt;
        unsigned mm = mask;
        for (unsigned z = 0; z < kk; ++z) mm &= mm - 1;
        const unsigned t = __ffs(mm) - 1;
        const float h = __ldcg(&a.hidden[((static_cast<size_t>(u) * S + si) * T + t) * 32 + lane]);
        if (ACT == FRC_ACT_Q8) {
          float amax = fabsf(h);
#pragma unroll
          for (unsigned o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
          const float scale = __fdiv_rn(amax, 127.0f);
          const int v = q8_value(h, amax, scale);
          const unsigned pos = down == kMXFP4 ? prmt_pos(lane) : lane;
          smem[a.sm.hq + idx * 32 + pos] = static_cast<uint8_t>(v & 0xff);
          if (lane == 0) reinterpret_cast<float*>(smem + a.sm.gs)[idx] = __fmul_rn(scale, s_ugate[u * T + t]);
        } else {
          reinterpret_cast<float*>(smem + a.sm.hq)[idx * 32 + lane] = h;
          if (lane == 0) reinterpret_cast<float*>(smem + a.sm.gs)[idx] = s_ugate[u * T + t];
        }
      }
      __syncthreads();
      const unsigned r = tid % kDnRows, q = tid / kDnRows;
      const float* gs = reinterpret_cast<const float*>(smem + a.sm.gs);
      float acc[MAXT];
#pragma unroll
      for (unsigned kk = 0; kk < MAXT; ++kk) acc[kk] = 0.0f;
      bool bad = false;
      const bool mx = down == kMXFP4;
      const unsigned hb = mx ? 1 : 2, ib = kDnRows * (mx ? 17 : 34);
      for (unsigned si = q; si < S; si += kDnSplit) {
        const uint8_t* it = stage + si * ib;
        if (ACT == FRC_ACT_Q8) {
          if (mx) {
            const unsigned e = it[r];
            bad |= e == 255;
            const float sw = pow2_m128(e);
            const uint4 w = *reinterpret_cast<const uint4*>(it + kDnRows * hb + 16 * r);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            uint32_t pw[8], nw[8];
#pragma unroll
            for (unsigned m = 0; m < 4; ++m) {
              pw[2 * m] = prmt(kE2M1Lo, kE2M1Hi, ww[m]);
              nw[2 * m] = prmt(kE2M1Lo, kE2M1Hi, ww[m] ^ 0x8888u);
              pw[2 * m + 1] = prmt(kE2M1Lo, kE2M1Hi, ww[m] >> 16);
              nw[2 * m + 1] = prmt(kE2M1Lo, kE2M1Hi, (ww[m] >> 16) ^ 0x8888u);
            }
#pragma unroll
            for (unsigned kk = 0; kk < MAXT; ++kk) {
              if (kk >= cnt) break;
              const uint4* hv = reinterpret_cast<const uint4*>(smem + a.sm.hq + (si * cnt + kk) * 32);
              const uint4 h0 = hv[0], h1 = hv[1];
              const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
              int ip = 0, in = 0;
#pragma unroll
              for (unsigned m = 0; m < 8; ++m) {
                ip = __dp4a(static_cast<int>(pw[m]), static_cast<int>(hw[m]), ip);
                in = __dp4a(static_cast<int>(nw[m]), static_cast<int>(hw[m]), in);
              }
              const float cterm = __fmul_rn(sw, i2f(ip - in));
              acc[kk] = __fmaf_rn(cterm, gs[si * cnt + kk], acc[kk]);
            }
          } else {
            const float sw = h2f(it[2 * r] | it[2 * r + 1] << 8);
            bad |= !isfinite(sw);
            const uint4* wv = reinterpret_cast<const uint4*>(it + kDnRows * hb + 32 * r);
            const uint4 w0 = wv[0], w1 = wv[1];
            const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (unsigned kk = 0; kk < MAXT; ++kk) {
              if (kk >= cnt) break;
              const uint4* hv = reinterpret_cast<const uint4*>(smem + a.sm.hq + (si * cnt + kk) * 32);
              const uint4 h0 = hv[0], h1 = hv[1];
              const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
              int iv = 0;
#pragma unroll
              for (unsigned m = 0; m < 8; ++m) iv = __dp4a(static_cast<int>(ww[m]), static_cast<int>(hw[m]), iv);
              const float cterm = __fmul_rn(sw, i2f(iv));
              acc[kk] = __fmaf_rn(cterm, gs[si * cnt + kk], acc[kk]);
            }
          }
        } else {
          // fp32: exact weights times fp32 hidden, neuron order
          float wrow[32];
          if (mx) {
            const unsigned e = it[r];
            bad |= e == 255;
            const float sc = __uint_as_float(e ? e << 23 : 0x00400000u);
            const uint8_t* qb = it + kDnRows + 16 * r;
#pragma unroll
            for (unsigned nn = 0; nn < 32; ++nn) wrow[nn] = __fmul_rn(sc, e2m1((qb[nn & 15] >> (nn >> 4 ? 4 : 0)) & 15));
          } else {
            const float sw = h2f(it[2 * r] | it[2 * r + 1] << 8);
            bad |= !isfinite(sw);
            const int8_t* qb = reinterpret_cast<const int8_t*>(it + 2 * kDnRows + 32 * r);
#pragma unroll
            for (unsigned nn = 0; nn < 32; ++nn) wrow[nn] = __fmul_rn(sw, static_cast<float>(qb[nn]));
          }
#pragma unroll
          for (unsigned kk = 0; kk < MAXT; ++kk) {
            if (kk >= cnt) break;
            const float* hv = reinterpret_cast<const float*>(smem + a.sm.hq) + (si * cnt + kk) * 32;
            float dot = 0.0f;
#pragma unroll
            for (unsigned nn = 0; nn < 32; ++nn) dot = __fmaf_rn(wrow[nn], hv[nn], dot);
            acc[kk] = __fmaf_rn(dot, gs[si * cnt + kk], acc[kk]);
          }
        }
      }
      if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.status, kStNumeric);
      __syncthreads();  // stage fully read: reuse it for the split sums
      float* red = reinterpret_cast<float*>(stage);  // [kDnSplit][cnt][64]
#pragma unroll
      for (unsigned kk = 0; kk < MAXT; ++kk)
        if (kk < cnt) red[(q * cnt + kk) * kDnRows + r] = acc[kk];
      __syncthreads();
      for (unsigned idx = tid; idx < cnt * kDnRows; idx += kThreads) {
        const unsigned kk = idx / kDnRows, rr = idx % kDnRows;
        float sum = red[kk * kDnRows + rr];
        for (unsigned z = 1; z < kDnSplit; ++z) sum = __fadd_rn(sum, red[(z * cnt + kk) * kDnRows + rr]);
        unsigned mm = mask;
        for (unsigned z = 0; z < kk; ++z) mm &= mm - 1;
        const unsigned t = __ffs(mm) - 1;
        a.partial[(static_cast<size_t>(u) * T + t) * d + c * kDnRows + rr] = sum;
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) misc[2] = atomicAdd(&a.ctl->chunk_done[c], 1u) == U - 1;
      __syncthreads();
      if (misc[2]) {
        __threadfence();
        bool nf = false;
        // each token sums its experts in its own routing order, then the
        // shared expert: a token's y does not depend on the rest of the burst
        for (unsigned idx = tid; idx < T * kDnRows; idx += kThreads) {
          const unsigned t = idx / kDnRows, rr = idx % kDnRows;
          const size_t col = static_cast<size_t>(t) * d + c * kDnRows + rr;
          float yv = 0.0f;
          for (unsigned e = 0; e < 10; ++e) {
            const unsigned id = s_ids[t * 10 + e];
            if (id >= 512) continue;
            const unsigned uu = static_cast<unsigned>(-1 - s_first[id]);
            yv = __fadd_rn(yv, __ldcg(&a.partial[static_cast<size_t>(uu) * T * d + col]));
          }
          if (s_g[t * 11 + 10] != 0.0f) yv = __fadd_rn(yv, __ldcg(&a.partial[static_cast<size_t>(misc[4]) * T * d + col]));
          nf |= !isfinite(yv);
          a.y[col] = yv;
        }
        if (nf) atomicOr(a.status, kStNumeric);
      }
    }
    __syncthreads();
    k = misc[(iter + 1) & 1];
    st ^= 1;
    ++iter;
  }

  // ---- leave: no bulk copy may still be writing this CTA's shared memory
  for (unsigned b2 = 0; b2 < 2; ++b2)
    if (inflight[b2] && !mbar_wait(&bar[b2], b2 ? ph1 : ph0) && tid == 0) atomicOr(a.status, kStTimeout);
  // ---- the last CTA out restores the counters for the next launch
  __syncthreads();
  if (tid == 0) misc[3] = atomicAdd(&a.ctl->exited, 1u) == gridDim.x - 1;
  __syncthreads();
  if (misc[3]) {
    __threadfence();
    for (unsigned i = tid; i < kMaxUnique + 3; i += kThreads) a.ctl->gu_done[i] = 0;
    for (unsigned i = tid; i < kMaxChunks; i += kThreads) a.ctl->chunk_done[i] = 0;
    if (tid == 0) {
      a.ctl->next = 0;
      a.ctl->exited = 0;
      a.ctl->abort = 0;
    }
  }
}

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

// ========================================================= host runtime

struct frc_context {
  int device = 0, sms = 0;
  frc_geometry g{};
  size_t row_bytes = 0, proj_bytes = 0, slice_bytes = 0, shared_row = 0, shared_proj = 0, shared_bytes = 0, layer_bytes = 0;
  uint8_t* layer_ptr[FRC_MAX_BLOCKS][FRC_MAX_LAYERS] = {};
  uint8_t* staging = nullptr;
  float* hidden = nullptr;
  float* partial = nullptr;
  Ctl* ctl = nullptr;
  unsigned* status = nullptr;
  uint16_t* d_expert = nullptr;
  float *d_gate = nullptr, *d_x = nullptr, *d_y = nullptr;
  uint16_t* h_expert = nullptr;
  float *h_gate = nullptr, *h_x = nullptr, *h_y = nullptr;
  unsigned* h_status = nullptr;
  cudaStream_t stream = nullptr;
  uint8_t* pool = nullptr;
  unsigned pool_count = 0;
  unsigned long long launches = 0;
  bool attr_set[2][3] = {};
  unsigned occ_smem[2][3] = {};
  int occ_val[2][3] = {};
  unsigned last_T = 0, last_S = 0;
  uint16_t last_expert[FRC_MAX_TOKENS * FRC_TOPK] = {};
  float last_gate[FRC_MAX_TOKENS * FRC_ACTIVE] = {};
  char err[256] = {};
};

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

static Smem smem_layout(const frc_context* c, unsigned T, unsigned S, int act) {
  const unsigned d = c->g.hidden, P = d / 64;
  Smem m{};
  unsigned o = 64 + 64;  // mbarriers + misc words
  auto take = [&](unsigned bytes) { unsigned at = o; o = align_up(o + bytes, 16); return at; };
  m.ids = take(2 * T * 10);
  m.gates = take(4 * T * 11);
  m.first = take(4 * 512);
  m.uid = take(2 * kMaxUnique);
  m.umask = take(4 * kMaxUnique);
  m.ugate = take(4 * kMaxUnique * T);
  m.rms = take(4 * T);
  if (act == FRC_ACT_Q8) {
    m.xq = take(T * d);
    m.xp = c->g.gate_type == FRC_MXFP4 ? take(T * d) : 0;
    m.xs = take(4 * T * P);
    m.xv = take(4 * T * 2 * P);
    m.xf = 0;
    m.hq = take(32 * S * T);
  } else {
    m.xq = m.xp = m.xs = m.xv = 0;
    m.xf = take(4 * T * d);
    m.hq = take(4 * 32 * S * T);
  }
  m.gs = take(4 * S * T);
  // A stage holds the largest unit: 16 gate/up rows, or one expert's 64 down
  // rows of every loaded slice; and later the down split sums.
  const unsigned gu = 2 * kGuNeurons * static_cast<unsigned>(c->row_bytes > c->shared_row ? c->row_bytes : c->shared_row);
  const unsigned dn = S * kDnRows * 34;  // the shared expert's Q8_0 rows bound the routed MXFP4 ones
  const unsigned red = 4 * kDnSplit * T * kDnRows;
  unsigned sb = gu > dn ? gu : dn;
  if (red > sb) sb = red;
  m.stage_bytes = align_up(sb, 128);
  o = align_up(o, 128);
  m.stage = o;
  m.total = o + 2 * m.stage_bytes;
  return m;
}

template <int ACT, int MAXT>
static int launch_layer(frc_context* c, const LayerArgs& a, unsigned units, cudaStream_t s) {
  auto kern = layer_kernel<ACT, MAXT>;
  const int ai = ACT == FRC_ACT_Q8, mi = MAXT == 1 ? 0 : MAXT == 4 ? 1 : 2;
  if (!c->attr_set[ai][mi]) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    c->attr_set[ai][mi] = true;
  }
  int per_sm = 0;
  if (c->occ_smem[ai][mi] == a.sm.total) {
    per_sm = c->occ_val[ai][mi];
  } else {
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, a.sm.total));
    c->occ_smem[ai][mi] = a.sm.total;
    c->occ_val[ai][mi] = per_sm;
  }
  if (per_sm < 1) return fail(c, FRC_INVALID, "layer needs %u bytes of shared memory", a.sm.total);
  unsigned grid = static_cast<unsigned>(per_sm) * c->sms;
  if (grid > units) grid = units;
  kern<<<grid, kThreads, a.sm.total, s>>>(a);
  CK(cudaGetLastError());
  ++c->launches;
  return FRC_OK;
}

static int run_device(frc_context* c, unsigned layer, unsigned T, const uint16_t* expert, const float* gate,
                      const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags,
                      cudaStream_t s) {
  if (!c || !expert || !gate || !x || !y) return fail(c, FRC_INVALID, "null argument");
  if (T < 1 || T > FRC_MAX_TOKENS || layer >= c->g.layers) return fail(c, FRC_INVALID, "tokens or layer out of range");
  if (act != FRC_ACT_Q8 && act != FRC_ACT_F32) return fail(c, FRC_INVALID, "unknown activation mode");
  LayerArgs a{};
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
  a.hidden = c->hidden; a.partial = c->partial; a.ctl = c->ctl; a.status = c->status;
  a.S = S; a.T = T; a.d = c->g.hidden;
  a.norm = flags & FRC_RUN_RMSNORM ? 1u : 0u;
  a.gate_type = c->g.gate_type; a.down_type = c->g.down_type;
  a.row_bytes = static_cast<unsigned>(c->row_bytes); a.proj_bytes = static_cast<unsigned>(c->proj_bytes);
  a.shared_row = static_cast<unsigned>(c->shared_row); a.shared_proj = static_cast<unsigned>(c->shared_proj);
  a.slice_bytes = static_cast<unsigned>(c->slice_bytes);
  a.sm = smem_layout(c, T, S, act);
  if (a.sm.total > 227 * 1024) return fail(c, FRC_INVALID, "%u tokens need too much shared memory", T);
  const unsigned umax = (10 * T < 512 ? 10 * T : 512) + 1;
  const unsigned units = umax * S * kGuUnits + umax * (c->g.hidden / kDnRows);
  c->last_S = S;
  const int maxt = T == 1 ? 1 : T <= 4 ? 4 : 16;
  if (act == FRC_ACT_Q8) {
    if (maxt == 1) return launch_layer<FRC_ACT_Q8, 1>(c, a, units, s);
    if (maxt == 4) return launch_layer<FRC_ACT_Q8, 4>(c, a, units, s);
    return launch_layer<FRC_ACT_Q8, 16>(c, a, units, s);
  }
  if (maxt == 1) return launch_layer<FRC_ACT_F32, 1>(c, a, units, s);
  if (maxt == 4) return launch_layer<FRC_ACT_F32, 4>(c, a, units, s);
  return launch_layer<FRC_ACT_F32, 16>(c, a, units, s);
}

static int status_code(unsigned st) {
  if (st & kStTimeout) return FRC_IO;
  if (st & kStInvalid) return FRC_INVALID;
  if (st & kStNumeric) return FRC_NUMERIC;
  return FRC_OK;
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
  alloc(reinterpret_cast<void**>(&c->hidden), sizeof(float) * kMaxUnique * kMaxBlocks * kMaxTokens * 32);
  alloc(reinterpret_cast<void**>(&c->partial), sizeof(float) * kMaxUnique * kMaxTokens * d);
  alloc(reinterpret_cast<void**>(&c->ctl), sizeof(Ctl));
  alloc(reinterpret_cast<void**>(&c->status), sizeof(unsigned));
  alloc(reinterpret_cast<void**>(&c->d_expert), sizeof(uint16_t) * kMaxTokens * 10);
  alloc(reinterpret_cast<void**>(&c->d_gate), sizeof(float) * kMaxTokens * 11);
  alloc(reinterpret_cast<void**>(&c->d_x), sizeof(float) * kMaxTokens * d);
  alloc(reinterpret_cast<void**>(&c->d_y), sizeof(float) * kMaxTokens * d);
  if (rc == FRC_OK) {
    if (cudaMallocHost(reinterpret_cast<void**>(&c->h_expert), sizeof(uint16_t) * kMaxTokens * 10) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&c->h_gate), sizeof(float) * kMaxTokens * 11) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&c->h_x), sizeof(float) * kMaxTokens * d) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&c->h_y), sizeof(float) * kMaxTokens * d) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&c->h_status), sizeof(unsigned)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess)
      rc = fail(c, FRC_IO, "pinned buffers or stream");
  }
  if (rc == FRC_OK && (cudaMemset(c->ctl, 0, sizeof(Ctl)) != cudaSuccess ||
                       cudaMemset(c->status, 0, sizeof(unsigned)) != cudaSuccess ||
                       cudaMemset(c->hidden, 0, sizeof(float) * kMaxUnique * kMaxBlocks * kMaxTokens * 32) != cudaSuccess))
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
  for (auto& b : c->layer_ptr)
    for (auto& p : b) if (p) cudaFree(p);
  cudaFree(c->staging); cudaFree(c->hidden); cudaFree(c->partial); cudaFree(c->ctl); cudaFree(c->status);
  cudaFree(c->d_expert); cudaFree(c->d_gate); cudaFree(c->d_x); cudaFree(c->d_y); cudaFree(c->pool);
  cudaFreeHost(c->h_expert); cudaFreeHost(c->h_gate); cudaFreeHost(c->h_x); cudaFreeHost(c->h_y); cudaFreeHost(c->h_status);
  if (c->stream) cudaStreamDestroy(c->stream);
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

static int ensure_layer(frc_context* c, int block, unsigned layer) {
  if (!c->layer_ptr[block][layer]) CK(cudaMalloc(&c->layer_ptr[block][layer], c->layer_bytes));
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
  return any ? FRC_OK : fail(c, FRC_STATE, "block %d not loaded", block);
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

int frc_run(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate, const float* x,
            float* y, int act) {
  if (!c || !expert || !gate || !x || !y || tokens < 1 || tokens > FRC_MAX_TOKENS || layer >= c->g.layers ||
      (act != FRC_ACT_Q8 && act != FRC_ACT_F32))
    return fail(c, FRC_INVALID, "bad run arguments");
  int rc = validate(c, tokens, expert, gate, x);
  if (rc) return fail(c, rc, "request rejected");
  CK(cudaSetDevice(c->device));
  const size_t xb = sizeof(float) * tokens * c->g.hidden;
  memcpy(c->h_expert, expert, sizeof(uint16_t) * tokens * FRC_TOPK);
  memcpy(c->h_gate, gate, sizeof(float) * tokens * FRC_ACTIVE);
  memcpy(c->h_x, x, xb);
  CK(cudaMemcpyAsync(c->d_expert, c->h_expert, sizeof(uint16_t) * tokens * FRC_TOPK, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(c->d_gate, c->h_gate, sizeof(float) * tokens * FRC_ACTIVE, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(c->d_x, c->h_x, xb, cudaMemcpyHostToDevice, c->stream));
  rc = run_device(c, layer, tokens, c->d_expert, c->d_gate, c->d_x, nullptr, nullptr, c->d_y, act, 0, c->stream);
  if (rc) return rc;
  c->last_T = tokens;
  memcpy(c->last_expert, expert, sizeof(uint16_t) * tokens * FRC_TOPK);
  memcpy(c->last_gate, gate, sizeof(float) * tokens * FRC_ACTIVE);
  CK(cudaMemcpyAsync(c->h_y, c->d_y, xb, cudaMemcpyDeviceToHost, c->stream));
  rc = frc_status(c, c->stream);
  if (rc) return rc;
  memcpy(y, c->h_y, xb);  // published only after the whole layer succeeded
  return FRC_OK;
}

int frc_run_device(frc_context* c, unsigned layer, unsigned tokens, const uint16_t* expert, const float* gate,
                   const float* x, const float* x_add, float* x_out, float* y, int act, unsigned flags, void* stream) {
  if (!c) return FRC_INVALID;
  if (cudaSetDevice(c->device) != cudaSuccess) return fail(c, FRC_IO, "cudaSetDevice");
  return run_device(c, layer, tokens, expert, gate, x, x_add, x_out, y, act, flags, static_cast<cudaStream_t>(stream));
}

int frc_status(frc_context* c, void* stream) {
  if (!c) return FRC_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemcpyAsync(c->h_status, c->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
  CK(cudaMemsetAsync(c->status, 0, sizeof(unsigned), s));
  CK(cudaStreamSynchronize(s));
  const int rc = status_code(*c->h_status);
  if (rc) return fail(c, rc, "device status 0x%x", *c->h_status);
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

}  // extern "C"
