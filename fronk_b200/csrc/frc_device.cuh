// frc_device.cuh - device building blocks of the expert-slice kernels (sm_100a).
//
// Exactness: every fp32 operation whose rounding the parity tests pin is
// written with an explicit _rn intrinsic, so nvcc's FMA contraction cannot
// change it.  Integer block dot products use dp4a and are exact.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace frc {

constexpr unsigned kDnSplit = 4;       // slice interleave of the down partial sums
constexpr unsigned kMaxTokens = 16;
constexpr unsigned kMaxUnique = kMaxTokens * 10 + 1;
constexpr unsigned kMaxPairs = kMaxTokens * 11;  // (expert, token) pairs of one call
constexpr unsigned kMaxBlocks = 20;

enum : unsigned { kQ80 = 8, kQ4K = 12, kMXFP4 = 39 };
enum : unsigned { kStNumeric = 1, kStInvalid = 2, kStTimeout = 4 };

// ------------------------------------------------------------------ PTX

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Bulk (untiled) TMA copy global -> shared; both 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// 16-byte LSU copy global -> shared (L2 only), for many small pieces where a
// bulk copy per piece would cost more than the bytes it moves.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same test, but a thread whose phase is incomplete may sleep up to `ns`
// nanoseconds (it wakes when the phase completes): a waiting warp then takes
// no issue slots from the warps that work beside it.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, unsigned parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitNs = 2000000000ull;  // every wait gives up after 2 s (the layer kernel: a context setting)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, uint64_t limit = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - start > limit) return false;
  return true;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Waits until *p >= target; gives up after `limit` ns or once *abort is set.
__device__ __forceinline__ bool spin_geq(const unsigned* p, unsigned target, const unsigned* abort,
                                        uint64_t limit = kWaitNs) {
  if (ld_acquire(p) >= target) return true;
  const uint64_t start = globaltimer();
  while (ld_acquire(p) < target) {
    if (globaltimer() - start > limit || ld_acquire(abort)) return false;
    __nanosleep(64);
  }
  return true;
}
// Division by a run-time divisor 1 <= dv < 2^16 through multiply-high:
// exact for dividends x < 2^16.
__host__ __device__ constexpr unsigned div_magic(unsigned v) { return v > 1 ? 0xffffffffu / v + 1 : 0u; }
struct Div {
  unsigned dv, m;
  __device__ __forceinline__ explicit Div(unsigned v) : dv(v), m(div_magic(v)) {}
  __device__ __forceinline__ Div(unsigned v, unsigned magic) : dv(v), m(magic) {}  // magic from div_magic(v)
  __device__ __forceinline__ unsigned q(unsigned x) const { return dv > 1 ? __umulhi(x, m) : x; }
  __device__ __forceinline__ unsigned r(unsigned x) const { return x - q(x) * dv; }
};

// Generic-form byte permute: msb of a selector nibble replicates the sign.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// ------------------------------------------------------------- numerics

__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}
// Exact int -> float for |v| < 2^22 (1.5 * 2^23 magic).
__device__ __forceinline__ float i2f(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}
// Byte k of w as a float, exact.
__device__ __forceinline__ float byte_f(uint32_t w, unsigned k) {
  return __fsub_rn(__int_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | k)), 8388608.0f);
}
// 2^(e-128) as fp32 (subnormal for e < 2); the MXFP4 scale of the doubled E2M1 table.
__device__ __forceinline__ float pow2_m128(unsigned e) {
  return __uint_as_float(e >= 2 ? (e - 1) << 23 : 0x00200000u << e);
}
// Doubled E2M1 magnitudes {0,1,2,3,4,6,8,12} for prmt lookups.
constexpr uint32_t kE2M1Lo = 0x03020100u, kE2M1Hi = 0x0C080604u;

// Stable SiLU(a) * u in double, narrowed to fp32 (backends/ref.c:81-83).
__device__ __forceinline__ bool swiglu(float a, float u, float* h) {
  const double ad = a;
  const double sig = a >= 0 ? 1.0 / (1.0 + exp(-ad)) : exp(ad) / (1.0 + exp(ad));
  const double v = ad * sig * (double)u;
  if (!isfinite(v) || fabs(v) > 3.4028234663852886e38) return false;
  *h = __double2float_rn(v);
  return true;
}

// Symmetric int8 quantization of one value of a group with absolute maximum
// amax (src/q4.c:37-61): scale = amax/127, multiplier 127/amax (x/amax*127 if
// that overflows), nearest-even, clamp.  Returns the int8 value.
// q8_round keeps the rounded float (its sign of zero is what the
// reference's dequantized output carries); q8_value is its integer.
__device__ __forceinline__ float q8_round(float x, float amax, float scale) {
  if (scale == 0.0f) return 0.0f;
  const float inv = __fdiv_rn(127.0f, amax);
  float v = isfinite(inv) ? __fmul_rn(x, inv) : __fmul_rn(__fdiv_rn(x, amax), 127.0f);
  v = rintf(v);
  return fminf(fmaxf(v, -127.0f), 127.0f);
}
__device__ __forceinline__ int q8_value(float x, float amax, float scale) {
  return static_cast<int>(q8_round(x, amax, scale));
}
// The same quantizer with the group's two divisions done once.
struct Q8Group {
  float amax, scale, inv;
  bool inv_ok;
  __device__ __forceinline__ explicit Q8Group(float m) : amax(m) {
    scale = __fdiv_rn(m, 127.0f);
    inv = scale != 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
    inv_ok = isfinite(inv);
  }
  __device__ __forceinline__ int q(float x) const {
    if (scale == 0.0f) return 0;
    float v = inv_ok ? __fmul_rn(x, inv) : __fmul_rn(__fdiv_rn(x, amax), 127.0f);
    v = rintf(v);
    return static_cast<int>(fminf(fmaxf(v, -127.0f), 127.0f));
  }
  // q(x) when mul_ok(): the multiply form alone.  Callers branch once per
  // group on mul_ok() so the division fallback stays out of the hot code.
  __device__ __forceinline__ bool mul_ok() const { return inv_ok && scale != 0.0f; }
  __device__ __forceinline__ int qm(float x) const {
    return static_cast<int>(fminf(fmaxf(rintf(__fmul_rn(x, inv)), -127.0f), 127.0f));
  }
};

// Position of element n (0..31) of a 32-weight block in the "prmt order" that
// matches an MXFP4 block's nibble bytes (byte j holds elements j and j+16).
__host__ __device__ __forceinline__ unsigned prmt_pos(unsigned n) {
  const unsigned j = n & 15, hi = n >> 4, m = j >> 2, r = j & 3;
  return 4 * (2 * m + (r >> 1)) + 2 * (r & 1) + hi;
}
// uint4 slot of quad q (0..3) of x group p in the activation layout.  Groups
// are stored span-interleaved, position (p % 4) * nspan + p / 4 (nspan = d /
// 256), so the eight lanes of a row reading group p % 4 of consecutive spans
// read consecutive positions; the four quads of a position are swizzled
// across the 128-byte bank window.  Conflict-free for those reads.
__device__ __forceinline__ unsigned xslot(unsigned p, unsigned q, unsigned nspan) {
  const unsigned pos = (p & 3) * nspan + (p >> 2);
  return 4 * pos + (q ^ ((pos >> 1) & 3));
}

// ------------------------------------------------------ gate/up row terms
// The reference multiplies every weight by the dequantized activation
// X_j = fl32(v_j * s) (src/q4.c:54-58) and sums the products in double
// (backends/ref.c:74-79).  With the group scale s = M * 2^E (M its 24-bit
// significand), X_j = v_j * s + r_j * 2^E for an integer |r_j| <= 64, so each
// block term sum_j w_j * X_j is an exact combination of two integer dots (v
// and r against the block's integer weights) and a few scales.  The terms
// below are formed exactly in double and accumulated in double: the gate/up
// value narrowed to fp32 is then the reference's own, and the Q8 rounding of
// the hidden slice sees the same inputs.

// Exact int32 -> double: 2^52 + 2^51 + k carries k in its low bits.
__device__ __forceinline__ double i2d(int k) {
  return __hiloint2double(0x43380000 + (k >> 31), k) - 6755399441055744.0;
}
// Exact int64 -> double for |z| < 2^51.
__device__ __forceinline__ double ll2d(long long z) {
  return __longlong_as_double(0x4338000000000000LL + z) - 6755399441055744.0;
}
// 2^e as a double, -1022 <= e <= 1023.
__device__ __forceinline__ double pow2d(int e) { return __hiloint2double((e + 1023) << 20, 0); }
// Exact small-int float -> int (|v| < 2^22).
__device__ __forceinline__ int f2i_small(float v) {
  return __float_as_int(__fadd_rn(v, 12582912.0f)) - 0x4B400000;
}
// Exponent field of a group scale with subnormals counted as 1: the scale's
// last significand bit is 2^(ef - 150).
__device__ __forceinline__ unsigned scale_ef(float s) { return max((__float_as_uint(s) >> 23) & 255u, 1u); }

// One token's quantized activations in shared memory.  v and r are stored in
// the same swizzled layout (xslot), in natural order for Q4_K / Q8_0 rows and
// in prmt order for MXFP4 rows; st[p] = {2^E_p, M_p (the low word)} per
// 64-group (its scale s_p = M_p 2^E_p); vr[p] = {V, RS} of its two 32-blocks
// (sums of v and of r).
struct XAct {
  const uint8_t* v;
  const uint8_t* r;
  const double2* st;
  const int4* vr;
};

__device__ __forceinline__ void load_x8(const uint8_t* xq, unsigned p, unsigned q0, unsigned nspan, uint32_t (&x)[8]) {
#pragma unroll
  for (unsigned q = 0; q < 2; ++q) {
    const uint4 w = *reinterpret_cast<const uint4*>(xq + 16 * xslot(p, q0 + q, nspan));
    x[4 * q] = w.x; x[4 * q + 1] = w.y; x[4 * q + 2] = w.z; x[4 * q + 3] = w.w;
  }
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K super-block header: fp16 d / dmin, and the eight 6-bit scales and
// mins (src/native.c:17-18) as bytes, sub-blocks 0-3 in sc[0]/mi[0] and 4-7
// in sc[1]/mi[1].
struct Q4KHead {
  float d, m;
  uint32_t sc[2], mi[2];
  __device__ __forceinline__ explicit Q4KHead(const uint4 h) {
    d = h2f(h.x & 0xffffu);
    m = h2f(h.x >> 16);
    sc[0] = h.y & 0x3f3f3f3fu;
    mi[0] = h.z & 0x3f3f3f3fu;
    sc[1] = (h.w & 0x0f0f0f0fu) | ((h.y >> 6) & 0x03030303u) << 4;
    mi[1] = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 6) & 0x03030303u) << 4;
  }
  __device__ __forceinline__ bool ok() const { return isfinite(d) && isfinite(m); }
};

// Integer dots of one Q4_K group (64 weights: the low nibbles are sub-block
// 2gp, the high nibbles 2gp+1) against v and r: I0, I1, R0, R1.
__device__ __forceinline__ void q4k_idots(const uint8_t* qs, const uint32_t (&xlo)[8], const uint32_t (&rlo)[8],
                                          const uint32_t (&xhi)[8], const uint32_t (&rhi)[8], int& i0, int& i1,
                                          int& r0, int& r1) {
  const uint4 qa = reinterpret_cast<const uint4*>(qs)[0], qb = reinterpret_cast<const uint4*>(qs)[1];
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  i0 = i1 = r0 = r1 = 0;
#pragma unroll
  for (unsigned m = 0; m < 8; ++m) {
    const uint32_t lo = w[m] & 0x0f0f0f0fu, hi = w[m] & 0xf0f0f0f0u;
    i0 = __dp4a(static_cast<int>(lo), static_cast<int>(xlo[m]), i0);
    r0 = __dp4a(static_cast<int>(lo), static_cast<int>(rlo[m]), r0);
    i1 = dp4a_us(hi, xhi[m], i1);  // 16x the high-nibble dot
    r1 = dp4a_us(hi, rhi[m], r1);
  }
  i1 >>= 4;  // exact: multiples of 16
  r1 >>= 4;
}

// MXFP4 device row: [e: nb bytes][qs: nb x 16 bytes]; x and r in prmt order.
__device__ __forceinline__ int idot_mxfp4_16(const uint4 q, const uint32_t* x) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  int ip = 0, in = 0;
#pragma unroll
  for (unsigned m = 0; m < 4; ++m) {
    const uint32_t lo = w[m], hi = w[m] >> 16, nlo = lo ^ 0x8888u, nhi = hi ^ 0x8888u;
    ip = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, lo)), static_cast<int>(x[2 * m]), ip);
    in = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, nlo)), static_cast<int>(x[2 * m]), in);
    ip = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, hi)), static_cast<int>(x[2 * m + 1]), ip);
    in = __dp4a(static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, nhi)), static_cast<int>(x[2 * m + 1]), in);
  }
  return ip - in;
}
// The same block against v and r at once (the E2M1 lookups are shared).
__device__ __forceinline__ void idot2_mxfp4_16(const uint4 q, const uint32_t* x, const uint32_t* r, int& I, int& R) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  int ip = 0, in = 0, rp = 0, rn = 0;
#pragma unroll
  for (unsigned m = 0; m < 4; ++m) {
    const uint32_t lo = w[m], hi = w[m] >> 16;
    const int pl = static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, lo)), nl = static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, lo ^ 0x8888u));
    const int ph = static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, hi)), nh = static_cast<int>(prmt(kE2M1Lo, kE2M1Hi, hi ^ 0x8888u));
    ip = __dp4a(pl, static_cast<int>(x[2 * m]), ip);
    in = __dp4a(nl, static_cast<int>(x[2 * m]), in);
    rp = __dp4a(pl, static_cast<int>(r[2 * m]), rp);
    rn = __dp4a(nl, static_cast<int>(r[2 * m]), rn);
    ip = __dp4a(ph, static_cast<int>(x[2 * m + 1]), ip);
    in = __dp4a(nh, static_cast<int>(x[2 * m + 1]), in);
    rp = __dp4a(ph, static_cast<int>(r[2 * m + 1]), rp);
    rn = __dp4a(nh, static_cast<int>(r[2 * m + 1]), rn);
  }
  I = ip - in;
  R = rp - rn;
}

// acc + c * (s * I + t * R): the inner value is exact (|s * I| < 2^40 ulps of
// t), one rounding in the fma.
__device__ __forceinline__ double block_acc(double acc, double c, const double2 st, int I, int R) {
  // Z = M I + R exactly (|Z| < 2^51) as the bits of Z + 1.5 * 2^52, then
  // acc += Z * (c 2^E) with one rounding (c 2^E exact: c is a power of two or
  // an fp16 value)
  const long long zm = static_cast<long long>(__double2loint(st.y)) * I + (0x4338000000000000LL + R);
  return fma(__longlong_as_double(zm) - 6755399441055744.0, c * st.x, acc);
}

// Exact group terms (64 weights = blocks 2p, 2p+1) of an MXFP4 row.
__device__ __forceinline__ double group_mxfp4(double acc, const uint8_t* row, unsigned nb, unsigned p,
                                              const uint32_t (&x)[16], const uint32_t (&r)[16], const double2 st,
                                              bool& bad) {
  const unsigned e0 = row[2 * p], e1 = row[2 * p + 1];
  bad |= e0 == 255 || e1 == 255;
  const uint4* qs = reinterpret_cast<const uint4*>(row + nb + 32 * p);
  int I0, R0, I1, R1;
  idot2_mxfp4_16(qs[0], x, r, I0, R0);
  idot2_mxfp4_16(qs[1], x + 8, r + 8, I1, R1);
  acc = block_acc(acc, pow2d(static_cast<int>(e0) - 128), st, I0, R0);
  return block_acc(acc, pow2d(static_cast<int>(e1) - 128), st, I1, R1);
}

// Q8_0 device row: [d: nb x 2 bytes][qs: nb x 32 bytes]; x and r in natural order.
__device__ __forceinline__ double group_q80(double acc, const uint8_t* row, unsigned nb, unsigned p,
                                            const uint32_t (&x)[16], const uint32_t (&r)[16], const double2 st,
                                            bool& bad) {
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(row + 4 * p);
  const float s0 = h2f(dd & 0xffffu), s1 = h2f(dd >> 16);
  bad |= !isfinite(s0) || !isfinite(s1);
  const uint4* qs = reinterpret_cast<const uint4*>(row + 2 * nb + 64 * p);
  int i0 = 0, i1 = 0, r0 = 0, r1 = 0;
#pragma unroll
  for (unsigned q = 0; q < 2; ++q) {
    const uint4 a = qs[q], b = qs[2 + q];
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
      i0 = __dp4a(static_cast<int>(wa[k]), static_cast<int>(x[4 * q + k]), i0);
      r0 = __dp4a(static_cast<int>(wa[k]), static_cast<int>(r[4 * q + k]), r0);
      i1 = __dp4a(static_cast<int>(wb[k]), static_cast<int>(x[8 + 4 * q + k]), i1);
      r1 = __dp4a(static_cast<int>(wb[k]), static_cast<int>(r[8 + 4 * q + k]), r1);
    }
  }
  acc = block_acc(acc, static_cast<double>(s0), st, i0, r0);
  return block_acc(acc, static_cast<double>(s1), st, i1, r1);
}

// ------------------------------------------------- exact fp32 weight decode
// The fp32 weight src/native.c:14-30 computes, element j of a device row.

__device__ __forceinline__ float weight_q4k(const uint8_t* row, unsigned j) {
  const uint8_t* b = row + (j / 256) * 144;
  const unsigned g = j % 256 / 32;
  const uint8_t* s = b + 4;
  unsigned sc, mi;
  if (g < 4) {
    sc = s[g] & 63; mi = s[g + 4] & 63;
  } else {
    sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
    mi = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
  }
  const float d = h2f(b[0] | b[1] << 8), m = h2f(b[2] | b[3] << 8);
  const unsigned q = (b[16 + (g / 2) * 32 + j % 32] >> ((g % 2) * 4)) & 15;
  // (d*sc)*q is exact, m*mi is exact: one rounding of their difference.
  return __fmaf_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q),
                   -__fmul_rn(m, static_cast<float>(mi)));
}
__device__ __forceinline__ float e2m1(unsigned nib) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = 0.0f;
#pragma unroll
  for (unsigned i = 0; i < 8; ++i) v = (nib & 7) == i ? mag[i] : v;
  return nib & 8 && v != 0.0f ? -v : v;  // nibble 8 is +0 in the reference table (src/native.c:10)
}
__device__ __forceinline__ float weight_mxfp4(const uint8_t* row, unsigned nb, unsigned j) {
  const unsigned blk = j / 32, n = j % 32, e = row[blk];
  if (e == 255) return __int_as_float(0x7fc00000);
  const unsigned nib = (row[nb + 16 * blk + (n & 15)] >> (n >> 4 ? 4 : 0)) & 15;
  return __fmul_rn(__uint_as_float(e ? e << 23 : 0x00400000u), e2m1(nib));
}
__device__ __forceinline__ float weight_q80(const uint8_t* row, unsigned nb, unsigned j) {
  const unsigned blk = j / 32;
  const float d = h2f(row[2 * blk] | row[2 * blk + 1] << 8);
  return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(row[2 * nb + j])));
}
__device__ __forceinline__ float weight_any(const uint8_t* row, unsigned type, unsigned n, unsigned j) {
  if (type == kQ4K) return weight_q4k(row, j);
  if (type == kMXFP4) return weight_mxfp4(row, n / 32, j);
  return weight_q80(row, n / 32, j);
}

// splitmix64 of (seed, index): the same function as frc_rand64 on the host.
__host__ __device__ __forceinline__ uint64_t rand64(uint64_t seed, uint64_t index) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (index + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace frc
