// rg_math.cuh -- scalar arithmetic of the Npu(Int8) path, shared by every kernel.
//
// Every function reproduces the reference's f32 arithmetic operation by
// operation (round-to-nearest, no contraction: the library is compiled with
// -fmad=false and the critical steps use explicit __f*_rn intrinsics), so
// the device results are bit-identical to the reference CPU path.
//
// Transcendentals: the reference calls Rust's f32::tanh / f32::exp, i.e.
// glibc 2.39's tanhf / expf on x86-64 linux-gnu.  glibc is not correctly
// rounded (tanhf differs from the correctly rounded result on ~2.8% of all
// floats), so the device uses restatements of glibc's own published methods:
//   * tanhf: the fdlibm method (Sun Microsystems, 1993), tanh via expm1 with
//     expm1 by argument reduction x = k ln2 + r and a rational approximation
//     of r (e^r + 1)/(e^r - 1);
//   * expf: the method of ARM's optimized-routines (Szabolcs Nagy, 2017) that
//     glibc ships since 2.27: x/ln2 split into k/32 + r, 2^(k/32) from a
//     32-entry table, a cubic for 2^r evaluated in double.  On x86-64 CPUs
//     with FMA glibc selects its FMA build, whose rounding the fma() calls
//     below reproduce.
// Both restatements match glibc 2.39 on all 2^32 f32 inputs (checked
// exhaustively on the host); the GPU tests re-check them on the device.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define RG_HD __host__ __device__ __forceinline__
#else
#define RG_HD inline
#endif

namespace rg {

enum : int32_t { ACT_NONE = 0, ACT_RELU = 1, ACT_SIGMOID = 2, ACT_TANH = 3, ACT_GELU = 4,
                 ACT_LEAKY_RELU = 5, ACT_SILU = 6 };

RG_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  union { float f; uint32_t u; } v; v.f = f; return v.u;
#endif
}
RG_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  union { float f; uint32_t u; } v; v.u = u; return v.f;
#endif
}
RG_HD uint64_t d2u(double d) {
#ifdef __CUDA_ARCH__
  return (uint64_t)__double_as_longlong(d);
#else
  union { double d; uint64_t u; } v; v.d = d; return v.u;
#endif
}
RG_HD double u2d(uint64_t u) {
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)u);
#else
  union { double d; uint64_t u; } v; v.u = u; return v.d;
#endif
}

#ifdef __CUDA_ARCH__
#define RG_MUL(a, b) __fmul_rn((a), (b))
#define RG_ADD(a, b) __fadd_rn((a), (b))
#define RG_SUB(a, b) __fsub_rn((a), (b))
#define RG_DIV(a, b) __fdiv_rn((a), (b))
#else
#define RG_MUL(a, b) ((a) * (b))
#define RG_ADD(a, b) ((a) + (b))
#define RG_SUB(a, b) ((a) - (b))
#define RG_DIV(a, b) ((a) / (b))
#endif

// Division rounded to nearest for the well-scaled operands of the tanh path
// (normal, finite divisor and quotient): Markstein's method -- a reciprocal
// estimate (PTX rcp.approx), one Newton-Raphson step y += y (1 - b y), the
// quotient q = a y, and one correction q += (a - b q) y with the remainder
// formed exactly by an FMA (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  Five
// FMA-pipe operations and one reciprocal estimate, against the IEEE division's
// range checks.  Its equality with the IEEE division on the path's whole input
// range (every f32 input of tanh_f32) is checked exhaustively on the device.
template <bool kNR>
RG_HD float div_path(float a, float b) {
#ifdef __CUDA_ARCH__
  if (kNR) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    y = __fmaf_rn(y, __fmaf_rn(-b, y, 1.0f), y);
    const float q = __fmul_rn(a, y);
    return __fmaf_rn(__fmaf_rn(-b, q, a), y, q);
  }
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}

RG_HD float fmax_ignore_nan(float a, float b) { return fmaxf(a, b); }  // IEEE maxNum == f32::max

// expm1 for the tanh argument range (|x| < 44); fdlibm method, f32 steps.
RG_HD float expm1_f32(float x) {
  const float ln2_hi = u2f(0x3f317180u), ln2_lo = u2f(0x3717f7d1u), invln2 = u2f(0x3fb8aa3bu);
  const float q1 = u2f(0xbd088889u), q2 = u2f(0x3ad00d01u), q3 = u2f(0xb8a670cdu),
              q4 = u2f(0x36867e54u), q5 = u2f(0xb457edbbu);
  uint32_t hx = f2u(x);
  const bool neg = (hx >> 31) != 0;
  hx &= 0x7fffffffu;
  if (hx >= 0x4195b844u) {  // |x| >= 27 ln2: saturates to -1 (negative side); tanh never asks above
    if (hx > 0x7f800000u) return RG_ADD(x, x);
    if (neg) return -1.0f;
  }
  float hi, lo, c = 0.0f, t;
  int k;
  if (hx > 0x3eb17218u) {                          // |x| > ln2 / 2: reduce
    if (hx < 0x3F851592u) {                        // |x| < 3 ln2 / 2
      if (!neg) { hi = RG_SUB(x, ln2_hi); lo = ln2_lo; k = 1; }
      else { hi = RG_ADD(x, ln2_hi); lo = -ln2_lo; k = -1; }
    } else {
      k = (int)RG_ADD(RG_MUL(invln2, x), neg ? -0.5f : 0.5f);
      t = (float)k;
      hi = RG_SUB(x, RG_MUL(t, ln2_hi));
      lo = RG_MUL(t, ln2_lo);
    }
    x = RG_SUB(hi, lo);
    c = RG_SUB(RG_SUB(hi, x), lo);
  } else if (hx < 0x33000000u) {
    return x;                                      // |x| < 2^-25
  } else {
    k = 0;
  }
  const float hfx = RG_MUL(0.5f, x);
  const float hxs = RG_MUL(x, hfx);
  float r1 = RG_MUL(hxs, q5);
  r1 = RG_MUL(hxs, RG_ADD(q4, r1));
  r1 = RG_MUL(hxs, RG_ADD(q3, r1));
  r1 = RG_MUL(hxs, RG_ADD(q2, r1));
  r1 = RG_MUL(hxs, RG_ADD(q1, r1));
  r1 = RG_ADD(1.0f, r1);
  t = RG_SUB(3.0f, RG_MUL(r1, hfx));
  float e = RG_MUL(hxs, RG_DIV(RG_SUB(r1, t), RG_SUB(6.0f, RG_MUL(x, t))));
  if (k == 0) return RG_SUB(x, RG_SUB(RG_MUL(x, e), hxs));
  e = RG_SUB(RG_MUL(x, RG_SUB(e, c)), c);
  e = RG_SUB(e, hxs);
  if (k == -1) return RG_SUB(RG_MUL(0.5f, RG_SUB(x, e)), 0.5f);
  if (k == 1) {
    if (x < -0.25f) return RG_MUL(-2.0f, RG_SUB(e, RG_ADD(x, 0.5f)));
    return RG_ADD(1.0f, RG_MUL(2.0f, RG_SUB(x, e)));
  }
  float y;
  if (k <= -2 || k > 56) {
    y = RG_SUB(1.0f, RG_SUB(e, x));
    y = u2f(f2u(y) + ((uint32_t)k << 23));
    return RG_SUB(y, 1.0f);
  }
  if (k < 23) {
    t = u2f(0x3f800000u - (0x1000000u >> k));     // 1 - 2^-k
    y = RG_SUB(t, RG_SUB(e, x));
  } else {
    t = u2f((uint32_t)(0x7f - k) << 23);           // 2^-k
    y = RG_SUB(x, RG_ADD(e, t));
    y = RG_ADD(y, 1.0f);
  }
  return u2f(f2u(y) + ((uint32_t)k << 23));
}

// expm1 on the arguments tanh_f32 gives it (a = 2|x| in [2, 44) or a = -2|x| in
// (-2, 0]), evaluated without divergent branches: the reduction x = k ln2 + (hi - lo)
// with t = (float)k reproduces expm1_f32's reduction cases exactly (k = 0 gives
// hi = a, lo = c = 0; k = -1 gives hi = a + ln2_hi, lo = -ln2_lo), and the
// reconstructions are computed side by side and selected by k.  On that domain k is
// never 1 (a >= 2 gives k >= 3), so that reconstruction is omitted.  Bit-identical
// to expm1_f32 on the domain.
template <bool kNR = true>
RG_HD float expm1_tanh_arg(float a) {
  const float ln2_hi = u2f(0x3f317180u), ln2_lo = u2f(0x3717f7d1u), invln2 = u2f(0x3fb8aa3bu);
  const float q1 = u2f(0xbd088889u), q2 = u2f(0x3ad00d01u), q3 = u2f(0xb8a670cdu),
              q4 = u2f(0x36867e54u), q5 = u2f(0xb457edbbu);
  const uint32_t hx = f2u(a) & 0x7fffffffu;
  const bool neg = a < 0.0f;
  int k = (int)RG_ADD(RG_MUL(invln2, a), neg ? -0.5f : 0.5f);
  k = hx < 0x3F851592u ? (neg ? -1 : 1) : k;
  k = hx > 0x3eb17218u ? k : 0;
  const float t = (float)k;
  const float hi = RG_SUB(a, RG_MUL(t, ln2_hi));
  const float lo = RG_MUL(t, ln2_lo);
  const float x = RG_SUB(hi, lo);
  const float c = RG_SUB(RG_SUB(hi, x), lo);
  const float hfx = RG_MUL(0.5f, x);
  const float hxs = RG_MUL(x, hfx);
  float r1 = RG_MUL(hxs, q5);
  r1 = RG_MUL(hxs, RG_ADD(q4, r1));
  r1 = RG_MUL(hxs, RG_ADD(q3, r1));
  r1 = RG_MUL(hxs, RG_ADD(q2, r1));
  r1 = RG_MUL(hxs, RG_ADD(q1, r1));
  r1 = RG_ADD(1.0f, r1);
  const float tt = RG_SUB(3.0f, RG_MUL(r1, hfx));
  const float e = RG_MUL(hxs, div_path<kNR>(RG_SUB(r1, tt), RG_SUB(6.0f, RG_MUL(x, tt))));
  const float res0 = RG_SUB(x, RG_SUB(RG_MUL(x, e), hxs));               // k == 0
  const float e2 = RG_SUB(RG_SUB(RG_MUL(x, RG_SUB(e, c)), c), hxs);
  const float res_m1 = RG_SUB(RG_MUL(0.5f, RG_SUB(x, e2)), 0.5f);         // k == -1
  const uint32_t kshift = (uint32_t)k << 23;
  const float ya = RG_SUB(1.0f, RG_SUB(e2, x));
  const float res_a = RG_SUB(u2f(f2u(ya) + kshift), 1.0f);                // k <= -2 or k > 56
  const int kc = k < 1 ? 1 : (k > 31 ? 31 : k);                           // in-range shifts only
  const float yb = RG_SUB(u2f(0x3f800000u - (0x1000000u >> kc)), RG_SUB(e2, x));
  const float res_b = u2f(f2u(yb) + kshift);                              // 2 <= k < 23
  const int kd = k < 0 ? 0 : (k > 126 ? 126 : k);
  const float yc = RG_ADD(RG_SUB(x, RG_ADD(e2, u2f((uint32_t)(0x7f - kd) << 23))), 1.0f);
  const float res_c = u2f(f2u(yc) + kshift);                              // 23 <= k <= 56
  float r = res_c;
  r = k < 23 ? res_b : r;
  r = (k <= -2 || k > 56) ? res_a : r;
  r = k == -1 ? res_m1 : r;
  r = k == 0 ? res0 : r;
  return hx < 0x33000000u ? a : r;                                        // |a| < 2^-25
}

// tanh, glibc/fdlibm method (identical on all 2^32 inputs to glibc 2.39 tanhf):
// |x| >= 1: 1 - 2 / (expm1(2|x|) + 2); else -expm1(-2|x|) / (expm1(-2|x|) + 2).
// One expm1 and one division per element, the cases resolved by selects.
template <bool kNR = true>
RG_HD float tanh_f32(float x) {
  const uint32_t jx = f2u(x), ix = jx & 0x7fffffffu;
  const bool big = ix >= 0x3f800000u;                 // |x| >= 1
  const float ax = ix < 0x41b00000u ? fabsf(x) : 1.0f;  // keep the main path finite
  const float two_ax = RG_MUL(2.0f, ax);
  const float t = expm1_tanh_arg<kNR>(big ? two_ax : -two_ax);
  const float q = div_path<kNR>(big ? 2.0f : -t, RG_ADD(t, 2.0f));
  float z = big ? RG_SUB(1.0f, q) : q;
  z = ix < 0x41b00000u ? z : 1.0f;                    // |x| >= 22 (and inf)
  z = (jx >> 31) ? -z : z;
  z = ix < 0x24000000u ? RG_MUL(x, RG_ADD(1.0f, x)) : z;  // |x| < 2^-55
  if (ix > 0x7f800000u) z = RG_ADD(x, x);             // NaN
  return z;
}

// tanh_f32 on its common range |x| in [2^-25, 7.5) (finite), with only the steps
// that range can take.  There the expm1 argument a = +-2|x| has 2^-24 <= |a| < 15,
// so the reduction's k lies in {-3, -2, -1, 0} (|x| < 1) or [3, 22] (|x| >= 1): the
// k = 0 and k = -1 reconstructions, and the k <= -2 and 2 <= k < 23 ones, which
// share their operand (e2 - x) and differ only in the constant it is subtracted from
// (1, or 1 - 2^-k) and in a final - 1; the |x| >= 22, |x| < 2^-55, |a| < 2^-25, NaN and
// 23 <= k <= 56 cases cannot occur.  Every value is computed by the same operations
// in the same order as tanh_f32, so the two agree bit for bit on the range (checked
// on every f32 of it, on the host and by the device self-test).
RG_HD bool tanh_common_range(float x) {
  const uint32_t ix = f2u(x) & 0x7fffffffu;
  return ix >= 0x33000000u && ix < 0x40f00000u;
}
template <bool kNR = true>
RG_HD float tanh_f32_common(float x) {
  const float ln2_hi = u2f(0x3f317180u), ln2_lo = u2f(0x3717f7d1u), invln2 = u2f(0x3fb8aa3bu);
  const float q1 = u2f(0xbd088889u), q2 = u2f(0x3ad00d01u), q3 = u2f(0xb8a670cdu),
              q4 = u2f(0x36867e54u), q5 = u2f(0xb457edbbu);
  const uint32_t jx = f2u(x), ix = jx & 0x7fffffffu;
  const bool big = ix >= 0x3f800000u;                 // |x| >= 1
  const float two_ax = RG_MUL(2.0f, fabsf(x));
  // expm1_tanh_arg(a) on 2^-24 <= |a| < 15
  const float a = big ? two_ax : -two_ax;
  const uint32_t hx = f2u(two_ax);
  int k = (int)RG_ADD(RG_MUL(invln2, a), big ? 0.5f : -0.5f);
  k = hx < 0x3F851592u ? (big ? 1 : -1) : k;
  k = hx > 0x3eb17218u ? k : 0;
  const float t = (float)k;
  const float hi = RG_SUB(a, RG_MUL(t, ln2_hi));
  const float lo = RG_MUL(t, ln2_lo);
  const float xr = RG_SUB(hi, lo);
  const float c = RG_SUB(RG_SUB(hi, xr), lo);
  const float hfx = RG_MUL(0.5f, xr);
  const float hxs = RG_MUL(xr, hfx);
  float r1 = RG_MUL(hxs, q5);
  r1 = RG_MUL(hxs, RG_ADD(q4, r1));
  r1 = RG_MUL(hxs, RG_ADD(q3, r1));
  r1 = RG_MUL(hxs, RG_ADD(q2, r1));
  r1 = RG_MUL(hxs, RG_ADD(q1, r1));
  r1 = RG_ADD(1.0f, r1);
  const float tt = RG_SUB(3.0f, RG_MUL(r1, hfx));
  const float e = RG_MUL(hxs, div_path<kNR>(RG_SUB(r1, tt), RG_SUB(6.0f, RG_MUL(xr, tt))));
  const float res0 = RG_SUB(xr, RG_SUB(RG_MUL(xr, e), hxs));                 // k == 0
  const float e2 = RG_SUB(RG_SUB(RG_MUL(xr, RG_SUB(e, c)), c), hxs);
  const float res_m1 = RG_SUB(RG_MUL(0.5f, RG_SUB(xr, e2)), 0.5f);          // k == -1
  const float base = k < 0 ? 1.0f : u2f(0x3f800000u - (0x1000000u >> (k & 31)));
  const float sc = u2f(f2u(RG_SUB(base, RG_SUB(e2, xr))) + ((uint32_t)k << 23));
  const float res_ab = k < 0 ? RG_SUB(sc, 1.0f) : sc;                       // k <= -2; 3 <= k <= 22
  const float em1 = k == 0 ? res0 : (k == -1 ? res_m1 : res_ab);
  // tanh from expm1
  const float q = div_path<kNR>(big ? 2.0f : -em1, RG_ADD(em1, 2.0f));
  const float z = big ? RG_SUB(1.0f, q) : q;
  return (jx >> 31) ? -z : z;
}

// 2^(i/32) rounded to double, minus i << 47 (the table of the expf method).
#define RG_EXP2_TABLE                                                                  \
  {0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full,                 \
   0x3fef9301d0125b51ull, 0x3fef72b83c7d517bull, 0x3fef54873168b9aaull,                 \
   0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, 0x3fef06fe0a31b715ull,                 \
   0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,                 \
   0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull,                 \
   0x3feea47eb03a5585ull, 0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull,                 \
   0x3feea11473eb0187ull, 0x3feea589994cce13ull, 0x3feeace5422aa0dbull,                 \
   0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,                 \
   0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull,                 \
   0x3fef3720dcef9069ull, 0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full,                 \
   0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull}

#ifdef __CUDACC__
static __constant__ const uint64_t k_exp2_table[32] = RG_EXP2_TABLE;
#endif
static const uint64_t h_exp2_table[32] = RG_EXP2_TABLE;
#ifdef __CUDA_ARCH__
#define RG_EXP2_T(i) k_exp2_table[(i)]
#else
#define RG_EXP2_T(i) h_exp2_table[(i)]
#endif

// The 2^(i/32) table read through the constant bank (host: the host copy).
struct ExpTableConst {
  RG_HD uint64_t operator()(uint32_t i) const { return RG_EXP2_T(i); }
};
// ... or through a pointer (a shared-memory copy serves lanes that index different
// entries in one access, where the constant bank serialises them).
struct ExpTablePtr {
  const uint64_t* p;
  RG_HD uint64_t operator()(uint32_t i) const { return p[i]; }
};

// exp, optimized-routines method in its FMA form (identical on all 2^32 inputs to glibc 2.39 expf
// on an x86-64 CPU with FMA).
template <class Tab>
RG_HD float exp_f32_with(float x, Tab tab) {
  const uint32_t ax = f2u(x) & 0x7fffffffu;
  if (ax >= 0x42b00000u) {                         // |x| >= 88
    if (f2u(x) == 0xff800000u) return 0.0f;
    if (ax >= 0x7f800000u) return RG_ADD(x, x);
    if (x > u2f(0x42b17217u)) return u2f(0x7f800000u);
    if (x < -u2f(0x42cff1b4u)) return 0.0f;
  }
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
  const double shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
  const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
#ifdef __CUDA_ARCH__
  const double z = __dmul_rn(inv_ln2_n, xd);
  double kd = __dadd_rn(z, shift);
  const uint64_t ki = d2u(kd);
  kd = __dsub_rn(kd, shift);
#else
  volatile double zv = inv_ln2_n * xd;
  const double z = zv;
  volatile double kdv = z + shift;
  double kd = kdv;
  const uint64_t ki = d2u(kd);
  kd = kd - shift;
#endif
  (void)z;
  const double r = fma(inv_ln2_n, xd, -kd);
  uint64_t t = tab((uint32_t)(ki % 32));
  t += ki << (52 - 5);
  const double s = u2d(t);
  const double zz = fma(c0, r, c1);
#ifdef __CUDA_ARCH__
  const double r2 = __dmul_rn(r, r);
#else
  const double r2 = r * r;
#endif
  double y = fma(c2, r, 1.0);
  y = fma(zz, r2, y);
#ifdef __CUDA_ARCH__
  y = __dmul_rn(y, s);
  return __double2float_rn(y);
#else
  y = y * s;
  return (float)y;
#endif
}

RG_HD float exp_f32(float x) { return exp_f32_with(x, ExpTableConst{}); }

// GELU (tanh form) of Activation::apply (src/device/backend.rs:61-68):
// 0.5 * x * (1 + tanh(u)) with u = GELU_C * (x + 0.044715 * x * x * x).
RG_HD float gelu_arg(float x) {
  const float gelu_c = 0.7978846f;                               // GELU_C (backend.rs:61)
  float c = RG_MUL(0.044715f, x);
  c = RG_MUL(c, x);
  c = RG_MUL(c, x);
  return RG_MUL(gelu_c, RG_ADD(x, c));
}
RG_HD float gelu_from_tanh(float x, float t) { return RG_MUL(RG_MUL(0.5f, x), RG_ADD(1.0f, t)); }
template <bool kNR = true>
RG_HD float gelu_f32(float x) {
  return gelu_from_tanh(x, tanh_f32<kNR>(gelu_arg(x)));
}

// round_fp16 (src/inference/quantize.rs:50-64), the FP16 arm's emulation of a
// binary16 value: exponent below -14 -> +0 (sign dropped), above 15 -> +-65504
// (infinities and NaN included), otherwise 10 mantissa bits kept with the 13th
// bit rounding the magnitude up (a carry may reach 65536).
RG_HD float round_fp16(float x) {
  const uint32_t bits = f2u(x);
  const int32_t e = (int32_t)((bits >> 23) & 0xffu) - 127;
  if (e < -14) return 0.0f;
  if (e > 15) return u2f((bits & 0x80000000u) | 0x477fe000u);
  return u2f((bits + (1u << 12)) & ~0x1fffu);
}

// Activation::apply (src/inference/mod.rs:38-53, src/device/backend.rs:61-78).
RG_HD float act_apply(int32_t act, float p, float x) {
  switch (act) {
    case ACT_RELU: return fmaxf(x, 0.0f);                       // x.max(0.0): NaN -> 0
    case ACT_SIGMOID: return RG_DIV(1.0f, RG_ADD(1.0f, exp_f32(-x)));
    case ACT_TANH: return tanh_f32(x);
    case ACT_GELU: return gelu_f32(x);
    case ACT_LEAKY_RELU: return x > 0.0f ? x : RG_MUL(p, x);
    // extension: nn::Silu (src/nn/layers.rs:337-346), x * sigmoid(x) with the sigmoid above
    case ACT_SILU: return RG_MUL(x, RG_DIV(1.0f, RG_ADD(1.0f, exp_f32(-x))));
    default: return x;
  }
}

// QuantTensor scale from an absmax (quantize.rs:20) and its reciprocal (quantize.rs:21).
// On the device the divisions use div_path<true> for finite operands (amax >= 1e-12
// and scale in [7.8e-15, 2.7e36]: normal dividends, divisors and quotients); the IEEE
// division handles infinities.  Equal to the IEEE results for every f32 absmax
// (checked exhaustively on the device).
template <bool kNR = true>
RG_HD float quant_scale(float amax) {
  if (amax < 1e-12f) return 1.0f;
#ifdef __CUDA_ARCH__
  if (kNR && isfinite(amax)) return div_path<true>(amax, 127.0f);
#endif
  return RG_DIV(amax, 127.0f);
}
template <bool kNR = true>
RG_HD float quant_inv(float scale) {
#ifdef __CUDA_ARCH__
  if (kNR && isfinite(scale)) return div_path<true>(1.0f, scale);
#endif
  return RG_DIV(1.0f, scale);
}

// (v * inv).round().clamp(-127, 127) as i8 (quantize.rs:22): half away from zero, NaN -> 0.
RG_HD int32_t quant1(float v, float inv) {
  const float t = roundf(RG_MUL(v, inv));
  if (t != t) return 0;
  return (int32_t)fminf(fmaxf(t, -127.0f), 127.0f);
}

// Round half away from zero to an integer, for |t| < 2^23 and NaN (-> 0):
// t + copysign(0.5 - 2^-25, t) rounds (to nearest even) past the next integer
// exactly when |frac(t)| >= 0.5, so truncating it gives roundf(t); the bias below
// one half keeps |t| = 0.5 - 2^-25 from rounding up.  The device conversion turns
// NaN into 0.  Equal to roundf + NaN -> 0 on every f32 with |t| < 2^23 (checked
// exhaustively on the device).
RG_HD int32_t round_half_away(float t) {
#ifdef __CUDA_ARCH__
  const float h = __uint_as_float((__float_as_uint(t) & 0x80000000u) | 0x3effffffu);
  return __float2int_rz(__fadd_rn(t, h));
#else
  const float r = roundf(t);
  return r != r ? 0 : (int32_t)r;
#endif
}

// quant1 for a value of the tensor whose absmax gave `inv` (|v| <= amax):
// |v * inv| <= 127 (1 + 3 * 2^-24) < 127.5, so the clamp never acts and is left out.
RG_HD int32_t quant1_bounded(float v, float inv) { return round_half_away(RG_MUL(v, inv)); }

// (acc as f32) * cs + bias, the pre-activation value of int8_gemm_fused's epilogue.
RG_HD float dequant(int32_t acc, float cs, float bias) {
#ifdef __CUDA_ARCH__
  const float a = __int2float_rn(acc);
#else
  const float a = (float)acc;
#endif
  return RG_ADD(RG_MUL(a, cs), bias);
}

// Epilogue of int8_gemm_fused (quantize.rs:109-111): act((acc as f32) * cs + bias).
RG_HD float epilogue(int32_t acc, float cs, float bias, int32_t act, float p) {
  return act_apply(act, p, dequant(acc, cs, bias));
}

// Same with the activation fixed at compile time: the switch folds away, so a
// kernel instantiated per activation carries only that activation's code.
template <int ACT>
RG_HD float epilogue_t(int32_t acc, float cs, float bias, float p) {
  return epilogue(acc, cs, bias, ACT, p);
}

// f32(acc) for |acc| < 2^22 without a conversion instruction: 1.5 * 2^23 + acc is an
// integer in [2^23, 2^24), where f32 spacing is exactly 1, so its bit pattern is
// 0x4B400000 + acc and subtracting 1.5 * 2^23 is exact.  Equal to the round-to-nearest
// conversion on that range (both exact).
RG_HD float small_i32_to_f32(int32_t acc) {
#ifdef __CUDA_ARCH__
  return __fsub_rn(__int_as_float(0x4B400000 + acc), 12582912.0f);
#else
  return (float)acc;
#endif
}

// epilogue_t for accumulators known to satisfy |acc| < 2^22.
template <int ACT>
RG_HD float epilogue_small_t(int32_t acc, float cs, float bias, float p) {
  return act_apply(ACT, p, RG_ADD(RG_MUL(small_i32_to_f32(acc), cs), bias));
}


}  // namespace rg
