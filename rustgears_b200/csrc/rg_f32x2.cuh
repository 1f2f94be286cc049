// rg_f32x2.cuh -- packed f32 pairs for the GEMM epilogue's GELU.
//
// sm_100a executes add/sub/mul/fma on two f32 values held in one 64-bit register
// pair as a single instruction (PTX .f32x2), each element rounded exactly as the
// scalar .rn operation would round it.  The exact tanh of the GELU epilogue
// (tanh_f32_common) issues about fifty IEEE operations per value; done on pairs, the
// epilogue issues a fifth fewer instructions.  Integer steps, conversions,
// reciprocal estimates and selects stay per element.
#pragma once
#include <stdint.h>
#include "rg_math.cuh"

namespace rg {

struct f32x2 { uint64_t v; };  // element 0 in the low 32 bits

__device__ __forceinline__ f32x2 pack2(float a, float b) {
  return f32x2{((uint64_t)f2u(b) << 32) | f2u(a)};
}
__device__ __forceinline__ float lo2(f32x2 r) { return u2f((uint32_t)r.v); }
__device__ __forceinline__ float hi2(f32x2 r) { return u2f((uint32_t)(r.v >> 32)); }
__device__ __forceinline__ f32x2 splat2(float c) { return pack2(c, c); }
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
// A product whose result feeds an addition or subtraction.  ptxas merges a packed
// multiply into a following packed add (an FMA, one rounding instead of two) even
// with --fmad=false, but not a flush-to-zero multiply into an IEEE add; every such
// product of the tanh path has normal (or exactly zero) operands and result, where
// flushing subnormals changes nothing.
__device__ __forceinline__ f32x2 mul2_ftz(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}

// a / b rounded to nearest for the tanh path's operands, given nb = -b: the
// Markstein sequence of div_path<true>, each step the same real operation
// (-b * y + 1 is nb * y + 1), so both elements equal div_path<true>(a, b).
__device__ __forceinline__ f32x2 div2_negden(f32x2 a, f32x2 nb) {
  float y0, y1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(-lo2(nb)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y1) : "f"(-hi2(nb)));
  f32x2 y = pack2(y0, y1);
  y = fma2(y, fma2(nb, y, splat2(1.0f)), y);
  const f32x2 q = mul2(a, y);
  return fma2(fma2(nb, q, a), y, q);
}

// tanh_f32_common on two values, its floating-point steps as packed pairs and its
// integer steps and selects per element: each result is bit-identical to
// tanh_f32_common<true> of that element.
__device__ __forceinline__ void tanh_f32_common_x2(float x0, float x1, float& z0, float& z1) {
  const float ln2_hi = u2f(0x3f317180u), ln2_lo = u2f(0x3717f7d1u), invln2 = u2f(0x3fb8aa3bu);
  const float q1 = u2f(0xbd088889u), q2 = u2f(0x3ad00d01u), q3 = u2f(0xb8a670cdu),
              q4 = u2f(0x36867e54u), q5 = u2f(0xb457edbbu);
  const uint32_t jx0 = f2u(x0), jx1 = f2u(x1);
  const bool big0 = (jx0 & 0x7fffffffu) >= 0x3f800000u, big1 = (jx1 & 0x7fffffffu) >= 0x3f800000u;
  const float tax0 = __fmul_rn(2.0f, fabsf(x0)), tax1 = __fmul_rn(2.0f, fabsf(x1));
  const f32x2 a = pack2(big0 ? tax0 : -tax0, big1 ? tax1 : -tax1);
  const f32x2 kv = add2(mul2_ftz(splat2(invln2), a), pack2(big0 ? 0.5f : -0.5f, big1 ? 0.5f : -0.5f));
  int k0 = (int)lo2(kv), k1 = (int)hi2(kv);
  const uint32_t hx0 = f2u(tax0), hx1 = f2u(tax1);
  k0 = hx0 < 0x3F851592u ? (big0 ? 1 : -1) : k0;
  k1 = hx1 < 0x3F851592u ? (big1 ? 1 : -1) : k1;
  k0 = hx0 > 0x3eb17218u ? k0 : 0;
  k1 = hx1 > 0x3eb17218u ? k1 : 0;
  const f32x2 t = pack2((float)k0, (float)k1);
  const f32x2 hi = sub2(a, mul2_ftz(t, splat2(ln2_hi)));
  const f32x2 lo = mul2_ftz(t, splat2(ln2_lo));
  const f32x2 xr = sub2(hi, lo);
  const f32x2 c = sub2(sub2(hi, xr), lo);
  const f32x2 hfx = mul2(splat2(0.5f), xr);
  const f32x2 hxs = mul2_ftz(xr, hfx);
  f32x2 r1 = mul2_ftz(hxs, splat2(q5));
  r1 = mul2_ftz(hxs, add2(splat2(q4), r1));
  r1 = mul2_ftz(hxs, add2(splat2(q3), r1));
  r1 = mul2_ftz(hxs, add2(splat2(q2), r1));
  r1 = mul2_ftz(hxs, add2(splat2(q1), r1));
  r1 = add2(splat2(1.0f), r1);
  const f32x2 tt = sub2(splat2(3.0f), mul2_ftz(r1, hfx));
  // e = hxs * ((r1 - tt) / (6 - xr * tt)), the divisor formed negated (xr * tt - 6)
  const f32x2 e = mul2_ftz(hxs, div2_negden(sub2(r1, tt), sub2(mul2_ftz(xr, tt), splat2(6.0f))));
  const f32x2 res0 = sub2(xr, sub2(mul2_ftz(xr, e), hxs));                      // k == 0
  const f32x2 e2 = sub2(sub2(mul2_ftz(xr, sub2(e, c)), c), hxs);
  const f32x2 res_m1 = sub2(mul2_ftz(splat2(0.5f), sub2(xr, e2)), splat2(0.5f));  // k == -1
  const float base0 = k0 < 0 ? 1.0f : u2f(0x3f800000u - (0x1000000u >> (k0 & 31)));
  const float base1 = k1 < 0 ? 1.0f : u2f(0x3f800000u - (0x1000000u >> (k1 & 31)));
  const f32x2 s = sub2(pack2(base0, base1), sub2(e2, xr));
  const float sc0 = u2f(f2u(lo2(s)) + ((uint32_t)k0 << 23)), sc1 = u2f(f2u(hi2(s)) + ((uint32_t)k1 << 23));
  const f32x2 scm1 = sub2(pack2(sc0, sc1), splat2(1.0f));
  const float ab0 = k0 < 0 ? lo2(scm1) : sc0, ab1 = k1 < 0 ? hi2(scm1) : sc1;  // k <= -2; 3 <= k <= 22
  const float em0 = k0 == 0 ? lo2(res0) : (k0 == -1 ? lo2(res_m1) : ab0);
  const float em1 = k1 == 0 ? hi2(res0) : (k1 == -1 ? hi2(res_m1) : ab1);
  // tanh from expm1: q = (big ? 2 : -em) / (em + 2), the divisor formed negated (-2 - em)
  const f32x2 q = div2_negden(pack2(big0 ? 2.0f : -em0, big1 ? 2.0f : -em1), sub2(splat2(-2.0f), pack2(em0, em1)));
  const f32x2 omq = sub2(splat2(1.0f), q);
  const float w0 = big0 ? lo2(omq) : lo2(q), w1 = big1 ? hi2(omq) : hi2(q);
  z0 = (jx0 >> 31) ? -w0 : w0;
  z1 = (jx1 >> 31) ? -w1 : w1;
}

// gelu_arg and gelu_from_tanh on a pair.
__device__ __forceinline__ f32x2 gelu_arg_x2(f32x2 x) {
  f32x2 c = mul2(splat2(0.044715f), x);
  c = mul2(c, x);
  c = mul2_ftz(c, x);  // 0.044715 x^3 is below half an ulp of x wherever it is subnormal
  return mul2(splat2(0.7978846f), add2(x, c));
}
__device__ __forceinline__ f32x2 gelu_from_tanh_x2(f32x2 x, f32x2 t) {
  return mul2(mul2(splat2(0.5f), x), add2(splat2(1.0f), t));
}
}  // namespace rg
