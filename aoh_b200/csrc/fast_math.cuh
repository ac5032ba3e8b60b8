// Packed f32x2 arithmetic (sm_100: one FMA-pipe instruction per pair of fp32
// lanes held in a 64-bit register), a three-input max, and a polynomial 2^x on
// the FMA pipe for the prefill softmax.
#pragma once

#include <stdint.h>

namespace aoh {

// Two fp32 lanes in one 64-bit register, for the packed f32x2 arithmetic of
// sm_100 (one instruction per pair on the FMA pipe).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair, on the FMA pipe, for -inf < x <= 8: x = j + f with
// j = round(x) (adding 1.5 * 2^23 rounds to an integer held in the low mantissa
// bits) and f in [-0.5, 0.5]; 2^f is a cubic fitted for least maximum relative
// error on that interval (7.5e-5, below half a bf16 ulp of P), and j is added
// to its exponent field.  x is clamped to -126 so the exponent stays in range
// (2^-126 then stands for anything smaller).
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& p0, float& p1) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const uint64_t x = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t magic = f2_pack(12582912.f, 12582912.f);
  const uint64_t t = f2_add(x, magic);
  const uint64_t f = f2_sub(x, f2_sub(t, magic));
  uint64_t p = f2_fma(f, f2_pack(0.05517132f, 0.05517132f), f2_pack(0.24261054f, 0.24261054f));
  p = f2_fma(p, f, f2_pack(0.69326097f, 0.69326097f));
  p = f2_fma(p, f, f2_pack(0.99992812f, 0.99992812f));
  float q0, q1, t0, t1;
  f2_unpack(p, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

}  // namespace aoh
