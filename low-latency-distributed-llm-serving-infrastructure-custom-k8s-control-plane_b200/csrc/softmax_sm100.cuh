// Softmax arithmetic shared by the tcgen05 prefill kernels: packed fp32 pairs (the sm_100 f32x2
// instructions do two lanes of math per issue slot), a three-input max, and 2^x by a cubic on the
// FMA pipe for the share of the exponentials that the SFU should not carry.
#pragma once

#include "common.cuh"

namespace b200 {
namespace {

// ---- packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for two lanes of math) -----
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for both lanes of a packed pair on the FMA and integer pipes, leaving the SFU (whose ex2
// throughput, shared by both softmax warpgroups, is what the softmax otherwise waits on) to the
// other pairs.  x = j + f with j = round(x) -- adding 1.5 * 2^23 rounds to an integer held in the
// low mantissa bits -- and f in [-0.5, 0.5]; 2^f comes from a cubic fitted here to 2^f on that
// interval by relative least squares (maximum relative error 7.5e-5, against bf16's 2^-9), and j
// is added to its exponent field.  Lanes are clamped to x >= -126 first, so masked (-inf) and
// vanishing terms give a result of at most 2^-126 instead of a wrapped exponent.
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& p0, float& p1) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x2 = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t = f2_add(x2, f2_pack(12582912.f, 12582912.f));
  const uint64_t r = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(r, f2_pack(-1.f, -1.f), x2);
  uint64_t p = f2_fma(f2_pack(0.0551716648f, 0.0551716648f), f, f2_pack(0.2426111251f, 0.2426111251f));
  p = f2_fma(p, f, f2_pack(0.6932609677f, 0.6932609677f));
  p = f2_fma(p, f, f2_pack(0.9999280572f, 0.9999280572f));
  float t0, t1, q0, q1;
  f2_unpack(t, t0, t1);
  f2_unpack(p, q0, q1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

}  // namespace
}  // namespace b200
