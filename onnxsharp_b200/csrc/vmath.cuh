// vmath.cuh — the reference engine's vector transcendental functions, restated
// for the device so that fused epilogues produce the same bits as the CPU
// path's AVX2 bulk loop.
//
// Reference: src/OnnxSharp/Tensors/VectorMath.cs:21-43 (Exp: clamp to
// [-87.3, 88.7], n = rint(x*log2e), two-step Cody-Waite reduction, degree-6
// Horner polynomial with explicit FMAs, 2^n built from exponent bits),
// :70-74 (Sigmoid = 1/(1+exp(-x)), the quotient correctly rounded as the
// reference's IEEE division), :77 (Silu = x*sigmoid(x)).
// Every operation uses an explicitly rounded intrinsic so nvcc cannot contract
// or reorder it.
#pragma once

#include <cuda_runtime.h>

namespace osc {

__device__ __forceinline__ float ref_exp(float x) {
  // Avx.Max(x, c) returns c for NaN x, as fmaxf does.
  x = fminf(fmaxf(x, -87.3f), 88.7f);
  // rint(x*log2e) by the round-to-nearest-even of an add to 1.5*2^23: for
  // |v| < 2^22 the sum lies in [2^23, 2^24) where the float spacing is 1, so
  // t = v + C rounds v to the nearest integer, ties to even, exactly as
  // rint, and t - C is exact; the integer n also sits in t's low mantissa
  // bits. Here |v| <= 128. Plain FP32 adds and integer ops instead of the
  // quarter-rate round/convert instructions.
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float t = __fadd_rn(__fmul_rn(x, 1.4426950408889634f), kRound);
  const float n = __fsub_rn(t, kRound);
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.4286067653e-6f, r);
  float p = 1.0f / 720.0f;
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int e = (__float_as_int(t) - 0x4B400000 + 127) << 23;  // (n + 127) << 23
  return __fmul_rn(p, __int_as_float(e));
}

// Correctly rounded 1/d for d in [1, 2^126) without a branch: hardware
// reciprocal approximation (rcp.approx.f32, relative error <= 2^-23), one
// Newton-Raphson step and Markstein's final FMA correction
// y = y1 + y1*(1 - d*y1) (P. Markstein, "IA-64 and Elementary Functions",
// 2000). The sigmoid's divisor 1 + exp(-x) always lies in this range (the
// exp argument is clamped to [-87.3, 88.7]), so the quotient is normal and
// the result equals the IEEE division 1/d; tests/test_vmath_gpu.py checks
// every float d in [1, 2^126) against __fdiv_rn(1, d).
__device__ __forceinline__ float recip_1up(float d) {
  float y;
  asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(d));
  const float e = __fmaf_rn(-d, y, 1.0f);
  y = __fmaf_rn(y, e, y);
  const float r = __fmaf_rn(-d, y, 1.0f);
  return __fmaf_rn(y, r, y);
}

__device__ __forceinline__ float ref_sigmoid(float x) {
  return recip_1up(__fadd_rn(1.0f, ref_exp(__fmul_rn(x, -1.0f))));
}

__device__ __forceinline__ float ref_silu(float x) { return __fmul_rn(x, ref_sigmoid(x)); }

// Activation codes shared by every fused epilogue (match osc_act in the C ABI).
// ACT_FAST may be OR-ed into SiLU / Sigmoid: the hardware-instruction form
// (fast_sigmoid below) instead of the exact restatement.
enum : int { ACT_NONE = 0, ACT_SILU = 1, ACT_RELU = 2, ACT_SIGMOID = 3, ACT_FAST = 16 };

// The activation as a compile-time constant: a loop over act_t<ACT> has no
// branch per element, so the compiler interleaves the independent exp /
// reciprocal chains of consecutive elements (with a runtime switch inside
// the loop each element's chain runs alone, latency-bound).

// Sigmoid and SiLU for the tensor-core conv epilogues: 1 / (1 + 2^(-x log2 e))
// from the hardware ex2.approx and rcp.approx instructions (relative errors
// 2^-22 and 2^-23), 5 instructions instead of the ~25 of the exact restatement
// above. The error of the result stays below 1e-6 relative for |x| < 10
// (beyond, the rounding of the exponent's argument grows with |x| while the
// sigmoid saturates, and SiLU's absolute error stays below 1e-7). Those
// epilogues take the sum of a 3xTF32 tensor-core product, which already
// differs from the reference's FMA-chain sum at the 1e-6 level, so the
// bit-exact polynomial cannot make their outputs bit-identical anyway; the
// CUDA-core kernels whose sums are bit-identical keep act_t.
__device__ __forceinline__ float fast_sigmoid(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(x, -1.4426950408889634f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
  return r;
}

template <int ACT>
__device__ __forceinline__ float act_fast(float v) {
  constexpr int A = ACT & ~ACT_FAST;
  if constexpr (A == ACT_SILU) return __fmul_rn(v, fast_sigmoid(v));
  else if constexpr (A == ACT_RELU) return v > 0.0f ? v : 0.0f;
  else if constexpr (A == ACT_SIGMOID) return fast_sigmoid(v);
  else return v;
}

// The activation as a compile-time constant: a loop over act_t<ACT> has no
// branch per element, so the compiler interleaves the independent exp /
// reciprocal chains of consecutive elements (with a runtime switch inside
// the loop each element's chain runs alone, latency-bound). ACT_FAST picks
// the hardware-instruction form.
template <int ACT>
__device__ __forceinline__ float act_t(float v) {
  if constexpr ((ACT & ACT_FAST) != 0) return act_fast<ACT>(v);
  else if constexpr (ACT == ACT_SILU) return ref_silu(v);
  else if constexpr (ACT == ACT_RELU) return v > 0.0f ? v : 0.0f;
  else if constexpr (ACT == ACT_SIGMOID) return ref_sigmoid(v);
  else return v;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_SILU: return ref_silu(v);
    case ACT_RELU:
    case ACT_RELU | ACT_FAST: return v > 0.0f ? v : 0.0f;
    case ACT_SIGMOID: return ref_sigmoid(v);
    case ACT_SILU | ACT_FAST: return act_fast<ACT_SILU>(v);
    case ACT_SIGMOID | ACT_FAST: return act_fast<ACT_SIGMOID>(v);
    default: return v;
  }
}

template <int A>
struct ActTag {
  static constexpr int value = A;
};

// Calls f(ActTag<ACT>{}) with the runtime code `act` turned into a constant;
// f is a generic lambda that reads decltype(tag)::value.
template <class F>
__host__ __device__ __forceinline__ void with_act(int act, F&& f) {
  switch (act) {
    case ACT_SILU: f(ActTag<ACT_SILU>{}); break;
    case ACT_RELU:
    case ACT_RELU | ACT_FAST: f(ActTag<ACT_RELU>{}); break;
    case ACT_SIGMOID: f(ActTag<ACT_SIGMOID>{}); break;
    case ACT_SILU | ACT_FAST: f(ActTag<ACT_SILU | ACT_FAST>{}); break;
    case ACT_SIGMOID | ACT_FAST: f(ActTag<ACT_SIGMOID | ACT_FAST>{}); break;
    default: f(ActTag<ACT_NONE>{}); break;
  }
}

}  // namespace osc
