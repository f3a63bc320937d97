// Exact-erf GELU of MLXNN.gelu (DeBERTa.swift:421), GELU(x) = x Phi(x) = 0.5 x (1 + erf(x / sqrt 2)),
// for the GEMM epilogues (FFN up-projection).
//
// Evaluated as GELU(x) = max(x, 0) - h(|x|) with h(a) = 0.5 a erfc(a / sqrt 2) (for x >= 0,
// x Phi(x) = x - 0.5 x erfc(x / sqrt 2); for x < 0, x Phi(x) = -0.5 |x| erfc(|x| / sqrt 2)), and
// erfc(z) = 2^(g(z) - z^2 log2 e) with g(z) = log2(erfcx(z)) = log2(erfc(z) e^(z^2)), a smooth
// function from 0 at z = 0 to -3.4 at z = 4.3. g is a degree-10 polynomial, the Chebyshev
// least-squares fit of log2 erfcx on [0, 4.3] converted to monomial form (coefficients below,
// fp32, Horner); beyond z = 4.3 (|x| > 6.08) the polynomial is held at its end value, where
// h < 4e-9 and rounds to zero in fp16 either way.
//
// Error (fp32 arithmetic, exact exp2): erfc relative error <= 2.7e-6 over the range, GELU
// absolute error <= 4.8e-7; 0.016% of fp16-rounded outputs differ by one unit from the correctly
// rounded GELU on a dense grid of [-12, 12]. The direct h avoids the cancellation of 1 + erf(x)
// for negative x. One exp2 per value is the only multi-function-unit operation.
#pragma once

#include <cuda_runtime.h>

namespace gdc {

constexpr float kGeluRsqrt2 = 0.70710678118654752f;
constexpr float kGeluLog2e = 1.4426950408889634f;
constexpr float kGeluZMax = 4.3f;
// g(z) = c0 + c1 z + ... + c10 z^10
constexpr float kGeluG0 = 1.367034429e-06f, kGeluG1 = -1.627950191e+00f, kGeluG2 = 5.245834589e-01f,
                kGeluG3 = -1.493996084e-01f, kGeluG4 = 2.961711027e-02f, kGeluG5 = -1.809923328e-03f,
                kGeluG6 = -1.146566938e-03f, kGeluG7 = 4.596806830e-04f, kGeluG8 = -8.494793292e-05f,
                kGeluG9 = 8.306016753e-06f, kGeluG10 = -3.448797088e-07f;

__device__ __forceinline__ float2 splat2(float c) { return make_float2(c, c); }

__device__ __forceinline__ float ex2_approx_f32(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two values at once with the packed fp32 instructions of sm_100 (__ffma2_rn / __fmul2_rn:
// one instruction, two IEEE fp32 results).
__device__ __forceinline__ float2 gelu_erf2(float2 v) {
  const float2 a = make_float2(fabsf(v.x), fabsf(v.y));
  const float2 z = __fmul2_rn(a, splat2(kGeluRsqrt2));
  const float2 zc = make_float2(fminf(z.x, kGeluZMax), fminf(z.y, kGeluZMax));
  float2 g = __ffma2_rn(splat2(kGeluG10), zc, splat2(kGeluG9));
  g = __ffma2_rn(g, zc, splat2(kGeluG8));
  g = __ffma2_rn(g, zc, splat2(kGeluG7));
  g = __ffma2_rn(g, zc, splat2(kGeluG6));
  g = __ffma2_rn(g, zc, splat2(kGeluG5));
  g = __ffma2_rn(g, zc, splat2(kGeluG4));
  g = __ffma2_rn(g, zc, splat2(kGeluG3));
  g = __ffma2_rn(g, zc, splat2(kGeluG2));
  g = __ffma2_rn(g, zc, splat2(kGeluG1));
  g = __ffma2_rn(g, zc, splat2(kGeluG0));
  const float2 e = __ffma2_rn(__fmul2_rn(z, z), splat2(-kGeluLog2e), g);  // log2 erfc(z)
  const float2 h = __fmul2_rn(__fmul2_rn(a, splat2(0.5f)), make_float2(ex2_approx_f32(e.x), ex2_approx_f32(e.y)));
  return __ffma2_rn(h, splat2(-1.0f), make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f)));
}

}  // namespace gdc
