// analytic.cuh — the Analytic functions (kernels.rs:293-388) as device code,
// shared by the fused-program interpreter and the unary kernels.
#pragma once
#include "common.cuh"

namespace tc {

// Analytic::value in f32 (kernels.rs:329-353).  The transcendentals are
// CUDA's single-precision functions (within 2 ulp of the exact value); Sec
// and Csc divide with the correctly rounded quotient; Sqrt is the IEEE root.
__device__ __forceinline__ float analytic(int op, float x) {
  switch (op) {
    case TC_SIN: return sinf(x);
    case TC_COS: return cosf(x);
    case TC_TAN: return tanf(x);
    case TC_SEC: return __fdiv_rn(1.0f, cosf(x));
    case TC_CSC: return __fdiv_rn(1.0f, sinf(x));
    case TC_ARCSIN: return asinf(x);
    case TC_ARCCOS: return acosf(x);
    case TC_ARCTAN: return atanf(x);
    case TC_EXP: return expf(x);
    case TC_LN: return logf(x);
    case TC_SINH: return sinhf(x);
    case TC_COSH: return coshf(x);
    case TC_TANH: return tanhf(x);
    default: return __fsqrt_rn(x);
  }
}

// v rounded to the element type T (the identity for f32).
template <class T> __device__ __forceinline__ float round_to(float v) { return T::load(T::store(v)); }

// Analytic::derivative (kernels.rs:357-387) computed in T: every value,
// product, sum, root and reciprocal of the rule is rounded to T, as the
// Host's `Real` arithmetic on T rounds each operation.
template <class T> __device__ __forceinline__ float analytic_derivative(int op, float x) {
  auto r = [](float v) { return round_to<T>(v); };
  auto recip = [&](float v) { return r(__fdiv_rn(1.0f, v)); };
  switch (op) {
    case TC_SIN: return r(analytic(TC_COS, x));
    case TC_COS: return -r(analytic(TC_SIN, x));
    case TC_TAN: {
      const float c = r(analytic(TC_COS, x));
      return recip(r(__fmul_rn(c, c)));
    }
    case TC_SEC: {
      const float c = r(analytic(TC_COS, x));
      return r(__fdiv_rn(r(analytic(TC_SIN, x)), r(__fmul_rn(c, c))));
    }
    case TC_CSC: {
      const float s = r(analytic(TC_SIN, x));
      return r(__fdiv_rn(-r(analytic(TC_COS, x)), r(__fmul_rn(s, s))));
    }
    case TC_ARCSIN: return recip(r(__fsqrt_rn(r(__fsub_rn(1.0f, r(__fmul_rn(x, x)))))));
    case TC_ARCCOS: return -recip(r(__fsqrt_rn(r(__fsub_rn(1.0f, r(__fmul_rn(x, x)))))));
    case TC_ARCTAN: return recip(r(__fadd_rn(1.0f, r(__fmul_rn(x, x)))));
    case TC_EXP: return r(analytic(TC_EXP, x));
    case TC_LN: return recip(x);
    case TC_SINH: return r(analytic(TC_COSH, x));
    case TC_COSH: return r(analytic(TC_SINH, x));
    case TC_TANH: {
      const float t = r(analytic(TC_TANH, x));
      return r(__fsub_rn(1.0f, r(__fmul_rn(t, t))));
    }
    default: return recip(r(__fmul_rn(2.0f, r(__fsqrt_rn(x)))));
  }
}

}  // namespace tc
