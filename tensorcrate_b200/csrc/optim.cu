// optim.cu — the optimizers' fused parameter updates (Adam's and Sgd's
// programs, src/optim.rs:1048-1099 and 773-787, which the Host runs through
// Kernels::fused).  One pass: p, g, m, v are read once and p, m, v written
// in place with 128-bit accesses.  Every operation rounds to the element
// type in the program's order, as the program computes in T
// (fused/mod.rs, "Storage types"): for f16/bf16 each f32 result is rounded
// before the next operation reads it.
#include <algorithm>

#include "common.cuh"

namespace tc {
namespace {

template <class T> __device__ __forceinline__ float rnd(float v) { return T::load(T::store(v)); }

struct AdamCoef {
  float rate, beta1, beta2, eps, c1, c2, first_share, second_share;
};

// The built program, per element:
//   fresh_first = g*(1-b1); squared = g*g; fresh_second = squared*(1-b2)
//   first  = resumed ? m*b1 + fresh_first  : fresh_first
//   second = resumed ? v*b2 + fresh_second : fresh_second
//   p = p - ((first*c1) / (sqrt(second*c2) + eps)) * rate
template <class T>
__device__ __forceinline__ void adam_one(float g, float &p, float &m, float &v, bool resumed, const AdamCoef &k) {
  float fresh_first = rnd<T>(__fmul_rn(g, k.first_share));
  float squared = rnd<T>(__fmul_rn(g, g));
  float fresh_second = rnd<T>(__fmul_rn(squared, k.second_share));
  float first = fresh_first, second = fresh_second;
  if (resumed) {
    first = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(m, k.beta1)), fresh_first));
    second = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(v, k.beta2)), fresh_second));
  }
  float cf = rnd<T>(__fmul_rn(first, k.c1));
  float cs = rnd<T>(__fmul_rn(second, k.c2));
  float root = rnd<T>(__fsqrt_rn(cs));
  float den = rnd<T>(__fadd_rn(root, k.eps));
  float step = rnd<T>(__fmul_rn(rnd<T>(__fdiv_rn(cf, den)), k.rate));
  p = rnd<T>(__fsub_rn(p, step));
  m = first;
  v = second;
}

template <class T>
__global__ void __launch_bounds__(256) adam_kernel(typename T::S *p, const typename T::S *g, typename T::S *m,
                                                   typename T::S *v, size_t n, bool resumed, AdamCoef k, bool vec) {
  using S = typename T::S;
  constexpr int N = 16 / int(sizeof(S));
  union Pk { uint4 raw; S e[N]; };
  size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x, stride = size_t(gridDim.x) * blockDim.x;
  size_t packs = vec ? n / N : 0;
  for (size_t q = tid; q < packs; q += stride) {
    Pk pp, gg, mm, vv;
    pp.raw = *reinterpret_cast<const uint4 *>(p + q * N);
    gg.raw = __ldg(reinterpret_cast<const uint4 *>(g + q * N));
    if (resumed) {
      mm.raw = *reinterpret_cast<const uint4 *>(m + q * N);
      vv.raw = *reinterpret_cast<const uint4 *>(v + q * N);
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float P = T::load(pp.e[j]), M = resumed ? T::load(mm.e[j]) : 0.0f, V = resumed ? T::load(vv.e[j]) : 0.0f;
      adam_one<T>(T::load(gg.e[j]), P, M, V, resumed, k);
      pp.e[j] = T::store(P);
      mm.e[j] = T::store(M);
      vv.e[j] = T::store(V);
    }
    *reinterpret_cast<uint4 *>(p + q * N) = pp.raw;
    *reinterpret_cast<uint4 *>(m + q * N) = mm.raw;
    *reinterpret_cast<uint4 *>(v + q * N) = vv.raw;
  }
  for (size_t i = packs * N + tid; i < n; i += stride) {
    float P = T::load(p[i]), M = resumed ? T::load(m[i]) : 0.0f, V = resumed ? T::load(v[i]) : 0.0f;
    adam_one<T>(T::load(g[i]), P, M, V, resumed, k);
    p[i] = T::store(P);
    m[i] = T::store(M);
    v[i] = T::store(V);
  }
}

// Sgd: step = g * rate (Builder::scale), p = p - step.
template <class T>
__global__ void __launch_bounds__(256) sgd_kernel(typename T::S *p, const typename T::S *g, size_t n, float rate) {
  size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float step = rnd<T>(__fmul_rn(T::load(g[i]), rate));
    p[i] = T::store(__fsub_rn(T::load(p[i]), step));
  }
}

bool aligned16(const void *q) { return (uintptr_t(q) & 15u) == 0; }

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_adam(int dtype, size_t n, void *p, const void *g, void *m, void *v, int resumed, double rate, double beta1,
            double beta2, double eps, double c1, double c2, void *stream) {
  if (n == 0) return TC_OK;
  if (!p || !g || !m || !v) return fail(TC_EINVAL, "adam: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    AdamCoef k;
    k.rate = float(rate);
    k.beta1 = float(beta1);
    k.beta2 = float(beta2);
    k.eps = float(eps);
    k.c1 = float(c1);
    k.c2 = float(c2);
    // `1 - beta` is folded into the program's constants, computed once in
    // the element type (optim.rs:1067-1072).
    auto round_host = [](float x) {
      if (T::code == TC_F32) return x;
      return T::code == TC_BF16 ? bf16_bits_to_f32(f32_to_bf16_bits(x)) : f16_bits_to_f32(f32_to_f16_bits(x));
    };
    k.first_share = round_host(1.0f - k.beta1);
    k.second_share = round_host(1.0f - k.beta2);
    bool vec = aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v);
    unsigned grid = grid_for((n + 7) / 8, 256, 8);
    adam_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<S *>(p), static_cast<const S *>(g),
                                                        static_cast<S *>(m), static_cast<S *>(v), n, resumed != 0,
                                                        k, vec);
    return check_launch("adam");
  });
}

int tc_sgd(int dtype, size_t n, void *p, const void *g, double rate, void *stream) {
  if (n == 0) return TC_OK;
  if (!p || !g) return fail(TC_EINVAL, "sgd: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    unsigned grid = grid_for(n, 256, 8);
    sgd_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<S *>(p), static_cast<const S *>(g), n,
                                                       float(rate));
    return check_launch("sgd");
  });
}

}  // extern "C"
