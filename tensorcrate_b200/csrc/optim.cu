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

// Two elements at a time: each rounding to a 16-bit type is one packed
// conversion (cvt.rn.bf16x2.f32 / cvt.rn.f16x2.f32) of the pair, which
// rounds each half to nearest even exactly as the single conversion does.
template <class T> __device__ __forceinline__ float2 rnd2(float x, float y) {
  if (T::code == TC_BF16) {
    const uint32_t u = pack2_bf16(x, y);
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
  if (T::code == TC_F16) {
    const uint32_t u = pack2_f16(x, y);
    __half2 h = *reinterpret_cast<const __half2 *>(&u);
    return __half22float2(h);
  }
  return make_float2(x, y);
}

#define TC_PAIR(expr_x, expr_y) rnd2<T>((expr_x), (expr_y))

template <class T>
__device__ __forceinline__ void adam_pair(float2 g, float2 &p, float2 &m, float2 &v, bool resumed, const AdamCoef &k) {
  const float2 fresh_first = TC_PAIR(__fmul_rn(g.x, k.first_share), __fmul_rn(g.y, k.first_share));
  const float2 squared = TC_PAIR(__fmul_rn(g.x, g.x), __fmul_rn(g.y, g.y));
  const float2 fresh_second = TC_PAIR(__fmul_rn(squared.x, k.second_share), __fmul_rn(squared.y, k.second_share));
  float2 first = fresh_first, second = fresh_second;
  if (resumed) {
    const float2 mb = TC_PAIR(__fmul_rn(m.x, k.beta1), __fmul_rn(m.y, k.beta1));
    first = TC_PAIR(__fadd_rn(mb.x, fresh_first.x), __fadd_rn(mb.y, fresh_first.y));
    const float2 vb = TC_PAIR(__fmul_rn(v.x, k.beta2), __fmul_rn(v.y, k.beta2));
    second = TC_PAIR(__fadd_rn(vb.x, fresh_second.x), __fadd_rn(vb.y, fresh_second.y));
  }
  const float2 cf = TC_PAIR(__fmul_rn(first.x, k.c1), __fmul_rn(first.y, k.c1));
  const float2 cs = TC_PAIR(__fmul_rn(second.x, k.c2), __fmul_rn(second.y, k.c2));
  const float2 root = TC_PAIR(__fsqrt_rn(cs.x), __fsqrt_rn(cs.y));
  const float2 den = TC_PAIR(__fadd_rn(root.x, k.eps), __fadd_rn(root.y, k.eps));
  const float2 q = TC_PAIR(__fdiv_rn(cf.x, den.x), __fdiv_rn(cf.y, den.y));
  const float2 step = TC_PAIR(__fmul_rn(q.x, k.rate), __fmul_rn(q.y, k.rate));
  p = TC_PAIR(__fsub_rn(p.x, step.x), __fsub_rn(p.y, step.y));
  m = first;
  v = second;
}
#undef TC_PAIR

// Several parameters in one launch (Adam::update runs the same program,
// with the same coefficients, on each parameter of a step).
constexpr int MAX_TENSORS = 16;
struct AdamSet {
  int count;
  long long start[MAX_TENSORS + 1];  // first 16-byte pack of each tensor in the flat pack space
  long long len[MAX_TENSORS];        // elements
  long long packs[MAX_TENSORS];      // whole packs (0 when the tensor is not 16-byte aligned)
  void *p[MAX_TENSORS], *m[MAX_TENSORS], *v[MAX_TENSORS];
  const void *g[MAX_TENSORS];
};

// Each thread walks the flat pack space with a grid stride, loading the
// next pack's four operands before it computes the current one.
template <class T>
__global__ void __launch_bounds__(256) adam_kernel(const __grid_constant__ AdamSet set, bool resumed, AdamCoef k) {
  using S = typename T::S;
  constexpr int N = 16 / int(sizeof(S));
  union Pk { uint4 raw; S e[N]; };
  const long long total = set.start[set.count];
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  auto locate = [&](long long q, int &t, long long &at) {
    t = 0;
    while (t + 1 < set.count && q >= set.start[t + 1]) ++t;
    at = (q - set.start[t]) * N;
  };
  auto load = [&](int t, long long at, Pk &pp, Pk &gg, Pk &mm, Pk &vv) {
    pp.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(set.p[t]) + at);
    gg.raw = __ldg(reinterpret_cast<const uint4 *>(static_cast<const S *>(set.g[t]) + at));
    if (resumed) {
      mm.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(set.m[t]) + at);
      vv.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(set.v[t]) + at);
    }
  };
  long long q = gid;
  int t = 0;
  long long at = 0;
  Pk pp, gg, mm, vv;
  if (q < total) {
    locate(q, t, at);
    load(t, at, pp, gg, mm, vv);
  }
  while (q < total) {
    const long long qn = q + stride;
    int tn = 0;
    long long atn = 0;
    Pk pn, gn, mn, vn;
    if (qn < total) {
      locate(qn, tn, atn);
      load(tn, atn, pn, gn, mn, vn);
    }
#pragma unroll
    for (int j = 0; j < N; j += 2) {
      float2 P = make_float2(T::load(pp.e[j]), T::load(pp.e[j + 1]));
      float2 M = resumed ? make_float2(T::load(mm.e[j]), T::load(mm.e[j + 1])) : make_float2(0.0f, 0.0f);
      float2 V = resumed ? make_float2(T::load(vv.e[j]), T::load(vv.e[j + 1])) : make_float2(0.0f, 0.0f);
      adam_pair<T>(make_float2(T::load(gg.e[j]), T::load(gg.e[j + 1])), P, M, V, resumed, k);
      pp.e[j] = T::store(P.x);
      pp.e[j + 1] = T::store(P.y);
      mm.e[j] = T::store(M.x);
      mm.e[j + 1] = T::store(M.y);
      vv.e[j] = T::store(V.x);
      vv.e[j + 1] = T::store(V.y);
    }
    *reinterpret_cast<uint4 *>(static_cast<S *>(set.p[t]) + at) = pp.raw;
    *reinterpret_cast<uint4 *>(static_cast<S *>(set.m[t]) + at) = mm.raw;
    *reinterpret_cast<uint4 *>(static_cast<S *>(set.v[t]) + at) = vv.raw;
    q = qn;
    t = tn;
    at = atn;
    pp = pn;
    gg = gn;
    mm = mn;
    vv = vn;
  }
  // Elements past each tensor's whole packs, one at a time.
  for (int u = 0; u < set.count; ++u) {
    S *P_ = static_cast<S *>(set.p[u]);
    const S *G_ = static_cast<const S *>(set.g[u]);
    S *M_ = static_cast<S *>(set.m[u]);
    S *V_ = static_cast<S *>(set.v[u]);
    for (long long i = set.packs[u] * N + gid; i < set.len[u]; i += stride) {
      float P = T::load(P_[i]), M = resumed ? T::load(M_[i]) : 0.0f, V = resumed ? T::load(V_[i]) : 0.0f;
      adam_one<T>(T::load(G_[i]), P, M, V, resumed, k);
      P_[i] = T::store(P);
      M_[i] = T::store(M);
      V_[i] = T::store(V);
    }
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

int tc_adam_multi(int dtype, const tc_adam_tensor *tensors, size_t count, int resumed, double rate, double beta1,
                  double beta2, double eps, double c1, double c2, void *stream) {
  if (count && !tensors) return fail(TC_EINVAL, "adam: null tensor list");
  for (size_t i = 0; i < count; ++i)
    if (tensors[i].n && (!tensors[i].p || !tensors[i].g || !tensors[i].m || !tensors[i].v))
      return fail(TC_EINVAL, "adam: null pointer in tensor %zu", i);
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    constexpr size_t N = 16 / sizeof(typename T::S);
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
    static int resident = 0;
    if (!resident) {
      int n = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, adam_kernel<T>, 256, 0);
      resident = std::max(1, n);
    }
    size_t i = 0;  // next tensor of the list; each goes in exactly one launch
    while (i < count) {
      AdamSet set{};
      long long elems = 0;
      for (; i < count && set.count < MAX_TENSORS; ++i) {
        const tc_adam_tensor &x = tensors[i];
        if (x.n == 0) continue;
        const int c = set.count++;
        set.p[c] = x.p;
        set.g[c] = x.g;
        set.m[c] = x.m;
        set.v[c] = x.v;
        set.len[c] = (long long)x.n;
        const bool vec = aligned16(x.p) && aligned16(x.g) && aligned16(x.m) && aligned16(x.v);
        set.packs[c] = vec ? (long long)(x.n / N) : 0;
        set.start[c + 1] = set.start[c] + set.packs[c];
        elems += (long long)x.n;
      }
      if (set.count == 0) continue;
      const long long work = std::max(set.start[set.count], (elems + (long long)N - 1) / (long long)N);
      const unsigned grid = unsigned(std::max(1LL, std::min<long long>((work + 255) / 256,
                                                                       (long long)sm_count() * resident)));
      adam_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(set, resumed != 0, k);
      if (int st = check_launch("adam")) return st;
    }
    return TC_OK;
  });
}

int tc_adam(int dtype, size_t n, void *p, const void *g, void *m, void *v, int resumed, double rate, double beta1,
            double beta2, double eps, double c1, double c2, void *stream) {
  if (n == 0) return TC_OK;
  if (!p || !g || !m || !v) return fail(TC_EINVAL, "adam: null pointer");
  const tc_adam_tensor one{p, g, m, v, n};
  return tc_adam_multi(dtype, &one, 1, resumed, rate, beta1, beta2, eps, c1, c2, stream);
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
