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

// Two 16-bit elements at a time, in packed bf16x2 / f16x2 arithmetic.  A
// packed multiply, add or subtract (the _rn forms, which the compiler may
// not contract into a fused multiply-add) rounds the exact result once to
// the element type; the program's f32 operation followed by a rounding to the
// element type gives the same value, because the exact product or sum of two
// such values either fits in f32 or lies too far from a tie of the element
// type for the f32 rounding to move it there (the operands' exponents are
// then more than 15 apart, 12 for f16).  The one exception is a bf16
// product below 2^-126, which f32 itself rounds as a subnormal.  Square root
// and division have no packed form: they run in f32 and round once, as the
// program does.
template <class T> struct Half2;
template <> struct Half2<BF16T> {
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) { return op(a, b, 0); }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) { return op(a, b, 1); }
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) { return op(a, b, 2); }
  __device__ __forceinline__ static uint32_t op(uint32_t a, uint32_t b, int which) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162 *>(&a), y = *reinterpret_cast<__nv_bfloat162 *>(&b);
    __nv_bfloat162 r = which == 0 ? __hmul2_rn(x, y) : which == 1 ? __hadd2_rn(x, y) : __hsub2_rn(x, y);
    return *reinterpret_cast<uint32_t *>(&r);
  }
  __device__ __forceinline__ static float2 widen(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t narrow(float2 f) { return pack2_bf16(f.x, f.y); }
};
template <> struct Half2<F16T> {
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) { return op(a, b, 0); }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) { return op(a, b, 1); }
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) { return op(a, b, 2); }
  __device__ __forceinline__ static uint32_t op(uint32_t a, uint32_t b, int which) {
    __half2 x = *reinterpret_cast<__half2 *>(&a), y = *reinterpret_cast<__half2 *>(&b);
    __half2 r = which == 0 ? __hmul2_rn(x, y) : which == 1 ? __hadd2_rn(x, y) : __hsub2_rn(x, y);
    return *reinterpret_cast<uint32_t *>(&r);
  }
  __device__ __forceinline__ static float2 widen(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&u));
  }
  __device__ __forceinline__ static uint32_t narrow(float2 f) { return pack2_f16(f.x, f.y); }
};

// The coefficients as packed pairs of the element type.
struct AdamCoef2 {
  uint32_t rate, beta1, beta2, eps, c1, c2, first_share, second_share;
};

template <class T>
__device__ __forceinline__ void adam_pair(uint32_t g, uint32_t &p, uint32_t &m, uint32_t &v, bool resumed,
                                          const AdamCoef2 &k) {
  using H = Half2<T>;
  const uint32_t fresh_first = H::mul(g, k.first_share);
  const uint32_t squared = H::mul(g, g);
  const uint32_t fresh_second = H::mul(squared, k.second_share);
  uint32_t first = fresh_first, second = fresh_second;
  if (resumed) {
    first = H::add(H::mul(m, k.beta1), fresh_first);
    second = H::add(H::mul(v, k.beta2), fresh_second);
  }
  const uint32_t cf = H::mul(first, k.c1);
  const float2 cs = H::widen(H::mul(second, k.c2));
  const uint32_t root = H::narrow(make_float2(__fsqrt_rn(cs.x), __fsqrt_rn(cs.y)));
  const float2 den = H::widen(H::add(root, k.eps));
  const float2 num = H::widen(cf);
  const uint32_t q = H::narrow(make_float2(__fdiv_rn(num.x, den.x), __fdiv_rn(num.y, den.y)));
  const uint32_t step = H::mul(q, k.rate);
  p = H::sub(p, step);
  m = first;
  v = second;
}

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
__global__ void __launch_bounds__(256) adam_kernel(const __grid_constant__ AdamSet set, bool resumed, AdamCoef k,
                                                   AdamCoef2 k2) {
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
    if constexpr (sizeof(S) == 2) {
      uint32_t *P2 = reinterpret_cast<uint32_t *>(&pp.raw), *M2 = reinterpret_cast<uint32_t *>(&mm.raw);
      uint32_t *V2 = reinterpret_cast<uint32_t *>(&vv.raw);
      const uint32_t *G2 = reinterpret_cast<const uint32_t *>(&gg.raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t m2 = resumed ? M2[j] : 0u, v2 = resumed ? V2[j] : 0u;
        adam_pair<T>(G2[j], P2[j], m2, v2, resumed, k2);
        M2[j] = m2;
        V2[j] = v2;
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float P = T::load(pp.e[j]), M = resumed ? T::load(mm.e[j]) : 0.0f, V = resumed ? T::load(vv.e[j]) : 0.0f;
        adam_one<T>(T::load(gg.e[j]), P, M, V, resumed, k);
        pp.e[j] = T::store(P);
        mm.e[j] = T::store(M);
        vv.e[j] = T::store(V);
      }
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
__global__ void __launch_bounds__(256) sgd_kernel(typename T::S *p, const typename T::S *g, size_t n, float rate,
                                                  bool vec) {
  // 16-byte packs of p and g when both are aligned, the tail (or all of an
  // unaligned update) element by element; the same operations either way.
  using S = typename T::S;
  constexpr int N = 16 / int(sizeof(S));
  union Pk {
    uint4 raw;
    S v[N];
  };
  const size_t stride = size_t(gridDim.x) * blockDim.x, tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t packs = vec ? n / N : 0;
  for (size_t q = tid; q < packs; q += stride) {
    Pk pp, gg;
    pp.raw = reinterpret_cast<const uint4 *>(p)[q];
    gg.raw = __ldg(reinterpret_cast<const uint4 *>(g) + q);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float step = rnd<T>(__fmul_rn(T::load(gg.v[j]), rate));
      pp.v[j] = T::store(__fsub_rn(T::load(pp.v[j]), step));
    }
    reinterpret_cast<uint4 *>(p)[q] = pp.raw;
  }
  for (size_t i = packs * N + tid; i < n; i += stride) {
    float step = rnd<T>(__fmul_rn(T::load(g[i]), rate));
    p[i] = T::store(__fsub_rn(T::load(p[i]), step));
  }
}

// The state-carrying rules of optim.rs whose programs the reference builds
// beside Sgd and Adam, each as the program computes it: every operation in
// f32 on values of T, its result rounded to T, in the builder's order.
//   Momentum (optim.rs:826-846): v' = v·μ + g; step = nesterov ? g + v'·μ : v';
//     p' = p - step·rate.
//   AdaGrad (optim.rs:892-904): s' = s + g·g; p' = p - (g / (√s' + ε))·rate.
//   RmsProp (optim.rs:948-964): s' = s·ρ + (g·g)·(1 - ρ); p' as AdaGrad.
// (`descend`, optim.rs:1146-1159, is the shared p' step.)  The coefficients
// arrive as values of T.
enum StateRule { R_MOMENTUM = 0, R_NESTEROV = 1, R_ADAGRAD = 2, R_RMSPROP = 3 };

struct StateCoef {
  float rate, a, b, c;  // momentum: μ; adagrad: ε; rmsprop: ρ, 1 - ρ, ε
};

template <class T, int RULE>
__device__ __forceinline__ void state_rule(float &p, float g, float &s, const StateCoef &k) {
  float step;
  if (RULE == R_MOMENTUM || RULE == R_NESTEROV) {
    s = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(s, k.a)), g));
    step = RULE == R_NESTEROV ? rnd<T>(__fadd_rn(g, rnd<T>(__fmul_rn(s, k.a)))) : s;
  } else {
    const float squared = rnd<T>(__fmul_rn(g, g));
    if (RULE == R_ADAGRAD) s = rnd<T>(__fadd_rn(s, squared));
    else s = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(s, k.a)), rnd<T>(__fmul_rn(squared, k.b))));
    const float eps = RULE == R_ADAGRAD ? k.a : k.c;
    const float denominator = rnd<T>(__fadd_rn(rnd<T>(__fsqrt_rn(s)), eps));
    step = rnd<T>(__fdiv_rn(g, denominator));
  }
  p = rnd<T>(__fsub_rn(p, rnd<T>(__fmul_rn(step, k.rate))));
}

// p and the state s updated in place, g read: 16-byte packs when all three
// are aligned, the tail (or all of an unaligned update) element by element.
template <class T, int RULE>
__global__ void __launch_bounds__(256) state_rule_kernel(typename T::S *p, const typename T::S *g,
                                                         typename T::S *s, size_t n, StateCoef k, bool vec) {
  using S = typename T::S;
  constexpr int N = 16 / int(sizeof(S));
  union Pk {
    uint4 raw;
    S v[N];
  };
  const size_t stride = size_t(gridDim.x) * blockDim.x, tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t packs = vec ? n / N : 0;
  for (size_t q = tid; q < packs; q += stride) {
    Pk pp, gg, ss;
    pp.raw = reinterpret_cast<const uint4 *>(p)[q];
    gg.raw = __ldg(reinterpret_cast<const uint4 *>(g) + q);
    ss.raw = reinterpret_cast<const uint4 *>(s)[q];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float pv = T::load(pp.v[j]), sv = T::load(ss.v[j]);
      state_rule<T, RULE>(pv, T::load(gg.v[j]), sv, k);
      pp.v[j] = T::store(pv);
      ss.v[j] = T::store(sv);
    }
    reinterpret_cast<uint4 *>(p)[q] = pp.raw;
    reinterpret_cast<uint4 *>(s)[q] = ss.raw;
  }
  for (size_t i = packs * N + tid; i < n; i += stride) {
    float pv = T::load(p[i]), sv = T::load(s[i]);
    state_rule<T, RULE>(pv, T::load(g[i]), sv, k);
    p[i] = T::store(pv);
    s[i] = T::store(sv);
  }
}

bool aligned16(const void *q) { return (uintptr_t(q) & 15u) == 0; }

// A 16-byte load that no cache on this GPU may answer from an older copy:
// another GPU wrote the line (peer memory over NVLink).
__device__ __forceinline__ uint4 load_fresh(const uint4 *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// The sharded data-parallel update of one block (see PeerAdam): each thread
// takes 16-byte packs of this rank's shard, loads the pack of every rank's
// gradient (peer memory over NVLink; all loads issued before any is used),
// sums them in rank order in f32 and rounds once to T, runs Adam's program
// on it with this rank's moments, and stores the new parameters to every
// rank's copy (NVLink stores) and the summed gradient to this rank's.
template <class T>
__global__ void __launch_bounds__(256) peer_adam_kernel(const __grid_constant__ PeerAdam x, bool resumed, AdamCoef k,
                                                        AdamCoef2 k2) {
  using S = typename T::S;
  constexpr int N = 16 / int(sizeof(S));
  union Pk { uint4 raw; S e[N]; };
  const long long packs = (long long)(x.count / N);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < packs; q += stride) {
    const size_t at = x.first + size_t(q) * N;
    uint4 parts[MAX_PEER_RANKS];
#pragma unroll
    for (int r = 0; r < MAX_PEER_RANKS; ++r)
      if (r < x.nranks) parts[r] = load_fresh(reinterpret_cast<const uint4 *>(static_cast<const S *>(x.grads[r]) + at));
    Pk pp, mm, vv, gg;
    pp.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(x.params[x.rank]) + at);
    if (resumed) {
      mm.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(x.m) + at);
      vv.raw = *reinterpret_cast<const uint4 *>(static_cast<const S *>(x.v) + at);
    }
    float sum[N];
#pragma unroll
    for (int r = 0; r < MAX_PEER_RANKS; ++r)
      if (r < x.nranks) {
        Pk part;
        part.raw = parts[r];
#pragma unroll
        for (int j = 0; j < N; ++j) sum[j] = r == 0 ? T::load(part.e[j]) : __fadd_rn(sum[j], T::load(part.e[j]));
      }
#pragma unroll
    for (int j = 0; j < N; ++j) gg.e[j] = T::store(sum[j]);
    if constexpr (sizeof(S) == 2) {
      uint32_t *P2 = reinterpret_cast<uint32_t *>(&pp.raw), *M2 = reinterpret_cast<uint32_t *>(&mm.raw);
      uint32_t *V2 = reinterpret_cast<uint32_t *>(&vv.raw);
      const uint32_t *G2 = reinterpret_cast<const uint32_t *>(&gg.raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t m2 = resumed ? M2[j] : 0u, v2 = resumed ? V2[j] : 0u;
        adam_pair<T>(G2[j], P2[j], m2, v2, resumed, k2);
        M2[j] = m2;
        V2[j] = v2;
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float P = T::load(pp.e[j]), M = resumed ? T::load(mm.e[j]) : 0.0f, V = resumed ? T::load(vv.e[j]) : 0.0f;
        adam_one<T>(T::load(gg.e[j]), P, M, V, resumed, k);
        pp.e[j] = T::store(P);
        mm.e[j] = T::store(M);
        vv.e[j] = T::store(V);
      }
    }
#pragma unroll
    for (int r = 0; r < MAX_PEER_RANKS; ++r)
      if (r < x.nranks) *reinterpret_cast<uint4 *>(static_cast<S *>(x.params[r]) + at) = pp.raw;
    *reinterpret_cast<uint4 *>(static_cast<S *>(x.m) + at) = mm.raw;
    *reinterpret_cast<uint4 *>(static_cast<S *>(x.v) + at) = vv.raw;
    *reinterpret_cast<uint4 *>(const_cast<S *>(static_cast<const S *>(x.grads[x.rank])) + at) = gg.raw;
  }
  // The stores to the peers are ordered before the flag that announces them.
  __threadfence_system();
}

}  // namespace
}  // namespace tc

using namespace tc;

namespace tc {
namespace {
template <class T>
void adam_coefficients(double rate, double beta1, double beta2, double eps, double c1, double c2, AdamCoef &k,
                       AdamCoef2 &k2) {
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
  // The same values as packed pairs (each already a value of T).
  auto pair = [](float x) -> uint32_t {
    if (T::code == TC_F32) return 0u;
    const uint32_t h = T::code == TC_BF16 ? f32_to_bf16_bits(x) : f32_to_f16_bits(x);
    return h | (h << 16);
  };
  k2 = AdamCoef2{pair(k.rate), pair(k.beta1), pair(k.beta2), pair(k.eps), pair(k.c1), pair(k.c2),
                 pair(k.first_share), pair(k.second_share)};
}
}  // namespace

int peer_adam_run(int dtype, const PeerAdam &x, int resumed, double rate, double beta1, double beta2, double eps,
                  double c1, double c2, cudaStream_t stream) {
  if (x.nranks < 1 || x.nranks > MAX_PEER_RANKS || x.rank < 0 || x.rank >= x.nranks)
    return fail(TC_EINVAL, "peer adam: rank %d of %d", x.rank, x.nranks);
  if (x.count == 0) return TC_OK;
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    constexpr size_t N = 16 / sizeof(typename T::S);
    if (x.count % N || x.first % N) return fail(TC_EINVAL, "peer adam: the shard is not whole 16-byte packs");
    AdamCoef k;
    AdamCoef2 k2;
    adam_coefficients<T>(rate, beta1, beta2, eps, c1, c2, k, k2);
    const unsigned grid = grid_for(x.count / N, 256, 8);
    peer_adam_kernel<T><<<grid, 256, 0, stream>>>(x, resumed != 0, k, k2);
    return check_launch("peer adam");
  });
}
}  // namespace tc

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
    AdamCoef2 k2;
    adam_coefficients<T>(rate, beta1, beta2, eps, c1, c2, k, k2);
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
      adam_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(set, resumed != 0, k, k2);
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
    const bool vec = aligned16(p) && aligned16(g);
    unsigned grid = grid_for(vec ? (n + 15 / sizeof(S)) / (16 / sizeof(S)) : n, 256, 8);
    sgd_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<S *>(p), static_cast<const S *>(g), n,
                                                       float(rate), vec);
    return check_launch("sgd");
  });
}

static int run_state_rule(const char *what, int dtype, int rule, size_t n, void *p, const void *g, void *s, double rate,
                          double a, double b, double c, void *stream) {
  if (n == 0) return TC_OK;
  if (!p || !g || !s) return fail(TC_EINVAL, "%s: null pointer", what);
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    auto in_t = [](double x) { return T::load(T::store(float(x))); };
    StateCoef k{in_t(rate), in_t(a), in_t(b), in_t(c)};
    if (rule == R_RMSPROP) k.b = in_t(1.0f - k.a);  // 1 - ρ, in T, as the rule computes it
    const bool vec = aligned16(p) && aligned16(g) && aligned16(s);
    const unsigned grid = grid_for(vec ? (n + 15 / sizeof(S)) / (16 / sizeof(S)) : n, 256, 8);
    cudaStream_t st = as_stream(stream);
    S *ps = static_cast<S *>(p), *ss = static_cast<S *>(s);
    const S *gs = static_cast<const S *>(g);
    switch (rule) {
      case R_MOMENTUM: state_rule_kernel<T, R_MOMENTUM><<<grid, 256, 0, st>>>(ps, gs, ss, n, k, vec); break;
      case R_NESTEROV: state_rule_kernel<T, R_NESTEROV><<<grid, 256, 0, st>>>(ps, gs, ss, n, k, vec); break;
      case R_ADAGRAD: state_rule_kernel<T, R_ADAGRAD><<<grid, 256, 0, st>>>(ps, gs, ss, n, k, vec); break;
      default: state_rule_kernel<T, R_RMSPROP><<<grid, 256, 0, st>>>(ps, gs, ss, n, k, vec);
    }
    return check_launch(what);
  });
}

int tc_momentum(int dtype, size_t n, void *p, const void *g, void *velocity, double rate, double momentum,
                int nesterov, void *stream) {
  return run_state_rule("momentum", dtype, nesterov ? R_NESTEROV : R_MOMENTUM, n, p, g, velocity, rate, momentum, 0.0,
                        0.0, stream);
}

int tc_adagrad(int dtype, size_t n, void *p, const void *g, void *total, double rate, double eps, void *stream) {
  return run_state_rule("adagrad", dtype, R_ADAGRAD, n, p, g, total, rate, eps, 0.0, 0.0, stream);
}

int tc_rmsprop(int dtype, size_t n, void *p, const void *g, void *mean_square, double rate, double decay, double eps,
               void *stream) {
  return run_state_rule("rmsprop", dtype, R_RMSPROP, n, p, g, mean_square, rate, decay, 0.0, eps, stream);
}

}  // extern "C"
