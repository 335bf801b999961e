// elementwise.cu — same-shape elementwise, scalar broadcast, comparisons,
// clamp (Kernels<T>::vector_* / matrix_*, src/tensors/kernels.rs:832-863)
// and the broadcasting strided binary (Kernels::strided_binary,
// kernels.rs:1162; Host strided::binary, strided.rs:29-78).
//
// All of it is HBM-bound: 128-bit loads and stores of whole 16-byte packs
// (4 f32 or 8 f16/bf16), grid-stride loops sized to the SM count, and the
// arithmetic done in f32 and rounded once per result with the explicit _rn
// intrinsics, so no a*b+c is ever contracted.
#include <algorithm>

#include "common.cuh"

namespace tc {
namespace {

// The operation a kernel applies, fixed at compile time: one instantiation
// per (Pairwise kind, operator), so the inner loops carry no branch.
template <int KIND, int OP> struct Fn {
  __device__ __forceinline__ float operator()(float a, float b) const {
    if (KIND == TC_PAIR_ARITHMETIC) return binary_value(OP, a, b);
    if (KIND == TC_PAIR_COMPARE) return compare_value(OP, a, b);
    return powf(a, b);
  }
};

// Call f(Fn<kind, op>{}) for a run-time (kind, op).
template <class G> int with_fn(int kind, int op, G &&g) {
  switch (kind) {
    case TC_PAIR_ARITHMETIC:
      switch (op) {
        case TC_ADD: return g(Fn<TC_PAIR_ARITHMETIC, TC_ADD>{});
        case TC_SUB: return g(Fn<TC_PAIR_ARITHMETIC, TC_SUB>{});
        case TC_MUL: return g(Fn<TC_PAIR_ARITHMETIC, TC_MUL>{});
        case TC_DIV: return g(Fn<TC_PAIR_ARITHMETIC, TC_DIV>{});
        default: return g(Fn<TC_PAIR_ARITHMETIC, TC_REM>{});
      }
    case TC_PAIR_COMPARE:
      switch (op) {
        case TC_MIN: return g(Fn<TC_PAIR_COMPARE, TC_MIN>{});
        case TC_MAX: return g(Fn<TC_PAIR_COMPARE, TC_MAX>{});
        case TC_MAX_SHARE: return g(Fn<TC_PAIR_COMPARE, TC_MAX_SHARE>{});
        case TC_LESS: return g(Fn<TC_PAIR_COMPARE, TC_LESS>{});
        case TC_LESS_EQUAL: return g(Fn<TC_PAIR_COMPARE, TC_LESS_EQUAL>{});
        case TC_GREATER: return g(Fn<TC_PAIR_COMPARE, TC_GREATER>{});
        default: return g(Fn<TC_PAIR_COMPARE, TC_GREATER_EQUAL>{});
      }
    default: return g(Fn<TC_PAIR_POWER, 0>{});
  }
}

struct Pair {
  int kind;  // tc_pairwise
  int op;
};

template <class T> struct Pack {
  using S = typename T::S;
  static constexpr int N = 16 / int(sizeof(S));
  union {
    uint4 raw;
    S v[N];
  };
};

template <class T>
__device__ __forceinline__ Pack<T> load_pack(const typename T::S *p) {
  Pack<T> k;
  k.raw = __ldg(reinterpret_cast<const uint4 *>(p));
  return k;
}
template <class T>
__device__ __forceinline__ void store_pack(typename T::S *p, const Pack<T> &k) {
  // (Cache-streaming stores, __stcs, measured no different on config 2.)
  *reinterpret_cast<uint4 *>(p) = k.raw;
}

bool aligned16(const void *p) { return (uintptr_t(p) & 15u) == 0; }

// out[i] = f(a[i], b[i]) — both operands whole.
template <class T, class F>
__global__ void __launch_bounds__(256) ew_same(const typename T::S *a, const typename T::S *b,
                                               typename T::S *out, size_t n, F f, bool vec) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x, stride = size_t(gridDim.x) * blockDim.x;
  size_t packs = vec ? n / N : 0;
  for (size_t p = tid; p < packs; p += stride) {
    Pack<T> x = load_pack<T>(a + p * N), y = load_pack<T>(b + p * N), r;
#pragma unroll
    for (int j = 0; j < N; ++j) r.v[j] = T::store(f(T::load(x.v[j]), T::load(y.v[j])));
    store_pack<T>(out + p * N, r);
  }
  for (size_t i = packs * N + tid; i < n; i += stride) out[i] = T::store(f(T::load(a[i]), T::load(b[i])));
}

// out[i] = f(a[i], s) or f(s, a[i]).
template <class T, class F>
__global__ void __launch_bounds__(256) ew_scalar(const typename T::S *a, float s, bool left,
                                                 typename T::S *out, size_t n, F f, bool vec) {
  constexpr int N = Pack<T>::N;
  size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x, stride = size_t(gridDim.x) * blockDim.x;
  size_t packs = vec ? n / N : 0;
  for (size_t p = tid; p < packs; p += stride) {
    Pack<T> x = load_pack<T>(a + p * N), r;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float v = T::load(x.v[j]);
      r.v[j] = T::store(left ? f(s, v) : f(v, s));
    }
    store_pack<T>(out + p * N, r);
  }
  for (size_t i = packs * N + tid; i < n; i += stride) {
    float v = T::load(a[i]);
    out[i] = T::store(left ? f(s, v) : f(v, s));
  }
}

// Vector::clamp (vector.rs:642-652): ordered_min(ordered_max(x, low), high);
// fmaxf returns `low` for a NaN element, as ordered_max does.
template <class T>
__global__ void __launch_bounds__(256) ew_clamp(const typename T::S *a, float lo, float hi,
                                                typename T::S *out, size_t n, bool vec) {
  constexpr int N = Pack<T>::N;
  size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x, stride = size_t(gridDim.x) * blockDim.x;
  size_t packs = vec ? n / N : 0;
  for (size_t p = tid; p < packs; p += stride) {
    Pack<T> x = load_pack<T>(a + p * N), r;
#pragma unroll
    for (int j = 0; j < N; ++j) r.v[j] = T::store(fminf(fmaxf(T::load(x.v[j]), lo), hi));
    store_pack<T>(out + p * N, r);
  }
  for (size_t i = packs * N + tid; i < n; i += stride) out[i] = T::store(fminf(fmaxf(T::load(a[i]), lo), hi));
}

// Broadcast over rows: out[r, c] = f(a[r*as + c*ac], b[r*bs + c*bc]) with
// ac, bc in {0, 1} — a [rows, inner] walk after coalescing, which is what
// `x + bias` over [64,512,1024] x [1,1,1024] becomes.  Packs along the
// inner axis when it allows.
template <class T, class F>
__global__ void __launch_bounds__(256) ew_rows(const typename T::S *a, long long as, int ac,
                                               const typename T::S *b, long long bs, int bc,
                                               typename T::S *out, long long rows, long long inner, F f,
                                               bool vec) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  long long per_row = vec ? inner / N : inner;
  long long total = rows * per_row;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    long long r = i / per_row, c = i - r * per_row;
    const S *ar = a + r * as;
    const S *br = b + r * bs;
    S *orow = out + r * inner;
    if (vec) {
      Pack<T> x, y, z;
      if (ac) x = load_pack<T>(ar + c * N);
      else {
        S s = ar[0];
#pragma unroll
        for (int j = 0; j < N; ++j) x.v[j] = s;
      }
      if (bc) y = load_pack<T>(br + c * N);
      else {
        S s = br[0];
#pragma unroll
        for (int j = 0; j < N; ++j) y.v[j] = s;
      }
#pragma unroll
      for (int j = 0; j < N; ++j) z.v[j] = T::store(f(T::load(x.v[j]), T::load(y.v[j])));
      store_pack<T>(orow + c * N, z);
    } else {
      orow[c] = T::store(f(T::load(ar[c * ac]), T::load(br[c * bc])));
    }
  }
}

// The same for long rows (a's inner step 1, packs): a block takes U rows
// at a time and its threads stride along them, so each thread has U loads
// in flight and no index division.
template <class T, class F, int U>
__global__ void __launch_bounds__(256) ew_rows_blocked(const typename T::S *a, long long as,
                                                       const typename T::S *b, long long bs, int bc,
                                                       typename T::S *out, long long rows, long long inner, F f) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  const int per_row = int(inner / N);
  for (long long r0 = (long long)blockIdx.x * U; r0 < rows; r0 += (long long)gridDim.x * U) {
    for (int c = threadIdx.x; c < per_row; c += blockDim.x) {
      Pack<T> x[U], y[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (r0 + u < rows) x[u] = load_pack<T>(a + (r0 + u) * as + (long long)c * N);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (r0 + u < rows) {
          if (bc) {
            y[u] = (u > 0 && bs == 0) ? y[0] : load_pack<T>(b + (r0 + u) * bs + (long long)c * N);
          } else {
            const S sb = b[(r0 + u) * bs];
#pragma unroll
            for (int j = 0; j < N; ++j) y[u].v[j] = sb;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (r0 + u < rows) {
          Pack<T> z;
#pragma unroll
          for (int j = 0; j < N; ++j) z.v[j] = T::store(f(T::load(x[u].v[j]), T::load(y[u].v[j])));
          store_pack<T>(out + (r0 + u) * inner + (long long)c * N, z);
        }
      }
    }
  }
}

// Any layout: one element per thread, coordinates from the flat index.
template <class T, class F>
__global__ void __launch_bounds__(256) ew_walk(const typename T::S *a, const typename T::S *b,
                                               typename T::S *out, Walk w, long long n, F f) {
  long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    long long pos[2];
    walk_positions<2>(w, i, pos);
    out[i] = T::store(f(T::load(a[pos[0]]), T::load(b[pos[1]])));
  }
}

int check_op(int kind, int op) {
  if (kind == TC_PAIR_ARITHMETIC && (op < TC_ADD || op > TC_REM)) return fail(TC_EINVAL, "bad BinaryOp %d", op);
  if (kind == TC_PAIR_COMPARE && (op < TC_MIN || op > TC_GREATER_EQUAL))
    return fail(TC_EINVAL, "bad Compare %d", op);
  if (kind < TC_PAIR_ARITHMETIC || kind > TC_PAIR_POWER) return fail(TC_EINVAL, "bad Pairwise kind %d", kind);
  return TC_OK;
}

int same(int dtype, Pair f, const void *a, const void *b, void *out, size_t n, void *stream) {
  if (int st = check_op(f.kind, f.op)) return st;
  if (n == 0) return TC_OK;
  if (!a || !b || !out) return fail(TC_EINVAL, "elementwise: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    return with_fn(f.kind, f.op, [&](auto fn) {
      bool vec = aligned16(a) && aligned16(b) && aligned16(out);
      unsigned grid = grid_for((n + Pack<T>::N - 1) / Pack<T>::N, 256, 8);
      ew_same<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const S *>(a), static_cast<const S *>(b),
                                                      static_cast<S *>(out), n, fn, vec);
      return check_launch("elementwise");
    });
  });
}

int scalar(int dtype, Pair f, const void *a, double s, int left, void *out, size_t n, void *stream) {
  if (int st = check_op(f.kind, f.op)) return st;
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "elementwise: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    return with_fn(f.kind, f.op, [&](auto fn) {
      bool vec = aligned16(a) && aligned16(out);
      unsigned grid = grid_for((n + Pack<T>::N - 1) / Pack<T>::N, 256, 8);
      ew_scalar<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const S *>(a), float(s), left != 0,
                                                        static_cast<S *>(out), n, fn, vec);
      return check_launch("elementwise scalar");
    });
  });
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_elementwise(int dtype, int op, const void *a, const void *b, void *out, size_t n, void *stream) {
  return same(dtype, Pair{TC_PAIR_ARITHMETIC, op}, a, b, out, n, stream);
}
int tc_broadcast_scalar(int dtype, int op, const void *a, double s, int left, void *out, size_t n, void *stream) {
  return scalar(dtype, Pair{TC_PAIR_ARITHMETIC, op}, a, s, left, out, n, stream);
}
int tc_compare(int dtype, int cmp, const void *a, const void *b, void *out, size_t n, void *stream) {
  return same(dtype, Pair{TC_PAIR_COMPARE, cmp}, a, b, out, n, stream);
}
int tc_compare_scalar(int dtype, int cmp, const void *a, double s, int left, void *out, size_t n, void *stream) {
  return scalar(dtype, Pair{TC_PAIR_COMPARE, cmp}, a, s, left, out, n, stream);
}

// vector_power / vector_power_scalar (kernels.rs:884-888; Host
// pow_elementwise, power_scalar): Pairwise::Power's powf.
int tc_power(int dtype, const void *a, const void *b, void *out, size_t n, void *stream) {
  return same(dtype, Pair{TC_PAIR_POWER, 0}, a, b, out, n, stream);
}
int tc_power_scalar(int dtype, const void *a, double s, int left, void *out, size_t n, void *stream) {
  return scalar(dtype, Pair{TC_PAIR_POWER, 0}, a, s, left, out, n, stream);
}

int tc_clamp(int dtype, const void *a, double low, double high, void *out, size_t n, void *stream) {
  if (!(low <= high)) return fail(TC_EINVAL, "clamp: low %g is not <= high %g", low, high);
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "clamp: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    bool vec = aligned16(a) && aligned16(out);
    unsigned grid = grid_for((n + Pack<T>::N - 1) / Pack<T>::N, 256, 8);
    ew_clamp<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const S *>(a), float(low), float(high),
                                                     static_cast<S *>(out), n, vec);
    return check_launch("clamp");
  });
}

int tc_strided_binary(int dtype, int kind, int op, uint32_t rank, const size_t *shape, const void *a,
                      size_t a_len, size_t a_offset, const size_t *a_strides, const void *b, size_t b_len,
                      size_t b_offset, const size_t *b_strides, void *out, void *stream) {
  if (int st = check_op(kind, op)) return st;
  if (int st = check_layout("strided binary (a)", a_len, rank, shape, a_offset, a_strides)) return st;
  if (int st = check_layout("strided binary (b)", b_len, rank, shape, b_offset, b_strides)) return st;
  size_t n = element_count(rank, shape);
  if (n == 0) return TC_OK;
  if (!a || !b || !out) return fail(TC_EINVAL, "strided binary: null pointer");
  size_t to[TC_MAX_RANK];
  contiguous_strides(rank, shape, to);
  const size_t *ops[3] = {a_strides, b_strides, to};
  Dims cs, cst[3];
  coalesce<3>(rank, shape, ops, cs, cst);
  Pair f{kind, op};
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    const S *pa = static_cast<const S *>(a) + a_offset;
    const S *pb = static_cast<const S *>(b) + b_offset;
    S *po = static_cast<S *>(out);
    cudaStream_t s = as_stream(stream);
    uint32_t r = cs.rank;
    // [rows, inner] with inner steps in {0, 1}: the row kernel.
    if (r <= 2) {
      long long inner = r ? (long long)cs.v[r - 1] : 1;
      long long rows = r == 2 ? (long long)cs.v[0] : 1;
      size_t ai = r ? cst[0].v[r - 1] : 0, bi = r ? cst[1].v[r - 1] : 0;
      if (ai <= 1 && bi <= 1) {
        long long as = r == 2 ? (long long)cst[0].v[0] : 0, bs = r == 2 ? (long long)cst[1].v[0] : 0;
        constexpr int N = Pack<T>::N;
        bool vec = inner % N == 0 && aligned16(po) && (!ai || (aligned16(pa) && as % N == 0)) &&
                   (!bi || (aligned16(pb) && bs % N == 0));
        long long work = rows * (vec ? inner / N : inner);
        unsigned grid = grid_for(size_t(work), 256, 8);
        if (vec && ai == 1 && inner / N >= 128) {
          unsigned g = unsigned(std::min<long long>((rows + 3) / 4, (long long)sm_count() * 8));
          return with_fn(f.kind, f.op, [&](auto fn) {
            ew_rows_blocked<T, decltype(fn), 4><<<std::max(1u, g), 256, 0, s>>>(pa, as, pb, bs, int(bi), po, rows,
                                                                                  inner, fn);
            return check_launch("strided binary (rows)");
          });
        }
        return with_fn(f.kind, f.op, [&](auto fn) {
          ew_rows<T><<<grid, 256, 0, s>>>(pa, as, int(ai), pb, bs, int(bi), po, rows, inner, fn, vec);
          return check_launch("strided binary");
        });
      }
    }
    Walk w{};
    w.rank = int(r);
    for (uint32_t ax = 0; ax < r; ++ax) {
      w.shape[ax] = (long long)cs.v[ax];
      w.stride[0][ax] = (long long)cst[0].v[ax];
      w.stride[1][ax] = (long long)cst[1].v[ax];
    }
    unsigned grid = grid_for(n, 256, 8);
    return with_fn(f.kind, f.op, [&](auto fn) {
      ew_walk<T><<<grid, 256, 0, s>>>(pa, pb, po, w, (long long)n, fn);
      return check_launch("strided binary (walk)");
    });
  });
}

}  // extern "C"
