// reduce.cu — axis reductions and arg-reductions (Kernels::reduce_axes,
// kernels.rs:1175; Kernels::arg_reduce, kernels.rs:1187; Host strided.rs:
// 105-225), plus the whole-vector fold and dot.
//
// Semantics (strided.rs): every slice folds in f32 and rounds to the element
// type once; Mean = total / depth; Variance = two passes, the f32 mean then
// the sum of squared deviations, / divisor; Min/Max pass over NaNs (fminf /
// fmaxf); arg-reductions keep the first position of the extreme, skip NaNs
// and answer 0 for a slice of only NaNs.  Sums are accumulated in a tree,
// so they agree with the Host's left-to-right fold to rounding, not bits;
// min, max and arg are exact.
//
// The host splits the layout into kept axes (one result each) and folded
// axes (coalesced separately), then picks a kernel:
//  - rows: the folded space ends in a contiguous run (innermost folded
//    stride 1).  A warp per (result, share of its slice); each lane issues
//    eight independent 128-bit loads before folding any.  When results are
//    few and slices long, the slice is split into shares whose partial
//    results land in a scratch buffer and are merged, in order, by a second
//    small kernel (by the share that finishes last, on the fast path).  A variance whose slice fits in registers is computed from
//    them in both passes, so the input is read from HBM once.
//    (A variant fed by 1-D TMA bulk copies through a shared-memory ring was
//    measured slower on B200 for 4 KB runs — 48 us against 30 us per
//    134 MB — and is not used.)
//  - columns: the innermost kept axis has stride 1 (results side by side).
//    Each thread owns four adjacent results (one vector load each) and a
//    share of the folded range; the shares combine in shared memory.
//  - walk: anything else; a warp per result over the decomposed folded
//    index.
// Every kernel is compiled per operation, so each carries only its own
// arithmetic.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace tc {
namespace {

enum Mode { M_SUM = 0, M_MIN = 1, M_MAX = 2, M_MEAN = 3, M_VAR = 4, M_ARGMIN = 5, M_ARGMAX = 6 };

template <int MODE> constexpr bool is_arg() { return MODE == M_ARGMIN || MODE == M_ARGMAX; }
// The fold a mode accumulates with.
template <int MODE> constexpr int fold_of() { return (MODE == M_MEAN || MODE == M_VAR) ? M_SUM : MODE; }

struct Acc {
  float v;
  uint32_t i;  // position (arg-reductions only)
};

template <int F> __device__ __forceinline__ Acc identity() {
  if (F == M_MIN) return {INFINITY, 0};
  if (F == M_MAX) return {-INFINITY, 0};
  if (is_arg<F>()) return {__int_as_float(0x7fc00000), 0};
  return {0.0f, 0};
}

// Fold one more element, at position `pos` along an arg-reduction's axis.
template <int F> __device__ __forceinline__ void push(Acc &a, float x, uint32_t pos) {
  if (F == M_MIN) a.v = fminf(a.v, x);
  else if (F == M_MAX) a.v = fmaxf(a.v, x);
  else if (F == M_ARGMIN) {
    // strided.rs:188-198 `replaces`: a number, and best is NaN or x is past it
    if (!isnan(x) && (isnan(a.v) || x < a.v)) { a.v = x; a.i = pos; }
  } else if (F == M_ARGMAX) {
    if (!isnan(x) && (isnan(a.v) || x > a.v)) { a.v = x; a.i = pos; }
  } else a.v = __fadd_rn(a.v, x);
}

// Combine partials; for an arg-reduction the lower position wins a tie.
template <int F> __device__ __forceinline__ Acc merge(Acc a, Acc b) {
  if (F == M_MIN) return {fminf(a.v, b.v), 0};
  if (F == M_MAX) return {fmaxf(a.v, b.v), 0};
  if (is_arg<F>()) {
    if (isnan(b.v)) return a;
    if (isnan(a.v)) return b;
    bool better = F == M_ARGMAX ? b.v > a.v : b.v < a.v;
    return (better || (b.v == a.v && b.i < a.i)) ? b : a;
  }
  return {__fadd_rn(a.v, b.v), 0};
}

template <int F> __device__ __forceinline__ Acc warp_merge(Acc a) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Acc b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, d);
    if (is_arg<F>()) b.i = __shfl_xor_sync(0xffffffffu, a.i, d);
    a = merge<F>(a, b);
  }
  return a;
}

// Storage position of flat index `r` of a one-operand walk; rank 0 and 1
// (the common cases) skip the division.
__device__ __forceinline__ long long walk_pos(const Walk &w, long long r) {
  if (w.rank == 0) return w.offset[0];
  if (w.rank == 1) return w.offset[0] + r * w.stride[0][0];
  long long p[1];
  walk_positions<1>(w, r, p);
  return p[0];
}

template <class T> struct Pack {
  using S = typename T::S;
  static constexpr int N = 16 / int(sizeof(S));
  union { uint4 raw; S v[N]; };
};

struct RowsArgs {
  Walk kept;          // result r -> slice base
  Walk folded;        // run o -> run offset within the slice
  long long results;  // kept results
  long long outer;    // runs per slice
  long long run;      // elements per run
  int splits;         // shares per slice (1 = no partials)
  long long share;    // runs (outer > 1) or units (outer == 1) per share
  float count, divisor;
  bool vec;
};

template <int MODE, class T>
__device__ __forceinline__ void write_result(const RowsArgs &a, long long r, Acc acc, typename T::S *out,
                                             uint32_t *arg_out) {
  if (is_arg<MODE>()) arg_out[r] = acc.i;
  else if (MODE == M_MEAN) out[r] = T::store(__fdiv_rn(acc.v, a.count));
  else out[r] = T::store(acc.v);
}

// ---------------------------------------------------------------------------
// rows: a warp per (result, share).  The slice is `outer` runs of `run`
// elements, read as units (16-byte packs when `vec`, else elements).
// ---------------------------------------------------------------------------
template <class T, int MODE>
__global__ void __launch_bounds__(256, 3) reduce_rows(const typename T::S *in, const RowsArgs a,
                                                      typename T::S *out, uint32_t *arg_out, Acc *partial) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  constexpr int F = fold_of<MODE>();
  constexpr int U = 8;
  const int lane = threadIdx.x & 31;
  const long long groups = a.results * a.splits;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long per_run = a.vec ? a.run / N : a.run;
  for (long long g = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
    const long long r = g / a.splits, s = g - r * a.splits;
    const S *base = in + walk_pos(a.kept, r);
    // A share is a range of whole runs, or (one run per slice) a range of
    // the run's units.
    long long o_lo = 0, o_hi = 1, c_lo = 0, c_hi = per_run;
    if (a.outer > 1) {
      o_lo = s * a.share;
      o_hi = min(a.outer, o_lo + a.share);
    } else {
      c_lo = s * a.share;
      c_hi = min(per_run, c_lo + a.share);
    }
    Acc acc = identity<F>();
    for (long long o = o_lo; o < o_hi; ++o) {
      const S *rp = base + walk_pos(a.folded, o);
      for (long long c0 = c_lo + lane; c0 < c_hi; c0 += 32 * U) {
        if (a.vec) {
          Pack<T> x[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < c_hi) x[u].raw = __ldg(reinterpret_cast<const uint4 *>(rp + (c0 + 32 * u) * N));
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < c_hi) {
              const uint32_t at = uint32_t((c0 + 32 * u) * N);
#pragma unroll
              for (int j = 0; j < N; ++j) push<F>(acc, T::load(x[u].v[j]), at + j);
            }
        } else {
          float x[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < c_hi) x[u] = T::load(rp[c0 + 32 * u]);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < c_hi) push<F>(acc, x[u], uint32_t(c0 + 32 * u));
        }
      }
    }
    acc = warp_merge<F>(acc);
    if (lane == 0) {
      if (a.splits > 1) partial[g] = acc;
      else write_result<MODE, T>(a, r, acc, out, arg_out);
    }
  }
}

// Merge each result's shares in order and finish it.
template <class T, int MODE>
__global__ void __launch_bounds__(256) reduce_finish(const RowsArgs a, const Acc *partial, typename T::S *out,
                                                     uint32_t *arg_out) {
  constexpr int F = fold_of<MODE>();
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < a.results; r += warps) {
    Acc acc = identity<F>();
    for (int s = lane; s < a.splits; s += 32) acc = merge<F>(acc, partial[r * a.splits + s]);
    acc = warp_merge<F>(acc);
    if (lane == 0) write_result<MODE, T>(a, r, acc, out, arg_out);
  }
}

// Two (count, sum, squared deviations from the mean) merged by the pairwise
// update of Chan, Golub and LeVeque (1979): M2 = M2a + M2b + d²·na·nb/n, d
// the difference of the two means.
__device__ __forceinline__ void chan_merge(float &n, float &sum, float &m2, float nb, float sum_b, float m2_b) {
  if (nb == 0.0f) return;
  if (n == 0.0f) {
    n = nb, sum = sum_b, m2 = m2_b;
    return;
  }
  const float d = __fsub_rn(__fdiv_rn(sum_b, nb), __fdiv_rn(sum, n));
  const float both = __fadd_rn(n, nb);
  m2 = __fadd_rn(__fadd_rn(m2, m2_b), __fmul_rn(__fmul_rn(d, d), __fdiv_rn(__fmul_rn(n, nb), both)));
  sum = __fadd_rn(sum, sum_b);
  n = both;
}

// Variance over rows: a warp per result.  When the slice is one run of at
// most 32*CACHE_PACKS packs it is held in registers between the passes; a
// longer single run is taken in sub-tiles of that size, each held in
// registers for its own sum and squared deviations from its own mean, merged
// pairwise (the run is read once); other slices take two passes.
constexpr int CACHE_PACKS = 8;
template <class T>
__global__ void __launch_bounds__(256, 2) reduce_rows_var(const typename T::S *in, const RowsArgs a,
                                                          typename T::S *out, typename T::S *mean_out) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const bool cache = a.vec && a.outer == 1 && a.run <= 32LL * N * CACHE_PACKS;
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < a.results; r += warps) {
    const S *base = in + walk_pos(a.kept, r);
    Acc sum = identity<M_SUM>(), dev = identity<M_SUM>();
    if (cache) {
      Pack<T> x[CACHE_PACKS];
#pragma unroll
      for (int k = 0; k < CACHE_PACKS; ++k)
        if ((32LL * k + lane) * N < a.run) x[k].raw = __ldg(reinterpret_cast<const uint4 *>(base + (32LL * k + lane) * N));
#pragma unroll
      for (int k = 0; k < CACHE_PACKS; ++k)
        if ((32LL * k + lane) * N < a.run) {
#pragma unroll
          for (int j = 0; j < N; ++j) sum.v = __fadd_rn(sum.v, T::load(x[k].v[j]));
        }
      sum = warp_merge<M_SUM>(sum);
      const float mean = __fdiv_rn(sum.v, a.count);
#pragma unroll
      for (int k = 0; k < CACHE_PACKS; ++k)
        if ((32LL * k + lane) * N < a.run) {
#pragma unroll
          for (int j = 0; j < N; ++j) {
            const float d = __fsub_rn(T::load(x[k].v[j]), mean);
            dev.v = __fadd_rn(dev.v, __fmul_rn(d, d));
          }
        }
    } else if (a.vec && a.outer == 1) {
      const long long packs = a.run / N;
      const uint4 *pp = reinterpret_cast<const uint4 *>(base);
      float n = 0.0f, s = 0.0f, m2 = 0.0f;
      for (long long t0 = 0; t0 < packs; t0 += 32 * CACHE_PACKS) {
        const long long in_tile = min((long long)(32 * CACHE_PACKS), packs - t0);
        Pack<T> x[CACHE_PACKS];
#pragma unroll
        for (int k = 0; k < CACHE_PACKS; ++k)
          if (32 * k + lane < in_tile) x[k].raw = __ldg(pp + t0 + 32 * k + lane);
        float ts = 0.0f;
#pragma unroll
        for (int k = 0; k < CACHE_PACKS; ++k)
          if (32 * k + lane < in_tile) {
#pragma unroll
            for (int j = 0; j < N; ++j) ts = __fadd_rn(ts, T::load(x[k].v[j]));
          }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) ts = __fadd_rn(ts, __shfl_xor_sync(0xffffffffu, ts, d));
        const float tn = float(in_tile * N), tm = __fdiv_rn(ts, tn);
        float tq = 0.0f;
#pragma unroll
        for (int k = 0; k < CACHE_PACKS; ++k)
          if (32 * k + lane < in_tile) {
#pragma unroll
            for (int j = 0; j < N; ++j) {
              const float d = __fsub_rn(T::load(x[k].v[j]), tm);
              tq = __fadd_rn(tq, __fmul_rn(d, d));
            }
          }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) tq = __fadd_rn(tq, __shfl_xor_sync(0xffffffffu, tq, d));
        chan_merge(n, s, m2, tn, ts, tq);
      }
      // every lane holds the totals: lane 0 carries them into the warp merge below
      dev.v = lane == 0 ? m2 : 0.0f;
      if (lane == 0 && mean_out) mean_out[r] = T::store(__fdiv_rn(s, a.count));
    } else {
      // Each pass: packs of the runs, four per lane in flight (the second
      // pass finds the slice in L2); element by element without packs.
      constexpr int U = 4;
      float mean = 0.0f;
      for (int pass = 0; pass < 2; ++pass) {
        Acc &acc = pass ? dev : sum;
        auto add = [&](float x) {
          if (pass) {
            const float d = __fsub_rn(x, mean);
            acc.v = __fadd_rn(acc.v, __fmul_rn(d, d));
          } else {
            acc.v = __fadd_rn(acc.v, x);
          }
        };
        for (long long o = 0; o < a.outer; ++o) {
          const S *rp = base + (a.outer > 1 ? walk_pos(a.folded, o) : 0);
          if (a.vec) {
            const long long packs = a.run / N;
            const uint4 *pp = reinterpret_cast<const uint4 *>(rp);
            for (long long c0 = lane; c0 < packs; c0 += 32 * U) {
              Pack<T> x[U];
#pragma unroll
              for (int u = 0; u < U; ++u)
                if (c0 + 32 * u < packs) x[u].raw = __ldg(pp + c0 + 32 * u);
#pragma unroll
              for (int u = 0; u < U; ++u)
                if (c0 + 32 * u < packs) {
#pragma unroll
                  for (int j = 0; j < N; ++j) add(T::load(x[u].v[j]));
                }
            }
          } else {
            for (long long c = lane; c < a.run; c += 32) add(T::load(rp[c]));
          }
        }
        if (!pass) {
          sum = warp_merge<M_SUM>(sum);
          mean = __fdiv_rn(sum.v, a.count);
        }
      }
      if (lane == 0 && mean_out) mean_out[r] = T::store(mean);
    }
    dev = warp_merge<M_SUM>(dev);
    if (lane == 0) {
      out[r] = T::store(__fdiv_rn(dev.v, a.divisor));
      if (cache && mean_out) mean_out[r] = T::store(__fdiv_rn(sum.v, a.count));
    }
  }
}


// ---------------------------------------------------------------------------
// columns: results r = (outer kept index) * K + k, k along the kept axis of
// stride 1.  blockDim = (32, 8): x walks 32*CPT adjacent results, y splits
// the folded range into 8 shares combined in shared memory in share order.
// ---------------------------------------------------------------------------
template <class T, int CPT> struct Cols {
  using S = typename T::S;
  using Raw = typename std::conditional<CPT * sizeof(S) == 16, uint4,
                                        typename std::conditional<CPT * sizeof(S) == 8, uint2, S>::type>::type;
  union { Raw raw; S v[CPT]; };
};

struct ColsArgs {
  Walk kept;    // kept outer index -> base
  Walk folded;  // folded flat index -> offset
  long long kept_outer, K, depth;
  float count, divisor;
  int kshares;         // shares of the folded range across blocks (1 = none)
  long long kchunk;    // folded positions per share
};

template <class T, int MODE, int CPT>
__global__ void __launch_bounds__(256, 3) reduce_cols(const typename T::S *in, const ColsArgs a, typename T::S *out,
                                                      uint32_t *arg_out, Acc *partial) {
  using S = typename T::S;
  using V = Cols<T, CPT>;
  constexpr int W = 32 * CPT;
  constexpr int U = 8;
  constexpr int F = fold_of<MODE>();
  __shared__ Acc part[8][W];
  const int Y = blockDim.y;
  const long long tiles_k = (a.K + W - 1) / W;
  const long long items = a.kept_outer * tiles_k * a.kshares;
  const long long results = a.kept_outer * a.K;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const long long t = it / a.kshares, ks = it - t * a.kshares;
    const long long ko = t / tiles_k;
    const long long k = (t - ko * tiles_k) * W + (long long)threadIdx.x * CPT;
    const bool live = k < a.K;  // CPT divides K when CPT > 1
    const S *base = in + walk_pos(a.kept, ko) + (live ? k : 0);
    // This block's share of the folded range, split again among the Y rows
    // of threads.
    const long long lo = ks * a.kchunk, hi = min(a.depth, lo + a.kchunk);
    const long long share = (hi - lo + Y - 1) / Y;
    const long long f0 = lo + (long long)threadIdx.y * share, f1 = min(hi, f0 + share);
    Acc acc[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[c] = identity<F>();
    if (live) {
      for (long long f = f0; f < f1; f += U) {
        V x[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (f + u < f1) x[u].raw = __ldg(reinterpret_cast<const typename V::Raw *>(base + walk_pos(a.folded, f + u)));
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (f + u < f1) {
#pragma unroll
            for (int c = 0; c < CPT; ++c) push<F>(acc[c], T::load(x[u].v[c]), uint32_t(f + u));
          }
      }
    }
#pragma unroll
    for (int c = 0; c < CPT; ++c) part[threadIdx.y][threadIdx.x * CPT + c] = acc[c];
    __syncthreads();
    Acc total[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      total[c] = part[0][threadIdx.x * CPT + c];
      for (int y = 1; y < Y; ++y) total[c] = merge<F>(total[c], part[y][threadIdx.x * CPT + c]);
    }
    __syncthreads();
    float result[CPT];
    if (MODE == M_VAR) {
      float mean[CPT];
      Acc d[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        mean[c] = __fdiv_rn(total[c].v, a.count);
        d[c] = identity<M_SUM>();
      }
      if (live)
        for (long long f = f0; f < f1; ++f) {
          V x;
          x.raw = __ldg(reinterpret_cast<const typename V::Raw *>(base + walk_pos(a.folded, f)));
#pragma unroll
          for (int c = 0; c < CPT; ++c) {
            const float dv = __fsub_rn(T::load(x.v[c]), mean[c]);
            d[c].v = __fadd_rn(d[c].v, __fmul_rn(dv, dv));
          }
        }
#pragma unroll
      for (int c = 0; c < CPT; ++c) part[threadIdx.y][threadIdx.x * CPT + c] = d[c];
      __syncthreads();
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        Acc dt = part[0][threadIdx.x * CPT + c];
        for (int y = 1; y < Y; ++y) dt = merge<M_SUM>(dt, part[y][threadIdx.x * CPT + c]);
        result[c] = __fdiv_rn(dt.v, a.divisor);
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int c = 0; c < CPT; ++c) result[c] = MODE == M_MEAN ? __fdiv_rn(total[c].v, a.count) : total[c].v;
    }
    if (live && threadIdx.y == 0) {
      const long long r = ko * a.K + k;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        if (a.kshares > 1) partial[ks * results + r + c] = total[c];
        else if (is_arg<MODE>()) arg_out[r + c] = total[c].i;
        else out[r + c] = T::store(result[c]);
      }
    }
  }
}

// Merge the column shares of each result, in share order.
template <class T, int MODE>
__global__ void __launch_bounds__(256) reduce_cols_finish(const Acc *partial, long long results, int kshares,
                                                          float count, typename T::S *out, uint32_t *arg_out) {
  constexpr int F = fold_of<MODE>();
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < results; r += (long long)gridDim.x * blockDim.x) {
    Acc acc = partial[r];
    for (int s = 1; s < kshares; ++s) acc = merge<F>(acc, partial[s * results + r]);
    if (is_arg<MODE>()) arg_out[r] = acc.i;
    else if (MODE == M_MEAN) out[r] = T::store(__fdiv_rn(acc.v, count));
    else out[r] = T::store(acc.v);
  }
}


// ---------------------------------------------------------------------------
// Fast paths for the common layouts (fixed strides, packs): lean kernels
// with 32-bit loop indices so that many warps stay resident.
//
// rows_fast: result r's slice is `outer` runs of `per_run` 16-byte packs at
// in + r*kept_stride + o*outer_stride; a warp per (result, share of runs).
// ---------------------------------------------------------------------------
struct FastRows {
  long long kept_stride, outer_stride;  // elements
  long long results;
  int outer, per_run;                   // runs per slice, packs per run
  int splits, share;                    // shares per slice, runs per share
  float count;
};

// An accumulator another block wrote in this launch, read past L1.
__device__ __forceinline__ Acc load_acc(const Acc *p) {
  const uint2 v = __ldcg(reinterpret_cast<const uint2 *>(p));
  return {__uint_as_float(v.x), v.y};
}

// With several shares per result, each publishes its accumulator and takes
// a ticket; the last to arrive merges them in share order (as
// reduce_finish does), writes the result and sets the ticket back to zero.
// (Requesting each warp's next 4 KB run into L2 before reading the current
// one measured slower on B200: config 2's sum 0.58 of HBM against 0.62.)
template <class T, int MODE>
__global__ void __launch_bounds__(256) reduce_rows_fast(const typename T::S *in, const FastRows a, typename T::S *out,
                                                        uint32_t *arg_out, Acc *partial, int *tickets) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  constexpr int F = fold_of<MODE>();
  constexpr int U = 8;
  const int lane = threadIdx.x & 31;
  const long long groups = a.results * a.splits;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long g = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
    const long long r = g / a.splits;
    const int s = int(g - r * a.splits);
    const int o_lo = s * a.share, o_hi = min(a.outer, o_lo + a.share);
    const uint4 *base = reinterpret_cast<const uint4 *>(in + r * a.kept_stride);
    Acc acc = identity<F>();
    for (int o = o_lo; o < o_hi; ++o) {
      const uint4 *rp = base + (o * a.outer_stride) / N;
      for (int c0 = lane; c0 < a.per_run; c0 += 32 * U) {
        Pack<T> x[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (c0 + 32 * u < a.per_run) x[u].raw = __ldg(rp + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (c0 + 32 * u < a.per_run) {
#pragma unroll
            for (int j = 0; j < N; ++j) push<F>(acc, T::load(x[u].v[j]), uint32_t((c0 + 32 * u) * N + j));
          }
      }
    }
    acc = warp_merge<F>(acc);
    if (a.splits > 1) {
      int ticket = 0;
      if (lane == 0) {
        partial[g] = acc;
        __threadfence();
        ticket = atomicAdd(&tickets[r], 1);
      }
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket != a.splits - 1) continue;
      __threadfence();
      acc = identity<F>();
      for (int q = lane; q < a.splits; q += 32) acc = merge<F>(acc, load_acc(partial + r * a.splits + q));
      acc = warp_merge<F>(acc);
      if (lane == 0) tickets[r] = 0;
    }
    if (lane == 0) {
      if (is_arg<MODE>()) arg_out[r] = acc.i;
      else if (MODE == M_MEAN) out[r] = T::store(__fdiv_rn(acc.v, a.count));
      else out[r] = T::store(acc.v);
    }
  }
}

// var_fast: a warp per result whose slice is one run of at most 32*8 packs
// at in + r*kept_stride, held in registers between the two passes.
template <class T>
__global__ void __launch_bounds__(256) reduce_rows_var_fast(const typename T::S *in, long long kept_stride,
                                                            long long results, int per_run, float count,
                                                            float divisor, typename T::S *out,
                                                            typename T::S *mean_out) {
  constexpr int N = Pack<T>::N;
  constexpr int K = CACHE_PACKS;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < results; r += warps) {
    const uint4 *base = reinterpret_cast<const uint4 *>(in + r * kept_stride);
    Pack<T> x[K];
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (32 * k + lane < per_run) x[k].raw = __ldg(base + 32 * k + lane);
    Acc sum = identity<M_SUM>();
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (32 * k + lane < per_run) {
#pragma unroll
        for (int j = 0; j < N; ++j) sum.v = __fadd_rn(sum.v, T::load(x[k].v[j]));
      }
    sum = warp_merge<M_SUM>(sum);
    const float mean = __fdiv_rn(sum.v, count);
    Acc dev = identity<M_SUM>();
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (32 * k + lane < per_run) {
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float d = __fsub_rn(T::load(x[k].v[j]), mean);
          dev.v = __fadd_rn(dev.v, __fmul_rn(d, d));
        }
      }
    dev = warp_merge<M_SUM>(dev);
    if (lane == 0) {
      out[r] = T::store(__fdiv_rn(dev.v, divisor));
      if (mean_out) mean_out[r] = T::store(mean);
    }
  }
}

// cols_fast: results r = ko*K + k (k along the stride-1 kept axis), in tiles
// of W = 256*CPT adjacent results of one kept-outer index; each thread owns
// CPT of them and reads them with one vector load per folded row (fixed
// folded stride).  The tiles' rows, laid end to end (tile-major), are cut
// into gridDim.x equal ranges, one per block, all resident at once, so
// every SM streams the same number of rows.  A tile whose rows fall in
// several blocks' ranges gets one partial from each: a block's range meets
// at most two tiles partly (its first and its last), so each block has two
// partial slots of W accumulators.  The last block to finish a tile merges
// its partials in block order and resets the tile's ticket.
struct FastCols {
  long long kept_stride, folded_stride;  // elements
  long long kept_outer, K, tiles_k, tiles;
  long long rows;                        // tiles * depth
  int depth;
  float count;
};

template <class T, int MODE, int CPT>
__global__ void __launch_bounds__(256, 3) reduce_cols_fast(const typename T::S *in, const FastCols a, typename T::S *out,
                                                           uint32_t *arg_out, Acc *partial, int *tickets) {
  // (Measured slower on B200 for config 2's argmax, against 37-40 us here:
  // a per-thread cp.async ring in shared memory with four blocks per SM,
  // 45.8 us; a warp-specialised ring fed by TMA bulk copies, one producer
  // warp and 4 stages of 16 KB per block, 45.5 us with DRAM 37% busy; TMA
  // bulk prefetches into L2 24 rows ahead of these loads, 40.2 us; four
  // loads per thread in flight with four blocks per SM, 41.6 us.)
  __shared__ int last;
  using S = typename T::S;
  using V = Cols<T, CPT>;
  constexpr int W = 256 * CPT;
  constexpr int U = sizeof(S) == 4 ? 6 : 8;  // loads in flight per thread, within 80 registers
  constexpr int F = fold_of<MODE>();
  const long long G = gridDim.x, b = blockIdx.x;
  long long x = b * a.rows / G;
  const long long x_end = (b + 1) * a.rows / G;
  while (x < x_end) {
    const long long t = x / a.depth;
    const int lo = int(x - t * a.depth);
    const int hi = int(min((long long)a.depth, (long long)lo + (x_end - x)));
    x += hi - lo;
    const long long ko = t / a.tiles_k;
    const long long k = (t - ko * a.tiles_k) * W + (long long)threadIdx.x * CPT;
    const bool live = k < a.K;  // CPT divides K
    const S *base = in + ko * a.kept_stride + (live ? k : 0);
    Acc acc[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[c] = identity<F>();
    if (live)
      for (int f = lo; f < hi; f += U) {
        V v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (f + u < hi)
            v[u].raw = __ldg(reinterpret_cast<const typename V::Raw *>(base + (long long)(f + u) * a.folded_stride));
        if (is_arg<MODE>()) {
          // The block's extreme per column first (fmaxf / fminf pass over
          // NaNs), then, only when it beats the running one, the first row
          // holding it: the same first-index, NaN-skipping result as folding
          // element by element, for about one instruction per element.
#pragma unroll
          for (int c = 0; c < CPT; ++c) {
            float x[U];
#pragma unroll
            for (int u = 0; u < U; ++u) x[u] = f + u < hi ? T::load(v[u].v[c]) : __int_as_float(0x7fc00000);
            float e = x[0];
#pragma unroll
            for (int u = 1; u < U; ++u) e = MODE == M_ARGMAX ? fmaxf(e, x[u]) : fminf(e, x[u]);
            const bool better = MODE == M_ARGMAX ? e > acc[c].v : e < acc[c].v;
            if (better || (isnan(acc[c].v) && !isnan(e))) {
              int first = U - 1;
#pragma unroll
              for (int u = U - 1; u >= 0; --u)
                if (x[u] == e) first = u;
              acc[c].v = e;
              acc[c].i = uint32_t(f + first);
            }
          }
        } else {
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (f + u < hi) {
#pragma unroll
              for (int c = 0; c < CPT; ++c) push<F>(acc[c], T::load(v[u].v[c]), uint32_t(f + u));
            }
        }
      }
    const long long r = ko * a.K + k;
    if (lo > 0 || hi < a.depth) {
      // Blocks first..first+n-1 hold the tile's rows (block(y), the one
      // whose range holds flat row y, is ((y + 1) * G - 1) / rows).  Block q
      // keeps its part of tile t in slot 0 when its range starts inside t,
      // else (t is its last tile) in slot 1.
      const long long t0 = t * a.depth;
      const long long first = ((t0 + 1) * G - 1) / a.rows;
      const int n = int(((t0 + a.depth) * G - 1) / a.rows - first + 1);
      const int side = b * a.rows / G < t0 ? 1 : 0;
      if (live) {
        Acc *mine = partial + (b * 2 + side) * W + threadIdx.x * CPT;
#pragma unroll
        for (int c = 0; c < CPT; ++c) mine[c] = acc[c];
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) last = atomicAdd(&tickets[t], 1) == n - 1;
      __syncthreads();
      if (!last) continue;
      __threadfence();
      if (live) {
        for (int q = 0; q < n; ++q) {
          const long long blk = first + q;
          const int sd = blk * a.rows / G < t0 ? 1 : 0;
          const Acc *theirs = partial + (blk * 2 + sd) * W + threadIdx.x * CPT;
#pragma unroll
          for (int c = 0; c < CPT; ++c) acc[c] = q ? merge<F>(acc[c], load_acc(theirs + c)) : load_acc(theirs + c);
        }
      }
      if (threadIdx.x == 0) tickets[t] = 0;
    }
    if (live) {
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        if (is_arg<MODE>()) arg_out[r + c] = acc[c].i;
        else if (MODE == M_MEAN) out[r + c] = T::store(__fdiv_rn(acc[c].v, a.count));
        else out[r + c] = T::store(acc[c].v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// walk: a warp per result over the decomposed folded index.
// ---------------------------------------------------------------------------
template <class T, int MODE>
__global__ void __launch_bounds__(256) reduce_walk(const typename T::S *in, const ColsArgs a, long long results,
                                                   typename T::S *out, uint32_t *arg_out) {
  constexpr int F = fold_of<MODE>();
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < results; r += warps) {
    const long long base = walk_pos(a.kept, r);
    Acc acc = identity<F>();
    for (long long f = lane; f < a.depth; f += 32) push<F>(acc, T::load(in[base + walk_pos(a.folded, f)]), uint32_t(f));
    acc = warp_merge<F>(acc);
    float result = acc.v;
    if (MODE == M_MEAN) result = __fdiv_rn(acc.v, a.count);
    if (MODE == M_VAR) {
      const float mean = __fdiv_rn(acc.v, a.count);
      Acc d = identity<M_SUM>();
      for (long long f = lane; f < a.depth; f += 32) {
        const float dv = __fsub_rn(T::load(in[base + walk_pos(a.folded, f)]), mean);
        d.v = __fadd_rn(d.v, __fmul_rn(dv, dv));
      }
      d = warp_merge<M_SUM>(d);
      result = __fdiv_rn(d.v, a.divisor);
    }
    if (lane == 0) {
      if (is_arg<MODE>()) arg_out[r] = acc.i;
      else out[r] = T::store(result);
    }
  }
}

// var_split: a variance whose slices are few and long, in chunks that fill
// the machine (a warp per slice would leave it nearly idle).  Slices that
// are one contiguous run take one pass (var_split_one below).  Otherwise
// pass 1 sums each (slice, chunk) with a block; the chunk sums, added in
// chunk order, give the f32 mean; pass 2 sums the squared deviations from
// it the same way; the chunk sums, added in order and divided, give the
// result.  The
// innermost folded axis is walked as a run (a step of run_stride), the
// others through their walk, recomputed only when the run changes.
struct VarSplit {
  Walk kept, outer;            // result -> base; folded outer index -> offset
  long long run, run_stride;   // the innermost folded axis
  long long results, depth, chunk;
  int chunks;
  float count, divisor;
};

template <class T, bool DEV>
__global__ void __launch_bounds__(256) var_split_pass(const typename T::S *in, const VarSplit a, const float *means,
                                                      float *partial) {
  __shared__ float warp_part[8];
  const long long groups = a.results * a.chunks;
  for (long long g = blockIdx.x; g < groups; g += gridDim.x) {
    const long long r = g / a.chunks;
    const long long f0 = (g - r * a.chunks) * a.chunk, f1 = min(a.depth, f0 + a.chunk);
    const typename T::S *base = in + walk_pos(a.kept, r);
    const float mean = DEV ? means[r] : 0.0f;
    float s = 0.0f;
    auto add = [&](float x) {
      if (DEV) {
        const float d = __fsub_rn(x, mean);
        s = __fadd_rn(s, __fmul_rn(d, d));
      } else {
        s = __fadd_rn(s, x);
      }
    };
    using P = Pack<T>;
    constexpr int N = P::N;
    if (a.outer.rank == 0 && a.run_stride == 1 && (reinterpret_cast<uintptr_t>(base + f0) & 15u) == 0) {
      // One contiguous run: 16-byte packs, two per thread in flight.
      const long long packs = (f1 - f0) / N;
      const uint4 *src = reinterpret_cast<const uint4 *>(base + f0);
      for (long long q = threadIdx.x; q < packs; q += 512) {
        P x0, x1;
        x0.raw = __ldg(src + q);
        const bool two = q + 256 < packs;
        if (two) x1.raw = __ldg(src + q + 256);
#pragma unroll
        for (int e = 0; e < N; ++e) add(T::load(x0.v[e]));
        if (two) {
#pragma unroll
          for (int e = 0; e < N; ++e) add(T::load(x1.v[e]));
        }
      }
      for (long long f = f0 + packs * N + threadIdx.x; f < f1; f += 256) add(T::load(base[f]));
    } else {
      long long f = f0 + threadIdx.x;
      if (f < f1) {
        long long o = f / a.run, j = f - o * a.run;
        const long long so = 256 / a.run, sj = 256 - so * a.run;
        long long last_o = o, opos = walk_pos(a.outer, o);
        for (; f < f1; f += 256) {
          if (o != last_o) {
            last_o = o;
            opos = walk_pos(a.outer, o);
          }
          add(T::load(base[opos + j * a.run_stride]));
          j += sj;
          o += so;
          if (j >= a.run) {
            j -= a.run;
            ++o;
          }
        }
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, d));
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = warp_part[0];
      for (int w = 1; w < 8; ++w) t = __fadd_rn(t, warp_part[w]);
      partial[g] = t;
    }
    __syncthreads();
  }
}

// The chunk sums of each slice (a block per slice: thread t adds chunks t,
// t+256, ... in order, then a fixed tree): the f32 mean (into means, and in
// T into out when asked), or the variance rounded to T (into out).
template <class T, bool DEV>
__global__ void __launch_bounds__(256) var_split_finish(const VarSplit a, const float *partial, float *means,
                                                        typename T::S *out) {
  __shared__ float warp_part[8];
  for (long long r = blockIdx.x; r < a.results; r += gridDim.x) {
    float t = 0.0f;
    for (int c = threadIdx.x; c < a.chunks; c += 256) t = __fadd_rn(t, partial[r * a.chunks + c]);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, d));
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
      float total = warp_part[0];
      for (int w = 1; w < 8; ++w) total = __fadd_rn(total, warp_part[w]);
      if (DEV) {
        out[r] = T::store(__fdiv_rn(total, a.divisor));
      } else {
        means[r] = __fdiv_rn(total, a.count);
        if (out) out[r] = T::store(means[r]);  // the mean in T, for moments
      }
    }
    __syncthreads();
  }
}

// var_split in one pass, for slices that are one contiguous run: each warp
// takes 16 elements per lane at a time (a sub-tile of 512, in 16-byte packs
// when the chunk starts on a 16-byte boundary), takes the sub-tile's sum and
// its squared deviations from its own mean (both warp trees), and merges
// that into its running (count, sum, squared deviations) with chan_merge.
// The block merges its warps in warp order into partial[g] = (sum, M2) of
// its chunk; the input is read once.
constexpr int VS_PER_LANE = 16;


template <class T>
__global__ void __launch_bounds__(256) var_split_one(const typename T::S *in, const VarSplit a, float2 *partial) {
  __shared__ float3 warp_part[8];  // (count, sum, M2) per warp
  using P = Pack<T>;
  constexpr int N = P::N, K = VS_PER_LANE / N, TILE = 32 * VS_PER_LANE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long groups = a.results * a.chunks;
  for (long long g = blockIdx.x; g < groups; g += gridDim.x) {
    const long long r = g / a.chunks;
    const long long f0 = (g - r * a.chunks) * a.chunk, len = min(a.depth, f0 + a.chunk) - f0;
    const typename T::S *base = in + walk_pos(a.kept, r) + f0;
    const bool vec = (reinterpret_cast<uintptr_t>(base) & 15u) == 0;
    float wn = 0.0f, ws = 0.0f, wm2 = 0.0f;
    for (long long t0 = (long long)warp * TILE; t0 < len; t0 += 8LL * TILE) {
      const int cnt = int(min((long long)TILE, len - t0));
      float v[VS_PER_LANE];
      bool ok[VS_PER_LANE];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        // pack k of the lane: elements t0 + (k*32 + lane)*N .. +N-1
        const long long at = t0 + (long long)(k * 32 + lane) * N;
        if (vec && at + N <= len) {
          P x;
          x.raw = __ldg(reinterpret_cast<const uint4 *>(base + at));
#pragma unroll
          for (int e = 0; e < N; ++e) v[k * N + e] = T::load(x.v[e]), ok[k * N + e] = true;
        } else {
#pragma unroll
          for (int e = 0; e < N; ++e) {
            ok[k * N + e] = at + e < len;
            v[k * N + e] = ok[k * N + e] ? T::load(base[at + e]) : 0.0f;
          }
        }
      }
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < VS_PER_LANE; ++i)
        if (ok[i]) s = __fadd_rn(s, v[i]);
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, d));
      const float mean = __fdiv_rn(s, float(cnt));
      float q = 0.0f;
#pragma unroll
      for (int i = 0; i < VS_PER_LANE; ++i)
        if (ok[i]) {
          const float d = __fsub_rn(v[i], mean);
          q = __fadd_rn(q, __fmul_rn(d, d));
        }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, d));
      chan_merge(wn, ws, wm2, float(cnt), s, q);
    }
    if (lane == 0) warp_part[warp] = make_float3(wn, ws, wm2);
    __syncthreads();
    if (threadIdx.x == 0) {
      float n = 0.0f, sum = 0.0f, m2 = 0.0f;
      for (int w = 0; w < 8; ++w) chan_merge(n, sum, m2, warp_part[w].x, warp_part[w].y, warp_part[w].z);
      partial[g] = make_float2(sum, m2);
    }
    __syncthreads();
  }
}

// The chunks of each slice merged (a block per slice: thread t merges chunks
// t, t+256, ... in order, then the threads' results meet in a fixed tree):
// the mean (the plain sum of the chunk sums over the count, in T into
// `mean_out` when asked) and the variance M2 / divisor in T into `out`.
template <class T>
__global__ void __launch_bounds__(256) var_split_one_finish(const VarSplit a, const float2 *partial,
                                                            typename T::S *mean_out, typename T::S *out) {
  __shared__ float3 part[256];
  for (long long r = blockIdx.x; r < a.results; r += gridDim.x) {
    float n = 0.0f, sum = 0.0f, m2 = 0.0f;
    for (int c = threadIdx.x; c < a.chunks; c += 256) {
      const float cn = float(min(a.chunk, a.depth - (long long)c * a.chunk));
      const float2 p = partial[r * a.chunks + c];
      chan_merge(n, sum, m2, cn, p.x, p.y);
    }
    part[threadIdx.x] = make_float3(n, sum, m2);
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
      if (threadIdx.x < stride) {
        float3 x = part[threadIdx.x];
        const float3 y = part[threadIdx.x + stride];
        chan_merge(x.x, x.y, x.z, y.x, y.y, y.z);
        part[threadIdx.x] = x;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      if (mean_out) mean_out[r] = T::store(__fdiv_rn(part[0].y, a.count));
      out[r] = T::store(__fdiv_rn(part[0].z, a.divisor));
    }
    __syncthreads();
  }
}

void fill_walk(Walk &w, const Dims &shape, const Dims &strides) {
  w = Walk{};
  w.rank = int(shape.rank);
  for (uint32_t a = 0; a < shape.rank; ++a) {
    w.shape[a] = (long long)shape.v[a];
    w.stride[0][a] = (long long)strides.v[a];
  }
}

int scratch_get(size_t bytes, void **out, cudaStream_t stream) { return scratch(bytes, out, stream); }

// A variance's slices' means in T, when the path computing the variance
// can write them too (`written` says whether it did).
struct MeanOut {
  void *ptr = nullptr;
  bool written = false;
};

template <class T, int MODE>
int launch_mode(const typename T::S *in, const Dims &kc, const Dims &kcs, const Dims &fc, const Dims &fcs,
                long long results, long long depth, float count, float divisor, void *out, uint32_t *arg_out,
                cudaStream_t stream, MeanOut *mean_out = nullptr) {
  using S = typename T::S;
  S *o = static_cast<S *>(out);
  S *mo = mean_out ? static_cast<S *>(mean_out->ptr) : nullptr;
  const int sms = sm_count();
  // rows: innermost folded axis contiguous (unless the kept axis is the
  // contiguous one and the runs are short).
  const bool kept_inner_contig = kc.rank && kcs.v[kc.rank - 1] == 1;
  if (MODE == M_VAR && fc.rank >= 1 && results < (long long)sms * 16 && depth >= 16384) {
    VarSplit v{};
    fill_walk(v.kept, kc, kcs);
    Dims fo = fc, fos = fcs;
    fo.rank = fos.rank = fc.rank - 1;
    fill_walk(v.outer, fo, fos);
    v.run = (long long)fc.v[fc.rank - 1];
    v.run_stride = (long long)fcs.v[fc.rank - 1];
    v.results = results;
    v.depth = depth;
    // chunks of at least 4096 elements, about 8 blocks' worth per SM in all
    const long long want = std::max(1LL, (long long)sms * 8 / results);
    v.chunk = std::max(4096LL, ((depth + want - 1) / want + 255) / 256 * 256);
    v.chunks = int((depth + v.chunk - 1) / v.chunk);
    v.count = count;
    v.divisor = divisor;
    void *p = nullptr;
    const size_t groups = size_t(results) * size_t(v.chunks);
    if (int st = scratch_get((2 * groups + size_t(results)) * sizeof(float), &p, stream)) return st;
    float *partial = static_cast<float *>(p), *means = partial + groups;
    const unsigned grid = unsigned(std::min<long long>((long long)groups, (long long)sms * 8));
    const unsigned fgrid = unsigned(std::min<long long>(results, (long long)sms * 8));
    if (v.outer.rank == 0 && v.run_stride == 1) {
      // contiguous slices: one read (partial holds (sum, M2) per chunk)
      var_split_one<T><<<grid, 256, 0, stream>>>(in, v, reinterpret_cast<float2 *>(partial));
      var_split_one_finish<T><<<fgrid, 256, 0, stream>>>(v, reinterpret_cast<const float2 *>(partial), mo, o);
      if (mean_out) mean_out->written = true;
      return check_launch("reduce (variance, split, one pass)");
    }
    var_split_pass<T, false><<<grid, 256, 0, stream>>>(in, v, nullptr, partial);
    var_split_finish<T, false><<<fgrid, 256, 0, stream>>>(v, partial, means, mo);
    if (mean_out) mean_out->written = true;
    var_split_pass<T, true><<<grid, 256, 0, stream>>>(in, v, means, partial);
    var_split_finish<T, true><<<fgrid, 256, 0, stream>>>(v, partial, means, o);
    return check_launch("reduce (variance, split)");
  }
  if (fc.rank >= 1 && fcs.v[fc.rank - 1] == 1 && !(kept_inner_contig && fc.v[fc.rank - 1] < 64)) {
    RowsArgs a{};
    fill_walk(a.kept, kc, kcs);
    Dims fo = fc, fos = fcs;
    fo.rank = fos.rank = fc.rank - 1;
    fill_walk(a.folded, fo, fos);
    a.results = results;
    a.outer = (long long)element_count(fo.rank, fo.v);
    a.run = (long long)fc.v[fc.rank - 1];
    a.count = count;
    a.divisor = divisor;
    constexpr int N = Pack<T>::N;
    a.vec = a.run % N == 0 && (uintptr_t(in) & 15u) == 0;
    for (uint32_t ax = 0; a.vec && ax < kc.rank; ++ax) a.vec = kcs.v[ax] % N == 0;
    for (uint32_t ax = 0; a.vec && ax < fo.rank; ++ax) a.vec = fos.v[ax] % N == 0;
    // The fast path: at most one kept and one outer folded axis, packs, and
    // index ranges that fit 32 bits.
    // (A few long single-run slices go to the general kernel, which splits
    // a run between warps; this one splits only across runs.)
    const bool few_long_runs = a.outer == 1 && results < (long long)sms * 16 && a.run / N >= 32LL * 8 * 4;
    if (MODE != M_VAR && a.vec && kc.rank <= 1 && fo.rank <= 1 && a.outer < (1LL << 30) &&
        a.run / N < (1LL << 30) && !few_long_runs) {
      FastRows f{};
      f.kept_stride = kc.rank ? (long long)kcs.v[0] : 0;
      f.outer_stride = fo.rank ? (long long)fos.v[0] : 0;
      f.results = results;
      f.outer = int(a.outer);
      f.per_run = int(a.run / N);
      f.count = count;
      long long splits = 1;
      while (results * splits < (long long)sms * 32 && a.outer / (splits * 2) >= 1 &&
             (a.outer / (splits * 2)) * f.per_run >= 32LL * 8 * 2)
        splits *= 2;
      f.splits = int(splits);
      f.share = int((a.outer + splits - 1) / splits);
      Acc *partial = nullptr;
      int *tickets = nullptr;
      if (splits > 1) {
        void *p = nullptr;
        if (int st = scratch_get(size_t(results * splits) * sizeof(Acc), &p, stream)) return st;
        partial = static_cast<Acc *>(p);
        if (int st = counters(size_t(results), &tickets, stream)) return st;
      }
      static int resident_fast[7] = {0, 0, 0, 0, 0, 0, 0};
      if (!resident_fast[MODE]) {
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_rows_fast<T, MODE>, 256, 0);
        resident_fast[MODE] = n > 0 ? n : 2;
      }
      const long long groups = results * splits;
      unsigned grid = unsigned(std::min<long long>((groups + 7) / 8, (long long)sms * resident_fast[MODE]));
      reduce_rows_fast<T, MODE><<<std::max(1u, grid), 256, 0, stream>>>(in, f, o, arg_out, partial, tickets);
      return check_launch("reduce (rows, fast)");
    }
    if (MODE == M_VAR && a.vec && kc.rank <= 1 && a.outer == 1 && a.run / N <= 32LL * CACHE_PACKS) {
      static int resident_var = 0;
      if (!resident_var) {
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_rows_var_fast<T>, 256, 0);
        resident_var = n > 0 ? n : 2;
      }
      unsigned grid = unsigned(std::min<long long>((results + 7) / 8, (long long)sms * resident_var));
      reduce_rows_var_fast<T><<<std::max(1u, grid), 256, 0, stream>>>(
          in, kc.rank ? (long long)kcs.v[0] : 0, results, int(a.run / N), count, divisor, o, mo);
      if (mean_out) mean_out->written = true;
      return check_launch("reduce (rows, variance, fast)");
    }
    if (MODE == M_VAR) {
      a.splits = 1;
      unsigned grid = unsigned(std::min<long long>((results + 7) / 8, (long long)sms * 8));
      reduce_rows_var<T><<<std::max(1u, grid), 256, 0, stream>>>(in, a, o, mo);
      if (mean_out) mean_out->written = true;
      return check_launch("reduce (rows, variance)");
    }
    // Split each slice into shares (of whole runs, or of its one run's
    // units) while there are fewer than ~16 warps of work per SM and a share
    // keeps at least two batches of loads per lane.
    const long long per_run = a.vec ? a.run / N : a.run;
    long long splits = 1;
    if (a.outer > 1) {
      while (results * splits < (long long)sms * 16 && a.outer / (splits * 2) >= 1 &&
             (a.outer / (splits * 2)) * per_run >= 32LL * 8 * 2)
        splits *= 2;
      a.share = (a.outer + splits - 1) / splits;
    } else {
      while (results * splits < (long long)sms * 16 && per_run / (splits * 2) >= 32LL * 8 * 2) splits *= 2;
      a.share = (per_run + splits - 1) / splits;
    }
    a.splits = int(splits);
    Acc *partial = nullptr;
    if (splits > 1) {
      void *p = nullptr;
      if (int st = scratch_get(size_t(results * splits) * sizeof(Acc), &p, stream)) return st;
      partial = static_cast<Acc *>(p);
    }
    const long long groups = results * splits;
    // As many blocks as stay resident (a persistent grid): each warp walks
    // its groups in turn instead of the grid running in waves.
    static int resident[7] = {0, 0, 0, 0, 0, 0, 0};
    if (!resident[MODE]) {
      int n = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_rows<T, MODE>, 256, 0);
      resident[MODE] = n > 0 ? n : 2;
    }
    unsigned grid = unsigned(std::min<long long>((groups + 7) / 8, (long long)sms * resident[MODE]));
    reduce_rows<T, MODE><<<std::max(1u, grid), 256, 0, stream>>>(in, a, o, arg_out, partial);
    if (splits > 1) {
      unsigned g2 = unsigned(std::min<long long>((results + 7) / 8, (long long)sms * 8));
      reduce_finish<T, MODE><<<std::max(1u, g2), 256, 0, stream>>>(a, partial, o, arg_out);
    }
    return check_launch("reduce (rows)");
  }
  ColsArgs a{};
  a.depth = depth;
  a.count = count;
  a.divisor = divisor;
  if (kept_inner_contig) {
    a.K = (long long)kc.v[kc.rank - 1];
    Dims ko = kc, kos = kcs;
    ko.rank = kos.rank = kc.rank - 1;
    a.kept_outer = (long long)element_count(ko.rank, ko.v);
    fill_walk(a.kept, ko, kos);
    fill_walk(a.folded, fc, fcs);
    // Four results per thread when every row of them starts 4-aligned.
    bool four = a.K % 4 == 0 && (uintptr_t(in) % (4 * sizeof(S))) == 0;
    for (uint32_t ax = 0; four && ax < ko.rank; ++ax) four = kos.v[ax] % 4 == 0;
    for (uint32_t ax = 0; four && ax < fc.rank; ++ax) four = fcs.v[ax] % 4 == 0;
    if (MODE != M_VAR && four && ko.rank <= 1 && fc.rank <= 1 && depth < (1LL << 30)) {
      FastCols f{};
      f.kept_stride = ko.rank ? (long long)kos.v[0] : 0;
      f.folded_stride = fc.rank ? (long long)fcs.v[0] : 0;
      f.kept_outer = a.kept_outer;
      f.K = a.K;
      f.depth = int(depth);
      f.count = count;
      f.tiles_k = (a.K + 1023) / 1024;
      f.tiles = a.kept_outer * f.tiles_k;
      f.rows = f.tiles * depth;
      static int resident_cols[7] = {0, 0, 0, 0, 0, 0, 0};
      if (!resident_cols[MODE]) {
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_cols_fast<T, MODE, 4>, 256, 0);
        resident_cols[MODE] = std::max(1, n);
      }
      // One resident wave of blocks, each with at least 16 rows.
      const long long grid = std::max(1LL, std::min((long long)sms * resident_cols[MODE], f.rows / 16));
      Acc *partial = nullptr;
      int *tickets = nullptr;
      if (grid > 1) {
        void *p = nullptr;
        if (int st = scratch_get(size_t(grid) * 2 * 1024 * sizeof(Acc), &p, stream)) return st;
        partial = static_cast<Acc *>(p);
        if (int st = counters(size_t(f.tiles), &tickets, stream)) return st;
      }
      reduce_cols_fast<T, MODE, 4><<<unsigned(grid), 256, 0, stream>>>(in, f, o, arg_out, partial, tickets);
      return check_launch("reduce (columns, fast)");
    }
    const int cpt = four ? 4 : 1;
    const long long tiles = a.kept_outer * ((a.K + 32 * cpt - 1) / (32 * cpt));
    // Split the folded range across blocks until the work items divide
    // evenly-ish over the resident blocks (3 per SM), keeping each share at
    // least 64 folded positions.  A variance needs its slice's mean, so it
    // is never split.
    const long long slots = (long long)sms * 3;
    int ks = 1;
    if (MODE != M_VAR)
      while (tiles * ks < 4 * slots && depth / (ks * 2) >= 64) ks *= 2;
    a.kshares = ks;
    a.kchunk = (depth + ks - 1) / ks;
    const long long items = tiles * ks;
    long long waves = (items + slots - 1) / slots;
    unsigned grid = unsigned(std::max<long long>(1, (items + waves - 1) / waves));
    Acc *partial = nullptr;
    if (ks > 1) {
      void *p = nullptr;
      if (int st = scratch_get(size_t(ks) * size_t(a.kept_outer * a.K) * sizeof(Acc), &p, stream)) return st;
      partial = static_cast<Acc *>(p);
    }
    if (four) reduce_cols<T, MODE, 4><<<grid, dim3(32, 8), 0, stream>>>(in, a, o, arg_out, partial);
    else reduce_cols<T, MODE, 1><<<grid, dim3(32, 8), 0, stream>>>(in, a, o, arg_out, partial);
    if (ks > 1) {
      const long long results_c = a.kept_outer * a.K;
      reduce_cols_finish<T, MODE><<<grid_for(size_t(results_c), 256, 4), 256, 0, stream>>>(partial, results_c, ks,
                                                                                            count, o, arg_out);
    }
    return check_launch("reduce (columns)");
  }
  fill_walk(a.kept, kc, kcs);
  fill_walk(a.folded, fc, fcs);
  unsigned grid = unsigned(std::min<long long>((results + 7) / 8, (long long)sms * 8));
  reduce_walk<T, MODE><<<std::max(1u, grid), 256, 0, stream>>>(in, a, results, o, arg_out);
  return check_launch("reduce (walk)");
}

// The shared driver of reduce_axes and arg_reduce.
int run_reduction(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t offset,
                  const size_t *strides, const bool *folded, int mode, size_t divisor, void *out,
                  uint32_t *arg_out, cudaStream_t stream, MeanOut *mean_out = nullptr) {
  // Split, layout.rs:370-414.
  size_t ks[TC_MAX_RANK], kst[TC_MAX_RANK], fs[TC_MAX_RANK], fst[TC_MAX_RANK];
  uint32_t nk = 0, nf = 0;
  for (uint32_t a = 0; a < rank; ++a) {
    if (folded[a]) { fs[nf] = shape[a]; fst[nf++] = strides[a]; }
    else { ks[nk] = shape[a]; kst[nk++] = strides[a]; }
  }
  const long long results = (long long)element_count(nk, ks), depth = (long long)element_count(nf, fs);
  if (results == 0) return TC_OK;
  if (depth == 0) return fail(TC_EINVAL, "reduction over an empty slice");
  // Kept axes coalesce against the contiguous result strides, so results
  // stay in row-major order; folded axes coalesce among themselves (an
  // arg-reduction's one axis stays one axis).
  size_t kout[TC_MAX_RANK];
  contiguous_strides(nk, ks, kout);
  const size_t *kops[2] = {kst, kout};
  Dims kc, kcs[2];
  coalesce<2>(nk, ks, kops, kc, kcs);
  const size_t *fops[1] = {fst};
  Dims fc, fcs[1];
  coalesce<1>(nf, fs, fops, fc, fcs);
  const float count = float(depth), div = float(double(divisor));
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    const typename T::S *in = static_cast<const typename T::S *>(input) + offset;
    switch (mode) {
      case M_SUM: return launch_mode<T, M_SUM>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
      case M_MIN: return launch_mode<T, M_MIN>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
      case M_MAX: return launch_mode<T, M_MAX>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
      case M_MEAN: return launch_mode<T, M_MEAN>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
      case M_VAR:
        return launch_mode<T, M_VAR>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream,
                                     mean_out);
      case M_ARGMIN: return launch_mode<T, M_ARGMIN>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
      case M_ARGMAX: return launch_mode<T, M_ARGMAX>(in, kc, kcs[0], fc, fcs[0], results, depth, count, div, out, arg_out, stream);
    }
    return fail(TC_EINVAL, "reduction mode %d", mode);
  });
}

// Whole-vector fold / dot: per-block partials, then one block folds them.
template <class T, int F>
__global__ void __launch_bounds__(256) vector_partials(const typename T::S *a, const typename T::S *b, size_t n,
                                                       float *partials, bool vec) {
  // 16-byte packs, U of them (and of b's) in flight per thread; the tail
  // element by element.  Each thread's order and the block's tree are fixed.
  __shared__ Acc sh[8];
  constexpr int N = Pack<T>::N, U = 4;
  Acc acc = identity<F>();
  const size_t stride = size_t(gridDim.x) * blockDim.x, tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t packs = vec ? n / N : 0;
  const uint4 *pa = reinterpret_cast<const uint4 *>(a), *pb = reinterpret_cast<const uint4 *>(b);
  for (size_t p0 = tid; p0 < packs; p0 += stride * U) {
    Pack<T> x[U], y[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (p0 + u * stride < packs) {
        x[u].raw = __ldg(pa + p0 + u * stride);
        if (b) y[u].raw = __ldg(pb + p0 + u * stride);
      }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (p0 + u * stride < packs) {
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float v = T::load(x[u].v[j]);
          if (b) v = __fmul_rn(v, T::load(y[u].v[j]));
          push<F>(acc, v, 0);
        }
      }
  }
  for (size_t i = packs * N + tid; i < n; i += stride) {
    float x = T::load(a[i]);
    if (b) x = __fmul_rn(x, T::load(b[i]));
    push<F>(acc, x, 0);
  }
  acc = warp_merge<F>(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    Acc r = sh[0];
    for (int w = 1; w < int(blockDim.x >> 5); ++w) r = merge<F>(r, sh[w]);
    partials[blockIdx.x] = r.v;
  }
}
template <class T, int F>
__global__ void __launch_bounds__(256) vector_finish(const float *partials, int count, typename T::S *out) {
  __shared__ Acc sh[8];
  Acc acc = identity<F>();
  for (int i = threadIdx.x; i < count; i += blockDim.x) push<F>(acc, partials[i], 0);
  acc = warp_merge<F>(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    Acc r = sh[0];
    for (int w = 1; w < int(blockDim.x >> 5); ++w) r = merge<F>(r, sh[w]);
    out[0] = T::store(r.v);
  }
}

template <int F>
int vector_fold(int dtype, const void *a, const void *b, size_t n, void *out, cudaStream_t stream) {
  if (!out) return fail(TC_EINVAL, "vector reduce: null output");
  const int max_blocks = 2048;
  void *p = nullptr;
  if (int st = scratch_get(max_blocks * sizeof(float), &p, stream)) return st;
  float *partials = static_cast<float *>(p);
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    using S = typename T::S;
    constexpr size_t N = size_t(Pack<T>::N);
    const bool vec = (uintptr_t(a) & 15u) == 0 && (!b || (uintptr_t(b) & 15u) == 0);
    const size_t units = vec ? (n + N - 1) / N : n;
    int blocks = int(std::min<size_t>(std::max<size_t>((units + 255) / 256, 1),
                                      std::min<size_t>(size_t(max_blocks), size_t(sm_count()) * 8)));
    vector_partials<T, F><<<blocks, 256, 0, stream>>>(static_cast<const S *>(a), static_cast<const S *>(b), n, partials,
                                                      vec);
    vector_finish<T, F><<<1, 256, 0, stream>>>(partials, blocks, static_cast<S *>(out));
    return check_launch("vector reduce");
  });
}

}  // namespace



// Means and sums of squared deviations of the slices of `input` folded over
// `axes` (both in T): the variance kernel with divisor 1, which writes the
// means too where it can; otherwise a mean reduction beside it.
int reduce_moments(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t offset,
                   const size_t *strides, uint32_t n_axes, const uint32_t *axes, void *means, void *deviations,
                   cudaStream_t stream) {
  bool folded[TC_MAX_RANK] = {false};
  for (uint32_t i = 0; i < n_axes; ++i) folded[axes[i]] = true;
  MeanOut m;
  m.ptr = means;
  if (int st = run_reduction(dtype, rank, shape, input, offset, strides, folded, M_VAR, 1, deviations, nullptr, stream,
                             &m))
    return st;
  if (m.written) return TC_OK;
  return run_reduction(dtype, rank, shape, input, offset, strides, folded, M_MEAN, 0, means, nullptr, stream);
}

}  // namespace tc

using namespace tc;

extern "C" {

int tc_reduce_axes(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t input_len, size_t offset,
                   const size_t *strides, uint32_t n_axes, const uint32_t *axes, int kind, int op, size_t divisor,
                   void *out, void *stream) {
  if (int st = check_layout("reduce_axes", input_len, rank, shape, offset, strides)) return st;
  if (n_axes > rank || (n_axes && !axes)) return fail(TC_EINVAL, "reduce_axes: bad axes");
  bool folded[TC_MAX_RANK] = {false};
  for (uint32_t i = 0; i < n_axes; ++i) {
    if (axes[i] >= rank || (i && axes[i] <= axes[i - 1]))
      return fail(TC_EINVAL, "reduce_axes: axes must be distinct, ascending axes of a rank-%u shape", rank);
    folded[axes[i]] = true;
  }
  int mode;
  if (kind == TC_AXIS_FOLD) {
    if (op < TC_SUM || op > TC_RMAX) return fail(TC_EINVAL, "reduce_axes: bad Reduce %d", op);
    mode = op == TC_SUM ? M_SUM : (op == TC_RMIN ? M_MIN : M_MAX);
  } else if (kind == TC_AXIS_MEAN) {
    mode = M_MEAN;
  } else if (kind == TC_AXIS_VARIANCE) {
    mode = M_VAR;
  } else {
    return fail(TC_EINVAL, "reduce_axes: bad AxisReduction %d", kind);
  }
  if (element_count(rank, shape) == 0) {
    size_t results = 1;
    for (uint32_t a = 0; a < rank; ++a)
      if (!folded[a]) results *= shape[a];
    return results == 0 ? TC_OK : fail(TC_EINVAL, "reduce_axes: slices are empty");
  }
  if (!input || !out) return fail(TC_EINVAL, "reduce_axes: null pointer");
  return run_reduction(dtype, rank, shape, input, offset, strides, folded, mode, divisor, out, nullptr,
                       as_stream(stream));
}

int tc_arg_reduce(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t input_len, size_t offset,
                  const size_t *strides, uint32_t axis, int op, uint32_t *out, void *stream) {
  if (int st = check_layout("arg_reduce", input_len, rank, shape, offset, strides)) return st;
  if (axis >= rank) return fail(TC_EINVAL, "arg_reduce: axis %u of a rank-%u shape", axis, rank);
  if (op != TC_RMIN && op != TC_RMAX) return fail(TC_EINVAL, "arg_reduce: op must be Min or Max");
  if (shape[axis] == 0) return fail(TC_EINVAL, "arg_reduce: axis %u is empty", axis);
  if (shape[axis] > 0xffffffffull) return fail(TC_EINVAL, "arg_reduce: axis longer than a u32 index reaches");
  if (element_count(rank, shape) == 0) return TC_OK;
  if (!input || !out) return fail(TC_EINVAL, "arg_reduce: null pointer");
  bool folded[TC_MAX_RANK] = {false};
  folded[axis] = true;
  return run_reduction(dtype, rank, shape, input, offset, strides, folded, op == TC_RMAX ? M_ARGMAX : M_ARGMIN, 0,
                       nullptr, out, as_stream(stream));
}

int tc_vector_reduce(int dtype, int op, const void *a, size_t n, void *out, void *stream) {
  if (op < TC_SUM || op > TC_RMAX) return fail(TC_EINVAL, "vector_reduce: bad Reduce %d", op);
  if (n && !a) return fail(TC_EINVAL, "vector_reduce: null input");
  if (op == TC_SUM) return vector_fold<M_SUM>(dtype, a, nullptr, n, out, as_stream(stream));
  if (op == TC_RMIN) return vector_fold<M_MIN>(dtype, a, nullptr, n, out, as_stream(stream));
  return vector_fold<M_MAX>(dtype, a, nullptr, n, out, as_stream(stream));
}

int tc_dot(int dtype, const void *a, const void *b, size_t n, void *out, void *stream) {
  if (n && (!a || !b)) return fail(TC_EINVAL, "dot: null input");
  return vector_fold<M_SUM>(dtype, a, b, n, out, as_stream(stream));
}

}  // extern "C"
