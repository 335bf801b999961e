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
//  - rows: the folded space ends in a contiguous run (the innermost folded
//    axis has stride 1).  A warp (short slices) or a 256-thread block (long
//    ones) per result, 128-bit loads along the run.  A variance whose slice
//    fits in registers is computed from them in both passes, so the input
//    is read from HBM once.
//  - columns: the innermost kept axis has stride 1 (results side by side in
//    memory).  Each thread owns one result and a share of the folded range;
//    neighbouring threads read neighbouring addresses, so each folded step
//    is a coalesced row read.  The shares combine in shared memory.
//  - walk: anything else; a warp per result over the decomposed folded
//    index.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace tc {
namespace {

enum Mode { FOLD_SUM = 0, FOLD_MIN = 1, FOLD_MAX = 2, MEAN = 3, VARIANCE = 4, ARG_MIN = 5, ARG_MAX = 6 };

// ---- accumulators ---------------------------------------------------------
struct Acc {
  float v;
  uint32_t i;  // position (arg-reductions only)
};

__device__ __forceinline__ Acc identity(int mode) {
  switch (mode) {
    case FOLD_MIN: return {INFINITY, 0};
    case FOLD_MAX: return {-INFINITY, 0};
    case ARG_MIN:
    case ARG_MAX: return {__int_as_float(0x7fc00000), 0};
    default: return {0.0f, 0};
  }
}

// Fold one more element (at position `pos` along an arg-reduction's axis).
__device__ __forceinline__ void push(int mode, Acc &a, float x, uint32_t pos) {
  switch (mode) {
    case FOLD_MIN: a.v = fminf(a.v, x); break;
    case FOLD_MAX: a.v = fmaxf(a.v, x); break;
    case ARG_MIN:
      // strided.rs:188-198 `replaces`: a number, and best is NaN or x is past it
      if (!isnan(x) && (isnan(a.v) || x < a.v)) { a.v = x; a.i = pos; }
      break;
    case ARG_MAX:
      if (!isnan(x) && (isnan(a.v) || x > a.v)) { a.v = x; a.i = pos; }
      break;
    default: a.v = __fadd_rn(a.v, x); break;
  }
}

// Combine two partial results; for an arg-reduction the lower position wins
// a tie, which is the first position overall.
__device__ __forceinline__ Acc merge(int mode, Acc a, Acc b) {
  switch (mode) {
    case FOLD_MIN: return {fminf(a.v, b.v), 0};
    case FOLD_MAX: return {fmaxf(a.v, b.v), 0};
    case ARG_MIN:
    case ARG_MAX: {
      if (isnan(b.v)) return a;
      if (isnan(a.v)) return b;
      bool better = mode == ARG_MAX ? b.v > a.v : b.v < a.v;
      if (better || (b.v == a.v && b.i < a.i)) return b;
      return a;
    }
    default: return {__fadd_rn(a.v, b.v), 0};
  }
}

__device__ __forceinline__ Acc warp_merge(int mode, Acc a) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Acc b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, d);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, d);
    a = merge(mode, a, b);
  }
  return a;
}

// Merge across a block of `nwarps` warps: every thread gets the result.
__device__ __forceinline__ Acc block_merge(int mode, Acc a, Acc *scratch) {
  a = warp_merge(mode, a);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = a;
  __syncthreads();
  Acc r = scratch[0];
  for (int w = 1; w < nwarps; ++w) r = merge(mode, r, scratch[w]);
  return r;
}

// Finish one result: Mean divides, everything else is already final.
__device__ __forceinline__ float finish(int mode, float total, float count) {
  return mode == MEAN ? __fdiv_rn(total, count) : total;
}

// The kept walk gives each result's base offset; the folded walk (outer
// axes) gives each run's offset within the slice.
struct Layout2 {
  Walk kept;    // operand 0: input strides; rank 0 = one result
  Walk folded;  // operand 0: input strides of the folded axes except the run
};

// Storage position of flat index `r` of a one-operand walk; rank 0 and 1
// (the common cases) skip the division.
__device__ __forceinline__ long long kept_base(const Walk &w, long long r) {
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

// ---------------------------------------------------------------------------
// rows: G threads per result (G = 32: a warp; G = blockDim: the block).
// The slice is `outer` runs of `run` contiguous elements.
// ---------------------------------------------------------------------------
constexpr int CACHE_PACKS = 8;

template <class T, bool BLOCK>
__global__ void __launch_bounds__(256, 2) reduce_rows(const typename T::S *in, Layout2 L, long long results,
                                                   long long outer, long long run, int mode, float count,
                                                   float divisor, typename T::S *out, uint32_t *arg_out,
                                                   bool vec) {
  using S = typename T::S;
  constexpr int N = Pack<T>::N;
  __shared__ Acc scratch[32];
  const int G = BLOCK ? blockDim.x : 32;
  const int lane = BLOCK ? threadIdx.x : (threadIdx.x & 31);
  const long long groups_per_block = BLOCK ? 1 : (blockDim.x >> 5);
  const long long group0 = (long long)blockIdx.x * groups_per_block + (BLOCK ? 0 : (threadIdx.x >> 5));
  const long long group_stride = (long long)gridDim.x * groups_per_block;
  const int fold_mode = (mode == MEAN || mode == VARIANCE) ? FOLD_SUM : mode;
  const bool cache = mode == VARIANCE && vec && outer == 1 && run <= (long long)G * N * CACHE_PACKS;

  for (long long r = group0; r < results; r += group_stride) {
    const S *base = in + kept_base(L.kept, r);
    Acc a = identity(fold_mode);
    Pack<T> cached[CACHE_PACKS];  // the slice, still in its storage form
    if (cache) {
      // Pass one from memory into registers: all loads first, then the sum.
#pragma unroll
      for (int k = 0; k < CACHE_PACKS; ++k) {
        long long p = (long long)k * G + lane;
        if (p * N < run) cached[k].raw = __ldg(reinterpret_cast<const uint4 *>(base + p * N));
      }
#pragma unroll
      for (int k = 0; k < CACHE_PACKS; ++k) {
        long long p = (long long)k * G + lane;
        if (p * N < run) {
#pragma unroll
          for (int j = 0; j < N; ++j) a.v = __fadd_rn(a.v, T::load(cached[k].v[j]));
        }
      }
    } else {
      // The slice as one flat run of units (packs when vectorised, else
      // elements): `outer` runs of `per_run` units.  U independent loads are
      // issued before any is folded, so each thread keeps U requests in
      // flight.
      constexpr int U = 8;
      const long long per_run = vec ? run / N : run;
      const long long total = outer * per_run;
      for (long long f0 = lane; f0 < total; f0 += (long long)G * U) {
        if (vec) {
          Pack<T> x[U];
          long long at[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            long long f = f0 + (long long)u * G;
            if (f < total) {
              long long o = outer > 1 ? f / per_run : 0, c = f - o * per_run;
              at[u] = c * N;
              x[u].raw = __ldg(reinterpret_cast<const uint4 *>(base + (outer > 1 ? kept_base(L.folded, o) : 0) + c * N));
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            if (f0 + (long long)u * G < total) {
#pragma unroll
              for (int j = 0; j < N; ++j) push(fold_mode, a, T::load(x[u].v[j]), uint32_t(at[u] + j));
            }
          }
        } else {
          float x[U];
          long long at[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            long long f = f0 + (long long)u * G;
            if (f < total) {
              long long o = outer > 1 ? f / per_run : 0, c = f - o * per_run;
              at[u] = c;
              x[u] = T::load(base[(outer > 1 ? kept_base(L.folded, o) : 0) + c]);
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (f0 + (long long)u * G < total) push(fold_mode, a, x[u], uint32_t(at[u]));
        }
      }
    }
    a = BLOCK ? block_merge(fold_mode, a, scratch) : warp_merge(fold_mode, a);
    float result;
    if (mode == VARIANCE) {
      float mean = __fdiv_rn(a.v, count);
      Acc d = identity(FOLD_SUM);
      if (cache) {
#pragma unroll
        for (int k = 0; k < CACHE_PACKS; ++k) {
          long long p = (long long)k * G + lane;
          if (p * N < run) {
#pragma unroll
            for (int j = 0; j < N; ++j) {
              float dev = __fsub_rn(T::load(cached[k].v[j]), mean);
              d.v = __fadd_rn(d.v, __fmul_rn(dev, dev));
            }
          }
        }
      } else {
        for (long long o = 0; o < outer; ++o) {
          const S *rp = base + (outer > 1 ? kept_base(L.folded, o) : 0);
          for (long long c = lane; c < run; c += G) {
            float dev = __fsub_rn(T::load(rp[c]), mean);
            d.v = __fadd_rn(d.v, __fmul_rn(dev, dev));
          }
        }
      }
      d = BLOCK ? block_merge(FOLD_SUM, d, scratch) : warp_merge(FOLD_SUM, d);
      result = __fdiv_rn(d.v, divisor);
    } else {
      result = finish(mode, a.v, count);
    }
    if (lane == 0) {
      if (mode >= ARG_MIN) arg_out[r] = a.i;
      else out[r] = T::store(result);
    }
    if (BLOCK) __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// columns: results r = (outer kept index) * K + k with k along the kept axis
// of stride 1.  blockDim = (32, Y): x walks 32*CPT adjacent results (CPT per
// thread, one vector load each), y splits the folded range into Y shares
// that combine in shared memory in share order.
// ---------------------------------------------------------------------------
template <class T, int CPT> struct Cols {
  using S = typename T::S;
  union { typename std::conditional<CPT * sizeof(S) == 16, uint4, typename std::conditional<CPT * sizeof(S) == 8, uint2, S>::type>::type raw; S v[CPT]; };
};

template <class T, int CPT>
__global__ void __launch_bounds__(256) reduce_cols(const typename T::S *in, Layout2 L, long long kept_outer,
                                                   long long K, long long depth, int mode, float count,
                                                   float divisor, typename T::S *out, uint32_t *arg_out) {
  using S = typename T::S;
  using V = Cols<T, CPT>;
  constexpr int W = 32 * CPT;
  constexpr int U = 8;
  __shared__ Acc part[8][W];
  const int Y = blockDim.y;
  const int fold_mode = (mode == MEAN || mode == VARIANCE) ? FOLD_SUM : mode;
  const long long tiles_k = (K + W - 1) / W;
  const long long tiles = kept_outer * tiles_k;
  const long long share = (depth + Y - 1) / Y;
  const long long f0 = (long long)threadIdx.y * share, f1 = min(depth, f0 + share);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const long long ko = t / tiles_k;
    const long long k = (t - ko * tiles_k) * W + (long long)threadIdx.x * CPT;
    const bool live = k < K;  // CPT divides K when CPT > 1
    const S *base = in + kept_base(L.kept, ko) + (live ? k : 0);
    Acc a[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) a[c] = identity(fold_mode);
    if (live) {
      for (long long f = f0; f < f1; f += U) {
        V x[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (f + u < f1) x[u].raw = __ldg(reinterpret_cast<const decltype(V::raw) *>(base + kept_base(L.folded, f + u)));
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (f + u < f1) {
#pragma unroll
            for (int c = 0; c < CPT; ++c) push(fold_mode, a[c], T::load(x[u].v[c]), uint32_t(f + u));
          }
      }
    }
    float result[CPT];
    Acc total[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) part[threadIdx.y][threadIdx.x * CPT + c] = a[c];
    __syncthreads();
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      total[c] = part[0][threadIdx.x * CPT + c];
      for (int y = 1; y < Y; ++y) total[c] = merge(fold_mode, total[c], part[y][threadIdx.x * CPT + c]);
    }
    __syncthreads();
    if (mode == VARIANCE) {
      float mean[CPT];
      Acc d[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        mean[c] = __fdiv_rn(total[c].v, count);
        d[c] = identity(FOLD_SUM);
      }
      if (live)
        for (long long f = f0; f < f1; ++f) {
          V x;
          x.raw = __ldg(reinterpret_cast<const decltype(V::raw) *>(base + kept_base(L.folded, f)));
#pragma unroll
          for (int c = 0; c < CPT; ++c) {
            float dev = __fsub_rn(T::load(x.v[c]), mean[c]);
            d[c].v = __fadd_rn(d[c].v, __fmul_rn(dev, dev));
          }
        }
#pragma unroll
      for (int c = 0; c < CPT; ++c) part[threadIdx.y][threadIdx.x * CPT + c] = d[c];
      __syncthreads();
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        Acc dt = part[0][threadIdx.x * CPT + c];
        for (int y = 1; y < Y; ++y) dt = merge(FOLD_SUM, dt, part[y][threadIdx.x * CPT + c]);
        result[c] = __fdiv_rn(dt.v, divisor);
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int c = 0; c < CPT; ++c) result[c] = finish(mode, total[c].v, count);
    }
    if (live && threadIdx.y == 0) {
      long long r = ko * K + k;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        if (mode >= ARG_MIN) arg_out[r + c] = total[c].i;
        else out[r + c] = T::store(result[c]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// walk: a warp per result over the decomposed folded index.
// ---------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(256) reduce_walk(const typename T::S *in, Layout2 L, long long results,
                                                   long long depth, int mode, float count, float divisor,
                                                   typename T::S *out, uint32_t *arg_out) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int fold_mode = (mode == MEAN || mode == VARIANCE) ? FOLD_SUM : mode;
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < results; r += warps) {
    long long base = kept_base(L.kept, r);
    Acc a = identity(fold_mode);
    for (long long f = lane; f < depth; f += 32) {
      push(fold_mode, a, T::load(in[base + kept_base(L.folded, f)]), uint32_t(f));
    }
    a = warp_merge(fold_mode, a);
    float result;
    if (mode == VARIANCE) {
      float mean = __fdiv_rn(a.v, count);
      Acc d = identity(FOLD_SUM);
      for (long long f = lane; f < depth; f += 32) {
        float dev = __fsub_rn(T::load(in[base + kept_base(L.folded, f)]), mean);
        d.v = __fadd_rn(d.v, __fmul_rn(dev, dev));
      }
      d = warp_merge(FOLD_SUM, d);
      result = __fdiv_rn(d.v, divisor);
    } else {
      result = finish(mode, a.v, count);
    }
    if (lane == 0) {
      if (mode >= ARG_MIN) arg_out[r] = a.i;
      else out[r] = T::store(result);
    }
  }
}

void fill_walk(Walk &w, const Dims &shape, const Dims &strides, long long offset) {
  w.rank = int(shape.rank);
  w.offset[0] = offset;
  for (uint32_t a = 0; a < shape.rank; ++a) {
    w.shape[a] = (long long)shape.v[a];
    w.stride[0][a] = (long long)strides.v[a];
  }
}

// The shared driver of reduce_axes and arg_reduce.
int run_reduction(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t offset,
                  const size_t *strides, const bool *folded, int mode, size_t divisor, void *out,
                  uint32_t *arg_out, cudaStream_t stream) {
  // Split, strided.rs / layout.rs:370-414.
  size_t ks[TC_MAX_RANK], kst[TC_MAX_RANK], fs[TC_MAX_RANK], fst[TC_MAX_RANK];
  uint32_t nk = 0, nf = 0;
  for (uint32_t a = 0; a < rank; ++a) {
    if (folded[a]) { fs[nf] = shape[a]; fst[nf++] = strides[a]; }
    else { ks[nk] = shape[a]; kst[nk++] = strides[a]; }
  }
  size_t results = element_count(nk, ks), depth = element_count(nf, fs);
  if (results == 0) return TC_OK;
  if (depth == 0) return fail(TC_EINVAL, "reduction over an empty slice");
  // Kept axes: coalesce input strides against the contiguous result
  // strides, so results stay in row-major order.
  size_t kout[TC_MAX_RANK];
  contiguous_strides(nk, ks, kout);
  const size_t *kops[2] = {kst, kout};
  Dims kc, kcs[2];
  coalesce<2>(nk, ks, kops, kc, kcs);
  const size_t *fops[1] = {fst};
  Dims fc, fcs[1];
  coalesce<1>(nf, fs, fops, fc, fcs);
  // An arg-reduction's position is the coordinate along its one axis; its
  // folded space is that axis alone (coalesce keeps it one axis).
  const float count = float(depth), div = float(double(divisor));

  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    using S = typename T::S;
    const S *in = static_cast<const S *>(input) + offset;
    S *o = static_cast<S *>(out);
    Layout2 L{};
    fill_walk(L.kept, kc, kcs[0], 0);

    // rows: innermost folded axis contiguous.
    if (fc.rank >= 1 && fcs[0].v[fc.rank - 1] == 1 && !(kc.rank && kcs[0].v[kc.rank - 1] == 1 && fc.v[fc.rank - 1] < 64)) {
      long long run = (long long)fc.v[fc.rank - 1];
      Dims fo = fc, fos = fcs[0];
      fo.rank = fos.rank = fc.rank - 1;
      long long outer = (long long)element_count(fo.rank, fo.v);
      fill_walk(L.folded, fo, fos, 0);
      constexpr int N = Pack<T>::N;
      bool vec = run % N == 0 && (uintptr_t(in) & 15u) == 0;
      for (uint32_t a = 0; vec && a < kc.rank; ++a) vec = kcs[0].v[a] % N == 0;
      for (uint32_t a = 0; vec && a < fo.rank; ++a) vec = fos.v[a] % N == 0;
      long long warps_total = (long long)sm_count() * 64;  // resident warps
      if ((long long)results >= warps_total / 2 || (long long)depth <= 4096) {
        unsigned grid = unsigned(std::min<long long>(((long long)results + 7) / 8, (long long)sm_count() * 8));
        reduce_rows<T, false><<<std::max(1u, grid), 256, 0, stream>>>(in, L, (long long)results, outer, run, mode,
                                                                      count, div, o, arg_out, vec);
      } else {
        unsigned grid = unsigned(std::min<long long>((long long)results, (long long)sm_count() * 8));
        reduce_rows<T, true><<<std::max(1u, grid), 256, 0, stream>>>(in, L, (long long)results, outer, run, mode,
                                                                     count, div, o, arg_out, vec);
      }
      return check_launch("reduce (rows)");
    }
    // columns: innermost kept axis contiguous.
    if (kc.rank >= 1 && kcs[0].v[kc.rank - 1] == 1) {
      long long K = (long long)kc.v[kc.rank - 1];
      Dims ko = kc, kos = kcs[0];
      ko.rank = kos.rank = kc.rank - 1;
      long long kept_outer = (long long)element_count(ko.rank, ko.v);
      fill_walk(L.kept, ko, kos, 0);
      fill_walk(L.folded, fc, fcs[0], 0);
      // Four results per thread when every row of them starts 4-aligned.
      bool four = K % 4 == 0 && (uintptr_t(in) % (4 * sizeof(S))) == 0;
      for (uint32_t a = 0; four && a < ko.rank; ++a) four = kos.v[a] % 4 == 0;
      for (uint32_t a = 0; four && a < fc.rank; ++a) four = fcs[0].v[a] % 4 == 0;
      const int cpt = four ? 4 : 1;
      long long tiles = kept_outer * ((K + 32 * cpt - 1) / (32 * cpt));
      int Y = 8;
      unsigned grid = unsigned(std::min<long long>(tiles, (long long)sm_count() * 8));
      if (four)
        reduce_cols<T, 4><<<std::max(1u, grid), dim3(32, Y), 0, stream>>>(in, L, kept_outer, K, (long long)depth,
                                                                           mode, count, div, o, arg_out);
      else
        reduce_cols<T, 1><<<std::max(1u, grid), dim3(32, Y), 0, stream>>>(in, L, kept_outer, K, (long long)depth,
                                                                           mode, count, div, o, arg_out);
      return check_launch("reduce (columns)");
    }
    fill_walk(L.folded, fc, fcs[0], 0);
    unsigned grid = unsigned(std::min<long long>(((long long)results + 7) / 8, (long long)sm_count() * 8));
    reduce_walk<T><<<std::max(1u, grid), 256, 0, stream>>>(in, L, (long long)results, (long long)depth, mode,
                                                            count, div, o, arg_out);
    return check_launch("reduce (walk)");
  });
}

// Whole-vector fold / dot: per-block partials, then one block folds them.
template <class T>
__global__ void __launch_bounds__(256) vector_partials(const typename T::S *a, const typename T::S *b, size_t n,
                                                       int mode, float *partials) {
  __shared__ Acc scratch[32];
  Acc acc = identity(mode);
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    float x = T::load(a[i]);
    if (b) x = __fmul_rn(x, T::load(b[i]));
    push(mode, acc, x, 0);
  }
  acc = block_merge(mode, acc, scratch);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc.v;
}
template <class T>
__global__ void __launch_bounds__(256) vector_finish(const float *partials, int count, int mode,
                                                     typename T::S *out) {
  __shared__ Acc scratch[32];
  Acc acc = identity(mode);
  for (int i = threadIdx.x; i < count; i += blockDim.x) push(mode, acc, partials[i], 0);
  acc = block_merge(mode, acc, scratch);
  if (threadIdx.x == 0) out[0] = T::store(acc.v);
}

int vector_fold(int dtype, int mode, const void *a, const void *b, size_t n, void *out, cudaStream_t stream) {
  if (!out) return fail(TC_EINVAL, "vector reduce: null output");
  const int max_blocks = 1024;
  static thread_local float *partials[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(TC_EINVAL, "device %d", dev);
  if (!partials[dev]) {
    if (int st = check_cuda(cudaMalloc(&partials[dev], max_blocks * sizeof(float)), "cudaMalloc")) return st;
  }
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    using S = typename T::S;
    int blocks = int(std::min<size_t>(std::max<size_t>((n + 255) / 256, 1), size_t(max_blocks)));
    vector_partials<T><<<blocks, 256, 0, stream>>>(static_cast<const S *>(a), static_cast<const S *>(b), n, mode,
                                                    partials[dev]);
    vector_finish<T><<<1, 256, 0, stream>>>(partials[dev], blocks, mode, static_cast<S *>(out));
    return check_launch("vector reduce");
  });
}

}  // namespace
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
    mode = op == TC_SUM ? FOLD_SUM : (op == TC_RMIN ? FOLD_MIN : FOLD_MAX);
  } else if (kind == TC_AXIS_MEAN) {
    mode = MEAN;
  } else if (kind == TC_AXIS_VARIANCE) {
    mode = VARIANCE;
  } else {
    return fail(TC_EINVAL, "reduce_axes: bad AxisReduction %d", kind);
  }
  if (element_count(rank, shape) == 0) {
    // Every result folds an empty slice: the front-end never asks; a
    // non-empty result set over an empty slice is an error.
    size_t results = 1;
    for (uint32_t a = 0; a < rank; ++a) if (!folded[a]) results *= shape[a];
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
  // A size-1 axis is dropped by coalescing; its answer is 0 everywhere.
  return run_reduction(dtype, rank, shape, input, offset, strides, folded, op == TC_RMAX ? ARG_MAX : ARG_MIN, 0,
                       nullptr, out, as_stream(stream));
}

int tc_vector_reduce(int dtype, int op, const void *a, size_t n, void *out, void *stream) {
  if (op < TC_SUM || op > TC_RMAX) return fail(TC_EINVAL, "vector_reduce: bad Reduce %d", op);
  if (n && !a) return fail(TC_EINVAL, "vector_reduce: null input");
  int mode = op == TC_SUM ? FOLD_SUM : (op == TC_RMIN ? FOLD_MIN : FOLD_MAX);
  return vector_fold(dtype, mode, a, nullptr, n, out, as_stream(stream));
}

int tc_dot(int dtype, const void *a, const void *b, size_t n, void *out, void *stream) {
  if (n && (!a || !b)) return fail(TC_EINVAL, "dot: null input");
  return vector_fold(dtype, FOLD_SUM, a, b, n, out, as_stream(stream));
}

}  // extern "C"
