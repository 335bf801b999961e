// window.cu — the windowed matrix methods of Kernels<T>: valid correlation
// and its two gradients (correlate, correlate_window_gradient,
// correlate_input_gradient, kernels.rs:998-1023), pad and flip
// (kernels.rs:1025-1028).
//
// Correlation follows the Host's loops (kernels.rs:1720-1788): each output
// is a sum over the window's taps in row-major tap order, `sum = sum + x*k`
// with the product and the sum each rounded (Rust does not contract), in
// f32 for f16/bf16 (widened exactly, the output rounded once).  A thread
// that owns an output and walks the taps in that order with __fmul_rn /
// __fadd_rn reproduces the Host's bits.  When the taps are many and the
// outputs few (the window gradient, whose "window" is the whole adjoint),
// a block shares one output instead: each thread sums its own stride of
// the taps in order and the partial sums meet in a fixed tree, which keeps
// the result deterministic but rounds within a sum's bound of the Host's.
#include <algorithm>

#include "common.cuh"

namespace tc {
namespace {

struct Window {
  long long in_rows, in_cols;    // the input read (correlate) or the adjoint (input gradient)
  long long win_rows, win_cols;  // the taps
  long long out_rows, out_cols;
  bool flip;
};

// The tap (wr, wc) of the sum, flipped or not, as the Host indexes it.
__device__ __forceinline__ long long tap_index(const Window &w, long long wr, long long wc) {
  return w.flip ? (w.win_rows - 1 - wr) * w.win_cols + (w.win_cols - 1 - wc) : wr * w.win_cols + wc;
}

// OUTS adjacent outputs of a row per thread, each summing its taps in the
// Host's order: for each window row the thread slides a register window of
// OUTS input values along the row, so a tap costs one input load and one
// (shared-memory, broadcast) tap read for OUTS products.  The taps are
// staged in shared memory when they fit (SMEM_TAPS), else read through L1.
constexpr int OUTS = 8, SMEM_TAPS = 4096;

template <class T>
__global__ void __launch_bounds__(256) correlate_direct(const typename T::S *in, const typename T::S *win,
                                                        typename T::S *out, Window w) {
  __shared__ float taps_sh[SMEM_TAPS];
  const long long taps = w.win_rows * w.win_cols;
  const bool staged = taps <= SMEM_TAPS;
  if (staged)
    for (long long t = threadIdx.x; t < taps; t += blockDim.x) taps_sh[t] = T::load(win[t]);
  __syncthreads();
  const long long groups = (w.out_cols + OUTS - 1) / OUTS, total = w.out_rows * groups;
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
       o += (long long)gridDim.x * blockDim.x) {
    const long long row = o / groups, c0 = (o - row * groups) * OUTS;
    const int n = int(min((long long)OUTS, w.out_cols - c0));
    float sum[OUTS];
#pragma unroll
    for (int j = 0; j < OUTS; ++j) sum[j] = 0.0f;
    for (long long wr = 0; wr < w.win_rows; ++wr) {
      const typename T::S *x = in + (row + wr) * w.in_cols + c0;
      const long long room = w.in_cols - c0;  // readable elements from x
      float v[OUTS];
#pragma unroll
      for (int j = 0; j < OUTS - 1; ++j) v[j] = j < room ? T::load(__ldg(x + j)) : 0.0f;
      for (long long wc = 0; wc < w.win_cols; ++wc) {
        v[OUTS - 1] = wc + OUTS - 1 < room ? T::load(__ldg(x + wc + OUTS - 1)) : 0.0f;
        const long long ti = tap_index(w, wr, wc);
        const float k = staged ? taps_sh[ti] : T::load(__ldg(win + ti));
#pragma unroll
        for (int j = 0; j < OUTS; ++j)
          if (j < n) sum[j] = __fadd_rn(sum[j], __fmul_rn(v[j], k));
#pragma unroll
        for (int j = 0; j < OUTS - 1; ++j) v[j] = v[j + 1];
      }
    }
#pragma unroll
    for (int j = 0; j < OUTS; ++j)
      if (j < n) out[row * w.out_cols + c0 + j] = T::store(sum[j]);
  }
}

// One block per output: thread t sums taps t, t+B, t+2B, ... in order; the
// partial sums meet in a fixed tree.
template <class T>
__global__ void __launch_bounds__(256) correlate_shared(const typename T::S *in, const typename T::S *win,
                                                        typename T::S *out, Window w) {
  __shared__ float part[8];
  const long long taps = w.win_rows * w.win_cols;
  for (long long o = blockIdx.x; o < w.out_rows * w.out_cols; o += gridDim.x) {
    const long long row = o / w.out_cols, col = o - row * w.out_cols;
    float sum = 0.0f;
    for (long long t = threadIdx.x; t < taps; t += blockDim.x) {
      const long long wr = t / w.win_cols, wc = t - wr * w.win_cols;
      sum = __fadd_rn(sum, __fmul_rn(T::load(__ldg(in + (row + wr) * w.in_cols + col + wc)),
                                     T::load(__ldg(win + tap_index(w, wr, wc)))));
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, d));
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = part[0];
      for (int k = 1; k < int(blockDim.x >> 5); ++k) s = __fadd_rn(s, part[k]);
      out[o] = T::store(s);
    }
    __syncthreads();
  }
}

// The input gradient (kernels.rs:1754-1788): output (p, q) sums adjoint
// (p-u, q-v) times tap (u, v) over the taps whose adjoint index is in range,
// in tap order, skipping the rest (they are not added as zeros).  OUTS
// adjacent outputs of a row per thread: for each window row the thread
// slides a register window of adjoint values (column q-v) leftwards as v
// grows, and each output adds a tap only where its column is in range.
template <class T>
__global__ void __launch_bounds__(256) correlate_input_gradient_direct(const typename T::S *adj,
                                                                       const typename T::S *win, typename T::S *out,
                                                                       Window w) {
  __shared__ float taps_sh[SMEM_TAPS];
  const long long taps = w.win_rows * w.win_cols;
  const bool staged = taps <= SMEM_TAPS;
  if (staged)
    for (long long t = threadIdx.x; t < taps; t += blockDim.x) taps_sh[t] = T::load(win[t]);
  __syncthreads();
  const long long groups = (w.out_cols + OUTS - 1) / OUTS, total = w.out_rows * groups;
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
       o += (long long)gridDim.x * blockDim.x) {
    const long long row = o / groups, c0 = (o - row * groups) * OUTS;
    const int n = int(min((long long)OUTS, w.out_cols - c0));
    float sum[OUTS];
#pragma unroll
    for (int j = 0; j < OUTS; ++j) sum[j] = 0.0f;
    const long long wr0 = max(0LL, row - (w.in_rows - 1)), wr1 = min(w.win_rows - 1, row);
    for (long long wr = wr0; wr <= wr1; ++wr) {
      const typename T::S *a = adj + (row - wr) * w.in_cols;
      // v[j] holds the adjoint at column c0 + j - wc (0 outside the row)
      auto at = [&](long long col) { return col >= 0 && col < w.in_cols ? T::load(__ldg(a + col)) : 0.0f; };
      float v[OUTS];
#pragma unroll
      for (int j = 1; j < OUTS; ++j) v[j] = at(c0 + j);
      for (long long wc = 0; wc < w.win_cols; ++wc) {
#pragma unroll
        for (int j = OUTS - 1; j > 0; --j) v[j] = wc ? v[j - 1] : v[j];
        v[0] = at(c0 - wc);
        const long long ti = tap_index(w, wr, wc);
        const float k = staged ? taps_sh[ti] : T::load(__ldg(win + ti));
#pragma unroll
        for (int j = 0; j < OUTS; ++j) {
          const long long col = c0 + j - wc;
          if (j < n && col >= 0 && col < w.in_cols) sum[j] = __fadd_rn(sum[j], __fmul_rn(v[j], k));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < OUTS; ++j)
      if (j < n) out[row * w.out_cols + c0 + j] = T::store(sum[j]);
  }
}

// Windows at most NARROW taps wide, the width WC a compile-time constant:
// the same sums in the same order as the kernels above, with the tap loop
// unrolled (no index arithmetic, no register shifts), the taps staged
// already flipped where the sum flips them (tap (wr, wc) of a flipped sum is
// staged tap taps-1-(wr·WC+wc)), and each window row's input values for a
// group loaded at once, four to a vector load when the rows are aligned.
constexpr int NARROW = 8;

// Four values of storage type S from a 16-byte (f32) or 8-byte (16-bit)
// aligned address.
template <class T> __device__ __forceinline__ void load4(const typename T::S *x, float *v) {
  if constexpr (sizeof(typename T::S) == 4) {
    const float4 q = __ldg(reinterpret_cast<const float4 *>(x));
    v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
  } else {
    const uint2 q = __ldg(reinterpret_cast<const uint2 *>(x));
    v[0] = T::load(uint16_t(q.x)), v[1] = T::load(uint16_t(q.x >> 16));
    v[2] = T::load(uint16_t(q.y)), v[3] = T::load(uint16_t(q.y >> 16));
  }
}

template <class T> __device__ __forceinline__ void stage_taps(const typename T::S *win, const Window &w, int wc,
                                                              float *taps_sh) {
  const int taps = int(w.win_rows) * wc;
  for (int t = threadIdx.x; t < taps; t += blockDim.x) taps_sh[t] = T::load(win[w.flip ? taps - 1 - t : t]);
  __syncthreads();
}

// Output (row, c0 + j) sums in(row + wr, c0 + j + wc) · tap(wr, wc); `vec`:
// rows start on the vector boundary (in_cols a multiple of 4, `in` aligned).
template <class T, int WC>
__global__ void __launch_bounds__(256) correlate_narrow(const typename T::S *in, const typename T::S *win,
                                                        typename T::S *out, Window w, bool vec) {
  __shared__ float taps_sh[SMEM_TAPS];
  stage_taps<T>(win, w, WC, taps_sh);
  constexpr int NV = (OUTS + WC - 1 + 3) / 4 * 4;  // values a group reads per window row, whole vectors
  const long long groups = (w.out_cols + OUTS - 1) / OUTS, total = w.out_rows * groups;
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
       o += (long long)gridDim.x * blockDim.x) {
    const long long row = o / groups, c0 = (o - row * groups) * OUTS;
    const int n = int(min((long long)OUTS, w.out_cols - c0));
    const bool fast = vec && n == OUTS && c0 + NV <= w.in_cols;
    float sum[OUTS];
#pragma unroll
    for (int j = 0; j < OUTS; ++j) sum[j] = 0.0f;
    for (long long wr = 0; wr < w.win_rows; ++wr) {
      const typename T::S *x = in + (row + wr) * w.in_cols + c0;
      float v[NV];
      if (fast) {
#pragma unroll
        for (int q = 0; q < NV / 4; ++q) load4<T>(x + 4 * q, v + 4 * q);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] = c0 + j < w.in_cols ? T::load(__ldg(x + j)) : 0.0f;
      }
      const float *k = taps_sh + wr * WC;
#pragma unroll
      for (int wc = 0; wc < WC; ++wc) {
        const float kk = k[wc];
#pragma unroll
        for (int j = 0; j < OUTS; ++j) sum[j] = __fadd_rn(sum[j], __fmul_rn(v[j + wc], kk));
      }
    }
#pragma unroll
    for (int j = 0; j < OUTS; ++j)
      if (j < n) out[row * w.out_cols + c0 + j] = T::store(sum[j]);
  }
}

// The input gradient for windows at most NARROW wide: output (row, c0 + j)
// sums adj(row - wr, c0 + j - wc) · tap(wr, wc) over the taps in order,
// skipping the taps whose adjoint column is outside the row (the fast path
// takes only groups whose columns are all inside: nothing to skip).
template <class T, int WC>
__global__ void __launch_bounds__(256) correlate_input_gradient_narrow(const typename T::S *adj,
                                                                       const typename T::S *win, typename T::S *out,
                                                                       Window w, bool vec) {
  __shared__ float taps_sh[SMEM_TAPS];
  stage_taps<T>(win, w, WC, taps_sh);
  // a group reads adjoint columns c0-(WC-1) .. c0+OUTS-1; loaded from c0-LEAD
  // (a vector boundary), the column c0 + j - wc sits at b[j - wc + LEAD]
  constexpr int LEAD = (WC - 1 + 3) / 4 * 4, NB = (LEAD + OUTS + 3) / 4 * 4, NV = OUTS + WC - 1;
  const long long groups = (w.out_cols + OUTS - 1) / OUTS, total = w.out_rows * groups;
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
       o += (long long)gridDim.x * blockDim.x) {
    const long long row = o / groups, c0 = (o - row * groups) * OUTS;
    const int n = int(min((long long)OUTS, w.out_cols - c0));
    const long long a0 = c0 - LEAD;
    const bool fast = vec && n == OUTS && a0 >= 0 && a0 + NB <= w.in_cols;
    float sum[OUTS];
#pragma unroll
    for (int j = 0; j < OUTS; ++j) sum[j] = 0.0f;
    const long long wr0 = max(0LL, row - (w.in_rows - 1)), wr1 = min(w.win_rows - 1, row);
    for (long long wr = wr0; wr <= wr1; ++wr) {
      const typename T::S *a = adj + (row - wr) * w.in_cols;
      const float *k = taps_sh + wr * WC;
      if (fast) {
        float b[NB];
#pragma unroll
        for (int q = 0; q < NB / 4; ++q) load4<T>(a + a0 + 4 * q, b + 4 * q);
#pragma unroll
        for (int wc = 0; wc < WC; ++wc) {
          const float kk = k[wc];
#pragma unroll
          for (int j = 0; j < OUTS; ++j) sum[j] = __fadd_rn(sum[j], __fmul_rn(b[j - wc + LEAD], kk));
        }
      } else {
        // b[i] holds column c0 - (WC-1) + i (0 outside the row, never added)
        float b[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const long long col = c0 - (WC - 1) + i;
          b[i] = col >= 0 && col < w.in_cols ? T::load(__ldg(a + col)) : 0.0f;
        }
#pragma unroll
        for (int wc = 0; wc < WC; ++wc) {
          const float kk = k[wc];
#pragma unroll
          for (int j = 0; j < OUTS; ++j) {
            const long long col = c0 + j - wc;
            if (j < n && col >= 0 && col < w.in_cols) sum[j] = __fadd_rn(sum[j], __fmul_rn(b[j - wc + WC - 1], kk));
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < OUTS; ++j)
      if (j < n) out[row * w.out_cols + c0 + j] = T::store(sum[j]);
  }
}

// f(width) with width = WC as a compile-time constant, 1 .. NARROW.
template <class F> int with_width(long long wc, F &&f) {
  switch (wc) {
    case 1: return f(std::integral_constant<int, 1>{});
    case 2: return f(std::integral_constant<int, 2>{});
    case 3: return f(std::integral_constant<int, 3>{});
    case 4: return f(std::integral_constant<int, 4>{});
    case 5: return f(std::integral_constant<int, 5>{});
    case 6: return f(std::integral_constant<int, 6>{});
    case 7: return f(std::integral_constant<int, 7>{});
    default: return f(std::integral_constant<int, 8>{});
  }
}

// Rows of `cols` elements of S starting at `p` all start on a 4-element
// vector boundary.
template <class S> bool rows_on_vectors(const void *p, long long cols) {
  return cols % 4 == 0 && (reinterpret_cast<uintptr_t>(p) & (4 * sizeof(S) - 1)) == 0;
}

// pad (kernels.rs:1575-1601): zeros around the input, bits moved; a block
// per output row in turn, its threads along the row (no division).
template <class E>
__global__ void __launch_bounds__(256) pad_kernel(const E *in, E *out, long long rows, long long cols,
                                                  long long pr, long long pc) {
  const long long ocols = cols + 2 * pc, orows = rows + 2 * pr;
  for (long long orow = blockIdx.x; orow < orows; orow += gridDim.x) {
    const long long r = orow - pr;
    const bool inside_row = r >= 0 && r < rows;
    E *dst = out + orow * ocols;
    const E *src = in + (inside_row ? r * cols : 0) - pc;
    for (long long c = threadIdx.x; c < ocols; c += blockDim.x)
      dst[c] = (inside_row && c >= pc && c < pc + cols) ? src[c] : E(0);
  }
}

// pad in 16-byte packs: the same rows when the padding, the row length and
// both buffers are whole packs (element size E, P = 16 / E per pack).
template <class E>
__global__ void __launch_bounds__(256) pad_packs(const E *in, E *out, long long rows, long long cols, long long pr,
                                                 long long pc) {
  constexpr long long P = 16 / sizeof(E);
  const long long ocols = cols + 2 * pc, orows = rows + 2 * pr;
  const long long oq = ocols / P, pq = pc / P, cq = cols / P;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (long long orow = blockIdx.x; orow < orows; orow += gridDim.x) {
    const long long r = orow - pr;
    uint4 *dst = reinterpret_cast<uint4 *>(out + orow * ocols);
    if (r < 0 || r >= rows) {
      for (long long q = threadIdx.x; q < oq; q += blockDim.x) dst[q] = zero;
      continue;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(in + r * cols);
    for (long long q = threadIdx.x; q < oq; q += blockDim.x)
      dst[q] = (q >= pq && q < pq + cq) ? __ldg(src + (q - pq)) : zero;
  }
}

// flip (kernels.rs:1531-1542): out[r][c] = in[rows-1-r][cols-1-c], which is
// the whole matrix reversed in storage order.
template <class E>
__global__ void __launch_bounds__(256) flip_kernel(const E *in, E *out, long long n) {
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < n; o += (long long)gridDim.x * blockDim.x)
    out[o] = __ldg(in + (n - 1 - o));
}

int run_correlate(int dtype, const Window &w, const void *in, const void *win, void *out, cudaStream_t s) {
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    const long long outputs = w.out_rows * w.out_cols, taps = w.win_rows * w.win_cols;
    if (taps >= 4096 && outputs < (long long)sm_count() * 64) {
      const unsigned grid = unsigned(std::min<long long>(outputs, (long long)sm_count() * 8));
      correlate_shared<T><<<grid, 256, 0, s>>>(static_cast<const S *>(in), static_cast<const S *>(win),
                                               static_cast<S *>(out), w);
    } else if (w.win_cols <= NARROW && taps <= SMEM_TAPS) {
      const bool vec = rows_on_vectors<S>(in, w.in_cols);
      return with_width(w.win_cols, [&](auto width) {
        correlate_narrow<T, decltype(width)::value><<<grid_for((outputs + OUTS - 1) / OUTS, 256, 8), 256, 0, s>>>(
            static_cast<const S *>(in), static_cast<const S *>(win), static_cast<S *>(out), w, vec);
        return check_launch("correlate");
      });
    } else {
      correlate_direct<T><<<grid_for((outputs + OUTS - 1) / OUTS, 256, 8), 256, 0, s>>>(static_cast<const S *>(in),
                                                                      static_cast<const S *>(win),
                                                                      static_cast<S *>(out), w);
    }
    return check_launch("correlate");
  });
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_correlate(int dtype, size_t rows, size_t cols, size_t window_rows, size_t window_cols, int flip,
                 const void *input, const void *window, void *out, void *stream) {
  if (window_rows > rows || window_cols > cols)
    return fail(TC_EINVAL, "correlate: a %zux%zu window does not fit in a %zux%zu input", window_rows, window_cols,
                rows, cols);
  if (window_rows == 0 || window_cols == 0)
    return fail(TC_EINVAL, "correlate: the window is empty");
  Window w{(long long)rows, (long long)cols, (long long)window_rows, (long long)window_cols,
           (long long)(rows - window_rows + 1), (long long)(cols - window_cols + 1), flip != 0};
  if (!input || !window || !out) return fail(TC_EINVAL, "correlate: null pointer");
  return run_correlate(dtype, w, input, window, out, as_stream(stream));
}

int tc_correlate_window_gradient(int dtype, size_t rows, size_t cols, size_t adjoint_rows, size_t adjoint_cols,
                                 const void *input, const void *adjoint, void *out, void *stream) {
  return tc_correlate(dtype, rows, cols, adjoint_rows, adjoint_cols, 0, input, adjoint, out, stream);
}

int tc_correlate_input_gradient(int dtype, size_t adjoint_rows, size_t adjoint_cols, size_t window_rows,
                                size_t window_cols, int forward_flip, const void *adjoint, const void *window,
                                void *out, void *stream) {
  if (window_rows == 0 || window_cols == 0 || adjoint_rows == 0 || adjoint_cols == 0)
    return fail(TC_EINVAL, "correlate_input_gradient: empty operand");
  Window w{(long long)adjoint_rows, (long long)adjoint_cols, (long long)window_rows, (long long)window_cols,
           (long long)(adjoint_rows + window_rows - 1), (long long)(adjoint_cols + window_cols - 1),
           forward_flip != 0};
  if (!adjoint || !window || !out) return fail(TC_EINVAL, "correlate_input_gradient: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    const unsigned grid = grid_for(w.out_rows * ((w.out_cols + OUTS - 1) / OUTS), 256, 8);
    if (w.win_cols <= NARROW && w.win_rows * w.win_cols <= SMEM_TAPS) {
      const bool vec = rows_on_vectors<S>(adjoint, w.in_cols);
      return with_width(w.win_cols, [&](auto width) {
        correlate_input_gradient_narrow<T, decltype(width)::value><<<grid, 256, 0, as_stream(stream)>>>(
            static_cast<const S *>(adjoint), static_cast<const S *>(window), static_cast<S *>(out), w, vec);
        return check_launch("correlate_input_gradient");
      });
    }
    correlate_input_gradient_direct<T><<<grid, 256, 0, as_stream(stream)>>>(
        static_cast<const S *>(adjoint), static_cast<const S *>(window), static_cast<S *>(out), w);
    return check_launch("correlate_input_gradient");
  });
}

int tc_pad(int dtype, size_t rows, size_t cols, size_t pad_rows, size_t pad_cols, const void *input, void *out,
           void *stream) {
  const size_t total = (rows + 2 * pad_rows) * (cols + 2 * pad_cols);
  if (total == 0) return TC_OK;
  if ((rows * cols && !input) || !out) return fail(TC_EINVAL, "pad: null pointer");
  return with_real(dtype, [&](auto t) {
    using S = typename decltype(t)::S;
    const unsigned grid = unsigned(std::min<long long>((long long)(rows + 2 * pad_rows), (long long)sm_count() * 16));
    constexpr size_t P = 16 / sizeof(S);
    if ((uintptr_t(input) & 15u) == 0 && (uintptr_t(out) & 15u) == 0 && cols % P == 0 && pad_cols % P == 0) {
      pad_packs<S><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const S *>(input), static_cast<S *>(out),
                                                        (long long)rows, (long long)cols, (long long)pad_rows,
                                                        (long long)pad_cols);
      return check_launch("pad");
    }
    pad_kernel<S><<<grid, 256, 0, as_stream(stream)>>>(
        static_cast<const S *>(input), static_cast<S *>(out), (long long)rows, (long long)cols,
        (long long)pad_rows, (long long)pad_cols);
    return check_launch("pad");
  });
}

int tc_flip(int dtype, size_t rows, size_t cols, const void *input, void *out, void *stream) {
  const size_t n = rows * cols;
  if (n == 0) return TC_OK;
  if (!input || !out) return fail(TC_EINVAL, "flip: null pointer");
  return with_real(dtype, [&](auto t) {
    using S = typename decltype(t)::S;
    flip_kernel<S><<<grid_for(n, 256, 8), 256, 0, as_stream(stream)>>>(static_cast<const S *>(input),
                                                                        static_cast<S *>(out), (long long)n);
    return check_launch("flip");
  });
}

}  // extern "C"
