// gemv.cu — matrix-vector products (Kernels::matvec / matvec_add,
// kernels.rs:901-908; Kernels::vecmat, kernels.rs:899) and the tc_matmul
// entry point that routes products to the GEMM kernels.
//
// Both GEMVs are HBM-bound: the matrix is read once with 128-bit loads.
//  - matvec: a warp per row, the row streamed in packs, a shuffle tree.
//  - vecmat: each thread owns adjacent output columns; the block's warps
//    split the rows and combine in shared memory, so every row read is
//    one coalesced segment.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace tc {
namespace {

template <class T> struct Pack {
  using S = typename T::S;
  static constexpr int N = 16 / int(sizeof(S));
  union { uint4 raw; S v[N]; };
};

// y[r] (+)= M[r, :] . x.  WPR warps per row (a block holds 8 / WPR rows),
// each over every WPR-th group of 32 packs of the row, four packs in flight
// per lane; the warps' partial sums meet in shared memory in warp order.
template <class T, int WPR>
__global__ void __launch_bounds__(256) matvec_rows(const typename T::S *m, const typename T::S *x,
                                                   typename T::S *y, long long rows, long long cols,
                                                   bool accumulate, bool vec) {
  constexpr int N = Pack<T>::N;
  constexpr int RPB = 8 / WPR;  // rows per block
  __shared__ float part[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = warp / WPR, wr = warp - g * WPR;  // row in block, warp in row
  for (long long r0 = (long long)blockIdx.x * RPB; r0 < rows; r0 += (long long)gridDim.x * RPB) {
    const long long r = r0 + g;
    float s = 0.0f;
    if (r < rows) {
      const typename T::S *row = m + r * cols;
      if (vec) {
        constexpr int U = 4;
        const long long packs = cols / N;
        for (long long p0 = (long long)wr * 32 + lane; p0 < packs; p0 += 32LL * WPR * U) {
          Pack<T> a[U], b[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (p0 + 32LL * WPR * u < packs) {
              a[u].raw = __ldg(reinterpret_cast<const uint4 *>(row + (p0 + 32LL * WPR * u) * N));
              b[u].raw = __ldg(reinterpret_cast<const uint4 *>(x + (p0 + 32LL * WPR * u) * N));
            }
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (p0 + 32LL * WPR * u < packs) {
#pragma unroll
              for (int j = 0; j < N; ++j) s = fmaf(T::load(a[u].v[j]), T::load(b[u].v[j]), s);
            }
        }
      } else {
        for (long long c = (long long)wr * 32 + lane; c < cols; c += 32LL * WPR)
          s = fmaf(T::load(row[c]), T::load(x[c]), s);
      }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    }
    if (WPR == 1) {
      if (lane == 0 && r < rows) {
        if (accumulate) s = __fadd_rn(T::load(y[r]), s);
        y[r] = T::store(s);
      }
    } else {
      if (lane == 0) part[warp] = s;
      __syncthreads();
      if (wr == 0 && lane == 0 && r < rows) {
        float t = part[warp];
#pragma unroll
        for (int k = 1; k < WPR; ++k) t += part[warp + k];
        if (accumulate) t = __fadd_rn(T::load(y[r]), t);
        y[r] = T::store(t);
      }
      __syncthreads();
    }
  }
}

// y[j] = sum_p x[p] * m[p, j].  blockDim = (32, 8): x walks 32*CPT
// adjacent columns (one 16-byte load each when CPT > 1), y splits a block's
// rows; blockIdx.y picks one of `shares` row ranges, whose f32 partial sums
// go to `partial` when shares > 1 (merged in order by vecmat_finish).
template <class T, int CPT>
__global__ void __launch_bounds__(256) vecmat_cols(const typename T::S *x, const typename T::S *m,
                                                   typename T::S *y, long long rows, long long cols,
                                                   long long rows_per_share, float *partial) {
  using S = typename T::S;
  __shared__ float part[8][32 * CPT + 1];
  const long long j0 = ((long long)blockIdx.x * 32 + threadIdx.x) * CPT;
  const long long r0 = (long long)blockIdx.y * rows_per_share, r1 = min(rows, r0 + rows_per_share);
  float s[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) s[c] = 0.0f;
  if (j0 < cols) {
    // Four rows in flight per thread, folded in row order as one at a time.
    constexpr int U = 4;
    for (long long p0 = r0 + threadIdx.y; p0 < r1; p0 += 8 * U) {
      if (CPT > 1) {
        union Pk { uint4 raw; S v[16 / sizeof(S)]; } pk[U];
        float xp[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (p0 + 8 * u < r1) {
            xp[u] = T::load(x[p0 + 8 * u]);
            pk[u].raw = __ldg(reinterpret_cast<const uint4 *>(m + (p0 + 8 * u) * cols + j0));
          }
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (p0 + 8 * u < r1) {
#pragma unroll
            for (int c = 0; c < CPT; ++c) s[c] = fmaf(xp[u], T::load(pk[u].v[c]), s[c]);
          }
      } else {
        for (int u = 0; u < U; ++u)
          if (p0 + 8 * u < r1) s[0] = fmaf(T::load(x[p0 + 8 * u]), T::load(__ldg(m + (p0 + 8 * u) * cols + j0)), s[0]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CPT; ++c) part[threadIdx.y][threadIdx.x * CPT + c] = s[c];
  __syncthreads();
  if (threadIdx.y == 0 && j0 < cols) {
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      float t = part[0][threadIdx.x * CPT + c];
      for (int k = 1; k < 8; ++k) t += part[k][threadIdx.x * CPT + c];
      if (gridDim.y > 1) partial[blockIdx.y * cols + j0 + c] = t;
      else y[j0 + c] = T::store(t);
    }
  }
}

// blockDim = (32, 8): x walks 32 columns, y takes every 8th share; the
// eight partial sums of a column then meet in shared memory.
template <class T>
__global__ void __launch_bounds__(256) vecmat_finish(const float *partial, int shares, long long cols,
                                                     typename T::S *y) {
  __shared__ float part[8][33];
  const long long j = (long long)blockIdx.x * 32 + threadIdx.x;
  float t = 0.0f;
  if (j < cols)
    for (int s = threadIdx.y; s < shares; s += 8) t += partial[s * cols + j];
  part[threadIdx.y][threadIdx.x] = t;
  __syncthreads();
  if (threadIdx.y == 0 && j < cols) {
    float r = part[0][threadIdx.x];
    for (int k = 1; k < 8; ++k) r += part[k][threadIdx.x];
    y[j] = T::store(r);
  }
}

// An inner dimension of one: C[i, j] (+)= a[i] * b[j], one rounding (the
// product of two stored values is exact in f32).  The tape's outer product
// b ⊗ ones is this (tape/mod.rs:1000-1005).  Packs of 16 bytes along j.
template <class T>
__global__ void __launch_bounds__(256) outer_rows(const typename T::S *a, const typename T::S *b, typename T::S *c,
                                                  long long rows, long long cols, bool accumulate, bool vec) {
  constexpr int N = Pack<T>::N;
  const long long per_row = vec ? cols / N : cols;
  const long long total = rows * per_row;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / per_row, q = i - r * per_row;
    const float ar = T::load(a[r]);
    if (vec) {
      Pack<T> bb, cc;
      bb.raw = __ldg(reinterpret_cast<const uint4 *>(b + q * N));
      if (accumulate) cc.raw = *reinterpret_cast<const uint4 *>(c + r * cols + q * N);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float v = __fmul_rn(ar, T::load(bb.v[j]));
        if (accumulate) v = __fadd_rn(T::load(cc.v[j]), v);
        cc.v[j] = T::store(v);
      }
      *reinterpret_cast<uint4 *>(c + r * cols + q * N) = cc.raw;
    } else {
      float v = __fmul_rn(ar, T::load(b[q]));
      if (accumulate) v = __fadd_rn(T::load(c[r * cols + q]), v);
      c[r * cols + q] = T::store(v);
    }
  }
}

// A dense layer's epilogue as a pass of its own, over a product already
// rounded to T: c = round(c * MaxShare(share_of, 0)); c = round(c +
// bias[row]); relu_out = max(c, 0).
template <class T>
__global__ void __launch_bounds__(256) epilogue_rows(typename T::S *c, const typename T::S *share_of,
                                                     const typename T::S *bias, typename T::S *relu_out,
                                                     long long rows, long long cols) {
  const long long total = rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    float v = T::load(c[i]);
    if (share_of) v = T::load(T::store(__fmul_rn(v, compare_value(TC_MAX_SHARE, T::load(share_of[i]), 0.0f))));
    if (bias) v = T::load(T::store(__fadd_rn(v, T::load(bias[i / cols]))));
    if (share_of || bias) c[i] = T::store(v);
    if (relu_out) relu_out[i] = T::store(fmaxf(v, 0.0f));
  }
}

}  // namespace
}  // namespace tc

// ---------------------------------------------------------------------------
// Static scratch for tc_vecmat_noalloc: the row split's f32 partial sums,
// in a device array that is part of the module, so the entry point
// allocates nothing.  Every call on a device shares it.  Nothing in it has
// to start at zero: each partial is written before it is read.
// ---------------------------------------------------------------------------
constexpr size_t VECMAT_NOALLOC_SCRATCH_BYTES = size_t(1) << 20;  // 1 MiB
static __device__ __align__(256) float vecmat_noalloc_scratch[VECMAT_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace tc {
namespace {
// The array's address on the current device, looked up once per device.
int vecmat_noalloc_scratch_address(float **out) {
  static std::mutex mu;
  static float *address[64] = {nullptr};
  int dev = 0;
  if (int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  if (dev < 0 || dev >= 64) return fail(TC_EINVAL, "vecmat_noalloc: device %d", dev);
  std::lock_guard<std::mutex> g(mu);
  if (!address[dev]) {
    void *p = nullptr;
    if (int st = check_cuda(cudaGetSymbolAddress(&p, vecmat_noalloc_scratch), "cudaGetSymbolAddress (vecmat scratch)"))
      return st;
    address[dev] = static_cast<float *>(p);
  }
  *out = address[dev];
  return TC_OK;
}
}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_matvec(int dtype, size_t rows, size_t cols, const void *m, const void *x, void *y, int accumulate,
              void *stream) {
  if (rows == 0) return TC_OK;
  if (!m || !x || !y) return fail(TC_EINVAL, "matvec: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    constexpr int N = Pack<T>::N;
    bool vec = cols % N == 0 && (uintptr_t(m) & 15u) == 0 && (uintptr_t(x) & 15u) == 0;
    // Warps per row: enough warps in all to cover the SMs (32 each), while
    // every warp still has a group of 32 units of its row.
    const long long units = vec ? (long long)cols / N : (long long)cols;
    int wpr = 1;
    while (wpr < 8 && (long long)rows * wpr < 32LL * sm_count() && units >= 32LL * wpr * 2) wpr *= 2;
    const long long rpb = 8 / wpr;
    unsigned grid = unsigned(std::max(1LL, std::min<long long>(((long long)rows + rpb - 1) / rpb, (long long)sm_count() * 8)));
    auto go = [&](auto kernel) {
      kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const S *>(m), static_cast<const S *>(x),
                                                  static_cast<S *>(y), (long long)rows, (long long)cols,
                                                  accumulate != 0, vec);
    };
    if (wpr == 8) go(matvec_rows<T, 8>);
    else if (wpr == 4) go(matvec_rows<T, 4>);
    else if (wpr == 2) go(matvec_rows<T, 2>);
    else go(matvec_rows<T, 1>);
    return check_launch("matvec");
  });
}

int tc_vecmat(int dtype, size_t rows, size_t cols, const void *x, const void *m, void *y, void *stream) {
  if (cols == 0) return TC_OK;
  if (!m || !x || !y) return fail(TC_EINVAL, "vecmat: null pointer");
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    using S = typename T::S;
    constexpr int CPT = 16 / int(sizeof(S));
    const bool vec = cols % CPT == 0 && (uintptr_t(m) & 15u) == 0;
    const int cpt = vec ? CPT : 1;
    const long long col_blocks = ((long long)cols + 32 * cpt - 1) / (32 * cpt);
    // Split the rows until there are ~4 blocks per SM, keeping 64+ rows each.
    long long shares = 1;
    while (col_blocks * shares < 4LL * sm_count() && (long long)rows / (shares * 2) >= 64) shares *= 2;
    const long long per = ((long long)rows + shares - 1) / shares;
    float *partial = nullptr;
    if (shares > 1) {
      void *p = nullptr;
      if (int st = scratch(size_t(shares) * cols * sizeof(float), &p, as_stream(stream))) return st;
      partial = static_cast<float *>(p);
    }
    dim3 grid((unsigned)col_blocks, (unsigned)shares);
    cudaStream_t s = as_stream(stream);
    if (vec)
      vecmat_cols<T, CPT><<<grid, dim3(32, 8), 0, s>>>(static_cast<const S *>(x), static_cast<const S *>(m),
                                                        static_cast<S *>(y), (long long)rows, (long long)cols, per,
                                                        partial);
    else
      vecmat_cols<T, 1><<<grid, dim3(32, 8), 0, s>>>(static_cast<const S *>(x), static_cast<const S *>(m),
                                                      static_cast<S *>(y), (long long)rows, (long long)cols, per,
                                                      partial);
    if (shares > 1)
      vecmat_finish<T><<<unsigned((cols + 31) / 32), dim3(32, 8), 0, s>>>(partial, int(shares), (long long)cols,
                                                                         static_cast<S *>(y));
    return check_launch("vecmat");
  });
}

// tc_vecmat with the same row split and kernels, so the same bits, but the
// partial sums in the static array above instead of the allocated scratch.
int tc_vecmat_noalloc(int dtype, size_t rows, size_t cols, const void *x, const void *m, void *y, void *stream) {
  if (cols == 0) return TC_OK;
  if (!m || !x || !y) return fail(TC_EINVAL, "vecmat_noalloc: null pointer");
  return with_real(dtype, [&](auto t) -> int {
    using T = decltype(t);
    using S = typename T::S;
    constexpr int CPT = 16 / int(sizeof(S));
    const bool vec = cols % CPT == 0 && (uintptr_t(m) & 15u) == 0;
    const int cpt = vec ? CPT : 1;
    const long long col_blocks = ((long long)cols + 32 * cpt - 1) / (32 * cpt);
    long long shares = 1;
    while (col_blocks * shares < 4LL * sm_count() && (long long)rows / (shares * 2) >= 64) shares *= 2;
    const long long per = ((long long)rows + shares - 1) / shares;
    float *partial = nullptr;
    if (shares > 1) {
      const size_t need = size_t(shares) * cols * sizeof(float);
      if (need > VECMAT_NOALLOC_SCRATCH_BYTES)
        return fail(TC_ERANGE,
                    "vecmat_noalloc: %zu x %zu splits into %lld row shares whose partial sums take %zu bytes, more "
                    "than its %zu-byte static scratch",
                    rows, cols, shares, need, VECMAT_NOALLOC_SCRATCH_BYTES);
      if (int st = vecmat_noalloc_scratch_address(&partial)) return st;
    }
    dim3 grid((unsigned)col_blocks, (unsigned)shares);
    cudaStream_t s = as_stream(stream);
    if (vec)
      vecmat_cols<T, CPT><<<grid, dim3(32, 8), 0, s>>>(static_cast<const S *>(x), static_cast<const S *>(m),
                                                        static_cast<S *>(y), (long long)rows, (long long)cols, per,
                                                        partial);
    else
      vecmat_cols<T, 1><<<grid, dim3(32, 8), 0, s>>>(static_cast<const S *>(x), static_cast<const S *>(m),
                                                      static_cast<S *>(y), (long long)rows, (long long)cols, per,
                                                      partial);
    if (shares > 1)
      vecmat_finish<T><<<unsigned((cols + 31) / 32), dim3(32, 8), 0, s>>>(partial, int(shares), (long long)cols,
                                                                         static_cast<S *>(y));
    return check_launch("vecmat_noalloc");
  });
}

int tc_matmul_epilogue(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a,
                       const void *b, const void *share_of, const void *bias, void *c, void *relu_out,
                       void *stream) {
  if (transposed < TC_TRANS_NONE || transposed > TC_TRANS_RIGHT)
    return fail(TC_EINVAL, "matmul_epilogue: bad Transposed %d", transposed);
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16)
    return fail(TC_EINVAL, "matmul_epilogue: element type %d", dtype);
  if (rows == 0 || cols == 0) return TC_OK;
  if (!c) return fail(TC_EINVAL, "matmul_epilogue: null output");
  cudaStream_t s = as_stream(stream);
  if (dtype != TC_F32 && inner >= 16 && a && b) {
    Epilogue e;
    e.share_of = share_of;
    e.bias = bias;
    e.relu_out = relu_out;
    int st = gemm_tc_run_full(dtype, transposed, rows, inner, cols, a, b, c, false, nullptr, 0, e, s);
    if (st != TC_ENOTSUP) return st;
  }
  // Otherwise the product, then the epilogue as its own pass (same bits).
  if (int st = tc_matmul(dtype, transposed, rows, inner, cols, a, b, c, 0, stream)) return st;
  if (!share_of && !bias && !relu_out) return TC_OK;
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    epilogue_rows<T><<<grid_for(rows * cols, 256, 8), 256, 0, s>>>(
        static_cast<S *>(c), static_cast<const S *>(share_of), static_cast<const S *>(bias),
        static_cast<S *>(relu_out), (long long)rows, (long long)cols);
    return check_launch("matmul_epilogue");
  });
}

int tc_matmul(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
              void *c, int accumulate, void *stream) {
  if (transposed < TC_TRANS_NONE || transposed > TC_TRANS_RIGHT)
    return fail(TC_EINVAL, "matmul: bad Transposed %d", transposed);
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16) return fail(TC_EINVAL, "matmul: element type %d", dtype);
  if (rows == 0 || cols == 0) return TC_OK;
  if (!c) return fail(TC_EINVAL, "matmul: null output");
  if (inner == 0) {
    // An empty inner dimension: the product is zero.
    if (accumulate) return TC_OK;
    return check_cuda(cudaMemsetAsync(c, 0, rows * cols * dtype_bytes(dtype), as_stream(stream)), "memset");
  }
  if (!a || !b) return fail(TC_EINVAL, "matmul: null operand");
  cudaStream_t s = as_stream(stream);
  if (inner == 1) {
    // [rows x 1]·[1 x cols]: every storage order of either operand is the same.
    return with_real(dtype, [&](auto t) {
      using T = decltype(t);
      using S = typename T::S;
      constexpr int N = Pack<T>::N;
      const bool vec = cols % N == 0 && (uintptr_t(b) & 15u) == 0 && (uintptr_t(c) & 15u) == 0;
      const long long work = (long long)rows * (vec ? (long long)cols / N : (long long)cols);
      outer_rows<T><<<grid_for(size_t(work), 256, 8), 256, 0, s>>>(static_cast<const S *>(a),
                                                                    static_cast<const S *>(b), static_cast<S *>(c),
                                                                    (long long)rows, (long long)cols,
                                                                    accumulate != 0, vec);
      return check_launch("matmul (outer)");
    });
  }
  if (dtype != TC_F32) {
    int st = gemm_tc_run(dtype, transposed, rows, inner, cols, a, b, c, accumulate != 0, s);
    if (st != TC_ENOTSUP) return st;
  } else if (double(rows) * double(cols) * double(inner) >= double(1 << 24) && rows >= 64 && cols >= 64 &&
             inner >= 32) {
    // f32 products big enough to fill the machine: three TF32 passes on the
    // tensor cores (relative error near 2^-21 per product, inside the f32
    // parity tolerance); small ones stay on the FP32 pipe.
    int st = gemm_tf32_run(transposed, rows, inner, cols, a, b, c, accumulate != 0, s);
    if (st != TC_ENOTSUP) return st;
  }
  return gemm_simt_run(dtype, transposed, rows, inner, cols, a, b, c, accumulate != 0, s);
}

}  // extern "C"
