// gemm_simt.cu — FP32 CUDA-core GEMM tiles: the f32 product (accuracy
// first: every product and sum in IEEE f32, no TF32), and the fallback for
// f16/bf16 shapes the tensor-core kernel does not tile (inner dimension
// below 16, or operands that break its 16-byte TMA alignment).
//
// C[rows x cols] (+)= op(A)·op(B): each operand is read through (row, col)
// element strides, so Transposed::{Left, Right} (kernels.rs:462-467) cost
// nothing: A^T is A read with its strides swapped.
//
// Register blocking: a BM x BN tile per block, BK-deep slices of A and B in
// shared memory (double-buffered), each thread an TM x TN micro-tile held in
// registers.
#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"

namespace tc {
namespace {

template <class T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_simt(const typename T::S *__restrict__ a, long long a_r, long long a_c, const typename T::S *__restrict__ b,
              long long b_r, long long b_c, typename T::S *__restrict__ c, long long M, long long N, long long K,
              bool accumulate) {
  constexpr int THREADS = (BM / TM) * (BN / TN);
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  const long long m0 = (long long)blockIdx.y * BM, n0 = (long long)blockIdx.x * BN;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  auto load_tiles = [&](int buf, long long k0) {
    for (int e = tid; e < BM * BK; e += THREADS) {
      // Consecutive threads walk the operand's contiguous direction when
      // it is the K direction (a_c == 1) or the M direction (a_r == 1).
      int mm, kk;
      if (a_c == 1) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
      long long gm = m0 + mm, gk = k0 + kk;
      As[buf][kk][mm] = (gm < M && gk < K) ? T::load(a[gm * a_r + gk * a_c]) : 0.0f;
    }
    for (int e = tid; e < BN * BK; e += THREADS) {
      int nn, kk;
      if (b_c == 1) { nn = e % BN; kk = e / BN; } else { kk = e % BK; nn = e / BK; }
      long long gn = n0 + nn, gk = k0 + kk;
      Bs[buf][kk][nn] = (gn < N && gk < K) ? T::load(b[gk * b_r + gn * b_c]) : 0.0f;
    }
  };

  load_tiles(0, 0);
  __syncthreads();
  int buf = 0;
  for (long long k0 = 0; k0 < K; k0 += BK) {
    if (k0 + BK < K) load_tiles(buf ^ 1, k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float ra[TM], rb[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) ra[i] = As[buf][kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) rb[j] = Bs[buf][kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(ra[i], rb[j], acc[i][j]);
    }
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    long long gm = m0 + ty * TM + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      long long gn = n0 + tx * TN + j;
      if (gn >= N) continue;
      typename T::S *p = c + gm * N + gn;
      float v = acc[i][j];
      if (accumulate) v = __fadd_rn(T::load(*p), v);
      *p = T::store(v);
    }
  }
}

template <class T>
int launch(const void *a, long long a_r, long long a_c, const void *b, long long b_r, long long b_c, void *c,
           long long M, long long N, long long K, bool accumulate, cudaStream_t s) {
  using S = typename T::S;
  const S *pa = static_cast<const S *>(a);
  const S *pb = static_cast<const S *>(b);
  S *pc = static_cast<S *>(c);
  long long big_tiles = ((M + 127) / 128) * ((N + 127) / 128);
  if (big_tiles >= sm_count()) {
    dim3 grid(unsigned((N + 127) / 128), unsigned((M + 127) / 128));
    gemm_simt<T, 128, 128, 8, 8, 8><<<grid, 256, 0, s>>>(pa, a_r, a_c, pb, b_r, b_c, pc, M, N, K, accumulate);
  } else {
    dim3 grid(unsigned((N + 63) / 64), unsigned((M + 63) / 64));
    gemm_simt<T, 64, 64, 16, 4, 4><<<grid, 256, 0, s>>>(pa, a_r, a_c, pb, b_r, b_c, pc, M, N, K, accumulate);
  }
  return check_launch("gemm (simt)");
}

}  // namespace

int gemm_simt_run(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                  void *c, bool accumulate, cudaStream_t stream) {
  long long M = (long long)rows, N = (long long)cols, K = (long long)inner;
  if ((M + 127) / 128 > 65535 && (M + 63) / 64 > 65535) return fail(TC_EINVAL, "gemm: %lld rows", M);
  // Element strides of op(A)(i, p) and op(B)(p, j).
  long long a_r = K, a_c = 1, b_r = N, b_c = 1;
  if (transposed == TC_TRANS_LEFT) { a_r = 1; a_c = M; }
  if (transposed == TC_TRANS_RIGHT) { b_r = 1; b_c = K; }
  return with_real(dtype, [&](auto t) {
    return launch<decltype(t)>(a, a_r, a_c, b, b_r, b_c, c, M, N, K, accumulate, stream);
  });
}

}  // namespace tc
