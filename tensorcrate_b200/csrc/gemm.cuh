// gemm.cuh — the product kernels behind tc_matmul: tcgen05 tensor-core tiles
// for f16/bf16 (gemm_sm100.cu) and FP32 CUDA-core tiles (gemm_simt.cu).
#pragma once
#include "common.cuh"

namespace tc {
// SMs the persistent tensor-core kernels leave free on this thread's
// launches (for kernels that must run beside them, such as a collective's).
void gemm_reserve_sms(int n);
int reserved_sms();
int gemm_simt_run(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                  void *c, bool accumulate, cudaStream_t stream);
// TC_ENOTSUP when the shape or alignment is not one the tensor-core kernel
// tiles; the caller then runs the SIMT kernel.
int gemm_tc_run(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                void *c, bool accumulate, cudaStream_t stream);
// The same product, each tile also stored to the `n_peers` (at most 7)
// buffers in peer_c: C as other GPUs hold it, at the same offset.
int gemm_tc_run_peers(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a,
                      const void *b, void *c, bool accumulate, void *const *peer_c, int n_peers,
                      cudaStream_t stream);
// What a dense layer's epilogue does to the rounded product P, in this
// order (all optional, none with accumulate or peers):
//   share_of: P = round(P * MaxShare(share_of[row, col], 0)), the ReLU's
//             backward rule (share_of laid out as C)
//   bias:     C = round(P + bias[row])
//   relu_out: relu_out = max(C, 0)
struct Epilogue {
  const void *bias = nullptr;
  void *relu_out = nullptr;
  const void *share_of = nullptr;
};
// The product with an epilogue: TC_ENOTSUP as gemm_tc_run.
int gemm_tc_run_full(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a,
                     const void *b, void *c, bool accumulate, void *const *peer_c, int n_peers, const Epilogue &e,
                     cudaStream_t stream);
// f32 products on the tensor cores as three TF32 passes: each operand split
// into a TF32 head and a TF32 tail (hi + lo), and C = hi.hi + hi.lo + lo.hi
// accumulated in f32, which leaves a relative error near 2^-21 per product.
// The halves go through the per-device scratch buffer.  TC_ENOTSUP beyond
// 32-bit tile coordinates.
int gemm_tf32_run(int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b, void *c,
                  bool accumulate, cudaStream_t stream);
}  // namespace tc
