/*
 * oracle.h — CPU restatement of tensorcrate's Host backend for the hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the CUDA backend is
 * compared against, and the timed CPU baseline; nothing in the product
 * (libtccuda, the tensorcrate_b200 package) links, loads or calls it.
 *
 * Each function restates the reference's Host algorithm it names
 * (file:line inside the tensorcrate crate), in the same arithmetic order, so
 * that integer, bit and comparison work is bit-identical and floating-point
 * work rounds where the reference rounds.  The enums, dtype codes and the
 * region struct are the public ones of include/tccuda.h.
 */
#ifndef TC_ORACLE_H
#define TC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/tccuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* f16/bf16 <-> f32, as crate `half` 2.7.1 converts (round to nearest even,
 * NaN kept quiet with its payload). */
void orc_narrow(int dtype, const float *in, void *out, size_t n);
void orc_widen(int dtype, const void *in, float *out, size_t n);

/* layout.rs */
int orc_coalesce(uint32_t rank, const size_t *shape, uint32_t n_ops, const size_t *strides,
                 uint32_t *out_rank, size_t *out_shape, size_t *out_strides);
int orc_broadcast_shape(uint32_t lrank, const size_t *left, uint32_t rrank, const size_t *right,
                        uint32_t *out_rank, size_t *out_shape);
int orc_broadcast_strides(uint32_t rank, const size_t *shape, const size_t *strides,
                          uint32_t trank, const size_t *target, size_t *out_strides);
/* The walk for_each_run makes: every storage position, in order. */
int orc_walk(uint32_t rank, const size_t *shape, size_t offset, const size_t *strides,
             size_t *out_positions);

/* backend.rs */
int orc_strided_copy(size_t elem_bytes, uint32_t rank, const size_t *shape, const void *src,
                     size_t src_len, size_t src_offset, const size_t *src_strides, void *dst);
int orc_strided_write(size_t elem_bytes, void *target, size_t target_len, const tc_region *region);
int orc_assemble(size_t elem_bytes, void *dst, size_t len, const tc_region *regions, size_t n);

/* kernels.rs / simd_dispatch.rs same-shape elementwise */
int orc_elementwise(int dtype, int op, const void *a, const void *b, void *out, size_t n);
int orc_broadcast_scalar(int dtype, int op, const void *a, double scalar, int scalar_left,
                         void *out, size_t n);
int orc_compare(int dtype, int cmp, const void *a, const void *b, void *out, size_t n);
int orc_compare_scalar(int dtype, int cmp, const void *a, double scalar, int scalar_left,
                       void *out, size_t n);
int orc_clamp(int dtype, const void *a, double low, double high, void *out, size_t n);
int orc_vector_reduce(int dtype, int op, const void *a, size_t n, void *out);
int orc_dot(int dtype, const void *a, const void *b, size_t n, void *out);

/* strided.rs */
int orc_strided_binary(int dtype, int kind, int op, uint32_t rank, const size_t *shape,
                       const void *a, size_t a_len, size_t a_offset, const size_t *a_strides,
                       const void *b, size_t b_len, size_t b_offset, const size_t *b_strides,
                       void *out);
int orc_reduce_axes(int dtype, uint32_t rank, const size_t *shape, const void *input,
                    size_t input_len, size_t offset, const size_t *strides, uint32_t n_axes,
                    const uint32_t *axes, int kind, int op, size_t divisor, void *out);
int orc_arg_reduce(int dtype, uint32_t rank, const size_t *shape, const void *input,
                   size_t input_len, size_t offset, const size_t *strides, uint32_t axis, int op,
                   uint32_t *out);

/* matrix.rs / simd_x86.rs / compact.rs products */
int orc_matmul(int dtype, int transposed, size_t rows, size_t inner, size_t cols,
               const void *a, const void *b, void *c, int accumulate);
/* The same product over a band of output rows [row0, row1) only: rows of
 * the i-p-j loop are independent, so a band times the whole. */
int orc_matmul_rows(int dtype, size_t rows, size_t inner, size_t cols, const void *a,
                    const void *b, void *c, int accumulate, size_t row0, size_t row1);
int orc_matvec(int dtype, size_t rows, size_t cols, const void *m, const void *x, void *y,
               int accumulate);
int orc_vecmat(int dtype, size_t rows, size_t cols, const void *x, const void *m, void *y);
int orc_transpose(int dtype, size_t rows, size_t cols, const void *m, void *out);

/* optim.rs */
int orc_adam(int dtype, size_t n, void *p, const void *g, void *m, void *v, int resumed,
             double rate, double beta1, double beta2, double eps, double c1, double c2);
int orc_sgd(int dtype, size_t n, void *p, const void *g, double rate);
/* Adam::update's host arithmetic (optim.rs:1106-1124): for step t, the two
 * corrections (1 - beta^t).recip() rounded in the element type, and the
 * element-type values of the coefficients.  out[0..6] = rate, beta1, beta2,
 * eps, c1, c2 as doubles holding element-type values. */
int orc_adam_coefficients(int dtype, double rate, double beta1, double beta2, double eps,
                          uint32_t step, double *out);

/* One MLP training step through the tape's rules and Adam (see oracle.cpp). */
void *orc_mlp_create(int dtype, uint32_t layers, const uint32_t *dims, uint32_t batch, uint32_t global_batch,
                     double rate, double beta1, double beta2, double eps);
void orc_mlp_destroy(void *mlp);
int orc_mlp_params(void *mlp, uint32_t layer, void *w, void *b, int dir);
int orc_mlp_grads(void *mlp, uint32_t layer, void *gw, void *gb);
int orc_mlp_step(void *mlp, const void *x, const void *y, void *loss_out, int skip_update);

/* Host threads the elementwise kernels may use (set_host_threads,
 * src/parallel.rs:40); 0 = all. */
void orc_set_threads(int threads);
void orc_set_matmul_threads(int threads);

/* Fused program (Kernels::fused; Host interpreter, fused/mod.rs:4055-4260)
 * over host buffers, as tc_fused takes them. */
int orc_fused(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
              const tc_place *places, uint32_t n_places, void *const *outputs, const int *out_dtypes,
              uint32_t n_outputs);

/* The other vector methods, as tc_unary, tc_unary_dual, tc_prefix_sum,
 * tc_sort, tc_power and tc_power_scalar take them (kernels.rs:870-891). */
int orc_unary(int dtype, int f, const void *a, void *out, size_t n);
int orc_unary_dual(int dtype, int f, const void *value, const void *tangent, void *out_value,
                   void *out_tangent, size_t n);
int orc_prefix_sum(int dtype, const void *a, void *out, size_t n);
int orc_sort(int dtype, int order, const void *a, void *out, size_t n);
int orc_power(int dtype, const void *a, const void *b, void *out, size_t n);
int orc_power_scalar(int dtype, const void *a, double scalar, int scalar_left, void *out, size_t n);

/* Windowed matrix methods, as tc_correlate, tc_correlate_input_gradient,
 * tc_pad and tc_flip take them (kernels.rs:998-1028). */
int orc_correlate(int dtype, size_t rows, size_t cols, size_t window_rows, size_t window_cols, int flip,
                  const void *input, const void *window, void *out);
int orc_correlate_input_gradient(int dtype, size_t adjoint_rows, size_t adjoint_cols, size_t window_rows,
                                 size_t window_cols, int forward_flip, const void *adjoint, const void *window,
                                 void *out);
int orc_pad(int dtype, size_t rows, size_t cols, size_t pad_rows, size_t pad_cols, const void *input, void *out);
int orc_flip(int dtype, size_t rows, size_t cols, const void *input, void *out);

/* Moments and distributions, as tc_moments, tc_axis_moments,
 * tc_distribution and tc_axis_distribution take them (host buffers). */
int orc_moments(int dtype, const void *a, size_t n, void *out);
int orc_axis_moments(int dtype, size_t rows, size_t cols, int axis, const void *a, void *means, void *devs);
int orc_distribution(int dtype, int family, int statistic, const void *a, size_t n, double first, double second,
                     void *out);
double orc_evaluate_f64(int family, int statistic, double x, double first, double second);
int orc_axis_distribution(int dtype, size_t rows, size_t cols, int axis, int family, int statistic, const void *a,
                          const void *first, const void *second, void *out);

/* Fused programs with row statistics and sums, as tc_row_moments,
 * tc_fused_with_statistics and tc_fused_sum take them (host buffers). */
int orc_row_moments(int dtype, const tc_place *place, size_t rows, size_t cols, void *means, void *devs);
int orc_fused_with_statistics(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                              const tc_place *places, uint32_t n_places, const tc_row_statistic *stats,
                              uint32_t n_stats, void *const *outputs, const int *out_dtypes, uint32_t n_outputs);
int orc_fused_sum(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                  const tc_place *places, uint32_t n_places, int axis, void *sums);

int orc_matmul_program(int dtype, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                       const tc_instr *code, uint32_t n_code, const tc_place *places, uint32_t n_places,
                       void *const *outputs, const int *out_dtypes, uint32_t n_outputs);

#ifdef __cplusplus
}
#endif
#endif
