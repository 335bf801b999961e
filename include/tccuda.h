/*
 * tccuda.h — the C ABI of the tensorcrate CUDA backend (sm_100a, B200).
 *
 * Each entry point is what the crate's `Cuda` implementation of the sealed
 * `Backend` and `Kernels<T>` traits binds over FFI (`extern "C"`, plain
 * pointers and sizes).  The comment above each one names the reference
 * interface it replaces, as `file:line` inside the tensorcrate crate.
 *
 * Conventions
 *  - Every call returns `int` status: TC_OK (0) or a TC_E* code.  The message
 *    of the last failure on the calling thread is read with tc_last_error().
 *    The Rust side maps a non-zero status to a panic naming the operation,
 *    as `require_metal` does for Metal (src/tensors/backend.rs:418-426).
 *  - Pointers named `*_dev` / device buffers come from tc_malloc (or any
 *    cudaMalloc'd memory); `stream` is a cudaStream_t passed as void*
 *    (NULL = the legacy default stream).  Every compute call is
 *    asynchronous on `stream`; nothing synchronises except tc_stream_sync and
 *    the tc_memcpy_* calls given a NULL stream.
 *  - Threads and streams.  Calls that keep partial results between kernels
 *    (split reductions, vecmat, split-K products, scans, sorts, fused sums)
 *    take that scratch, and the ticket counters some of them use, from
 *    blocks owned by the (device, stream) pair they are called with.  Calls
 *    on different streams, from any threads, therefore share nothing and may
 *    run at the same time.  A stream belongs to one host thread at a time,
 *    as Metal's per-thread device and queue do (src/tensors/backend.rs:
 *    410-412): two threads enqueueing on one stream could interleave one
 *    call's kernels with another's.  tc_ctx_create gives a thread a stream
 *    of its own; tc_ctx_destroy frees that stream's blocks.  The scratch of
 *    a stream grows on demand with cudaMalloc, which must not happen while
 *    the stream is being captured into a CUDA graph: make one call of each
 *    size before capturing.
 *  - Sizes, offsets and strides count ELEMENTS (as `Strided` does,
 *    src/tensors/backend.rs:196-203), never bytes, except where named `bytes`.
 *  - Shapes have at most TC_MAX_RANK axes (src/tensors/layout.rs:16).
 *  - Scalars of the element type travel as `double`: every f32, f16 and bf16
 *    value is exact in f64, and the callee rounds nothing on the way in.
 */
#ifndef TCCUDA_H
#define TCCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TC_MAX_RANK 6

/* ---- status codes ------------------------------------------------------ */
enum tc_status {
  TC_OK = 0,
  TC_EINVAL = 1,   /* bad argument: shape, stride, dtype, op or size      */
  TC_ERANGE = 2,   /* a layout reads or writes past its storage           */
  TC_ENOMEM = 3,   /* device or pinned allocation failed                  */
  TC_ECUDA = 4,    /* a CUDA runtime/driver call or kernel launch failed  */
  TC_ENCCL = 5,    /* an NCCL call failed or NCCL could not be loaded     */
  TC_ETIMEOUT = 6, /* a bounded device-side wait gave up                  */
  TC_ENOTSUP = 7   /* the combination is not provided by this build       */
};

/* ---- element types ----------------------------------------------------- */
/* The `Real` element types the Cuda backend implements Kernels<T> for
 * (src/tensors/kernels.rs:808-829): f32, f16, bf16.  U32 is the index type
 * arg_reduce returns (src/tensors/kernels.rs:1187). */
enum tc_dtype { TC_F32 = 0, TC_F16 = 1, TC_BF16 = 2, TC_U32 = 3 };

/* ---- operation enums: the discriminants of the reference's enums -------- */
/* BinaryOp, src/tensors/kernels.rs:32-38 */
enum tc_binary_op { TC_ADD = 0, TC_SUB = 1, TC_MUL = 2, TC_DIV = 3, TC_REM = 4 };
/* Compare, src/tensors/kernels.rs:106-121 */
enum tc_compare {
  TC_MIN = 0, TC_MAX = 1, TC_MAX_SHARE = 2, TC_LESS = 3,
  TC_LESS_EQUAL = 4, TC_GREATER = 5, TC_GREATER_EQUAL = 6
};
/* Reduce, src/tensors/kernels.rs:183-188 */
enum tc_reduce { TC_SUM = 0, TC_RMIN = 1, TC_RMAX = 2 };
/* Pairwise, src/tensors/kernels.rs:411-416: which enum `op` belongs to */
enum tc_pairwise { TC_PAIR_ARITHMETIC = 0, TC_PAIR_COMPARE = 1, TC_PAIR_POWER = 2 };
/* AxisReduction, src/tensors/kernels.rs:449-457 */
enum tc_axis_reduction { TC_AXIS_FOLD = 0, TC_AXIS_MEAN = 1, TC_AXIS_VARIANCE = 2 };
/* Transposed, src/tensors/kernels.rs:462-467, plus "neither" */
enum tc_transposed { TC_TRANS_NONE = 0, TC_TRANS_LEFT = 1, TC_TRANS_RIGHT = 2 };

/* One block of an assemble or strided write: `shape` copied from `source`
 * (holding `source_len` elements) at (from_offset, from_strides) to the
 * target at (to_offset, to_strides).  Mirrors `Region`
 * (src/tensors/backend.rs:205-221) with `Strided` flattened in. */
typedef struct tc_region {
  const void *source;
  size_t source_len;
  uint32_t rank;
  size_t shape[TC_MAX_RANK];
  size_t from_offset;
  size_t from_strides[TC_MAX_RANK];
  size_t to_offset;
  size_t to_strides[TC_MAX_RANK];
} tc_region;

/* ---- errors, devices, memory, streams ----------------------------------- */
/* The message of this thread's last failure (NUL-terminated, truncated to
 * `len`).  Returns the status of that failure. */
int tc_last_error(char *buf, size_t len);
/* Library build string: version, arch, and which kernels are compiled in. */
const char *tc_build_info(void);
/* Make `device` current for this thread (Metal's per-thread device,
 * src/metal/device.rs; env TC_CUDA_DEVICE picks the default). */
int tc_set_device(int device);
int tc_device_count(int *count);

/* SMs of the current device (148 on B200): the launch geometry's unit. */
int tc_sm_count(int *count);

/* A device and a stream of its own for one host thread (Metal's per-thread
 * device and command queue, src/tensors/backend.rs:391-412 and
 * src/metal/device.rs).  Pass the stream tc_ctx_stream gives to every call
 * the thread makes; the stream keys its own scratch, ticket counters and
 * stream-ordered pool frees.  tc_ctx_destroy waits for the stream, frees its
 * scratch and counters, and destroys it. */
typedef struct tc_ctx tc_ctx;
int tc_ctx_create(int device, tc_ctx **out);
int tc_ctx_stream(tc_ctx *ctx, void **stream);
int tc_ctx_device(tc_ctx *ctx, int *device);
int tc_ctx_destroy(tc_ctx *ctx);

/* Device storage: `Backend::Storage<T>` (src/tensors/backend.rs:84).
 * Served from a per-device caching pool, as Metal's src/metal/pool.rs.
 * tc_free returns a block for immediate reuse: no queued work may still use
 * it.  tc_free_async returns it in `stream`'s order (work queued on `stream`
 * before the call may still use it): a later tc_malloc_async on the same
 * stream may take it at once, a request on another stream only with that
 * stream made to wait for the freeing stream's work, and tc_malloc only once
 * that work has completed.  This is how a storage dropped while its
 * kernels are queued (Drop of `CudaStorage`) goes back to the pool. */
int tc_malloc(void **out_dev, size_t bytes);
int tc_malloc_async(void **out_dev, size_t bytes, void *stream);
int tc_free(void *dev);
int tc_free_async(void *dev, void *stream);
/* Release every cached block back to CUDA. */
int tc_pool_trim(void);
/* Counters since the library loaded: cudaMalloc calls the library made
 * (pool misses, scratch and counter growth, peer buffers), and requests for
 * a stream's scratch.  The counterpart of the reference's allocation
 * counters (src/counters.rs:100-160). */
int tc_alloc_counts(uint64_t *device_allocations, uint64_t *scratch_requests);
/* Pinned host staging, for the lazily filled host mirror behind
 * `Backend::as_slice` (src/tensors/backend.rs:96-99). */
int tc_host_alloc(void **out_host, size_t bytes);
int tc_host_free(void *host);

/* `Backend::store`/`from_vec` (src/tensors/backend.rs:88-93): upload. */
int tc_memcpy_h2d(void *dst_dev, const void *src_host, size_t bytes, void *stream);
/* `Backend::as_slice`/`as_mut_slice` (src/tensors/backend.rs:96-104):
 * download; with a NULL stream it returns after the copy is complete. */
int tc_memcpy_d2h(void *dst_host, const void *src_dev, size_t bytes, void *stream);
/* `Backend::duplicate` (src/tensors/backend.rs:111): device copy, no wait. */
int tc_memcpy_d2d(void *dst_dev, const void *src_dev, size_t bytes, void *stream);
int tc_memset(void *dst_dev, int value, size_t bytes, void *stream);
int tc_stream_sync(void *stream);

/* ---- layout copies (bits; any element width 1, 2, 4, 8 or 16 bytes) ---- */
/* `Backend::strided_copy` (src/tensors/backend.rs:141-145; Host
 * strided_copy_slice :255-274): the elements a layout of `shape` reads from
 * `src` (`src_len` elements) at (src_offset, src_strides), written row-major
 * into `dst` (prod(shape) elements).  TC_ERANGE if the layout reaches past
 * src_len (check_strided, :225-252). */
int tc_strided_copy(size_t elem_bytes, uint32_t rank, const size_t *shape,
                    const void *src, size_t src_len, size_t src_offset,
                    const size_t *src_strides, void *dst, void *stream);

/* `Backend::strided_write` (src/tensors/backend.rs:170-173; Host
 * strided_write_slice :277-300): copy one region into `target`
 * (`target_len` elements) in place. */
int tc_strided_write(size_t elem_bytes, void *target, size_t target_len,
                     const tc_region *region, void *stream);

/* `Backend::assemble` (src/tensors/backend.rs:157-160; Host assemble_slices
 * :303-323): a new storage of `len` elements built from `n` regions.
 * Regions whose targets are disjoint boxes (a concatenation's) may share a
 * launch; otherwise they are written in order, so where two overlap the
 * later one's values remain, as the Host leaves them.  Elements no region
 * writes are left as they were in `dst` (the reference leaves them
 * unspecified). */
int tc_assemble(size_t elem_bytes, void *dst, size_t len, const tc_region *regions,
                size_t n, void *stream);

/* ---- same-shape elementwise (Kernels<T>, src/tensors/kernels.rs:832-863) */
/* `vector_elementwise`/`matrix_elementwise`: out = a op b. */
int tc_elementwise(int dtype, int op, const void *a, const void *b, void *out,
                   size_t n, void *stream);
/* `vector_broadcast`/`matrix_broadcast`: out = a op s, or s op a when
 * scalar_left. */
int tc_broadcast_scalar(int dtype, int op, const void *a, double scalar,
                        int scalar_left, void *out, size_t n, void *stream);
/* `vector_compare`/`matrix_compare` (Compare::value, kernels.rs:138-153). */
int tc_compare(int dtype, int cmp, const void *a, const void *b, void *out,
               size_t n, void *stream);
/* `vector_compare_scalar`/`matrix_compare_scalar`. */
int tc_compare_scalar(int dtype, int cmp, const void *a, double scalar,
                      int scalar_left, void *out, size_t n, void *stream);
/* `vector_clamp`/`matrix_clamp` (kernels.rs:863): TC_EINVAL unless
 * low <= high. */
int tc_clamp(int dtype, const void *a, double low, double high, void *out,
             size_t n, void *stream);
/* `vector_reduce` (kernels.rs:867): the whole vector folded into
 * out_dev[0] (one element of `dtype`); an empty vector gives the identity. */
int tc_vector_reduce(int dtype, int op, const void *a, size_t n, void *out_dev,
                     void *stream);
/* `dot` (kernels.rs:897): sum of a[i]*b[i], f32 accumulate, into out_dev[0]. */
int tc_dot(int dtype, const void *a, const void *b, size_t n, void *out_dev,
           void *stream);

/* ---- the other vector/matrix methods (kernels.rs:870-891, 941-1070) ----- */
/* SortOrder, src/tensors/kernels.rs:252-255 */
enum tc_sort_order { TC_ASCENDING = 0, TC_DESCENDING = 1 };
/* `vector_prefix_sum` (kernels.rs:870; Host vector.rs:578-589,
 * compact::prefix_sum): out[i] = a[0] + ... + a[i], an f32 running total
 * rounded once per output to `dtype`.  Three launches; uses the stream's
 * scratch. */
int tc_prefix_sum(int dtype, const void *a, void *out, size_t n, void *stream);
/* `vector_sort` (kernels.rs:873; Host vector.rs:874-886): the n values in
 * SortOrder's total order (f32::total_cmp / half's total_cmp: -NaN < -inf <
 * ... < -0 < +0 < ... < +inf < +NaN).  TC_EINVAL beyond 2^31-1 elements.
 * `out` may be `a` (sorted in place).  Uses the stream's scratch. */
int tc_sort(int dtype, int order, const void *a, void *out, size_t n, void *stream);
/* `vector_unary`/`matrix_unary` (kernels.rs:876, 941; Host 1257-1268):
 * out = f(a), f a tc_analytic, computed in f32 and rounded once. */
int tc_unary(int dtype, int f, const void *a, void *out, size_t n, void *stream);
/* `vector_unary_dual`/`matrix_unary_dual` (kernels.rs:891, 950; Host
 * 1284-1304): out_value = f(value), out_tangent = f'(value) * tangent,
 * the derivative's rule (Analytic::derivative, kernels.rs:357-387) and the
 * product each rounded to `dtype` per operation. */
int tc_unary_dual(int dtype, int f, const void *value, const void *tangent, void *out_value,
                  void *out_tangent, size_t n, void *stream);
/* `vector_power`/`matrix_power` (kernels.rs:884, 944; Host
 * pow_elementwise): out = powf(a, b), rounded once. */
int tc_power(int dtype, const void *a, const void *b, void *out, size_t n, void *stream);
/* `vector_power_scalar`/`matrix_power_scalar` (kernels.rs:888, 947):
 * out = powf(a, scalar), or powf(scalar, a) when scalar_left. */
int tc_power_scalar(int dtype, const void *a, double scalar, int scalar_left, void *out,
                    size_t n, void *stream);

/* ---- windowed matrix methods (kernels.rs:998-1028) ----------------------- */
/* `correlate` (kernels.rs:998; Host correlate_values, kernels.rs:1720-1751):
 * the valid cross-correlation of the rows x cols `input` with the
 * window_rows x window_cols `window` (reversed in both axes when `flip`),
 * into the (rows-window_rows+1) x (cols-window_cols+1) `out`.  Each output
 * sums its taps in row-major order with a rounded product and a rounded sum
 * per tap, in f32 for f16/bf16 with one rounding at the end: the Host's
 * bits, except when the taps number 4096 or more and the outputs are few,
 * where a block shares each output's sum (deterministic, within an f32
 * sum's rounding).  TC_EINVAL unless the window fits and is not empty. */
int tc_correlate(int dtype, size_t rows, size_t cols, size_t window_rows, size_t window_cols,
                 int flip, const void *input, const void *window, void *out, void *stream);
/* `correlate_window_gradient` (kernels.rs:1008, 1544-1551): correlate of
 * the input with the adjoint as the window, no flip; `out` has the
 * window's shape (rows-adjoint_rows+1) x (cols-adjoint_cols+1). */
int tc_correlate_window_gradient(int dtype, size_t rows, size_t cols, size_t adjoint_rows,
                                 size_t adjoint_cols, const void *input, const void *adjoint,
                                 void *out, void *stream);
/* `correlate_input_gradient` (kernels.rs:1017; Host 1754-1788): the full
 * correlation of the adjoint with the window, the taps reversed when the
 * forward pass did not reverse them, into the (adjoint_rows+window_rows-1)
 * x (adjoint_cols+window_cols-1) `out`; taps whose adjoint index falls
 * outside are skipped, as on the Host, so the bits are the Host's. */
int tc_correlate_input_gradient(int dtype, size_t adjoint_rows, size_t adjoint_cols,
                                size_t window_rows, size_t window_cols, int forward_flip,
                                const void *adjoint, const void *window, void *out, void *stream);
/* `pad` (kernels.rs:1025; Host 1575-1601): `input` surrounded by pad_rows
 * and pad_cols zeros on every side, (rows+2*pad_rows) x (cols+2*pad_cols). */
int tc_pad(int dtype, size_t rows, size_t cols, size_t pad_rows, size_t pad_cols,
           const void *input, void *out, void *stream);
/* `flip` (kernels.rs:1028; Host 1531-1542): both axes reversed. */
int tc_flip(int dtype, size_t rows, size_t cols, const void *input, void *out, void *stream);

/* ---- moments and distributions (kernels.rs:1035-1070) -------------------- */
/* Axis, src/tensors/kernels.rs:482-487: Rows folds each row (one result per
 * row), Columns each column. */
enum tc_axis { TC_ROWS = 0, TC_COLUMNS = 1 };
/* Family and Statistic, src/tensors/kernels.rs:536-576. */
enum tc_family { TC_NORMAL = 0, TC_INVERSE_GAUSSIAN = 1 };
enum tc_statistic { TC_PDF = 0, TC_CDF = 1, TC_PPF = 2 };
/* `vector_moments`/`matrix_moments` (kernels.rs:1035-1038; Host
 * statistics/mod.rs:419-441): out_dev[0] = the mean of the n elements,
 * out_dev[1] = the sum of their squared deviations from it (two passes, f32
 * for every type, each rounded once to `dtype`); NaNs when n is 0. */
int tc_moments(int dtype, const void *a, size_t n, void *out_dev, void *stream);
/* `matrix_axis_moments` (kernels.rs:1042; Host statistics/mod.rs:451-520):
 * one mean and one deviation sum per row (TC_ROWS, `rows` results) or per
 * column (TC_COLUMNS, `cols` results) of the row-major rows x cols `a`. */
int tc_axis_moments(int dtype, size_t rows, size_t cols, int axis, const void *a, void *means,
                    void *deviations, void *stream);
/* `vector_distribution`/`matrix_distribution` (kernels.rs:1046-1061; Host
 * Distribution::evaluate, statistics/mod.rs:285-303): the pdf, cdf or ppf
 * of the Normal(first = mean, second = stddev) or InverseGaussian(first =
 * mean, second = shape) distribution at each element, evaluated in f64
 * (statistics/special.rs) and rounded once to `dtype`.  first and second are
 * element-type values. */
int tc_distribution(int dtype, int family, int statistic, const void *a, size_t n, double first,
                    double second, void *out, void *stream);
/* `matrix_axis_distribution` (kernels.rs:1063): the same with one parameter
 * pair per row (TC_ROWS) or per column (TC_COLUMNS), read from the device
 * vectors `first` and `second` of the element type. */
int tc_axis_distribution(int dtype, size_t rows, size_t cols, int axis, int family, int statistic,
                         const void *a, const void *first, const void *second, void *out, void *stream);

/* ---- strided kernels (src/tensors/kernels.rs:1162-1187) ------------------ */
/* `strided_binary` (kernels.rs:1162; Host strided::binary, strided.rs:29):
 * op(a, b) over the common `shape`, each operand read through its own
 * offset and strides (a zero stride repeats an element), into a new
 * row-major `out`.  `kind` is tc_pairwise; `op` a tc_binary_op or
 * tc_compare (ignored for TC_PAIR_POWER).  a_len/b_len bound the reads. */
int tc_strided_binary(int dtype, int kind, int op, uint32_t rank, const size_t *shape,
                      const void *a, size_t a_len, size_t a_offset, const size_t *a_strides,
                      const void *b, size_t b_len, size_t b_offset, const size_t *b_strides,
                      void *out, void *stream);

/* `reduce_axes` (kernels.rs:1175; Host strided::reduce, strided.rs:105-184):
 * `input` folded over `axes` (distinct, ascending, n_axes of them), one
 * result per index of the kept axes in row-major order.  `kind` is
 * tc_axis_reduction; `op` the tc_reduce of a fold; `divisor` the
 * Variance divisor.  f32/f16/bf16 accumulate in f32 and round once.  Every
 * slice holds at least one element (the front-end, reduction.rs:126-143,
 * fills empty results itself). */
int tc_reduce_axes(int dtype, uint32_t rank, const size_t *shape, const void *input,
                   size_t input_len, size_t offset, const size_t *strides,
                   uint32_t n_axes, const uint32_t *axes, int kind, int op,
                   size_t divisor, void *out, void *stream);

/* `arg_reduce` (kernels.rs:1187; Host strided::arg_reduce, strided.rs:201):
 * the u32 position along `axis` of each slice's max (op = TC_RMAX) or min
 * (TC_RMIN): first position on ties, NaNs passed over, all-NaN -> 0. */
int tc_arg_reduce(int dtype, uint32_t rank, const size_t *shape, const void *input,
                  size_t input_len, size_t offset, const size_t *strides, uint32_t axis,
                  int op, uint32_t *out, void *stream);

/* ---- products ------------------------------------------------------------ */
/* `matmul` (kernels.rs:956), `matmul_add` (:963) and `matmul_transposed_add`
 * (:975-985), row-major:  C[rows x cols] (+)= op(A)·op(B) with inner
 * dimension `inner`.  transposed = TC_TRANS_NONE: A is rows x inner, B is
 * inner x cols; TC_TRANS_LEFT: A is stored inner x rows (Aᵀ·B);
 * TC_TRANS_RIGHT: B is stored cols x inner (A·Bᵀ).  accumulate != 0 adds
 * into C (the moved-in addend); otherwise C is overwritten.  f32 runs FP32
 * CUDA-core tiles; f16/bf16 run the tcgen05 tensor-core kernel with f32
 * accumulation, rounding each output once (compact::matmul,
 * src/compact.rs:232-253). */
int tc_matmul(int dtype, int transposed, size_t rows, size_t inner, size_t cols,
              const void *a, const void *b, void *c, int accumulate, void *stream);
/* `matmul_epilogue` (kernels.rs:1137-1150, reached through
 * Program::run_matmul, fused/mod.rs:1143) for the programs a dense layer's
 * forward and backward build, applied in this order to the product P:
 *   share_of (not null): P = P * MaxShare(share_of, 0), the ReLU's backward
 *     rule (Compare::MaxShare, kernels.rs:138-153; tape/mod.rs:1110-1130);
 *     share_of is laid out as c
 *   bias (not null): P = P + bias[row] (the add of b ⊗ ones)
 *   c = P, and relu_out (not null) = max(P, 0) (Compare::Max against 0).
 * Each step rounds to the element type as the separate operations do: the
 * product once (as tc_matmul), then each op; max is exact.  f16/bf16 run
 * it inside the tensor-core GEMM's epilogue; f32, and shapes the
 * tensor-core tiles refuse, run the product and then one pass over it. */
int tc_matmul_epilogue(int dtype, int transposed, size_t rows, size_t inner, size_t cols,
                       const void *a, const void *b, const void *share_of, const void *bias,
                       void *c, void *relu_out, void *stream);

/* `matvec`/`matvec_add` (kernels.rs:901-908; matrix.rs:675-730):
 * y[rows] (+)= M[rows x cols]·x[cols]. */
int tc_matvec(int dtype, size_t rows, size_t cols, const void *m, const void *x,
              void *y, int accumulate, void *stream);
/* `vecmat` (kernels.rs:899; vector.rs:491-505): y[cols] = xᵀ[rows]·M. */
int tc_vecmat(int dtype, size_t rows, size_t cols, const void *x, const void *m,
              void *y, void *stream);
/* tc_vecmat for callers that cannot allocate device memory.  No counterpart
 * in the reference.  Some callers' device memory is already claimed by
 * another allocator (a framework's caching allocator that holds the GPU's
 * memory, or a fixed arena sized at start-up), so a cudaMalloc from this
 * library would fail or break that allocator's budget; others run under a
 * hard latency budget, where cudaMalloc may block and synchronise the
 * device.  Same row split, kernels and bits as tc_vecmat, but the split's
 * f32 partial sums (shares x cols x 4 bytes) live in a 1 MiB static device
 * array of the library, which every GPU that loads the library holds until
 * exit, instead of the stream's scratch; the call makes no cudaMalloc,
 * cudaFree or other allocating call (its first call on a device looks the
 * array's address up once, with cudaGetSymbolAddress).  TC_ERANGE, before
 * any launch, when a shape's partials would not fit in 1 MiB.  Every call on
 * a device shares the array and it keeps the last call's partials: calls
 * that overlap on the GPU (other streams, other threads) race on it, so
 * order them, e.g. on one stream.  Nothing in the array has to start at
 * zero: each partial is written before it is read. */
int tc_vecmat_noalloc(int dtype, size_t rows, size_t cols, const void *x,
                      const void *m, void *y, void *stream);

/* ---- optimizer updates (the fused programs of src/optim.rs) ------------- */
/* Adam's fused program (optim.rs:1048-1099), run in place over n elements:
 * resumed = 0 is the first step (m, v are written fresh), resumed = 1 every
 * later one.  rate, beta1, beta2, eps and the two corrections
 * 1/(1-beta^t) are values of the element type, computed on the host as
 * Adam::update does (optim.rs:1106-1124).  Every operation rounds to the
 * element type, in the program's order. */
int tc_adam(int dtype, size_t n, void *p, const void *g, void *m, void *v, int resumed,
            double rate, double beta1, double beta2, double eps, double first_correction,
            double second_correction, void *stream);
/* The same program over several parameters in one launch, as Adam::update
 * steps every parameter with the same coefficients (optim.rs:1106-1140);
 * each tensor's result is the one tc_adam gives it.  At most 16 tensors go
 * in one launch; longer lists take several. */
typedef struct tc_adam_tensor {
  void *p;
  const void *g;
  void *m;
  void *v;
  size_t n;
} tc_adam_tensor;
int tc_adam_multi(int dtype, const tc_adam_tensor *tensors, size_t count, int resumed,
                  double rate, double beta1, double beta2, double eps, double c1, double c2,
                  void *stream);
/* Sgd's fused program (optim.rs:773-787): p <- p - g·rate. */
int tc_sgd(int dtype, size_t n, void *p, const void *g, double rate, void *stream);
/* The other rules' fused programs, one pass each, p and the state updated in
 * place; every operation rounded to `dtype` in the order the rule's builder
 * gives it; the coefficients are values of `dtype`.
 * Momentum (optim.rs:826-846): v <- v·momentum + g; p <- p - step·rate with
 * step = v, or g + v·momentum when `nesterov`. */
int tc_momentum(int dtype, size_t n, void *p, const void *g, void *velocity, double rate,
                double momentum, int nesterov, void *stream);
/* AdaGrad (optim.rs:892-904, descend 1146-1159): s <- s + g·g;
 * p <- p - (g / (sqrt(s) + eps))·rate (the rule's eps is 1e-8 in dtype). */
int tc_adagrad(int dtype, size_t n, void *p, const void *g, void *total, double rate, double eps,
               void *stream);
/* RmsProp (optim.rs:948-964): s <- s·decay + (g·g)·(1 - decay), 1 - decay
 * rounded to dtype; p as AdaGrad (the rule's decay is 0.9, eps 1e-8). */
int tc_rmsprop(int dtype, size_t n, void *p, const void *g, void *mean_square, double rate,
               double decay, double eps, void *stream);

/* Status of bounded device-side waits since the library loaded: TC_ETIMEOUT
 * (and *fault = 1) if a tensor-core GEMM gave up waiting on its pipeline, or
 * a data-parallel step gave up waiting for another rank's flag, and
 * returned early; TC_OK otherwise.  No counterpart in the reference
 * (Metal reports async errors at the next sync, src/metal/mod.rs:17-21). */
int tc_device_status(int *fault);
/* Clear those records.  No counterpart in the reference. */
int tc_device_status_reset(void);
/* How long a pipeline wait of the tensor-core GEMM lasts before its CTA
 * gives up (ns; 0 restores the default of 2 s).  Waits for in-flight copies
 * and products while giving up always allow 2 s.  Lets a test make a wait
 * run out on purpose; no counterpart in the reference. */
int tc_set_wait_limit(unsigned long long ns);
/* How long a data-parallel step's kernels wait for another rank's flag
 * (ns; 0 restores the default of 5 s); on expiry they record the fault and
 * return, and the step's results are not valid.  Lets a test make a wait
 * run out on purpose; no counterpart in the reference. */
int tc_set_peer_wait_limit(unsigned long long ns);

/* ---- layout helpers (host only; src/tensors/layout.rs) ------------------ */
/* `coalesce` (layout.rs:419-446) for n_ops operands whose strides are
 * strides[op*rank + axis]; writes the merged shape and strides (same
 * packing, out_rank axes).  Exposed so the descriptor builder can be tested
 * without a GPU. */
int tc_coalesce(uint32_t rank, const size_t *shape, uint32_t n_ops, const size_t *strides,
                uint32_t *out_rank, size_t *out_shape, size_t *out_strides);

/* ---- the tape and the optimizer, run natively (host-side mirror) --------- */
/* One training step of a dense ReLU network exactly as the reference's
 * reverse-mode tape and Adam rule run it on any backend
 * (benches/nn_ops.rs:877-921; tape rules src/tensors/tape/mod.rs:979-988,
 * 1026-1033, 1110-1130, 1174, 1195-1216, 1286-1300; Adam src/optim.rs:
 * 1001-1140), driven from C++ through the kernels above.  There is no
 * single-call counterpart in the reference: it is the Rust code above the
 * Kernels<T> boundary, restated so the path can run where no Rust toolchain
 * exists.  dims[0..layers] are the widths, inputs first; activations are
 * [width x batch], one column per sample.  global_batch scales the loss (the
 * sum over ranks of a data-parallel step's gradients is then the global
 * gradient). */
typedef struct tc_mlp tc_mlp;
typedef struct tc_comm tc_comm;
int tc_mlp_create(int dtype, uint32_t layers, const uint32_t *dims, uint32_t batch,
                  uint32_t global_batch, double rate, double beta1, double beta2, double eps,
                  tc_mlp **out);
int tc_mlp_destroy(tc_mlp *mlp);
/* dir = 0 uploads layer `layer`'s weight [dims[l+1] x dims[l]] and bias from
 * the host, dir = 1 downloads them. */
int tc_mlp_params(tc_mlp *mlp, uint32_t layer, void *w_host, void *b_host, int dir);
/* The gradients the last step computed.  After a step with a communicator
 * of more than 8 ranks they are summed over the ranks; after a sharded step
 * (2-8 ranks) only this rank's shard of each layer's block holds the sum
 * (tc_mlp_block says where), the rest this rank's own part of it. */
int tc_mlp_grads(tc_mlp *mlp, uint32_t layer, void *gw_host, void *gb_host);
/* Layer `layer`'s block of the flat parameter, gradient and moment buffers:
 * [W (row-major) | b], b starting at element *bias_at, the block *len
 * elements long (padding zero).  Rank r of P (P <= 8) owns elements
 * [r*len/P, (r+1)*len/P) of it in a sharded step. */
int tc_mlp_block(tc_mlp *mlp, uint32_t layer, size_t *len, size_t *bias_at);
/* Skip the adjoints nothing reads (inputs', targets', ones'); off by
 * default, as the tape computes them. */
int tc_mlp_prune_leaves(tc_mlp *mlp, int prune);
/* Forward, loss into loss_dev[0] if not NULL, backward, then Adam.  With a
 * communicator of 2-8 ranks the optimizer is sharded: as soon as the
 * backward pass is done with a layer, a second stream has this rank update
 * its shard of the layer's block with the gradient summed over the ranks,
 * and every rank receives every shard's new parameters, beside the rest of
 * the pass.  After tc_mlp_attach to that communicator one kernel per layer
 * does this over NVLink peer memory: it loads every rank's gradient of this
 * rank's shard (peer loads), sums them in rank order in f32, rounds once,
 * runs Adam on the shard and stores the new parameters into every rank's
 * copy (peer stores); flags in memory every rank maps order the steps
 * between the ranks, with bounded waits that report through
 * tc_device_status.  Otherwise NCCL reduce-scatters the gradients and
 * all-gathers the parameters (NCCL's bf16 sums round per hop).  With more
 * ranks each layer's gradients are all-reduced and every rank runs Adam on
 * everything.  x, y are device buffers.  The products'
 * split-K partials, vecmat's row split and the loss's sum use the scratch of
 * `stream` and of the handle's own side stream. */
int tc_mlp_step(tc_mlp *mlp, const void *x_dev, const void *y_dev, tc_comm *comm, void *loss_dev,
                void *stream);
/* Move the handle's flat parameters and gradients into buffers every rank
 * of `comm` (2-8 ranks) maps over NVLink (CUDA IPC), for steps over `comm`
 * that exchange through peer memory.  Collective: every rank attaches, in
 * the same order as its other collectives.  An attached handle's
 * tc_mlp_destroy is collective too, and `comm` must outlive it.  No
 * counterpart in the reference, which runs on one device. */
int tc_mlp_attach(tc_mlp *mlp, tc_comm *comm);

/* ---- a reverse-mode tape over device tensors (src/tensors/tape) --------- */
/* The tensor-level rules of tensorcrate's tape, recorded in creation order
 * and replayed backwards through the kernels above, for callers that drive
 * the backend without the Rust tape (Tape, tape/mod.rs:349-549).  Every var
 * is a tensor of the tape's element type; values and adjoints are device
 * buffers the tape owns (a leaf's value is the caller's), all work on the
 * tape's stream.  Shapes broadcast as layout.rs:330-363 (right-aligned,
 * extents equal or one).  Each call returns its result's var id in *out. */
typedef struct tc_tape tc_tape;
int tc_tape_create(int dtype, void *stream, tc_tape **out);
int tc_tape_destroy(tc_tape *tape);
/* A leaf (a parameter or an input): the tape reads `dev` in place. */
int tc_tape_leaf(tc_tape *tape, const void *dev, uint32_t rank, const size_t *shape, uint32_t *out);
/* a op b, op = TC_ADD/SUB/MUL/DIV, broadcast; backward sums each operand's
 * share to its shape (TensorVar::binary and sum_to_shape, tape/tensor.rs:
 * 23-37, 128-160). */
int tc_tape_binary(tc_tape *tape, int op, uint32_t a, uint32_t b, uint32_t *out);
/* max(a, 0); backward weights the adjoint by MaxShare(a, 0): 1, 1/2 at 0,
 * 0 (relu / select_scalar, tape/tensor.rs:272-300). */
int tc_tape_relu(tc_tape *tape, uint32_t a, uint32_t *out);
/* a * factor, factor a value of the element type (tape/tensor.rs:317). */
int tc_tape_scale(tc_tape *tape, uint32_t a, double factor, uint32_t *out);
/* The sum (mean != 0: the mean) over `axes` (distinct, ascending), the
 * folded axes dropped or kept at one; backward spreads the adjoint over each
 * slice, a mean's scaled first by `share` = 1/count as a value of the
 * element type (sum_axes / mean_axes, tape/tensor.rs:581-620). */
int tc_tape_sum_axes(tc_tape *tape, uint32_t a, uint32_t n_axes, const uint32_t *axes, int mean, int keep_dims,
                     double share, uint32_t *out);
/* [m x k]·[k x n]; backward Ā += C̄·Bᵀ, B̄ += Aᵀ·C̄ into the current adjoint
 * or zeros (MatrixVar::matmul, tape/mod.rs:1190-1216). */
int tc_tape_matmul(tc_tape *tape, uint32_t a, uint32_t b, uint32_t *out);
/* The sum of every element, a one-element var; backward fills (MatrixVar::
 * sum, tape/mod.rs:1286-1296). */
int tc_tape_sum(tc_tape *tape, uint32_t a, uint32_t *out);
/* A var's value: device pointer, rank and shape (shape may be NULL). */
int tc_tape_value(tc_tape *tape, uint32_t var, const void **dev, uint32_t *rank, size_t *shape);
/* Clear every adjoint, seed the one-element `var` with one and apply every
 * rule from it back to the first node (Var::backward_with, tape/mod.rs:
 * 507-521). */
int tc_tape_backward(tc_tape *tape, uint32_t var);
/* A var's adjoint after backward; NULL when no contribution reached it. */
int tc_tape_adjoint(tc_tape *tape, uint32_t var, const void **dev);

/* ---- fused elementwise programs (Kernels::fused, kernels.rs:1077-1082) --- */
/* One instruction of a fused::Program (fused/mod.rs:290-313).  `code` is a
 * tc_instr_code; registers are below 16.  Load reads place `slot` (one per
 * distinct load of the program, in the program's order of them, as
 * Space::places lists them); Store writes output `slot`; Const's `value` is
 * a value of the program's type; `op` is a tc_binary_op, tc_compare or
 * tc_analytic. */
enum tc_instr_code {
  TC_I_LOAD = 0, TC_I_CONST = 1, TC_I_BINARY = 2, TC_I_UNARY = 3, TC_I_CMP = 4, TC_I_STORE = 5
};
/* Analytic, src/tensors/kernels.rs:293-308 */
enum tc_analytic {
  TC_SIN = 0, TC_COS = 1, TC_TAN = 2, TC_SEC = 3, TC_CSC = 4, TC_ARCSIN = 5, TC_ARCCOS = 6,
  TC_ARCTAN = 7, TC_EXP = 8, TC_LN = 9, TC_SINH = 10, TC_COSH = 11, TC_TANH = 12, TC_SQRT = 13
};
typedef struct tc_instr {
  uint8_t code, dst, a, b, op, slot;
  uint16_t reserved;
  float value;
} tc_instr;
/* Where one load reads (fused::Place, fused/mod.rs:3229-3238): element
 * (row, col) of the rows x cols space is data[offset + col*col_step + sum_k
 * c_k*steps[k]], c the row index decomposed over dims[0..lead) (outermost
 * first); `dtype` is the storage type of `data` (f32, f16 or bf16). */
typedef struct tc_place {
  const void *data;
  int dtype;
  uint32_t lead;
  size_t offset, col_step;
  size_t dims[TC_MAX_RANK - 1], steps[TC_MAX_RANK - 1];
} tc_place;
/* Run `program` (n_code instructions, at most 256) over a rows x cols space
 * in the program's type `dtype`: every instruction's result rounds to that
 * type, loads convert from their storage type to it, stores from it to
 * each output's storage type (out_dtypes), as the Host's interpreter does
 * (fused/mod.rs:4055-4260).  Outputs are row-major rows x cols.  An output
 * may be the storage a load reads (a tensor updated in place) when that
 * load reads it in order.  Unary functions other than Sqrt use CUDA's f32
 * functions (within 2 ulp of the exact value for f32; sec and csc are 1/cos
 * and 1/sin); everything else is exact.  At most 16 places and 8 outputs.
 * TC_ENOTSUP for an f64 storage or program type. */
int tc_fused(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
             const tc_place *places, uint32_t n_places, void *const *outputs,
             const int *out_dtypes, uint32_t n_outputs, void *stream);
/* RowStatistic, src/tensors/fused/mod.rs:544-553. */
enum tc_row_statistic_kind { TC_ROW_MEAN = 0, TC_ROW_DEVIATIONS = 1 };
/* One statistic a program reads (Builder::row_statistic,
 * fused/mod.rs:1832): loads of place `into_place` read, for each row of the
 * space, the mean or the sum of squared deviations of that row of place
 * `of_place` (as Kernels::row_moments gives them, rounded to the program's
 * type).  `into_place` needs no data. */
typedef struct tc_row_statistic {
  uint32_t of_place, into_place;
  int statistic;
} tc_row_statistic;
/* `fused_with_statistics` (kernels.rs:1103-1117): `program` with its row
 * statistics computed in the same launch, one warp per row: the warp reduces
 * the row's statistics (two passes, f32, as row_moments), then runs the
 * program over the row's elements, which read them.  At most 8 places may
 * be the source of statistics. */
int tc_fused_with_statistics(int dtype, size_t rows, size_t cols, const tc_instr *code,
                             uint32_t n_code, const tc_place *places, uint32_t n_places,
                             const tc_row_statistic *stats, uint32_t n_stats,
                             void *const *outputs, const int *out_dtypes, uint32_t n_outputs,
                             void *stream);
/* `fused_sum` (kernels.rs:1120-1135; Program::run_sum, fused/mod.rs:1048):
 * a program with one output of its own type, that output summed along
 * `axis` (TC_ROWS: one sum per row, `rows` results; TC_COLUMNS: one per
 * column) without being stored: each value rounded to the type, the sums
 * in f32, rounded once.  Columns with many rows use the stream's scratch
 * for their bands' partial sums. */
int tc_fused_sum(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                 const tc_place *places, uint32_t n_places, int axis, void *sums, void *stream);
/* `matmul_epilogue` for any program (kernels.rs:1137-1150; Host
 * host_matmul, fused/mod.rs:4754-4764): C = a.b (rows x inner by inner x
 * cols, rounded once to `dtype`, as tc_matmul), then `program` over the
 * rows x cols space with C as its input 0: places[0] says how input 0 is
 * read and its data is ignored (the product goes there).  The dense-layer
 * programs (bias, ReLU, ReLU's backward rule) run inside the GEMM's
 * epilogue instead: tc_matmul_epilogue. */
int tc_matmul_program(int dtype, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                      const tc_instr *code, uint32_t n_code, const tc_place *places, uint32_t n_places,
                      void *const *outputs, const int *out_dtypes, uint32_t n_outputs, void *stream);
/* `row_moments` (kernels.rs:1090-1101; Host fused/mod.rs:4030-4043): the
 * mean and sum of squared deviations of each row of the rows x cols matrix
 * `place` reads, converted to `dtype`, in f32, each rounded once. */
int tc_row_moments(int dtype, const tc_place *place, size_t rows, size_t cols, void *means,
                   void *deviations, void *stream);

/* ---- multi-GPU (NCCL over NVLink; no counterpart in the reference) ------ */
/* 128 opaque bytes (ncclUniqueId) for rank 0 to share with the others. */
int tc_comm_unique_id(uint8_t id[128]);
int tc_comm_init(int rank, int nranks, const uint8_t id[128], tc_comm **out);
int tc_comm_destroy(tc_comm *comm);
/* Concatenate every rank's `count` elements into recv (nranks*count). */
int tc_allgather(tc_comm *comm, int dtype, const void *send, void *recv, size_t count,
                 void *stream);
/* In-place all-reduce of `count` elements; op is tc_reduce. */
int tc_allreduce(tc_comm *comm, int dtype, void *buf, size_t count, int op, void *stream);
/* Reduce nranks*count elements of `send` over the ranks, rank r keeping
 * elements [r*count, (r+1)*count) of the result in `recv` (which may be
 * send + r*count); op is tc_reduce. */
int tc_reducescatter(tc_comm *comm, int dtype, const void *send, void *recv, size_t count, int op,
                     void *stream);
/* This rank and the number of ranks. */
int tc_comm_rank(tc_comm *comm, int *rank, int *nranks);

/* A device buffer of `bytes` on every rank, each rank also mapping every
 * other rank's (CUDA IPC over NVLink).  Create and destroy are collective:
 * every rank calls them, in the same order. */
typedef struct tc_peer_buffer tc_peer_buffer;
int tc_peer_buffer_create(tc_comm *comm, size_t bytes, tc_peer_buffer **out);
int tc_peer_buffer_pointer(tc_peer_buffer *buf, void **local_dev);
int tc_peer_buffer_destroy(tc_peer_buffer *buf);
/* Row-panel product with its all-gather fused into the GEMM (the sharded
 * form of Kernels::matmul, kernels.rs:956, for one large f16/bf16 product).
 * Collective: rank r passes its panel A_r [rows x inner] and the whole
 * B [inner x cols]; the tensor-core kernel stores each tile of
 * C_r = A_r.B into row block r of every rank's `c`, so that when the call's
 * work on `stream` completes, every rank's `c` holds the whole
 * C [nranks*rows x cols] (rounded once, as tc_matmul rounds).  The call ends
 * with a collective on `stream` that every rank's product precedes.  Every
 * rank writes every rank's `c`: a rank must be done with `c` from an earlier
 * call before any rank starts the next.  TC_ENOTSUP for f32 or a shape the
 * tensor-core tiles do not take (inner < 16, rows of A or B not 16-byte
 * aligned); TC_ERANGE when `c` is smaller than nranks*rows*cols elements. */
int tc_matmul_allgather(tc_comm *comm, int dtype, size_t rows, size_t inner, size_t cols,
                        const void *a, const void *b, tc_peer_buffer *c, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TCCUDA_H */
