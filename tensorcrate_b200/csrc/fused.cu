// fused.cu — fused elementwise programs (Kernels::fused, fused_sum,
// row_moments and fused_with_statistics, kernels.rs:1077-1135; fused::Program
// and Instr, fused/mod.rs:290-340, 502): a bytecode interpreter.
//
// Semantics follow the Host's interpreter (fused/mod.rs:4055-4260): the
// program computes in its type T, so every instruction's result is rounded
// to T (an f16 or bf16 program computes each operation in f32 and rounds);
// a load converts its storage type to T, a store converts T to the output's
// storage type; Binary and Cmp are the unfused kernels' scalar rules
// (BinaryOp, Compare::value), Unary the Analytic functions.
//
// The program (at most 256 instructions of 12 bytes) and the places travel
// as one kernel parameter block.  The 16 registers are a per-thread array,
// as in the reference's Metal shader.  Three launch shapes:
//   - fused: one thread per element of the rows x cols space;
//   - rows: one warp per row, for programs that read statistics of their
//     rows (fused_with_statistics: each row's mean and squared deviations
//     are reduced by the warp first, then the row's elements read them, so
//     the input crosses HBM once) and for fused_sum along rows;
//   - columns: fused_sum along columns, each thread a column over a band of
//     rows, the bands' partial sums added in band order by a second launch.
// This is the general path; the optimizers' programs have kernels of their
// own (optim.cu), and dense layers' epilogues run inside the GEMM.
#include <algorithm>

#include "analytic.cuh"

namespace tc {
namespace {

constexpr int MAX_CODE = 256, MAX_PLACES = 16, MAX_OUTPUTS = 8, REGISTERS = 16, MAX_STAT_SOURCES = 8;

struct Place {
  const void *data;
  int dtype;
  int lead;
  int in_order;  // element (row, col) is data[offset + row*cols + col]
  int stat;      // -1: read from memory; else 2*k + (0 mean, 1 deviations) of statistic source k
  long long offset, col_step;
  long long dims[TC_MAX_RANK - 1], steps[TC_MAX_RANK - 1];
};

struct Program {
  int n_code, n_places, n_outputs, n_stat_sources;
  long long rows, cols;
  tc_instr code[MAX_CODE];
  Place places[MAX_PLACES];
  int stat_source[MAX_STAT_SOURCES];  // the place each statistic source reads
  void *out[MAX_OUTPUTS];
  int out_dtype[MAX_OUTPUTS];
};

__device__ __forceinline__ float load_as(const void *p, int dtype, long long i) {
  if (dtype == TC_F32) return static_cast<const float *>(p)[i];
  const uint16_t h = static_cast<const uint16_t *>(p)[i];
  return dtype == TC_BF16 ? BF16T::load(h) : F16T::load(h);
}

__device__ __forceinline__ void store_as(void *p, int dtype, long long i, float v) {
  if (dtype == TC_F32) static_cast<float *>(p)[i] = v;
  else if (dtype == TC_BF16) static_cast<uint16_t *>(p)[i] = BF16T::store(v);
  else static_cast<uint16_t *>(p)[i] = F16T::store(v);
}

// Where a place reads element i = (row, col) of the space.
__device__ __forceinline__ long long place_at(const Place &pl, long long i, long long row, long long col) {
  if (pl.in_order) return pl.offset + i;
  long long at = pl.offset + col * pl.col_step;
  long long rest = row;
  for (int a = pl.lead - 1; a >= 0; --a) {
    const long long q = rest / pl.dims[a];
    at += (rest - q * pl.dims[a]) * pl.steps[a];
    rest = q;
  }
  return at;
}

// The value a place holds at (row, col), converted to T.
template <class T>
__device__ __forceinline__ float load_place(const Place &pl, long long i, long long row, long long col) {
  return T::load(T::store(load_as(pl.data, pl.dtype, place_at(pl, i, row, col))));
}

// Run the program on element i = (row, col).  `stats` holds the row's
// statistics (2 per source) for places that read one; `sink(slot, value)`
// receives every store.
template <class T, class Sink>
__device__ __forceinline__ void run_element(const Program &p, long long i, long long row, long long col,
                                            const float *stats, Sink &&sink) {
  float reg[REGISTERS];
  for (int k = 0; k < p.n_code; ++k) {
    const tc_instr in = p.code[k];
    float v;
    switch (in.code) {
      case TC_I_LOAD: {
        const Place &pl = p.places[in.slot];
        v = pl.stat >= 0 ? stats[pl.stat] : load_place<T>(pl, i, row, col);
        break;
      }
      case TC_I_CONST: v = T::load(T::store(in.value)); break;
      case TC_I_BINARY: v = T::load(T::store(binary_value(in.op, reg[in.a], reg[in.b]))); break;
      case TC_I_UNARY: v = T::load(T::store(analytic(in.op, reg[in.a]))); break;
      case TC_I_CMP: v = compare_value(in.op, reg[in.a], reg[in.b]); break;
      default:  // store
        sink(in.slot, reg[in.a]);
        continue;
    }
    reg[in.dst] = v;
  }
}

template <class T>
__global__ void __launch_bounds__(256) fused_kernel(const __grid_constant__ Program p) {
  const long long total = p.rows * p.cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / p.cols, col = i - row * p.cols;
    run_element<T>(p, i, row, col, nullptr,
                   [&](int slot, float v) { store_as(p.out[slot], p.out_dtype[slot], i, v); });
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// The mean and the sum of squared deviations of row `row` as `pl` reads it
// (converted to T), in f32, two passes over the row by one warp; both
// rounded to T, as Kernels::row_moments returns them (fused/mod.rs:4030-4043,
// statistics/mod.rs:451-491).
template <class T>
__device__ __forceinline__ void row_moments_of(const Place &pl, long long row, long long cols, float &mean,
                                               float &dev) {
  const int lane = threadIdx.x & 31;
  float s = 0.0f;
  for (long long c = lane; c < cols; c += 32) s = __fadd_rn(s, load_place<T>(pl, row * cols + c, row, c));
  const float m = __fdiv_rn(warp_sum(s), float(cols));
  float d = 0.0f;
  for (long long c = lane; c < cols; c += 32) {
    const float e = __fsub_rn(load_place<T>(pl, row * cols + c, row, c), m);
    d = __fadd_rn(d, __fmul_rn(e, e));
  }
  mean = T::load(T::store(m));
  dev = T::load(T::store(warp_sum(d)));
}

// One warp per row.  SUM: the row's values of output 0 are added (f32,
// rounded once to T) into sums[row] instead of stored.
template <class T, bool SUM>
__global__ void __launch_bounds__(256) fused_rows_kernel(const __grid_constant__ Program p, void *sums) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < p.rows; row += warps) {
    float stats[2 * MAX_STAT_SOURCES];
    for (int k = 0; k < p.n_stat_sources; ++k)
      row_moments_of<T>(p.places[p.stat_source[k]], row, p.cols, stats[2 * k], stats[2 * k + 1]);
    float acc = 0.0f;
    for (long long col = lane; col < p.cols; col += 32) {
      const long long i = row * p.cols + col;
      if (SUM) {
        run_element<T>(p, i, row, col, stats, [&](int, float v) { acc = __fadd_rn(acc, v); });
      } else {
        run_element<T>(p, i, row, col, stats,
                       [&](int slot, float v) { store_as(p.out[slot], p.out_dtype[slot], i, v); });
      }
    }
    if (SUM) {
      acc = warp_sum(acc);
      if (lane == 0) static_cast<typename T::S *>(sums)[row] = T::store(acc);
    }
  }
}

// fused_sum along columns: thread = column, block row = a band of `band`
// rows; partial[band][col] in f32 (or the rounded sum itself with one band).
template <class T>
__global__ void __launch_bounds__(256) fused_cols_kernel(const __grid_constant__ Program p, long long band,
                                                         float *partial, void *sums) {
  const long long col = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= p.cols) return;
  const long long r0 = (long long)blockIdx.y * band, r1 = min(p.rows, r0 + band);
  float acc = 0.0f;
  for (long long row = r0; row < r1; ++row)
    run_element<T>(p, row * p.cols + col, row, col, nullptr, [&](int, float v) { acc = __fadd_rn(acc, v); });
  if (gridDim.y == 1) static_cast<typename T::S *>(sums)[col] = T::store(acc);
  else partial[(long long)blockIdx.y * p.cols + col] = acc;
}

template <class T>
__global__ void __launch_bounds__(256) cols_finish(const float *partial, long long bands, long long cols, void *sums) {
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (long long)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (long long b = 0; b < bands; ++b) acc = __fadd_rn(acc, partial[b * cols + c]);
    static_cast<typename T::S *>(sums)[c] = T::store(acc);
  }
}

template <class T>
__global__ void __launch_bounds__(256) row_moments_kernel(const __grid_constant__ Place pl, long long rows,
                                                          long long cols, void *means, void *devs) {
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    float m, d;
    row_moments_of<T>(pl, row, cols, m, d);
    if ((threadIdx.x & 31) == 0) {
      static_cast<typename T::S *>(means)[row] = T::store(m);
      static_cast<typename T::S *>(devs)[row] = T::store(d);
    }
  }
}

bool storage_type(int d) { return d == TC_F32 || d == TC_F16 || d == TC_BF16; }

// Check one tc_place against the rows x cols space and fill `pl`.
int take_place(const tc_place &q, uint32_t j, size_t rows, size_t cols, Place &pl) {
  if (!storage_type(q.dtype)) return fail(TC_ENOTSUP, "fused: storage type %d", q.dtype);
  if (!q.data || q.lead > uint32_t(TC_MAX_RANK - 1)) return fail(TC_EINVAL, "fused: place %u", j);
  pl.data = q.data;
  pl.dtype = q.dtype;
  pl.lead = int(q.lead);
  pl.stat = -1;
  pl.offset = (long long)q.offset;
  pl.col_step = (long long)q.col_step;
  long long rows_folded = 1;
  for (uint32_t a = 0; a < q.lead; ++a) {
    pl.dims[a] = (long long)std::max<size_t>(q.dims[a], 1);
    pl.steps[a] = (long long)q.steps[a];
    rows_folded *= pl.dims[a];
  }
  if (q.lead == 0) {
    if (rows != 1) return fail(TC_EINVAL, "fused: place %u folds no rows over %zu rows", j, rows);
  } else if (rows_folded != (long long)rows) {
    return fail(TC_EINVAL, "fused: place %u folds %lld rows, the space has %zu", j, rows_folded, rows);
  }
  // In order: a step of one along the row and each row right after the last.
  bool in_order = cols == 1 || q.col_step == 1;
  long long step = (long long)cols;
  for (int a = int(q.lead) - 1; in_order && a >= 0; --a) {
    if (pl.dims[a] != 1 && pl.steps[a] != step) in_order = false;
    step *= pl.dims[a];
  }
  pl.in_order = in_order;
  return TC_OK;
}

// Validate a program and fill `p`.  Places listed as statistics (`stats`)
// need no data: their loads read the row's statistic instead.
int build_program(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                  const tc_place *places, uint32_t n_places, const tc_row_statistic *stats, uint32_t n_stats,
                  void *const *outputs, const int *out_dtypes, uint32_t n_outputs, Program &p) {
  if (!storage_type(dtype)) return fail(TC_ENOTSUP, "fused: program type %d (f32, f16 and bf16 only)", dtype);
  if (n_code > uint32_t(MAX_CODE) || n_places > uint32_t(MAX_PLACES) || n_outputs > uint32_t(MAX_OUTPUTS))
    return fail(TC_EINVAL, "fused: %u instructions, %u places, %u outputs (at most %d, %d, %d)", n_code, n_places,
                n_outputs, MAX_CODE, MAX_PLACES, MAX_OUTPUTS);
  if ((n_code && !code) || (n_places && !places) || (n_outputs && (!outputs || !out_dtypes)) || (n_stats && !stats))
    return fail(TC_EINVAL, "fused: null program part");
  p = Program{};
  p.n_code = int(n_code);
  p.n_places = int(n_places);
  p.n_outputs = int(n_outputs);
  p.rows = (long long)rows;
  p.cols = (long long)cols;
  bool written[REGISTERS] = {false};
  for (uint32_t k = 0; k < n_code; ++k) {
    const tc_instr &in = code[k];
    const bool reads_a = in.code == TC_I_BINARY || in.code == TC_I_UNARY || in.code == TC_I_CMP || in.code == TC_I_STORE;
    const bool reads_b = in.code == TC_I_BINARY || in.code == TC_I_CMP;
    if (in.code > TC_I_STORE) return fail(TC_EINVAL, "fused: instruction %u has code %u", k, in.code);
    if ((reads_a && (in.a >= REGISTERS || !written[in.a])) || (reads_b && (in.b >= REGISTERS || !written[in.b])))
      return fail(TC_EINVAL, "fused: instruction %u reads a register no earlier instruction wrote", k);
    if (in.code == TC_I_LOAD && in.slot >= n_places) return fail(TC_EINVAL, "fused: load of place %u", in.slot);
    if (in.code == TC_I_STORE && in.slot >= n_outputs) return fail(TC_EINVAL, "fused: store to output %u", in.slot);
    if ((in.code == TC_I_BINARY && in.op > TC_REM) || (in.code == TC_I_CMP && in.op > TC_GREATER_EQUAL) ||
        (in.code == TC_I_UNARY && in.op > TC_SQRT))
      return fail(TC_EINVAL, "fused: instruction %u has operation %u", k, in.op);
    if (in.code != TC_I_STORE) {
      if (in.dst >= REGISTERS) return fail(TC_EINVAL, "fused: register %u", in.dst);
      written[in.dst] = true;
    }
    p.code[k] = in;
  }
  bool is_stat[MAX_PLACES] = {false};
  for (uint32_t s = 0; s < n_stats; ++s) {
    if (stats[s].into_place >= n_places || stats[s].of_place >= n_places ||
        (stats[s].statistic != TC_ROW_MEAN && stats[s].statistic != TC_ROW_DEVIATIONS))
      return fail(TC_EINVAL, "fused: row statistic %u", s);
    is_stat[stats[s].into_place] = true;
  }
  for (uint32_t j = 0; j < n_places; ++j) {
    if (is_stat[j]) {
      p.places[j] = Place{};
      continue;
    }
    if (int st = take_place(places[j], j, rows, cols, p.places[j])) return st;
  }
  for (uint32_t s = 0; s < n_stats; ++s) {
    const uint32_t of = stats[s].of_place;
    if (is_stat[of]) return fail(TC_EINVAL, "fused: row statistic %u is of a statistic", s);
    int k = 0;
    while (k < p.n_stat_sources && p.stat_source[k] != int(of)) ++k;
    if (k == p.n_stat_sources) {
      if (k == MAX_STAT_SOURCES) return fail(TC_EINVAL, "fused: statistics of more than %d inputs", MAX_STAT_SOURCES);
      p.stat_source[p.n_stat_sources++] = int(of);
    }
    p.places[stats[s].into_place].stat = 2 * k + (stats[s].statistic == TC_ROW_DEVIATIONS ? 1 : 0);
  }
  for (uint32_t j = 0; j < n_outputs; ++j) {
    if (!outputs[j] || !storage_type(out_dtypes[j])) return fail(TC_EINVAL, "fused: output %u", j);
    p.out[j] = outputs[j];
    p.out_dtype[j] = out_dtypes[j];
  }
  return TC_OK;
}

unsigned row_grid(long long rows) {
  return unsigned(std::max(1LL, std::min<long long>((rows + 7) / 8, (long long)sm_count() * 8)));
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_fused(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code, const tc_place *places,
             uint32_t n_places, void *const *outputs, const int *out_dtypes, uint32_t n_outputs, void *stream) {
  Program p;
  if (int st = build_program(dtype, rows, cols, code, n_code, places, n_places, nullptr, 0, outputs, out_dtypes,
                             n_outputs, p))
    return st;
  if (rows == 0 || cols == 0) return TC_OK;
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    fused_kernel<T><<<grid_for(rows * cols, 256, 8), 256, 0, as_stream(stream)>>>(p);
    return check_launch("fused program");
  });
}

int tc_fused_with_statistics(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                             const tc_place *places, uint32_t n_places, const tc_row_statistic *stats,
                             uint32_t n_stats, void *const *outputs, const int *out_dtypes, uint32_t n_outputs,
                             void *stream) {
  Program p;
  if (int st = build_program(dtype, rows, cols, code, n_code, places, n_places, stats, n_stats, outputs, out_dtypes,
                             n_outputs, p))
    return st;
  if (rows == 0 || cols == 0) return TC_OK;
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    fused_rows_kernel<T, false><<<row_grid((long long)rows), 256, 0, as_stream(stream)>>>(p, nullptr);
    return check_launch("fused program with statistics");
  });
}

int tc_fused_sum(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code, const tc_place *places,
                 uint32_t n_places, int axis, void *sums, void *stream) {
  if (axis != TC_ROWS && axis != TC_COLUMNS) return fail(TC_EINVAL, "bad Axis %d", axis);
  // One output of the program's own type; its values are summed, not kept.
  void *placeholder = sums;
  const int out_dtype = dtype;
  Program p;
  if (int st = build_program(dtype, rows, cols, code, n_code, places, n_places, nullptr, 0, &placeholder, &out_dtype,
                             1, p))
    return st;
  const size_t results = axis == TC_ROWS ? rows : cols;
  if (results == 0) return TC_OK;
  if (!sums) return fail(TC_EINVAL, "fused_sum: null output");
  cudaStream_t s = as_stream(stream);
  if (rows == 0 || cols == 0) {
    // Sums of nothing: zeros.
    return check_cuda(cudaMemsetAsync(sums, 0, results * dtype_bytes(dtype), s), "fused_sum (empty)");
  }
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    if (axis == TC_ROWS) {
      fused_rows_kernel<T, true><<<row_grid((long long)rows), 256, 0, s>>>(p, sums);
      return check_launch("fused sum (rows)");
    }
    const long long col_blocks = ((long long)cols + 255) / 256;
    const long long want = std::max(1LL, (long long)sm_count() * 8 / col_blocks);
    const long long band = std::max(16LL, ((long long)rows + want - 1) / want);
    const long long bands = ((long long)rows + band - 1) / band;
    float *partial = nullptr;
    if (bands > 1)
      if (int st = scratch(size_t(bands) * cols * sizeof(float), reinterpret_cast<void **>(&partial))) return st;
    fused_cols_kernel<T><<<dim3(unsigned(col_blocks), unsigned(bands)), 256, 0, s>>>(p, band, partial, sums);
    if (int st = check_launch("fused sum (columns)")) return st;
    if (bands > 1) {
      cols_finish<T><<<grid_for(cols, 256, 4), 256, 0, s>>>(partial, bands, (long long)cols, sums);
      return check_launch("fused sum (columns, finish)");
    }
    return int(TC_OK);
  });
}

int tc_matmul_program(int dtype, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                      const tc_instr *code, uint32_t n_code, const tc_place *places, uint32_t n_places,
                      void *const *outputs, const int *out_dtypes, uint32_t n_outputs, void *stream) {
  if (n_places == 0 || !places) return fail(TC_EINVAL, "matmul_program: place 0 (the product) is missing");
  if (n_places > uint32_t(MAX_PLACES)) return fail(TC_EINVAL, "matmul_program: %u places", n_places);
  if (!storage_type(dtype)) return fail(TC_ENOTSUP, "matmul_program: type %d", dtype);
  if (rows == 0 || cols == 0) return TC_OK;
  // The product, rounded once to T (a.matmul(b)), in a pooled block that
  // the program reads as its input 0 and that goes back to the pool after
  // the launch (later work on this stream is ordered after it).
  void *product = nullptr;
  if (int st = tc_malloc(&product, rows * cols * dtype_bytes(dtype))) return st;
  int st = tc_matmul(dtype, TC_TRANS_NONE, rows, inner, cols, a, b, product, 0, stream);
  if (st == TC_OK) {
    tc_place all[MAX_PLACES];
    for (uint32_t j = 0; j < n_places; ++j) all[j] = places[j];
    all[0].data = product;
    all[0].dtype = dtype;
    st = tc_fused(dtype, rows, cols, code, n_code, all, n_places, outputs, out_dtypes, n_outputs, stream);
  }
  tc_free(product);
  return st;
}

int tc_row_moments(int dtype, const tc_place *place, size_t rows, size_t cols, void *means, void *deviations,
                   void *stream) {
  if (!storage_type(dtype)) return fail(TC_ENOTSUP, "row_moments: type %d", dtype);
  if (!place) return fail(TC_EINVAL, "row_moments: null place");
  if (rows == 0) return TC_OK;
  if (!means || !deviations) return fail(TC_EINVAL, "row_moments: null output");
  if (cols == 0) return tc_axis_moments(dtype, rows, 0, TC_ROWS, nullptr, means, deviations, stream);
  Place pl;
  if (int st = take_place(*place, 0, rows, cols, pl)) return st;
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    row_moments_kernel<T><<<row_grid((long long)rows), 256, 0, as_stream(stream)>>>(pl, (long long)rows,
                                                                                  (long long)cols, means, deviations);
    return check_launch("row moments");
  });
}

}  // extern "C"
