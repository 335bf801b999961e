// fused.cu — fused elementwise programs (Kernels::fused, kernels.rs:1077-1082;
// fused::Program and Instr, fused/mod.rs:290-340, 502): a bytecode
// interpreter, one thread per element of the rows x cols space.
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
// as in the reference's Metal shader.  This is the general path; the
// optimizers' programs have kernels of their own (optim.cu).
#include <algorithm>

#include "analytic.cuh"

namespace tc {
namespace {

constexpr int MAX_CODE = 256, MAX_PLACES = 16, MAX_OUTPUTS = 8, REGISTERS = 16;

struct Place {
  const void *data;
  int dtype;
  int lead;
  int in_order;  // element (row, col) is data[offset + row*cols + col]
  long long offset, col_step;
  long long dims[TC_MAX_RANK - 1], steps[TC_MAX_RANK - 1];
};

struct Program {
  int n_code, n_places, n_outputs;
  long long rows, cols;
  tc_instr code[MAX_CODE];
  Place places[MAX_PLACES];
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

template <class T>
__global__ void __launch_bounds__(256) fused_kernel(const __grid_constant__ Program p) {
  const long long total = p.rows * p.cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / p.cols, col = i - row * p.cols;
    float reg[REGISTERS];
    for (int k = 0; k < p.n_code; ++k) {
      const tc_instr in = p.code[k];
      float v;
      switch (in.code) {
        case TC_I_LOAD: {
          const Place &pl = p.places[in.slot];
          long long at;
          if (pl.in_order) {
            at = pl.offset + i;
          } else {
            at = pl.offset + col * pl.col_step;
            long long rest = row;
            for (int a = pl.lead - 1; a >= 0; --a) {
              const long long q = rest / pl.dims[a];
              at += (rest - q * pl.dims[a]) * pl.steps[a];
              rest = q;
            }
          }
          v = T::load(T::store(load_as(pl.data, pl.dtype, at)));
          break;
        }
        case TC_I_CONST: v = T::load(T::store(in.value)); break;
        case TC_I_BINARY: v = T::load(T::store(binary_value(in.op, reg[in.a], reg[in.b]))); break;
        case TC_I_UNARY: v = T::load(T::store(analytic(in.op, reg[in.a]))); break;
        case TC_I_CMP: v = compare_value(in.op, reg[in.a], reg[in.b]); break;
        default:  // store
          store_as(p.out[in.slot], p.out_dtype[in.slot], i, reg[in.a]);
          continue;
      }
      reg[in.dst] = v;
    }
  }
}

bool storage_type(int d) { return d == TC_F32 || d == TC_F16 || d == TC_BF16; }

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" int tc_fused(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                        const tc_place *places, uint32_t n_places, void *const *outputs, const int *out_dtypes,
                        uint32_t n_outputs, void *stream) {
  if (!storage_type(dtype)) return fail(TC_ENOTSUP, "fused: program type %d (f32, f16 and bf16 only)", dtype);
  if (n_code > uint32_t(MAX_CODE) || n_places > uint32_t(MAX_PLACES) || n_outputs > uint32_t(MAX_OUTPUTS))
    return fail(TC_EINVAL, "fused: %u instructions, %u places, %u outputs (at most %d, %d, %d)", n_code, n_places,
                n_outputs, MAX_CODE, MAX_PLACES, MAX_OUTPUTS);
  if ((n_code && !code) || (n_places && !places) || (n_outputs && (!outputs || !out_dtypes)))
    return fail(TC_EINVAL, "fused: null program part");
  if (rows == 0 || cols == 0) return TC_OK;
  Program p{};
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
  for (uint32_t j = 0; j < n_places; ++j) {
    const tc_place &q = places[j];
    if (!storage_type(q.dtype)) return fail(TC_ENOTSUP, "fused: storage type %d", q.dtype);
    if (!q.data || q.lead > uint32_t(TC_MAX_RANK - 1)) return fail(TC_EINVAL, "fused: place %u", j);
    Place &pl = p.places[j];
    pl.data = q.data;
    pl.dtype = q.dtype;
    pl.lead = int(q.lead);
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
  }
  for (uint32_t j = 0; j < n_outputs; ++j) {
    if (!outputs[j] || !storage_type(out_dtypes[j])) return fail(TC_EINVAL, "fused: output %u", j);
    p.out[j] = outputs[j];
    p.out_dtype[j] = out_dtypes[j];
  }
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    fused_kernel<T><<<grid_for(rows * cols, 256, 8), 256, 0, as_stream(stream)>>>(p);
    return check_launch("fused program");
  });
}
