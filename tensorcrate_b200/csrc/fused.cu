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
#include <vector>

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
  int source;    // -1, or k when this place is statistic source k (its row may be staged on chip)
  int packs;     // in order, offset a multiple of 4, data aligned for 4-element vector loads
  long long offset, col_step;
  long long dims[TC_MAX_RANK - 1], steps[TC_MAX_RANK - 1];
};

struct Program {
  int n_code, n_places, n_outputs, n_stat_sources;
  int n_regs;    // rows of the register file: the registers that pass through it (at least 1)
  int needs_rc;  // some place is read out of order: elements need their (row, col)
  int n_ahead;   // places read in order, whose next group is requested into L2 ahead
  int ahead[4];
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

// E elements of the space run through the program together: flat indices
// i0 .. i0+n-1 (n <= E), the first at (row, col) of a space `cols` wide
// (row and col are set only for programs that read a place out of order).
// Registers hold E values; a load of an in-order place whose E elements are
// 16-byte (f32) or 8-byte (f16/bf16) aligned is one vector load per 4, and
// so is the store of a group.
template <int E> struct Group {
  long long i0;
  int n;
  long long row, col, cols;
};

template <int E>
__device__ __forceinline__ Group<E> make_group(long long i0, int n, long long cols, bool with_rc = true) {
  Group<E> g;
  g.i0 = i0;
  g.n = n;
  g.cols = cols;
  if (with_rc) {
    g.row = i0 / cols;
    g.col = i0 - g.row * cols;
  }
  return g;
}

__device__ __forceinline__ bool aligned_to(const void *p, unsigned bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

template <class T, int E>
__device__ __forceinline__ void load_group(const Place &pl, const Group<E> &g, float v[E]) {
  if (pl.in_order) {
    const long long at = pl.offset + g.i0;
    if (E % 4 == 0 && pl.packs && g.n == E && (g.i0 & 3) == 0) {
      if (pl.dtype == TC_F32) {
        const float4 *src = reinterpret_cast<const float4 *>(pl.data) + at / 4;
        float4 q[E / 4 > 0 ? E / 4 : 1];
#pragma unroll
        for (int k = 0; k < E / 4; ++k) q[k] = __ldg(src + k);
#pragma unroll
        for (int k = 0; k < E / 4; ++k) {
          v[4 * k] = q[k].x;
          v[4 * k + 1] = q[k].y;
          v[4 * k + 2] = q[k].z;
          v[4 * k + 3] = q[k].w;
        }
        goto convert;
      }
      {
        const uint2 *src = reinterpret_cast<const uint2 *>(pl.data) + at / 4;
        uint2 q[E / 4 > 0 ? E / 4 : 1];
#pragma unroll
        for (int k = 0; k < E / 4; ++k) q[k] = __ldg(src + k);
#pragma unroll
        for (int k = 0; k < E / 4; ++k) {
          const uint16_t h[4] = {uint16_t(q[k].x), uint16_t(q[k].x >> 16), uint16_t(q[k].y), uint16_t(q[k].y >> 16)};
#pragma unroll
          for (int j = 0; j < 4; ++j) v[4 * k + j] = pl.dtype == TC_BF16 ? BF16T::load(h[j]) : F16T::load(h[j]);
        }
        goto convert;
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (e < g.n) v[e] = load_as(pl.data, pl.dtype, at + e);
  } else {
    long long r = g.row, c = g.col;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (e < g.n) v[e] = load_as(pl.data, pl.dtype, place_at(pl, g.i0 + e, r, c));
      if (++c == g.cols) c = 0, ++r;
    }
  }
convert:
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = T::load(T::store(v[e]));
}

// Store a group's values of one output (laid out as the space, in order).
template <int E>
__device__ __forceinline__ void store_group(void *out, int dtype, const Group<E> &g, const float v[E]) {
  if (E % 4 == 0 && g.n == E && (g.i0 & 3) == 0) {
    if (dtype == TC_F32 && aligned_to(out, 16)) {
#pragma unroll
      for (int k = 0; k < E / 4; ++k)
        reinterpret_cast<float4 *>(out)[g.i0 / 4 + k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      return;
    }
    if (dtype != TC_F32 && aligned_to(out, 8)) {
#pragma unroll
      for (int k = 0; k < E / 4; ++k) {
        uint16_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = dtype == TC_BF16 ? BF16T::store(v[4 * k + j]) : F16T::store(v[4 * k + j]);
        reinterpret_cast<uint2 *>(out)[g.i0 / 4 + k] =
            make_uint2(uint32_t(h[0]) | (uint32_t(h[1]) << 16), uint32_t(h[2]) | (uint32_t(h[3]) << 16));
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e)
    if (e < g.n) store_as(out, dtype, g.i0 + e, v[e]);
}

// What a group's loads may read on chip instead of from memory (the row
// kernels): the row's statistics, 2 per source (mean, deviations), and the
// row of each statistic source staged in shared memory, `stage_cols` floats
// apart, with the group's first element at column `col0` (a multiple of 4).
struct OnChip {
  const float *stats;
  const float *stage;  // null: nothing staged
  int stage_cols;
  int col0;
};

// Run the program on a group; `sink(slot, values)` receives every store.
// The interpreter's blocks are INTERP_BLOCK threads; each thread's
// registers live in dynamic shared memory (registers indexed by the program
// cannot be machine registers and would otherwise go to local memory), as
// many as the program writes: register r of thread t holds its E elements
// at file[(r * INTERP_BLOCK + t) * E ...], one 16-byte access for E = 4.
constexpr int INTERP_BLOCK = 128;

template <int E> struct RegFile {
  float *base;  // this thread's register 0
  __device__ __forceinline__ float *row(int r) const { return base + r * (INTERP_BLOCK * E); }
  __device__ __forceinline__ void get(int r, float v[E]) const {
    const float *at = base + r * (INTERP_BLOCK * E);
    if constexpr (E % 4 == 0) {
#pragma unroll
      for (int k = 0; k < E / 4; ++k) {
        const float4 q = reinterpret_cast<const float4 *>(at)[k];
        v[4 * k] = q.x, v[4 * k + 1] = q.y, v[4 * k + 2] = q.z, v[4 * k + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = at[e];
    }
  }
  __device__ __forceinline__ void put(int r, const float v[E]) const {
    float *at = base + r * (INTERP_BLOCK * E);
    if constexpr (E % 4 == 0) {
#pragma unroll
      for (int k = 0; k < E / 4; ++k)
        reinterpret_cast<float4 *>(at)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) at[e] = v[e];
    }
  }
};

__device__ __forceinline__ float *interp_shared() {
  extern __shared__ float4 interp_smem[];
  return reinterpret_cast<float *>(interp_smem);
}

template <int E> __device__ __forceinline__ RegFile<E> thread_registers() {
  return RegFile<E>{interp_shared() + threadIdx.x * E};
}

// A load of a staged statistic source reads the row's copy on chip.
template <int E> __device__ __forceinline__ bool read_stage(const OnChip &chip, const Place &pl, float v[E]) {
  if constexpr (E % 4 == 0) {
    if (chip.stage && pl.source >= 0) {
      const float4 *at = reinterpret_cast<const float4 *>(chip.stage + pl.source * chip.stage_cols + chip.col0);
#pragma unroll
      for (int k = 0; k < E / 4; ++k) {
        const float4 q = at[k];
        v[4 * k] = q.x, v[4 * k + 1] = q.y, v[4 * k + 2] = q.z, v[4 * k + 3] = q.w;
      }
      return true;
    }
  }
  return false;
}

// How a value moves between instructions (in the program's copy of each
// instruction, the `reserved` field; worked out by build_program): operand a
// or b is the result of the instruction just before (held in registers, not
// read from the file), and the result is also needed later than the next
// instruction (written to the file).  A unary operation other than the root
// works between the file's rows: its operand is always in the file and its
// result always goes there.
enum : uint16_t { A_PREV = 1, B_PREV = 2, SPILL = 4, A_STAT = 8, B_STAT = 16 };
// With A_STAT (B_STAT), operand a (b) is a row statistic, read where the row
// kernel keeps it (its index in bits 8-11, for b 12-15), not from the file.

template <int E> __device__ __forceinline__ void operand(const RegFile<E> &reg, const OnChip &chip, int r,
                                                         uint16_t f, bool is_b, const float prev[E], float x[E]) {
  if (f & (is_b ? B_PREV : A_PREV)) {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = prev[e];
  } else if (f & (is_b ? B_STAT : A_STAT)) {
    const float v = chip.stats[(f >> (is_b ? 12 : 8)) & 15];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = v;
  } else {
    reg.get(r, x);
  }
}

template <class T, int E, class Sink>
__device__ __forceinline__ void run_group(const Program &p, const Group<E> &g, const OnChip &chip, Sink &&sink) {
  const RegFile<E> reg = thread_registers<E>();
  float prev[E];  // the last instruction's result
#pragma unroll
  for (int e = 0; e < E; ++e) prev[e] = 0.0f;
  for (int k = 0; k < p.n_code; ++k) {
    const tc_instr in = p.code[k];
    const uint16_t f = in.reserved;
    float v[E];
    switch (in.code) {
      case TC_I_LOAD: {
        const Place &pl = p.places[in.slot];
        if (pl.stat >= 0) {
#pragma unroll
          for (int e = 0; e < E; ++e) v[e] = chip.stats[pl.stat];
        } else if (!read_stage<E>(chip, pl, v)) {
          load_group<T, E>(pl, g, v);
        }
        break;
      }
      case TC_I_CONST: {
        const float c = T::load(T::store(in.value));
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = c;
        break;
      }
      case TC_I_BINARY: {
        float x[E], y[E];
        operand<E>(reg, chip, in.a, f, false, prev, x);
        operand<E>(reg, chip, in.b, f, true, prev, y);
        // one branch per instruction, not per element
        switch (in.op) {
          case TC_ADD:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = __fadd_rn(x[e], y[e]);
            break;
          case TC_SUB:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = __fsub_rn(x[e], y[e]);
            break;
          case TC_MUL:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = __fmul_rn(x[e], y[e]);
            break;
          case TC_DIV:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = __fdiv_rn(x[e], y[e]);
            break;
          default:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = fmodf(x[e], y[e]);
        }
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = T::load(T::store(v[e]));
        break;
      }
      case TC_I_UNARY: {
        if (in.op == TC_SQRT) {  // normalisations' root: a few instructions, unrolled
          float x[E];
          operand<E>(reg, chip, in.a, f, false, prev, x);
#pragma unroll
          for (int e = 0; e < E; ++e) v[e] = T::load(T::store(__fsqrt_rn(x[e])));
          break;
        }
        // element by element between the register file's rows: the analytic
        // functions' code appears once, not once per element
        const float *x = reg.row(in.a);
        float *y = reg.row(in.dst);
#pragma unroll 1
        for (int e = 0; e < E; ++e) y[e] = T::load(T::store(analytic(in.op, x[e])));
        continue;
      }
      case TC_I_CMP: {
        float x[E], y[E];
        operand<E>(reg, chip, in.a, f, false, prev, x);
        operand<E>(reg, chip, in.b, f, true, prev, y);
        switch (in.op) {
          case TC_MIN:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = fminf(x[e], y[e]);
            break;
          case TC_MAX:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = fmaxf(x[e], y[e]);
            break;
          default:
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = compare_value(in.op, x[e], y[e]);
        }
        break;
      }
      default: {  // store
        operand<E>(reg, chip, in.a, f, false, prev, v);
        sink(int(in.slot), v);
        continue;
      }
    }
    if (f & SPILL) reg.put(in.dst, v);
#pragma unroll
    for (int e = 0; e < E; ++e) prev[e] = v[e];
  }
}

// Elements per lane and step in the row kernels (program and statistics),
// and columns per thread in the column sums.
constexpr int ROW_GROUP = 8, COL_GROUP = 4;

// Ask L2 for the group at flat index i0 of each in-order place the program
// loads: a thread's next group arrives while it runs the current one.
__device__ __forceinline__ void request_ahead(const Program &p, long long i0) {
  for (int k = 0; k < p.n_ahead; ++k) {
    const Place &pl = p.places[p.ahead[k]];
    const char *at = static_cast<const char *>(pl.data) + (pl.offset + i0) * (pl.dtype == TC_F32 ? 4 : 2);
    asm volatile("prefetch.global.L2 [%0];" ::"l"(at));
  }
}

// Ask L2 for row `row` of an in-order place: the row's `lanes` threads take
// its 128-byte lines in turn.  Allocations start on 256-byte boundaries, so
// the lines that hold the row's first and last bytes lie inside the place's
// allocation.
__device__ __forceinline__ void request_place_row(const Place &pl, long long row, long long cols, int lane,
                                                  int lanes) {
  const long long size = pl.dtype == TC_F32 ? 4 : 2;
  const uintptr_t first = reinterpret_cast<uintptr_t>(pl.data) + uintptr_t((pl.offset + row * cols) * size);
  const uintptr_t last = first + uintptr_t(cols * size) - 1;
  for (uintptr_t at = (first & ~uintptr_t(127)) + uintptr_t(lane) * 128; at <= last; at += uintptr_t(lanes) * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(at));
}

// The same for each in-order place the program loads.
__device__ __forceinline__ void request_row(const Program &p, long long row, int lane, int lanes) {
  for (int k = 0; k < p.n_ahead; ++k) request_place_row(p.places[p.ahead[k]], row, p.cols, lane, lanes);
}

// The flat kernel's elements per thread and step: each program instruction
// is decoded once for FLAT_GROUP elements.
constexpr int FLAT_GROUP = 8;

template <class T>
__global__ void __launch_bounds__(INTERP_BLOCK) fused_kernel(const __grid_constant__ Program p) {
  constexpr int E = FLAT_GROUP;
  const OnChip none{nullptr, nullptr, 0, 0};
  const long long total = p.rows * p.cols;
  const long long groups = (total + E - 1) / E;
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < groups;
       q += (long long)gridDim.x * blockDim.x) {
    const long long i0 = q * E;
    const long long next = i0 + (long long)gridDim.x * blockDim.x * E;
    if (next < total) request_ahead(p, next);
    const Group<E> g = make_group<E>(i0, int(min((long long)E, total - i0)), p.cols, p.needs_rc != 0);
    run_group<T, E>(p, g, none, [&](int slot, const float *v) { store_group<E>(p.out[slot], p.out_dtype[slot], g, v); });
  }
}

// The sum of v over the LANES threads that share a row (LANES a power of
// two): each warp's share by an xor tree, then, above 32 lanes, the row's
// warps in order through `scratch` (a float per warp of the block).  Every
// thread of the block calls it the same number of times.
template <int LANES> __device__ __forceinline__ float row_sum(float v, float *scratch) {
  constexpr int W = LANES < 32 ? LANES : 32;
#pragma unroll
  for (int d = W / 2; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
  if constexpr (LANES > 32) {
    const int warp = threadIdx.x >> 5, first = warp / (LANES / 32) * (LANES / 32);
    __syncthreads();  // the previous sum's reads of scratch are done
    if ((threadIdx.x & 31) == 0) scratch[warp] = v;
    __syncthreads();
    v = scratch[first];
#pragma unroll
    for (int w = 1; w < LANES / 32; ++w) v = __fadd_rn(v, scratch[first + w]);
  }
  return v;
}

// The mean and the sum of squared deviations of row `row` as `pl` reads it
// (converted to T), in f32, two passes over the row by its LANES threads;
// both rounded to T, as Kernels::row_moments returns them
// (fused/mod.rs:4030-4043, statistics/mod.rs:451-491).  Lane l adds columns
// 8l + 8·LANES·j onwards, 8 at a time, in order, then the lanes' sums are
// added (row_sum).  With `stage`, the first pass also keeps the row on chip
// (lane l's columns at stage[8l + 8·LANES·j ...], read back only by lane l,
// which takes the same columns in the program) and the second reads
// it there: the row crosses memory once.  A thread whose row is past the
// end (`live` false) reads nothing but takes part in the sums.
template <class T, int LANES>
__device__ __forceinline__ void row_moments_of(const Place &pl, long long row, long long cols, bool live,
                                               float &mean, float &dev, float *stage, float *scratch) {
  const int lane = threadIdx.x & (LANES - 1);
  const long long n = live ? cols : 0;
  float s = 0.0f;
#pragma unroll 2
  for (long long c0 = (long long)lane * ROW_GROUP; c0 < n; c0 += LANES * ROW_GROUP) {
    Group<ROW_GROUP> g =
        make_group<ROW_GROUP>(row * cols + c0, int(min((long long)ROW_GROUP, cols - c0)), cols, !pl.in_order);
    float v[ROW_GROUP];
    load_group<T, ROW_GROUP>(pl, g, v);
    if (stage)
#pragma unroll
      for (int k = 0; k < ROW_GROUP / 4; ++k)
        reinterpret_cast<float4 *>(stage + c0)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
#pragma unroll
    for (int e = 0; e < ROW_GROUP; ++e)
      if (e < g.n) s = __fadd_rn(s, v[e]);
  }
  const float m = __fdiv_rn(row_sum<LANES>(s, scratch), float(cols));
  float d = 0.0f;
  for (long long c0 = (long long)lane * ROW_GROUP; c0 < n; c0 += LANES * ROW_GROUP) {
    const int k = int(min((long long)ROW_GROUP, cols - c0));
    float v[ROW_GROUP];
    if (stage) {
#pragma unroll
      for (int j = 0; j < ROW_GROUP / 4; ++j) {
        const float4 q = reinterpret_cast<const float4 *>(stage + c0)[j];
        v[4 * j] = q.x, v[4 * j + 1] = q.y, v[4 * j + 2] = q.z, v[4 * j + 3] = q.w;
      }
    } else {
      Group<ROW_GROUP> g = make_group<ROW_GROUP>(row * cols + c0, k, cols, !pl.in_order);
      load_group<T, ROW_GROUP>(pl, g, v);
    }
#pragma unroll
    for (int e = 0; e < ROW_GROUP; ++e)
      if (e < k) {
        const float x = __fsub_rn(v[e], m);
        d = __fadd_rn(d, __fmul_rn(x, x));
      }
  }
  mean = T::load(T::store(m));
  dev = T::load(T::store(row_sum<LANES>(d, scratch)));
}

// LANES threads per row (8, 32 or a block of 128, by the row's length),
// INTERP_BLOCK / LANES rows per block at once, each row's next one requested
// into L2 while it runs.  With `sums`, the row's values of output 0 are added
// (f32, rounded once to T) into sums[row] instead of stored (fused_sum's
// programs read no statistics).  With stage_cols > 0, each statistic
// source's row is kept on chip after its statistics are taken (stage_cols
// floats per source per row, after the register file), and the program's
// loads of it read it there.
template <class T, int LANES>
__global__ void __launch_bounds__(INTERP_BLOCK, 6) fused_rows_kernel(const __grid_constant__ Program p, void *sums,
                                                                     int stage_cols) {
  constexpr int SLOTS = INTERP_BLOCK / LANES;
  __shared__ float scratch[INTERP_BLOCK / 32];
  const int slot = threadIdx.x / LANES, lane = threadIdx.x & (LANES - 1);
  float *stage = nullptr;
  if (stage_cols > 0)
    stage = interp_shared() + p.n_regs * INTERP_BLOCK * ROW_GROUP + slot * p.n_stat_sources * stage_cols;
  for (long long r0 = (long long)blockIdx.x * SLOTS; r0 < p.rows; r0 += (long long)gridDim.x * SLOTS) {
    const long long row = r0 + slot;
    const bool live = row < p.rows;
    const long long next = row + (long long)gridDim.x * SLOTS;
    if (next < p.rows) request_row(p, next, lane, LANES);
    float stats[2 * MAX_STAT_SOURCES];
    for (int k = 0; k < p.n_stat_sources; ++k)
      row_moments_of<T, LANES>(p.places[p.stat_source[k]], row, p.cols, live, stats[2 * k], stats[2 * k + 1],
                               stage ? stage + k * stage_cols : nullptr, scratch);
    OnChip chip{stats, stage, stage_cols, 0};
    float acc = 0.0f;
    const long long n = live ? p.cols : 0;
    for (long long c0 = (long long)lane * ROW_GROUP; c0 < n; c0 += LANES * ROW_GROUP) {
      const Group<ROW_GROUP> g = make_group<ROW_GROUP>(row * p.cols + c0, int(min((long long)ROW_GROUP, p.cols - c0)),
                                                       p.cols, p.needs_rc != 0);
      chip.col0 = int(c0);
      run_group<T, ROW_GROUP>(p, g, chip, [&](int slot, const float *v) {
        if (sums) {
#pragma unroll
          for (int e = 0; e < ROW_GROUP; ++e)
            if (e < g.n) acc = __fadd_rn(acc, v[e]);
        } else {
          store_group<ROW_GROUP>(p.out[slot], p.out_dtype[slot], g, v);
        }
      });
    }
    if (sums) {
      acc = row_sum<LANES>(acc, scratch);
      if (live && lane == 0) static_cast<typename T::S *>(sums)[row] = T::store(acc);
    }
  }
}

// fused_sum along columns: a thread takes COL_GROUP consecutive columns over
// a band of `band` rows.  A block holds `groups` column groups side by side
// and INTERP_BLOCK / groups bands of them one under another (narrow matrices
// fill the block with bands); band b = blockIdx.y * (INTERP_BLOCK / groups)
// + the thread's place in the block, for b < bands.  partial[b][col] in f32,
// or the rounded sums themselves when there is one band.  Each column's
// values are added row after row (the row four ahead requested into L2),
// then the bands' sums in band order.
template <class T>
__global__ void __launch_bounds__(INTERP_BLOCK) fused_cols_kernel(const __grid_constant__ Program p, int groups,
                                                                  long long band, long long bands, float *partial,
                                                                  void *sums) {
  const int per_block = INTERP_BLOCK / groups, sub = threadIdx.x / groups;
  const long long c0 = ((long long)blockIdx.x * groups + threadIdx.x % groups) * COL_GROUP;
  if (sub >= per_block || c0 >= p.cols) return;
  const int n = int(min((long long)COL_GROUP, p.cols - c0));
  const OnChip none{nullptr, nullptr, 0, 0};
  const long long b = (long long)blockIdx.y * per_block + sub;
  if (b >= bands) return;
  const long long r0 = b * band, r1 = min(p.rows, r0 + band);
  float acc[COL_GROUP] = {};
  for (long long row = r0; row < r1; ++row) {
    if (row + 4 < r1) request_ahead(p, (row + 4) * p.cols + c0);
    Group<COL_GROUP> g;
    g.i0 = row * p.cols + c0;
    g.n = n;
    g.row = row, g.col = c0, g.cols = p.cols;
    run_group<T, COL_GROUP>(p, g, none, [&](int, const float *v) {
#pragma unroll
      for (int e = 0; e < COL_GROUP; ++e) acc[e] = __fadd_rn(acc[e], v[e]);
    });
  }
  for (int e = 0; e < n; ++e) {
    if (bands == 1) static_cast<typename T::S *>(sums)[c0 + e] = T::store(acc[e]);
    else partial[b * p.cols + c0 + e] = acc[e];
  }
}

template <class T>
__global__ void __launch_bounds__(256) cols_finish(const float *partial, long long bands, long long cols, void *sums) {
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (long long)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (long long b = 0; b < bands; ++b) acc = __fadd_rn(acc, partial[b * cols + c]);
    static_cast<typename T::S *>(sums)[c] = T::store(acc);
  }
}

// tc_row_moments: LANES threads per row, as the row kernels.
template <class T, int LANES>
__global__ void __launch_bounds__(INTERP_BLOCK) row_moments_kernel(const __grid_constant__ Place pl, long long rows,
                                                                   long long cols, void *means, void *devs) {
  constexpr int SLOTS = INTERP_BLOCK / LANES;
  __shared__ float scratch[INTERP_BLOCK / 32];
  const int slot = threadIdx.x / LANES, lane = threadIdx.x & (LANES - 1);
  for (long long r0 = (long long)blockIdx.x * SLOTS; r0 < rows; r0 += (long long)gridDim.x * SLOTS) {
    const long long row = r0 + slot;
    const bool live = row < rows;
    const long long next = row + (long long)gridDim.x * SLOTS;
    if (next < rows && pl.in_order) request_place_row(pl, next, cols, lane, LANES);
    float m, d;
    row_moments_of<T, LANES>(pl, row, cols, live, m, d, nullptr, scratch);
    if (live && lane == 0) {
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
  pl.source = -1;
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
  const uintptr_t align = q.dtype == TC_F32 ? 16 : 8;
  pl.packs = in_order && q.offset % 4 == 0 && (reinterpret_cast<uintptr_t>(q.data) & (align - 1)) == 0;
  return TC_OK;
}

// Which values the interpreter forwards in registers (A_PREV, B_PREV) and
// which it writes to the register file (SPILL), from the registers each
// instruction reads and writes; then the file's rows (n_regs).  A row
// statistic's readers (other than a transcendental unary, which works
// between file rows) read it where the row kernel keeps it (A_STAT, B_STAT).  A result that only the next instruction
// reads stays in registers; one read later, before the register is written
// again, goes to the file; a unary operation other than the root neither
// takes its operand from registers nor leaves its result there.
void mark_forwarding(Program &p) {
  auto writes = [](const tc_instr &in) { return in.code != TC_I_STORE; };
  auto reads_a = [](const tc_instr &in) {
    return in.code == TC_I_BINARY || in.code == TC_I_UNARY || in.code == TC_I_CMP || in.code == TC_I_STORE;
  };
  auto reads_b = [](const tc_instr &in) { return in.code == TC_I_BINARY || in.code == TC_I_CMP; };
  auto generic_unary = [](const tc_instr &in) { return in.code == TC_I_UNARY && in.op != TC_SQRT; };
  for (int k = 0; k < p.n_code; ++k) {
    tc_instr &in = p.code[k];
    if (!writes(in) || generic_unary(in)) continue;  // no result, or one that goes to the file itself
    const int r = in.dst;
    // a row statistic stays where the row kernel keeps it: its readers take it from there
    const int stat = in.code == TC_I_LOAD ? p.places[in.slot].stat : -1;
    bool to_file = false;
    for (int j = k + 1; j < p.n_code; ++j) {
      tc_instr &next = p.code[j];
      const bool by_a = reads_a(next) && next.a == r, by_b = reads_b(next) && next.b == r;
      if (by_a || by_b) {
        if (j == k + 1 && !generic_unary(next)) {
          next.reserved |= (by_a ? A_PREV : 0) | (by_b ? B_PREV : 0);
        } else if (stat >= 0 && !generic_unary(next)) {
          if (by_a) next.reserved |= A_STAT | uint16_t(stat << 8);
          if (by_b) next.reserved |= B_STAT | uint16_t(stat << 12);
        } else {
          to_file = true;
        }
      }
      if (writes(next) && next.dst == r) break;  // read (if at all) before it is written again
    }
    if (to_file) in.reserved |= SPILL;
  }
  // The file keeps rows only for the registers that pass through it (a
  // result written there, an operand read from there, a generic unary's
  // operand and result); its register fields are renumbered to those rows.
  // Fields that never reach the file keep row 0.
  int row_of[REGISTERS];
  for (int r = 0; r < REGISTERS; ++r) row_of[r] = -1;
  int rows = 0;
  auto use = [&](int r) {
    if (row_of[r] < 0) row_of[r] = rows++;
  };
  for (int k = 0; k < p.n_code; ++k) {
    const tc_instr &in = p.code[k];
    if (generic_unary(in)) {
      use(in.a);
      use(in.dst);
      continue;
    }
    if (reads_a(in) && !(in.reserved & (A_PREV | A_STAT))) use(in.a);
    if (reads_b(in) && !(in.reserved & (B_PREV | B_STAT))) use(in.b);
    if (in.reserved & SPILL) use(in.dst);
  }
  for (int k = 0; k < p.n_code; ++k) {
    tc_instr &in = p.code[k];
    in.a = uint8_t(std::max(row_of[in.a < REGISTERS ? in.a : 0], 0));
    in.b = uint8_t(std::max(row_of[in.b < REGISTERS ? in.b : 0], 0));
    in.dst = uint8_t(std::max(row_of[in.dst < REGISTERS ? in.dst : 0], 0));
  }
  p.n_regs = std::max(rows, 1);
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
  p.n_regs = 1;
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
    p.code[k].reserved = 0;
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
      p.places[j].stat = -1;
      p.places[j].source = -1;
      continue;
    }
    if (int st = take_place(places[j], j, rows, cols, p.places[j])) return st;
    if (!p.places[j].in_order) p.needs_rc = 1;
    else if (p.n_ahead < 4) p.ahead[p.n_ahead++] = int(j);
  }
  for (uint32_t s = 0; s < n_stats; ++s) {
    const uint32_t of = stats[s].of_place;
    if (is_stat[of]) return fail(TC_EINVAL, "fused: row statistic %u is of a statistic", s);
    int k = 0;
    while (k < p.n_stat_sources && p.stat_source[k] != int(of)) ++k;
    if (k == p.n_stat_sources) {
      if (k == MAX_STAT_SOURCES) return fail(TC_EINVAL, "fused: statistics of more than %d inputs", MAX_STAT_SOURCES);
      p.stat_source[p.n_stat_sources++] = int(of);
      p.places[of].source = k;
    }
    p.places[stats[s].into_place].stat = 2 * k + (stats[s].statistic == TC_ROW_DEVIATIONS ? 1 : 0);
  }
  for (uint32_t j = 0; j < n_outputs; ++j) {
    if (!outputs[j] || !storage_type(out_dtypes[j])) return fail(TC_EINVAL, "fused: output %u", j);
    p.out[j] = outputs[j];
    p.out_dtype[j] = out_dtypes[j];
  }
  mark_forwarding(p);  // after the places: a statistic's loads are known
  return TC_OK;
}

// The register file of a block of the interpreter: the program's registers,
// E elements per thread.
size_t register_file_bytes(const Program &p, int E) { return size_t(p.n_regs) * INTERP_BLOCK * E * sizeof(float); }

// Blocks for an interpreter kernel with `smem` bytes of dynamic shared
// memory: as many as fit on every SM at once, at most `wanted`.
template <class K> unsigned interp_grid(K kernel, size_t smem, long long wanted) {
  // above 48 KB with the kernel's own static shared memory, a launch needs
  // the kernel's limit raised first
  if (smem > 40 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, INTERP_BLOCK, smem) != cudaSuccess) {
    cudaGetLastError();
    per_sm = 1;
  }
  return unsigned(std::max(1LL, std::min(wanted, (long long)sm_count() * std::max(per_sm, 1))));
}

// The row kernels stage each statistic source's row on chip while the
// block's shared memory stays within this bound (four blocks per SM).
constexpr size_t STAGE_LIMIT = 54 * 1024;

// Threads per row for rows of `cols` elements: 8 lanes up to 4 groups of
// ROW_GROUP each, a warp up to 8 groups each, else a block of INTERP_BLOCK.  f(lanes) with lanes a
// compile-time constant.
template <class F> int with_lanes(long long cols, F &&f) {
  if (cols <= 4 * 8 * ROW_GROUP) return f(std::integral_constant<int, 8>{});
  if (cols <= 8 * 32 * ROW_GROUP) return f(std::integral_constant<int, 32>{});
  return f(std::integral_constant<int, INTERP_BLOCK>{});
}

// Launch the row kernel (statistics, or sums along rows) for `p`.
// With `sums`: fused_sum along rows.
template <class T> int launch_rows(const Program &p, void *sums, cudaStream_t s, const char *what) {
  return with_lanes(p.cols, [&](auto lanes) {
    constexpr int LANES = decltype(lanes)::value, SLOTS = INTERP_BLOCK / LANES;
    const long long wanted = (p.rows + SLOTS - 1) / SLOTS;
    const size_t regs = register_file_bytes(p, ROW_GROUP);
    const int stage_cols = int((p.cols + ROW_GROUP - 1) / ROW_GROUP * ROW_GROUP);
    const size_t staged = regs + size_t(SLOTS) * p.n_stat_sources * stage_cols * sizeof(float);
    auto k = fused_rows_kernel<T, LANES>;
    if (p.n_stat_sources > 0 && p.cols <= (1LL << 30) && staged <= STAGE_LIMIT)
      k<<<interp_grid(k, staged, wanted), INTERP_BLOCK, staged, s>>>(p, sums, stage_cols);
    else
      k<<<interp_grid(k, regs, wanted), INTERP_BLOCK, regs, s>>>(p, sums, 0);
    return check_launch(what);
  });
}

// ---------------------------------------------------------------------------
// Programs the optimizers build, run by their dedicated kernels.  The
// reference's rules reach a backend as fused programs (Rule::update calls
// P::fused with the rule's program, optim.rs:773-787, 826-846, 892-904,
// 948-964, 1048-1099).  A program whose computation is one of those updates
// (the same operations on the same operands, each rounded to the program's
// type, so the same bits) over in-order places of the program's type, with
// the updated places written in place, runs as the rule's kernel instead of
// the interpreter.  The match is on the dataflow, not on the instructions'
// order or registers; commutative operations match either way round.
// ---------------------------------------------------------------------------
struct Expr {
  int kind, op, a, b, place;
  float value;
};

struct Dataflow {
  std::vector<Expr> e;
  int out[MAX_OUTPUTS];
  int n_out;
  int dtype;

  float in_type(float x) const {
    if (dtype == TC_F32) return x;
    return dtype == TC_BF16 ? bf16_bits_to_f32(f32_to_bf16_bits(x)) : f16_bits_to_f32(f32_to_f16_bits(x));
  }
  bool load(int n, int &place) const {
    if (n < 0 || e[n].kind != TC_I_LOAD) return false;
    place = e[n].place;
    return true;
  }
  bool is_load(int n, int place) const { return n >= 0 && e[n].kind == TC_I_LOAD && e[n].place == place; }
  bool cnst(int n, float &v) const {
    if (n < 0 || e[n].kind != TC_I_CONST) return false;
    v = e[n].value;
    return true;
  }
  bool bin(int n, int op, int &x, int &y) const {
    if (n < 0 || e[n].kind != TC_I_BINARY || e[n].op != op) return false;
    x = e[n].a, y = e[n].b;
    return true;
  }
  // n = x·c (either way round) with c a constant
  bool mul_const(int n, int &x, float &c) const {
    int a, b;
    if (!bin(n, TC_MUL, a, b)) return false;
    if (cnst(b, c)) return x = a, true;
    if (cnst(a, c)) return x = b, true;
    return false;
  }
  // n = g·g with g a load of `place`
  bool square(int n, int place) const {
    int a, b;
    return bin(n, TC_MUL, a, b) && is_load(a, place) && is_load(b, place);
  }
  bool same(int a, int b) const {
    if (a == b) return true;
    if (a < 0 || b < 0) return false;
    const Expr &x = e[a], &y = e[b];
    if (x.kind != y.kind || x.op != y.op) return false;
    switch (x.kind) {
      case TC_I_LOAD: return x.place == y.place;
      case TC_I_CONST: return x.value == y.value;
      case TC_I_UNARY: return same(x.a, y.a);
      default: {
        if (same(x.a, y.a) && same(x.b, y.b)) return true;
        const bool comm = x.kind == TC_I_BINARY && (x.op == TC_ADD || x.op == TC_MUL);
        return comm && same(x.a, y.b) && same(x.b, y.a);
      }
    }
  }
  // n = l + r with one side matching `first` and the other `second`
  template <class F, class G> bool add_of(int n, F &&first, G &&second) const {
    int a, b;
    if (!bin(n, TC_ADD, a, b)) return false;
    return (first(a) && second(b)) || (first(b) && second(a));
  }
  // p' = p - ((g / (sqrt(s) + eps)) · rate), s matching `state` (descend)
  bool descend(int n, int p_place, int g_place, int state, float &eps, float &rate) const {
    int x, y, q, num, den;
    if (!bin(n, TC_SUB, x, y) || !is_load(x, p_place) || !mul_const(y, q, rate)) return false;
    if (!bin(q, TC_DIV, num, den) || !is_load(num, g_place)) return false;
    return add_of(den,
                  [&](int r) { return r >= 0 && e[r].kind == TC_I_UNARY && e[r].op == TC_SQRT && same(e[r].a, state); },
                  [&](int c) { return cnst(c, eps); });
  }
};

bool build_dataflow(int dtype, const tc_instr *code, uint32_t n_code, uint32_t n_outputs, Dataflow &d) {
  d.dtype = dtype;
  d.n_out = int(n_outputs);
  int reg[REGISTERS];
  for (int &r : reg) r = -1;
  for (int &o : d.out) o = -1;
  for (uint32_t k = 0; k < n_code; ++k) {
    const tc_instr &in = code[k];
    Expr x{int(in.code), int(in.op), -1, -1, -1, 0.0f};
    switch (in.code) {
      case TC_I_LOAD: x.op = 0, x.place = in.slot; break;
      case TC_I_CONST: x.op = 0, x.value = d.in_type(in.value); break;
      case TC_I_UNARY: x.a = reg[in.a]; break;
      case TC_I_STORE:
        if (d.out[in.slot] >= 0) return false;  // an output stored twice
        d.out[in.slot] = reg[in.a];
        continue;
      default: x.a = reg[in.a], x.b = reg[in.b];
    }
    d.e.push_back(x);
    reg[in.dst] = int(d.e.size()) - 1;
  }
  for (uint32_t j = 0; j < n_outputs; ++j)
    if (d.out[j] < 0) return false;
  return true;
}

// TC_OK or an error if a rule's kernel ran; -1 if the program is no rule's.
int run_as_rule(int dtype, size_t n, const tc_instr *code, uint32_t n_code, const Program &p,
                void *const *outputs, const int *out_dtypes, uint32_t n_outputs, void *stream) {
  if (n_outputs < 1 || n_outputs > 3) return -1;
  Dataflow d;
  if (!build_dataflow(dtype, code, n_code, n_outputs, d)) return -1;
  const size_t esz = dtype_bytes(dtype);
  auto at = [&](int j) { return static_cast<char *>(const_cast<void *>(p.places[j].data)) + p.places[j].offset * esz; };
  // every place read in order, in the program's type; outputs of that type
  for (int j = 0; j < p.n_places; ++j)
    if (!p.places[j].in_order || p.places[j].dtype != dtype || p.places[j].stat >= 0) return -1;
  for (uint32_t k = 0; k < n_outputs; ++k)
    if (out_dtypes[k] != dtype) return -1;
  // `place` is updated in place as output k; `g` is read only
  auto in_place = [&](int place, int k) { return outputs[k] == at(place); };
  auto read_only = [&](int place) {
    for (uint32_t k = 0; k < n_outputs; ++k)
      if (outputs[k] == at(place)) return false;
    return true;
  };
  int pp = -1, pg = -1, ps = -1;
  float rate = 0.0f, c = 0.0f, eps = 0.0f;
  if (n_outputs == 1) {  // Sgd: p - g·rate
    int x, y, u;
    if (d.bin(d.out[0], TC_SUB, x, y) && d.load(x, pp) && d.mul_const(y, u, rate) && d.load(u, pg) && pp != pg &&
        in_place(pp, 0) && read_only(pg))
      return tc_sgd(dtype, n, outputs[0], at(pg), rate, stream);
    return -1;
  }
  if (n_outputs == 2) {
    const int s = d.out[1];
    int x, y, step;
    // Momentum: v' = v·mu + g; p' = p - step·rate, step = v' or g + v'·mu
    if (d.add_of(s, [&](int a) { return d.load(a, pg); },
                 [&](int b) { int v; return d.mul_const(b, v, c) && d.load(v, ps); }) &&
        d.bin(d.out[0], TC_SUB, x, y) && d.load(x, pp) && d.mul_const(y, step, rate) && pp != pg && ps != pg &&
        pp != ps && in_place(pp, 0) && in_place(ps, 1) && read_only(pg)) {
      if (d.same(step, s)) return tc_momentum(dtype, n, outputs[0], at(pg), outputs[1], rate, c, 0, stream);
      float c2;
      if (d.add_of(step, [&](int a) { return d.is_load(a, pg); },
                   [&](int b) { int v; return d.mul_const(b, v, c2) && c2 == c && d.same(v, s); }))
        return tc_momentum(dtype, n, outputs[0], at(pg), outputs[1], rate, c, 1, stream);
      return -1;
    }
    // AdaGrad: s' = s + g·g, RmsProp: s' = s·rho + (g·g)·(1 - rho); p' by descend
    int sub_x, sub_y;
    if (!d.bin(d.out[0], TC_SUB, sub_x, sub_y) || !d.load(sub_x, pp)) return -1;
    int num, den, q;
    if (!d.mul_const(sub_y, q, rate) || !d.bin(q, TC_DIV, num, den) || !d.load(num, pg)) return -1;
    if (pp == pg || !in_place(pp, 0) || !read_only(pg)) return -1;
    float rho = 0.0f, share = 0.0f;
    const bool adagrad =
        d.add_of(s, [&](int a) { return d.load(a, ps); }, [&](int b) { return d.square(b, pg); });
    const bool rmsprop =
        !adagrad && d.add_of(s, [&](int a) { int v; return d.mul_const(a, v, rho) && d.load(v, ps); },
                             [&](int b) { int v; return d.mul_const(b, v, share) && d.square(v, pg); });
    if ((!adagrad && !rmsprop) || ps == pp || ps == pg || !in_place(ps, 1)) return -1;
    if (!d.descend(d.out[0], pp, pg, s, eps, rate)) return -1;
    if (adagrad) return tc_adagrad(dtype, n, outputs[0], at(pg), outputs[1], rate, eps, stream);
    if (share != d.in_type(1.0f - rho)) return -1;  // the kernel takes 1 - rho in the type from rho
    return tc_rmsprop(dtype, n, outputs[0], at(pg), outputs[1], rate, rho, eps, stream);
  }
  // Adam: m' = m·b1 + g·s1 and v' = v·b2 + (g·g)·s2 (resumed), or g·s1 and
  // (g·g)·s2 (the first step, into fresh outputs); p' = p - ((m'·c1) /
  // (sqrt(v'·c2) + eps))·rate, with s = 1 - b in the type.
  int pm = -1, pv = -1;
  float b1 = 0.0f, b2 = 0.0f, s1 = 0.0f, s2 = 0.0f, c1 = 0.0f, c2 = 0.0f;
  const int m = d.out[1], v = d.out[2];
  auto fresh_first = [&](int r) { int u; return d.mul_const(r, u, s1) && d.load(u, pg); };
  auto fresh_second = [&](int r) { int u; return d.mul_const(r, u, s2) && d.square(u, pg); };
  bool resumed = d.add_of(m, [&](int a) { int u; return d.mul_const(a, u, b1) && d.load(u, pm); }, fresh_first) &&
                 d.add_of(v, [&](int a) { int u; return d.mul_const(a, u, b2) && d.load(u, pv); }, fresh_second);
  if (!resumed) {
    if (!fresh_first(m) || !fresh_second(v)) return -1;
    // the kernel derives the shares from the betas: the betas that give them
    b1 = d.in_type(1.0f - s1), b2 = d.in_type(1.0f - s2);
  }
  if (s1 != d.in_type(1.0f - b1) || s2 != d.in_type(1.0f - b2)) return -1;
  int x, y, q, num, den, mx, vx;
  if (!d.bin(d.out[0], TC_SUB, x, y) || !d.load(x, pp) || !d.mul_const(y, q, rate) || !d.bin(q, TC_DIV, num, den))
    return -1;
  if (!d.mul_const(num, mx, c1) || !d.same(mx, m)) return -1;
  if (!d.add_of(den,
                [&](int r) {
                  return r >= 0 && d.e[r].kind == TC_I_UNARY && d.e[r].op == TC_SQRT && d.mul_const(d.e[r].a, vx, c2) &&
                         d.same(vx, v);
                },
                [&](int r) { return d.cnst(r, eps); }))
    return -1;
  if (pp == pg || !in_place(pp, 0) || !read_only(pg)) return -1;
  if (resumed) {
    if (pm == pv || pm == pp || pv == pp || pm == pg || pv == pg || !in_place(pm, 1) || !in_place(pv, 2)) return -1;
  } else {
    // fresh outputs: none of them may be a place the program reads
    for (int j = 0; j < p.n_places; ++j)
      if (outputs[1] == at(j) || outputs[2] == at(j)) return -1;
    if (outputs[1] == outputs[2] || outputs[1] == outputs[0] || outputs[2] == outputs[0]) return -1;
  }
  return tc_adam(dtype, n, outputs[0], at(pg), outputs[1], outputs[2], resumed ? 1 : 0, rate, b1, b2, eps, c1, c2,
                 stream);
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
  if (int st = run_as_rule(dtype, rows * cols, code, n_code, p, outputs, out_dtypes, n_outputs, stream); st != -1)
    return st;
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    const size_t regs = register_file_bytes(p, FLAT_GROUP);
    auto k = fused_kernel<T>;
    const long long wanted = ((long long)(rows * cols) + FLAT_GROUP * INTERP_BLOCK - 1) / (FLAT_GROUP * INTERP_BLOCK);
    k<<<interp_grid(k, regs, wanted), INTERP_BLOCK, regs, as_stream(stream)>>>(p);
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
    return launch_rows<T>(p, nullptr, as_stream(stream), "fused program with statistics");
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
      return launch_rows<T>(p, sums, s, "fused sum (rows)");
    }
    // column groups side by side in a block, the rest of the block bands
    const long long col_groups = ((long long)cols + COL_GROUP - 1) / COL_GROUP;
    const int groups = int(std::min<long long>(INTERP_BLOCK, col_groups)), per_block = INTERP_BLOCK / groups;
    const long long col_blocks = (col_groups + groups - 1) / groups;
    // about 8 blocks per SM, each band 16 rows or more
    const long long want = std::max(1LL, (long long)sm_count() * 8 / col_blocks) * per_block;
    const long long band = std::max(16LL, ((long long)rows + want - 1) / want);
    const long long bands = ((long long)rows + band - 1) / band;
    const long long band_rows = (bands + per_block - 1) / per_block;  // blockIdx.y
    float *partial = nullptr;
    if (bands > 1)
      if (int st = scratch(size_t(bands) * cols * sizeof(float), reinterpret_cast<void **>(&partial), s)) return st;
    fused_cols_kernel<T><<<dim3(unsigned(col_blocks), unsigned(band_rows)), INTERP_BLOCK,
                           register_file_bytes(p, COL_GROUP), s>>>(p, groups, band, bands, partial, sums);
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
    return with_lanes((long long)cols, [&](auto lanes) {
      constexpr int LANES = decltype(lanes)::value, SLOTS = INTERP_BLOCK / LANES;
      auto k = row_moments_kernel<T, LANES>;
      k<<<interp_grid(k, 0, ((long long)rows + SLOTS - 1) / SLOTS), INTERP_BLOCK, 0, as_stream(stream)>>>(
          pl, (long long)rows, (long long)cols, means, deviations);
      return check_launch("row moments");
    });
  });
}

}  // extern "C"
