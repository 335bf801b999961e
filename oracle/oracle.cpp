// oracle.cpp — CPU restatement of tensorcrate's Host backend (test
// infrastructure only: the checker and the timed CPU baseline, never part of
// the product).  Built with -ffp-contract=off so that a*b+c is two roundings
// unless a function below calls std::fma or an FMA intrinsic where the
// reference does.
#include "oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// f16 / bf16 <-> f32.  Crate `half` 2.7.1 (Cargo.lock:51-54) converts with
// round-to-nearest-even and keeps a NaN quiet with the top of its payload;
// the compact types compute every operation in f32 and round once
// (src/compact.rs:5-22).
// ---------------------------------------------------------------------------
inline uint32_t bits_of(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float float_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

inline uint16_t f32_to_bf16(float f) {
  uint32_t x = bits_of(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return uint16_t((x >> 16) | 0x0040u);
  const uint32_t round_bit = 0x8000u;
  if ((x & round_bit) && (x & (3u * round_bit - 1u))) return uint16_t((x >> 16) + 1u);
  return uint16_t(x >> 16);
}
inline float bf16_to_f32(uint16_t h) { return float_of(uint32_t(h) << 16); }

inline uint16_t f32_to_f16(float f) {
  uint32_t x = bits_of(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) {
    if (man == 0) return uint16_t(sign | 0x7c00u);
    return uint16_t(sign | 0x7c00u | 0x0200u | (man >> 13));
  }
  int e = int(exp) - 127 + 15;
  if (e >= 0x1f) return uint16_t(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    man |= 0x800000u;
    uint32_t shift = uint32_t(14 - e);
    uint32_t half_man = man >> shift;
    uint32_t round_bit = 1u << (shift - 1);
    if ((man & round_bit) && (man & (3u * round_bit - 1u))) half_man++;
    return uint16_t(sign | half_man);
  }
  uint32_t out = sign | (uint32_t(e) << 10) | (man >> 13);
  const uint32_t round_bit = 0x1000u;
  if ((man & round_bit) && (man & (3u * round_bit - 1u))) out++;
  return uint16_t(out);
}
inline float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0x1fu) return float_of(sign | 0x7f800000u | (man << 13));
  if (exp == 0) {
    if (man == 0) return float_of(sign);
    // subnormal: value = man * 2^-24, exact in f32
    float v = float(man) * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  return float_of(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

// Element access: load widens exactly, store rounds once.
struct F32 { using S = float;
  static float load(const void *p, size_t i) { return static_cast<const float *>(p)[i]; }
  static void store(void *p, size_t i, float v) { static_cast<float *>(p)[i] = v; }
  static float round(float v) { return v; } };
struct F16 { using S = uint16_t;
  static float load(const void *p, size_t i) { return f16_to_f32(static_cast<const uint16_t *>(p)[i]); }
  static void store(void *p, size_t i, float v) { static_cast<uint16_t *>(p)[i] = f32_to_f16(v); }
  static float round(float v) { return f16_to_f32(f32_to_f16(v)); } };
struct BF16 { using S = uint16_t;
  static float load(const void *p, size_t i) { return bf16_to_f32(static_cast<const uint16_t *>(p)[i]); }
  static void store(void *p, size_t i, float v) { static_cast<uint16_t *>(p)[i] = f32_to_bf16(v); }
  static float round(float v) { return bf16_to_f32(f32_to_bf16(v)); } };

template <class F> int with_dtype(int dtype, F &&f) {
  switch (dtype) {
    case TC_F32: return f(F32{});
    case TC_F16: return f(F16{});
    case TC_BF16: return f(BF16{});
    default: return int(TC_EINVAL);
  }
}

// ---------------------------------------------------------------------------
// Scalar semantics, src/tensors/kernels.rs.
// ---------------------------------------------------------------------------
// f32::min / f32::max: IEEE minNum/maxNum, a number beats a NaN.
inline float min_num(float a, float b) { if (std::isnan(a)) return b; if (std::isnan(b)) return a; return b < a ? b : a; }
inline float max_num(float a, float b) { if (std::isnan(a)) return b; if (std::isnan(b)) return a; return b > a ? b : a; }

// Compare::value, kernels.rs:138-153.
inline float compare_value(int op, float a, float b) {
  switch (op) {
    case TC_MIN: return min_num(a, b);
    case TC_MAX: return max_num(a, b);
    case TC_MAX_SHARE: return a > b ? 1.0f : (a < b ? 0.0f : 0.5f);
    case TC_LESS: return a < b ? 1.0f : 0.0f;
    case TC_LESS_EQUAL: return a <= b ? 1.0f : 0.0f;
    case TC_GREATER: return a > b ? 1.0f : 0.0f;
    case TC_GREATER_EQUAL: return a >= b ? 1.0f : 0.0f;
  }
  return NAN;
}
// BinaryOp as Pairwise::value computes it, kernels.rs:431-441 (Rem is the
// truncated remainder, Rust's `%` on floats = fmod).
inline float binary_value(int op, float a, float b) {
  switch (op) {
    case TC_ADD: return a + b;
    case TC_SUB: return a - b;
    case TC_MUL: return a * b;
    case TC_DIV: return a / b;
    case TC_REM: return std::fmod(a, b);
  }
  return NAN;
}
// Pairwise::Power: f32::powf (src/numbers/primitive.rs:133-153).
inline float power_value(float a, float b) { return std::pow(a, b); }

inline bool valid_binary(int op) { return op >= TC_ADD && op <= TC_REM; }
inline bool valid_compare(int op) { return op >= TC_MIN && op <= TC_GREATER_EQUAL; }

// ---------------------------------------------------------------------------
// Layout, src/tensors/layout.rs.
// ---------------------------------------------------------------------------
struct Dims { uint32_t rank = 0; size_t v[TC_MAX_RANK] = {0}; };

// coalesce, layout.rs:419-446: drop axes of extent 1, merge an axis into the
// previous one wherever every operand steps across the pair as across one.
template <int N>
void coalesce(uint32_t rank, const size_t *shape, const size_t *const *strides, Dims &out_shape,
              Dims *out) {
  out_shape.rank = 0;
  for (int o = 0; o < N; ++o) out[o].rank = 0;
  for (uint32_t axis = 0; axis < rank; ++axis) {
    size_t extent = shape[axis];
    if (extent == 1) continue;
    uint32_t r = out_shape.rank;
    bool joins = r > 0;
    for (int o = 0; o < N && joins; ++o) joins = out[o].v[r - 1] == strides[o][axis] * extent;
    if (joins) {
      out_shape.v[r - 1] *= extent;
      for (int o = 0; o < N; ++o) out[o].v[r - 1] = strides[o][axis];
    } else {
      out_shape.v[r] = extent;
      out_shape.rank++;
      for (int o = 0; o < N; ++o) { out[o].v[r] = strides[o][axis]; out[o].rank++; }
    }
  }
}

// for_each_run, layout.rs:457-498: call run(starts, len, steps) for each
// innermost run of a row-major walk.
template <int N, class Run>
void for_each_run(uint32_t rank, const size_t *shape, const size_t *offsets,
                  const size_t *const *strides, Run &&run) {
  for (uint32_t a = 0; a < rank; ++a) if (shape[a] == 0) return;
  Dims cs; Dims cst[N];
  coalesce<N>(rank, shape, strides, cs, cst);
  size_t at[N];
  for (int o = 0; o < N; ++o) at[o] = offsets[o];
  uint32_t r = cs.rank;
  if (r == 0) { size_t steps[N] = {0}; run(at, size_t(1), steps); return; }
  size_t inner = cs.v[r - 1];
  size_t steps[N];
  for (int o = 0; o < N; ++o) steps[o] = cst[o].v[r - 1];
  size_t index[TC_MAX_RANK] = {0};
  for (;;) {
    run(at, inner, steps);
    uint32_t axis = r - 1;
    for (;;) {
      if (axis == 0) return;
      axis -= 1;
      index[axis] += 1;
      for (int o = 0; o < N; ++o) at[o] += cst[o].v[axis];
      if (index[axis] < cs.v[axis]) break;
      for (int o = 0; o < N; ++o) at[o] -= cst[o].v[axis] * cs.v[axis];
      index[axis] = 0;
    }
  }
}

// reach, layout.rs:136-149: one past the last element read, or 0 if none;
// SIZE_MAX on overflow.
size_t reach(uint32_t rank, const size_t *shape, size_t offset, const size_t *strides) {
  for (uint32_t a = 0; a < rank; ++a) if (shape[a] == 0) return 0;
  size_t end = offset;
  for (uint32_t a = 0; a < rank; ++a) {
    size_t span;
    if (__builtin_mul_overflow(shape[a] - 1, strides[a], &span)) return SIZE_MAX;
    if (__builtin_add_overflow(end, span, &end)) return SIZE_MAX;
  }
  if (end == SIZE_MAX) return SIZE_MAX;
  return end + 1;
}

size_t element_count(uint32_t rank, const size_t *shape) {
  size_t n = 1;
  for (uint32_t a = 0; a < rank; ++a) n *= shape[a];
  return n;
}

// check_strided, backend.rs:226-252.
bool check_strided(size_t len, uint32_t rank, const size_t *shape, size_t offset,
                   const size_t *strides) {
  if (rank > TC_MAX_RANK) return false;
  return reach(rank, shape, offset, strides) <= len;
}

void contiguous_strides(uint32_t rank, const size_t *shape, size_t *out) {
  size_t step = 1;
  for (int a = int(rank) - 1; a >= 0; --a) { out[a] = step; step *= shape[a]; }
}

// ---------------------------------------------------------------------------
// Threads for the same-shape elementwise kernels, as simd_dispatch::split
// (src/tensors/simd_dispatch.rs:54-76): windows of PARALLEL_GRAIN elements
// over all host threads once the output holds at least two of them.
// ---------------------------------------------------------------------------
int g_threads = 0;
constexpr size_t PARALLEL_GRAIN = 32 * 1024;

template <class K> void split(size_t n, K &&kernel) {
  int threads = g_threads > 0 ? g_threads : int(std::max(1u, std::thread::hardware_concurrency()));
  if (n < 2 * PARALLEL_GRAIN || threads == 1) { kernel(size_t(0), n); return; }
  size_t windows = (n + PARALLEL_GRAIN - 1) / PARALLEL_GRAIN;
  std::atomic<size_t> next{0};
  auto worker = [&] {
    for (;;) {
      size_t w = next.fetch_add(1);
      if (w >= windows) return;
      size_t lo = w * PARALLEL_GRAIN, hi = std::min(n, lo + PARALLEL_GRAIN);
      kernel(lo, hi);
    }
  };
  std::vector<std::thread> pool;
  int spawn = int(std::min<size_t>(size_t(threads), windows)) - 1;
  for (int t = 0; t < spawn; ++t) pool.emplace_back(worker);
  worker();
  for (auto &t : pool) t.join();
}

// ---------------------------------------------------------------------------
// f32 products, src/simd_x86.rs.  The Host dispatches on CPU features at run
// time; so does this.
// ---------------------------------------------------------------------------
bool has_avx2_fma() {
  static int cached = -1;
  if (cached < 0) cached = (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) ? 1 : 0;
  return cached == 1;
}

// matmul_avx, simd_x86.rs:1303-1327: for i, for p, broadcast a[i,p] and FMA
// it with b[p, j..j+8] into out[i, j..j+8]; the column tail is
// `out += a*b`, two roundings (Rust does not contract).
__attribute__((target("avx2,fma")))
void matmul_avx(const float *a, const float *b, size_t, size_t k, size_t n, float *out,
                size_t row0, size_t row1) {
  for (size_t i = row0; i < row1; ++i) {
    size_t arow = i * k, orow = i * n;
    for (size_t p = 0; p < k; ++p) {
      float value = a[arow + p];
      __m256 broadcast = _mm256_set1_ps(value);
      size_t brow = p * n;
      size_t j = 0;
      for (; j + 8 <= n; j += 8) {
        __m256 rhs = _mm256_loadu_ps(b + brow + j);
        __m256 cur = _mm256_loadu_ps(out + orow + j);
        _mm256_storeu_ps(out + orow + j, _mm256_fmadd_ps(broadcast, rhs, cur));
      }
      for (; j < n; ++j) out[orow + j] += value * b[brow + j];
    }
  }
}
void matmul_sse(const float *a, const float *b, size_t m, size_t k, size_t n, float *out, size_t row0, size_t row1);
// The same products per output element, for the tests' large cases only:
// each out[i, j] still runs p = 0..k in order with the same FMA (or, in the
// column tail, the same unfused multiply-add), so the bits are matmul_avx's.
// Only the loop nest differs (column blocks that stay in cache across rows,
// row bands over threads).  The timed CPU baseline never takes this path.
int g_matmul_threads = 1;
__attribute__((target("avx2,fma")))
void matmul_avx_blocked(const float *a, const float *b, size_t k, size_t n, float *out, size_t row0,
                        size_t row1) {
  constexpr size_t JB = 64;
  const size_t body = n / 8 * 8;
  for (size_t j0 = 0; j0 < body; j0 += JB) {
    const size_t j1 = std::min(body, j0 + JB);
    for (size_t i = row0; i < row1; ++i) {
      const size_t arow = i * k, orow = i * n;
      __m256 acc[JB / 8];
      const size_t lanes = (j1 - j0) / 8;
      for (size_t q = 0; q < lanes; ++q) acc[q] = _mm256_loadu_ps(out + orow + j0 + 8 * q);
      for (size_t p = 0; p < k; ++p) {
        const __m256 broadcast = _mm256_set1_ps(a[arow + p]);
        const float *brow = b + p * n + j0;
        for (size_t q = 0; q < lanes; ++q) acc[q] = _mm256_fmadd_ps(broadcast, _mm256_loadu_ps(brow + 8 * q), acc[q]);
      }
      for (size_t q = 0; q < lanes; ++q) _mm256_storeu_ps(out + orow + j0 + 8 * q, acc[q]);
    }
  }
  if (body < n)
    for (size_t i = row0; i < row1; ++i)
      for (size_t p = 0; p < k; ++p) {
        const float value = a[i * k + p];
        for (size_t j = body; j < n; ++j) out[i * n + j] += value * b[p * n + j];
      }
}
// Rows [row0, row1) of the SIMD product: matmul_avx as the Host runs it, or,
// when the tests asked for threads, the blocked form over row bands.
void matmul_simd_rows(const float *a, const float *b, size_t m, size_t k, size_t n, float *out, size_t row0,
                      size_t row1) {
  if (!has_avx2_fma()) { matmul_sse(a, b, m, k, n, out, row0, row1); return; }
  const size_t rows = row1 - row0;
  if (g_matmul_threads <= 1 || rows < 2) { matmul_avx(a, b, m, k, n, out, row0, row1); return; }
  const size_t bands = std::min<size_t>(size_t(g_matmul_threads), rows);
  std::vector<std::thread> pool;
  for (size_t t = 0; t < bands; ++t) {
    const size_t lo = row0 + rows * t / bands, hi = row0 + rows * (t + 1) / bands;
    pool.emplace_back([=] { matmul_avx_blocked(a, b, k, n, out, lo, hi); });
  }
  for (auto &t : pool) t.join();
}
// matmul_sse, simd_x86.rs:1334-1358: the same, unfused throughout.
void matmul_sse(const float *a, const float *b, size_t m, size_t k, size_t n, float *out,
                size_t row0, size_t row1) {
  (void)m;
  for (size_t i = row0; i < row1; ++i) {
    size_t arow = i * k, orow = i * n;
    for (size_t p = 0; p < k; ++p) {
      float value = a[arow + p];
      size_t brow = p * n;
      for (size_t j = 0; j < n; ++j) out[orow + j] = out[orow + j] + value * b[brow + j];
    }
  }
}

// dot_avx, simd_x86.rs:72-104: four 8-lane FMA accumulators over blocks of
// 32, summed pairwise lane by lane, then the 8 lanes in order; then 8-lane
// blocks of unfused products; then a scalar tail.
__attribute__((target("avx2,fma")))
float dot_avx(const float *a, const float *b, size_t len) {
  size_t i = 0;
  __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
  while (i + 32 <= len) {
    for (int lane = 0; lane < 4; ++lane) {
      size_t off = i + size_t(lane) * 8;
      acc[lane] = _mm256_fmadd_ps(_mm256_loadu_ps(a + off), _mm256_loadu_ps(b + off), acc[lane]);
    }
    i += 32;
  }
  __m256 total = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
  float lanes[8];
  _mm256_storeu_ps(lanes, total);
  // Rust's `Sum for f32` folds from -0.0.
  float sum = -0.0f;
  for (int l = 0; l < 8; ++l) sum += lanes[l];
  while (i + 8 <= len) {
    _mm256_storeu_ps(lanes, _mm256_mul_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i)));
    float part = -0.0f;
    for (int l = 0; l < 8; ++l) part += lanes[l];
    sum += part;
    i += 8;
  }
  for (; i < len; ++i) sum += a[i] * b[i];
  return sum;
}
// dot_sse, simd_x86.rs:110-135: four 4-lane unfused accumulators.
float dot_sse(const float *a, const float *b, size_t len) {
  size_t i = 0;
  float acc[4][4] = {{0}};
  while (i + 16 <= len) {
    for (int lane = 0; lane < 4; ++lane)
      for (int l = 0; l < 4; ++l) acc[lane][l] = acc[lane][l] + a[i + lane * 4 + l] * b[i + lane * 4 + l];
    i += 16;
  }
  float sum = -0.0f;
  for (int l = 0; l < 4; ++l) sum += (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  while (i + 4 <= len) {
    float part = -0.0f;
    for (int l = 0; l < 4; ++l) part += a[i + l] * b[i + l];
    sum += part;
    i += 4;
  }
  for (; i < len; ++i) sum += a[i] * b[i];
  return sum;
}
float dot_f32(const float *a, const float *b, size_t len) {
  return has_avx2_fma() ? dot_avx(a, b, len) : dot_sse(a, b, len);
}

constexpr size_t MIN_MATMUL_OPS = 512;  // HOST_MATMUL_DISPATCH_OPS, src/tensors/mod.rs:167

// Matrix<f32, Host>::matmul / matmul_add over output rows [row0, row1)
// (matrix.rs:580-666): the SIMD i-p-j path at or above 512 multiply-adds,
// else the scalar loops (i-j-p running sum for matmul, i-p-j for matmul_add).
void matmul_f32(const float *a, const float *b, size_t m, size_t k, size_t n, float *out,
                bool accumulate, size_t row0, size_t row1) {
  if (m * k * n >= MIN_MATMUL_OPS) {
    if (!accumulate)
      for (size_t i = row0; i < row1; ++i) std::fill(out + i * n, out + (i + 1) * n, 0.0f);
    matmul_simd_rows(a, b, m, k, n, out, row0, row1);
    return;
  }
  if (!accumulate) {
    for (size_t i = row0; i < row1; ++i)
      for (size_t j = 0; j < n; ++j) {
        float sum = 0.0f;
        for (size_t p = 0; p < k; ++p) sum = sum + a[i * k + p] * b[p * n + j];
        out[i * n + j] = sum;
      }
  } else {
    for (size_t i = row0; i < row1; ++i)
      for (size_t p = 0; p < k; ++p)
        for (size_t j = 0; j < n; ++j) out[i * n + j] = out[i * n + j] + a[i * k + p] * b[p * n + j];
  }
}

// Real::from_f64 (src/numbers/mod.rs:76-86): an f64 rounded to the element
// type once (crate half rounds f64 -> f16/bf16 directly).  Rounding to f32 by
// round-to-odd first keeps that single rounding exact, since f32 carries more
// than twice the compact types' precision plus two bits.
template <class T> float from_f64(double d) {
  float f = float(d);
  if (std::is_same<T, F32>::value) return f;
  if (std::isfinite(d) && double(f) != d && std::isfinite(f)) {
    uint32_t u = bits_of(f);
    if (std::fabs(double(f)) > std::fabs(d)) u -= 1;
    f = float_of(u | 1u);
  }
  return T::round(f);
}

template <class T> std::vector<float> widen_all(const void *p, size_t n) {
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = T::load(p, i);
  return out;
}

// A transposed copy, as Kernels::transpose then matmul_add is the default
// matmul_transposed_add (kernels.rs:975-985).
template <class T> std::vector<typename T::S> transposed_copy(const void *m, size_t rows, size_t cols) {
  using S = typename T::S;
  const S *src = static_cast<const S *>(m);
  std::vector<S> out(rows * cols);
  for (size_t i = 0; i < rows; ++i)
    for (size_t j = 0; j < cols; ++j) out[j * rows + i] = src[i * cols + j];
  return out;
}

template <class T>
int matmul_rows(size_t rows, size_t inner, size_t cols, const void *a, const void *b, void *c,
                bool accumulate, size_t row0, size_t row1) {
  if (std::is_same<T, F32>::value) {
    matmul_f32(static_cast<const float *>(a), static_cast<const float *>(b), rows, inner, cols,
               static_cast<float *>(c), accumulate, row0, row1);
    return int(TC_OK);
  }
  // compact::matmul, src/compact.rs:232-253: widen once, the f32 product
  // (addend widened too when accumulating), round each output once.
  std::vector<float> left(( row1 - row0) * inner);
  for (size_t i = row0; i < row1; ++i)
    for (size_t p = 0; p < inner; ++p) left[(i - row0) * inner + p] = T::load(a, i * inner + p);
  std::vector<float> right = widen_all<T>(b, inner * cols);
  std::vector<float> out((row1 - row0) * cols, 0.0f);
  if (accumulate)
    for (size_t i = row0; i < row1; ++i)
      for (size_t j = 0; j < cols; ++j) out[(i - row0) * cols + j] = T::load(c, i * cols + j);
  // The band is a matrix of its own; the MIN_MATMUL_OPS choice is made on
  // the whole product, as the reference makes it.
  size_t band = row1 - row0;
  if (rows * inner * cols >= MIN_MATMUL_OPS) {
    matmul_simd_rows(left.data(), right.data(), band, inner, cols, out.data(), 0, band);
  } else {
    matmul_f32(left.data(), right.data(), band, inner, cols, out.data(), accumulate, 0, band);
  }
  for (size_t i = row0; i < row1; ++i)
    for (size_t j = 0; j < cols; ++j) T::store(c, i * cols + j, out[(i - row0) * cols + j]);
  return int(TC_OK);
}

}  // namespace

// ===========================================================================
// exported
// ===========================================================================
extern "C" {

void orc_set_threads(int threads) { g_threads = threads; }
// Threads for the large products of the tests (same bits; see
// matmul_avx_blocked).  1, the default, is the Host's single thread.
void orc_set_matmul_threads(int threads) { g_matmul_threads = threads < 1 ? 1 : threads; }

void orc_narrow(int dtype, const float *in, void *out, size_t n) {
  with_dtype(dtype, [&](auto t) { using T = decltype(t); for (size_t i = 0; i < n; ++i) T::store(out, i, in[i]); return 0; });
}
void orc_widen(int dtype, const void *in, float *out, size_t n) {
  with_dtype(dtype, [&](auto t) { using T = decltype(t); for (size_t i = 0; i < n; ++i) out[i] = T::load(in, i); return 0; });
}

int orc_coalesce(uint32_t rank, const size_t *shape, uint32_t n_ops, const size_t *strides,
                 uint32_t *out_rank, size_t *out_shape, size_t *out_strides) {
  if (rank > TC_MAX_RANK || n_ops < 1 || n_ops > 3) return int(TC_EINVAL);
  const size_t *ops[3] = {strides, strides + rank, strides + 2 * rank};
  Dims cs; Dims cst[3];
  if (n_ops == 1) coalesce<1>(rank, shape, ops, cs, cst);
  else if (n_ops == 2) coalesce<2>(rank, shape, ops, cs, cst);
  else coalesce<3>(rank, shape, ops, cs, cst);
  *out_rank = cs.rank;
  for (uint32_t a = 0; a < cs.rank; ++a) out_shape[a] = cs.v[a];
  for (uint32_t o = 0; o < n_ops; ++o)
    for (uint32_t a = 0; a < cs.rank; ++a) out_strides[o * cs.rank + a] = cst[o].v[a];
  return int(TC_OK);
}

// broadcast_shape, layout.rs:330-341.
int orc_broadcast_shape(uint32_t lrank, const size_t *left, uint32_t rrank, const size_t *right,
                        uint32_t *out_rank, size_t *out_shape) {
  uint32_t rank = std::max(lrank, rrank);
  if (rank > TC_MAX_RANK) return int(TC_EINVAL);
  for (uint32_t axis = 0; axis < rank; ++axis) {
    uint32_t from_end = rank - axis;
    size_t l = lrank >= from_end ? left[lrank - from_end] : 1;
    size_t r = rrank >= from_end ? right[rrank - from_end] : 1;
    if (l == r) out_shape[axis] = l;
    else if (l == 1) out_shape[axis] = r;
    else if (r == 1) out_shape[axis] = l;
    else return int(TC_EINVAL);
  }
  *out_rank = rank;
  return int(TC_OK);
}

// broadcast_strides, layout.rs:347-363.
int orc_broadcast_strides(uint32_t rank, const size_t *shape, const size_t *strides,
                          uint32_t trank, const size_t *target, size_t *out_strides) {
  if (trank < rank || trank > TC_MAX_RANK) return int(TC_EINVAL);
  uint32_t added = trank - rank;
  for (uint32_t a = 0; a < trank; ++a) out_strides[a] = 0;
  for (uint32_t axis = 0; axis < rank; ++axis) {
    size_t wanted = target[added + axis];
    if (shape[axis] == wanted) out_strides[added + axis] = strides[axis];
    else if (shape[axis] == 1) out_strides[added + axis] = 0;
    else return int(TC_EINVAL);
  }
  return int(TC_OK);
}

int orc_walk(uint32_t rank, const size_t *shape, size_t offset, const size_t *strides,
             size_t *out_positions) {
  if (rank > TC_MAX_RANK) return int(TC_EINVAL);
  size_t k = 0;
  const size_t *st[1] = {strides};
  size_t off[1] = {offset};
  for_each_run<1>(rank, shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
    for (size_t i = 0; i < len; ++i) out_positions[k++] = at[0] + i * steps[0];
  });
  return int(TC_OK);
}

// strided_copy_slice, backend.rs:255-274.
int orc_strided_copy(size_t elem, uint32_t rank, const size_t *shape, const void *src,
                     size_t src_len, size_t src_offset, const size_t *src_strides, void *dst) {
  if (!check_strided(src_len, rank, shape, src_offset, src_strides)) return int(TC_ERANGE);
  const char *s = static_cast<const char *>(src);
  char *d = static_cast<char *>(dst);
  size_t k = 0;
  const size_t *st[1] = {src_strides};
  size_t off[1] = {src_offset};
  for_each_run<1>(rank, shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
    if (steps[0] == 1) {
      std::memcpy(d + k * elem, s + at[0] * elem, len * elem);
      k += len;
    } else {
      for (size_t i = 0; i < len; ++i, ++k) std::memcpy(d + k * elem, s + (at[0] + i * steps[0]) * elem, elem);
    }
  });
  return int(TC_OK);
}

// strided_write_slice, backend.rs:277-300.
int orc_strided_write(size_t elem, void *target, size_t target_len, const tc_region *r) {
  if (r->rank > TC_MAX_RANK) return int(TC_EINVAL);
  if (!check_strided(r->source_len, r->rank, r->shape, r->from_offset, r->from_strides)) return int(TC_ERANGE);
  if (!check_strided(target_len, r->rank, r->shape, r->to_offset, r->to_strides)) return int(TC_ERANGE);
  const char *s = static_cast<const char *>(r->source);
  char *d = static_cast<char *>(target);
  const size_t *st[2] = {r->from_strides, r->to_strides};
  size_t off[2] = {r->from_offset, r->to_offset};
  for_each_run<2>(r->rank, r->shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
    if (steps[0] == 1 && steps[1] == 1) std::memcpy(d + at[1] * elem, s + at[0] * elem, len * elem);
    else
      for (size_t i = 0; i < len; ++i)
        std::memcpy(d + (at[1] + i * steps[1]) * elem, s + (at[0] + i * steps[0]) * elem, elem);
  });
  return int(TC_OK);
}

// assemble_slices, backend.rs:303-323: fill with the first element of the
// first non-empty region, then one strided write per region in order.
int orc_assemble(size_t elem, void *dst, size_t len, const tc_region *regions, size_t n) {
  const void *fill = nullptr;
  for (size_t i = 0; i < n; ++i) {
    const tc_region &r = regions[i];
    if (r.rank > TC_MAX_RANK) return int(TC_EINVAL);
    if (!check_strided(r.source_len, r.rank, r.shape, r.from_offset, r.from_strides)) return int(TC_ERANGE);
    if (!fill && element_count(r.rank, r.shape) != 0)
      fill = static_cast<const char *>(r.source) + r.from_offset * elem;
  }
  if (!fill) return len == 0 ? TC_OK : TC_EINVAL;
  char *d = static_cast<char *>(dst);
  for (size_t k = 0; k < len; ++k) std::memcpy(d + k * elem, fill, elem);
  for (size_t i = 0; i < n; ++i) {
    int st = orc_strided_write(elem, dst, len, &regions[i]);
    if (st) return st;
  }
  return int(TC_OK);
}

// Same-shape elementwise: Host vector_elementwise (kernels.rs:1193-1206)
// through simd_dispatch::elementwise (split across threads).
int orc_elementwise(int dtype, int op, const void *a, const void *b, void *out, size_t n) {
  if (!valid_binary(op)) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) T::store(out, i, binary_value(op, T::load(a, i), T::load(b, i)));
    });
    return int(TC_OK);
  });
}

// vector_broadcast (kernels.rs:1208-1220): a op s, or s op a.
int orc_broadcast_scalar(int dtype, int op, const void *a, double scalar, int scalar_left,
                         void *out, size_t n) {
  if (!valid_binary(op)) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float s = float(scalar);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) {
        float x = T::load(a, i);
        T::store(out, i, scalar_left ? binary_value(op, s, x) : binary_value(op, x, s));
      }
    });
    return int(TC_OK);
  });
}

int orc_compare(int dtype, int cmp, const void *a, const void *b, void *out, size_t n) {
  if (!valid_compare(cmp)) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) T::store(out, i, compare_value(cmp, T::load(a, i), T::load(b, i)));
    });
    return int(TC_OK);
  });
}

int orc_compare_scalar(int dtype, int cmp, const void *a, double scalar, int scalar_left,
                       void *out, size_t n) {
  if (!valid_compare(cmp)) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float s = float(scalar);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) {
        float x = T::load(a, i);
        T::store(out, i, scalar_left ? compare_value(cmp, s, x) : compare_value(cmp, x, s));
      }
    });
    return int(TC_OK);
  });
}

// Vector::clamp, src/tensors/vector.rs:642-652: ordered_min(ordered_max(x,
// low), high) (src/tensors/order.rs:10-29); a NaN element becomes `low`.
int orc_clamp(int dtype, const void *a, double low, double high, void *out, size_t n) {
  if (!(low <= high)) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float lo_v = float(low), hi_v = float(high);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) {
        float x = T::load(a, i);
        float m = std::isnan(x) ? lo_v : (x < lo_v ? lo_v : x);
        m = m > hi_v ? hi_v : m;
        T::store(out, i, m);
      }
    });
    return int(TC_OK);
  });
}

// Reduce::fold (kernels.rs:217-226; compact::fold, compact.rs:196-205): left
// to right in f32 from the identity, rounded once.
int orc_vector_reduce(int dtype, int op, const void *a, size_t n, void *out) {
  if (op < TC_SUM || op > TC_RMAX) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float acc = op == TC_SUM ? 0.0f : (op == TC_RMIN ? INFINITY : -INFINITY);
    for (size_t i = 0; i < n; ++i) {
      float x = T::load(a, i);
      acc = op == TC_SUM ? acc + x : (op == TC_RMIN ? min_num(acc, x) : max_num(acc, x));
    }
    T::store(out, 0, acc);
    return int(TC_OK);
  });
}

// dot: f32 through simd::f32k::dot (simd_x86.rs:58-104); f16/bf16 through
// compact::dot (compact.rs:162-178), a running f32 sum of exact products.
int orc_dot(int dtype, const void *a, const void *b, size_t n, void *out) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (std::is_same<T, F32>::value) {
      const float *x = static_cast<const float *>(a), *y = static_cast<const float *>(b);
      float s;
      if (n >= 16) s = dot_f32(x, y, n);
      else { s = 0.0f; for (size_t i = 0; i < n; ++i) s = s + x[i] * y[i]; }
      T::store(out, 0, s);
    } else {
      float s = 0.0f;
      for (size_t i = 0; i < n; ++i) s = s + T::load(a, i) * T::load(b, i);
      T::store(out, 0, s);
    }
    return int(TC_OK);
  });
}

// strided::binary + zip, strided.rs:29-78: op over the common shape in
// row-major order, each operand read through its strides.  Single-threaded,
// as the Host runs it.
int orc_strided_binary(int dtype, int kind, int op, uint32_t rank, const size_t *shape,
                       const void *a, size_t a_len, size_t a_offset, const size_t *a_strides,
                       const void *b, size_t b_len, size_t b_offset, const size_t *b_strides,
                       void *out) {
  if (rank > TC_MAX_RANK) return int(TC_EINVAL);
  if (kind == TC_PAIR_ARITHMETIC && !valid_binary(op)) return int(TC_EINVAL);
  if (kind == TC_PAIR_COMPARE && !valid_compare(op)) return int(TC_EINVAL);
  if (kind < 0 || kind > TC_PAIR_POWER) return int(TC_EINVAL);
  if (!check_strided(a_len, rank, shape, a_offset, a_strides)) return int(TC_ERANGE);
  if (!check_strided(b_len, rank, shape, b_offset, b_strides)) return int(TC_ERANGE);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    auto f = [&](float x, float y) {
      return kind == TC_PAIR_ARITHMETIC ? binary_value(op, x, y)
           : kind == TC_PAIR_COMPARE ? compare_value(op, x, y) : power_value(x, y);
    };
    size_t k = 0;
    const size_t *st[2] = {a_strides, b_strides};
    size_t off[2] = {a_offset, b_offset};
    for_each_run<2>(rank, shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
      for (size_t i = 0; i < len; ++i, ++k)
        T::store(out, k, f(T::load(a, at[0] + i * steps[0]), T::load(b, at[1] + i * steps[1])));
    });
    return int(TC_OK);
  });
}

// strided::reduce / reduce_in / fold, strided.rs:105-184: one row-major walk
// of the input, each element (widened to f32) folded into the accumulator
// of its result; Mean = total / depth; Variance = a second walk over squared
// deviations from the f32 mean, divided by `divisor`; each result rounded
// to the element type once.
int orc_reduce_axes(int dtype, uint32_t rank, const size_t *shape, const void *input,
                    size_t input_len, size_t offset, const size_t *strides, uint32_t n_axes,
                    const uint32_t *axes, int kind, int op, size_t divisor, void *out) {
  if (rank > TC_MAX_RANK || n_axes > rank) return int(TC_EINVAL);
  if (kind < TC_AXIS_FOLD || kind > TC_AXIS_VARIANCE) return int(TC_EINVAL);
  if (kind == TC_AXIS_FOLD && (op < TC_SUM || op > TC_RMAX)) return int(TC_EINVAL);
  if (!check_strided(input_len, rank, shape, offset, strides)) return int(TC_ERANGE);
  bool folded[TC_MAX_RANK] = {false};
  for (uint32_t i = 0; i < n_axes; ++i) {
    if (axes[i] >= rank || (i > 0 && axes[i] <= axes[i - 1])) return int(TC_EINVAL);
    folded[axes[i]] = true;
  }
  // result_strides, strided.rs:83-100.
  size_t kept[TC_MAX_RANK]; uint32_t nk = 0;
  for (uint32_t a = 0; a < rank; ++a) if (!folded[a]) kept[nk++] = shape[a];
  size_t kept_strides[TC_MAX_RANK] = {0, 0, 0, 0, 0, 0};
  contiguous_strides(nk, kept, kept_strides);
  size_t to[TC_MAX_RANK]; uint32_t next = 0;
  for (uint32_t a = 0; a < rank; ++a) to[a] = folded[a] ? 0 : kept_strides[next++];
  size_t results = element_count(nk, kept);
  size_t depth = 1;
  for (uint32_t i = 0; i < n_axes; ++i) depth *= shape[axes[i]];
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const size_t *st[2] = {strides, to};
    size_t off[2] = {offset, 0};
    auto walk = [&](auto &&combine) {
      for_each_run<2>(rank, shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
        for (size_t i = 0; i < len; ++i) {
          size_t slot = at[1] + i * steps[1];
          combine(slot, T::load(input, at[0] + i * steps[0]));
        }
      });
    };
    std::vector<float> totals(results);
    float count = float(depth);
    auto means = [&] {
      std::vector<float> m(results, 0.0f);
      walk([&](size_t slot, float x) { m[slot] = m[slot] + x; });
      for (auto &v : m) v = v / count;
      return m;
    };
    if (kind == TC_AXIS_FOLD) {
      float id = op == TC_SUM ? 0.0f : (op == TC_RMIN ? INFINITY : -INFINITY);
      std::fill(totals.begin(), totals.end(), id);
      walk([&](size_t slot, float x) {
        totals[slot] = op == TC_SUM ? totals[slot] + x
                     : op == TC_RMIN ? min_num(totals[slot], x) : max_num(totals[slot], x);
      });
    } else if (kind == TC_AXIS_MEAN) {
      totals = means();
    } else {
      std::vector<float> m = means();
      std::fill(totals.begin(), totals.end(), 0.0f);
      walk([&](size_t slot, float x) {
        float d = x - m[slot];
        totals[slot] = totals[slot] + d * d;
      });
      float div = float(double(divisor));
      for (auto &v : totals) v = v / div;
    }
    for (size_t r = 0; r < results; ++r) T::store(out, r, totals[r]);
    return int(TC_OK);
  });
}

// strided::arg_reduce + replaces, strided.rs:186-225.
int orc_arg_reduce(int dtype, uint32_t rank, const size_t *shape, const void *input,
                   size_t input_len, size_t offset, const size_t *strides, uint32_t axis, int op,
                   uint32_t *out) {
  if (rank > TC_MAX_RANK || axis >= rank) return int(TC_EINVAL);
  if (op != TC_RMIN && op != TC_RMAX) return int(TC_EINVAL);
  if (!check_strided(input_len, rank, shape, offset, strides)) return int(TC_ERANGE);
  size_t kept[TC_MAX_RANK]; uint32_t nk = 0;
  for (uint32_t a = 0; a < rank; ++a) if (a != axis) kept[nk++] = shape[a];
  size_t kept_strides[TC_MAX_RANK];
  contiguous_strides(nk, kept, kept_strides);
  size_t to[TC_MAX_RANK]; uint32_t next = 0;
  for (uint32_t a = 0; a < rank; ++a) to[a] = a == axis ? 0 : kept_strides[next++];
  size_t along[TC_MAX_RANK] = {0};
  along[axis] = 1;
  size_t results = element_count(nk, kept);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    std::vector<float> best(results, NAN);
    for (size_t r = 0; r < results; ++r) out[r] = 0;
    const size_t *st[3] = {strides, to, along};
    size_t off[3] = {offset, 0, 0};
    for_each_run<3>(rank, shape, off, st, [&](const size_t *at, size_t len, const size_t *steps) {
      for (size_t i = 0; i < len; ++i) {
        size_t slot = at[1] + i * steps[1];
        float x = T::load(input, at[0] + i * steps[0]);
        bool replaces = !std::isnan(x) &&
                        (std::isnan(best[slot]) || (op == TC_RMIN ? x < best[slot] : x > best[slot]));
        if (replaces) { best[slot] = x; out[slot] = uint32_t(at[2] + i * steps[2]); }
      }
    });
    return int(TC_OK);
  });
}

int orc_matmul_rows(int dtype, size_t rows, size_t inner, size_t cols, const void *a,
                    const void *b, void *c, int accumulate, size_t row0, size_t row1) {
  if (row1 > rows || row0 > row1) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    return matmul_rows<decltype(t)>(rows, inner, cols, a, b, c, accumulate != 0, row0, row1);
  });
}

// Kernels::matmul / matmul_add / matmul_transposed_add on Host
// (kernels.rs:1441-1507): the transposed forms copy the operand transposed
// first (the trait default, kernels.rs:975-985).
int orc_matmul(int dtype, int transposed, size_t rows, size_t inner, size_t cols,
               const void *a, const void *b, void *c, int accumulate) {
  if (transposed < TC_TRANS_NONE || transposed > TC_TRANS_RIGHT) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    bool acc = accumulate != 0;
    if (transposed == TC_TRANS_LEFT) {
      auto at = transposed_copy<T>(a, inner, rows);
      return matmul_rows<T>(rows, inner, cols, at.data(), b, c, acc, 0, rows);
    }
    if (transposed == TC_TRANS_RIGHT) {
      auto bt = transposed_copy<T>(b, cols, inner);
      return matmul_rows<T>(rows, inner, cols, a, bt.data(), c, acc, 0, rows);
    }
    return matmul_rows<T>(rows, inner, cols, a, b, c, acc, 0, rows);
  });
}

// Matrix::matvec / matvec_add (matrix.rs:675-730): f16/bf16 through
// compact::matmul with one column (the i-p-j tail: a running `out += a*x`
// per row, from the widened addend when accumulating); f32 through
// simd_dispatch::matvec (a SIMD dot per row, simd_dispatch.rs:626-660) at or
// above 512 elements, else the scalar running sum.
int orc_matvec(int dtype, size_t rows, size_t cols, const void *m, const void *x, void *y,
               int accumulate) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (!std::is_same<T, F32>::value)
      return matmul_rows<T>(rows, cols, 1, m, x, y, accumulate != 0, 0, rows);
    const float *mm = static_cast<const float *>(m), *xx = static_cast<const float *>(x);
    float *yy = static_cast<float *>(y);
    bool simd = rows * cols >= MIN_MATMUL_OPS;
    for (size_t i = 0; i < rows; ++i) {
      float s;
      if (simd) s = dot_f32(mm + i * cols, xx, cols);
      else { s = 0.0f; for (size_t p = 0; p < cols; ++p) s = s + mm[i * cols + p] * xx[p]; }
      yy[i] = accumulate ? yy[i] + s : s;
    }
    return int(TC_OK);
  });
}

// Vector::vecmat (vector.rs:491-515): compact::matmul / simd vecmat = the
// (1 x rows)·(rows x cols) i-p-j product; else the scalar per-column sum.
int orc_vecmat(int dtype, size_t rows, size_t cols, const void *x, const void *m, void *y) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (!std::is_same<T, F32>::value || rows * cols >= MIN_MATMUL_OPS)
      return matmul_rows<T>(1, rows, cols, x, m, y, false, 0, 1);
    const float *xx = static_cast<const float *>(x), *mm = static_cast<const float *>(m);
    float *yy = static_cast<float *>(y);
    for (size_t j = 0; j < cols; ++j) {
      float s = 0.0f;
      for (size_t p = 0; p < rows; ++p) s = s + xx[p] * mm[p * cols + j];
      yy[j] = s;
    }
    return int(TC_OK);
  });
}

// Matrix::transpose (matrix.rs:740-745): moves bits.
int orc_transpose(int dtype, size_t rows, size_t cols, const void *m, void *out) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    auto tr = transposed_copy<T>(m, rows, cols);
    std::memcpy(out, tr.data(), tr.size() * sizeof(typename T::S));
    return int(TC_OK);
  });
}

// Adam's program as built (optim.rs:1048-1099), every operation in the
// element type, in the program's order:
//   first_share = 1 - beta1; second_share = 1 - beta2      (constants)
//   fresh_first = g*first_share; squared = g*g; fresh_second = squared*second_share
//   resumed: first = m*beta1 + fresh_first; second = v*beta2 + fresh_second
//   else:    first = fresh_first; second = fresh_second
//   step = (first*c1) / (sqrt(second*c2) + eps) * rate;  p = p - step
int orc_adam(int dtype, size_t n, void *p, const void *g, void *m, void *v, int resumed,
             double rate, double beta1, double beta2, double eps, double c1, double c2) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const float one = 1.0f;
    float r = float(rate), b1 = float(beta1), b2 = float(beta2), e = float(eps);
    float k1 = float(c1), k2 = float(c2);
    float first_share = T::round(one - b1), second_share = T::round(one - b2);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) {
        float gi = T::load(g, i);
        float fresh_first = T::round(gi * first_share);
        float squared = T::round(gi * gi);
        float fresh_second = T::round(squared * second_share);
        float first, second;
        if (resumed) {
          first = T::round(T::round(T::load(m, i) * b1) + fresh_first);
          second = T::round(T::round(T::load(v, i) * b2) + fresh_second);
        } else {
          first = fresh_first;
          second = fresh_second;
        }
        float cf = T::round(first * k1);
        float cs = T::round(second * k2);
        float root = T::round(std::sqrt(cs));
        float den = T::round(root + e);
        float step = T::round(T::round(cf / den) * r);
        T::store(p, i, T::load(p, i) - step);
        T::store(m, i, first);
        T::store(v, i, second);
      }
    });
    return int(TC_OK);
  });
}

// Sgd's program (optim.rs:773-787): step = g·rate (Builder::scale), p - step.
int orc_sgd(int dtype, size_t n, void *p, const void *g, double rate) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float r = float(rate);
    split(n, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) {
        float step = T::round(T::load(g, i) * r);
        T::store(p, i, T::load(p, i) - step);
      }
    });
    return int(TC_OK);
  });
}

// Adam::update's host arithmetic (optim.rs:1106-1124).  The coefficients are
// values of the element type (Adam::new rounds 0.9/0.999/1e-8 into it,
// optim.rs:1029-1035); `powi` is f32 powi then a rounding for f16/bf16
// (crate half) and compiler-rt's __powisf2 square-and-multiply for f32;
// `one - x` and `.recip()` round in the element type.
int orc_adam_coefficients(int dtype, double rate, double beta1, double beta2, double eps,
                          uint32_t step, double *out) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    auto powi = [](float a, int b) {
      bool recip = b < 0;
      float r = 1.0f;
      for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
      }
      return recip ? 1.0f / r : r;
    };
    float r = from_f64<T>(rate), b1 = from_f64<T>(beta1), b2 = from_f64<T>(beta2);
    float e = from_f64<T>(eps);
    float c1 = T::round(1.0f - T::round(powi(b1, int(step))));
    float c2 = T::round(1.0f - T::round(powi(b2, int(step))));
    out[0] = r; out[1] = b1; out[2] = b2; out[3] = e;
    out[4] = T::round(1.0f / c1);
    out[5] = T::round(1.0f / c2);
    return int(TC_OK);
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// One MLP training step as the reference's tape runs it (benches/nn_ops.rs:
// 877-921 with any number of layers; tape rules tape/mod.rs:979-988, 1026-
// 1033, 1110-1130, 1174, 1195-1216, 1286-1300), through the Host functions
// above, then Adam on every parameter (optim.rs:1106-1140).
// ---------------------------------------------------------------------------
struct OrcMlp {
  int dtype;
  size_t esz;
  int layers;
  std::vector<size_t> dims;
  size_t batch, global_batch;
  double rate, beta1, beta2, eps;
  uint32_t steps = 0;
  std::vector<std::vector<uint8_t>> W, b, gW, gb, mW, vW, mb, vb;
};

extern "C" {

void *orc_mlp_create(int dtype, uint32_t layers, const uint32_t *dims, uint32_t batch, uint32_t global_batch,
                     double rate, double beta1, double beta2, double eps) {
  OrcMlp *m = new OrcMlp;
  m->dtype = dtype;
  m->esz = dtype == TC_F32 ? 4 : 2;
  m->layers = int(layers);
  m->dims.assign(dims, dims + layers + 1);
  m->batch = batch;
  m->global_batch = global_batch ? global_batch : batch;
  m->rate = rate; m->beta1 = beta1; m->beta2 = beta2; m->eps = eps;
  for (int l = 0; l < m->layers; ++l) {
    size_t nw = m->dims[l + 1] * m->dims[l], nb = m->dims[l + 1];
    for (auto *v : {&m->W, &m->gW, &m->mW, &m->vW}) v->emplace_back(nw * m->esz, 0);
    for (auto *v : {&m->b, &m->gb, &m->mb, &m->vb}) v->emplace_back(nb * m->esz, 0);
  }
  return m;
}

void orc_mlp_destroy(void *p) { delete static_cast<OrcMlp *>(p); }

int orc_mlp_params(void *p, uint32_t l, void *w, void *b, int dir) {
  OrcMlp *m = static_cast<OrcMlp *>(p);
  if (int(l) >= m->layers) return int(TC_EINVAL);
  if (dir == 0) {
    if (w) std::memcpy(m->W[l].data(), w, m->W[l].size());
    if (b) std::memcpy(m->b[l].data(), b, m->b[l].size());
  } else {
    if (w) std::memcpy(w, m->W[l].data(), m->W[l].size());
    if (b) std::memcpy(b, m->b[l].data(), m->b[l].size());
  }
  return int(TC_OK);
}

int orc_mlp_grads(void *p, uint32_t l, void *gw, void *gb) {
  OrcMlp *m = static_cast<OrcMlp *>(p);
  if (int(l) >= m->layers) return int(TC_EINVAL);
  if (gw) std::memcpy(gw, m->gW[l].data(), m->gW[l].size());
  if (gb) std::memcpy(gb, m->gb[l].data(), m->gb[l].size());
  return int(TC_OK);
}

// x: [dims[0] x batch], y: [dims[L] x batch]; loss_out (one element) if
// not null.  `skip_update` leaves the parameters as they are (gradients
// only), for checking a data-parallel gradient sum.
int orc_mlp_step(void *p, const void *x, const void *y, void *loss_out, int skip_update) {
  OrcMlp *m = static_cast<OrcMlp *>(p);
  const int d = m->dtype, L = m->layers;
  const size_t B = m->batch, e = m->esz;
  using Bytes = std::vector<uint8_t>;
  auto buf = [&](size_t n) { return Bytes(n * e, 0); };
  Bytes ones = buf(B);
  {
    std::vector<float> one(B, 1.0f);
    if (d == TC_F32) std::memcpy(ones.data(), one.data(), B * 4);
    else orc_narrow(d, one.data(), ones.data(), B);
  }
  std::vector<Bytes> Z, O, A, H;
  for (int l = 0; l < L; ++l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    const void *input = l == 0 ? x : H[l - 1].data();
    Z.push_back(buf(outd * B));
    O.push_back(buf(outd * B));
    A.push_back(buf(outd * B));
    H.push_back(buf(outd * B));
    orc_matmul(d, TC_TRANS_NONE, outd, in, B, m->W[l].data(), input, Z[l].data(), 0);
    orc_matmul(d, TC_TRANS_NONE, outd, 1, B, m->b[l].data(), ones.data(), O[l].data(), 0);
    orc_elementwise(d, TC_ADD, Z[l].data(), O[l].data(), A[l].data(), outd * B);
    if (l + 1 < L) orc_compare_scalar(d, TC_MAX, A[l].data(), 0.0, 0, H[l].data(), outd * B);
  }
  const size_t last = m->dims[L];
  Bytes R = buf(last * B), S = buf(last * B);
  orc_elementwise(d, TC_SUB, A[L - 1].data(), y, R.data(), last * B);
  orc_elementwise(d, TC_MUL, R.data(), R.data(), S.data(), last * B);
  // scale factor in the element type
  double f = 1.0 / (double(last) * double(m->global_batch));
  double coef[6];
  orc_adam_coefficients(d, f, 0.5, 0.5, 0.5, 1, coef);  // coef[0] = f rounded to T
  const double factor = coef[0];
  if (loss_out) {
    Bytes total = buf(1);
    orc_vector_reduce(d, TC_SUM, S.data(), last * B, total.data());
    orc_broadcast_scalar(d, TC_MUL, total.data(), factor, 0, loss_out, 1);
  }
  // backward
  Bytes Sbar = buf(last * B), T1 = buf(last * B), T2 = buf(last * B), Rbar = buf(last * B);
  {
    std::vector<float> fill(last * B, float(factor));
    if (d == TC_F32) std::memcpy(Sbar.data(), fill.data(), fill.size() * 4);
    else orc_narrow(d, fill.data(), Sbar.data(), fill.size());
  }
  orc_elementwise(d, TC_MUL, Sbar.data(), R.data(), T1.data(), last * B);
  orc_elementwise(d, TC_MUL, Sbar.data(), R.data(), T2.data(), last * B);
  orc_elementwise(d, TC_ADD, T1.data(), T2.data(), Rbar.data(), last * B);
  Bytes abar = Rbar;
  for (int l = L - 1; l >= 0; --l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    const void *input = l == 0 ? x : H[l - 1].data();
    orc_matvec(d, outd, B, abar.data(), ones.data(), m->gb[l].data(), 0);
    orc_matmul(d, TC_TRANS_RIGHT, outd, B, in, abar.data(), input, m->gW[l].data(), 0);
    if (l > 0) {
      Bytes inbar = buf(in * B), share = buf(in * B), next = buf(in * B);
      orc_matmul(d, TC_TRANS_LEFT, in, outd, B, m->W[l].data(), abar.data(), inbar.data(), 0);
      orc_compare_scalar(d, TC_MAX_SHARE, A[l - 1].data(), 0.0, 0, share.data(), in * B);
      orc_elementwise(d, TC_MUL, inbar.data(), share.data(), next.data(), in * B);
      abar.swap(next);
    }
  }
  if (skip_update) return int(TC_OK);
  m->steps += 1;
  double k[6];
  orc_adam_coefficients(d, m->rate, m->beta1, m->beta2, m->eps, m->steps, k);
  const int resumed = m->steps > 1;
  for (int l = 0; l < L; ++l) {
    orc_adam(d, m->W[l].size() / e, m->W[l].data(), m->gW[l].data(), m->mW[l].data(), m->vW[l].data(), resumed,
             k[0], k[1], k[2], k[3], k[4], k[5]);
    orc_adam(d, m->b[l].size() / e, m->b[l].data(), m->gb[l].data(), m->mb[l].data(), m->vb[l].data(), resumed,
             k[0], k[1], k[2], k[3], k[4], k[5]);
  }
  return int(TC_OK);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Fused programs: the Host's interpreter (fused/mod.rs:4055-4260), element by
// element.  Every instruction's result rounds to the program's type; loads
// convert from their storage type, stores to the output's.  The analytic
// functions are the C library's f32 ones (the reference uses its own
// vmath; both are within an ulp or two of the exact value).
// ---------------------------------------------------------------------------
static float orc_analytic(int op, float x) {
  switch (op) {
    case TC_SIN: return std::sin(x);
    case TC_COS: return std::cos(x);
    case TC_TAN: return std::tan(x);
    case TC_SEC: return 1.0f / std::cos(x);
    case TC_CSC: return 1.0f / std::sin(x);
    case TC_ARCSIN: return std::asin(x);
    case TC_ARCCOS: return std::acos(x);
    case TC_ARCTAN: return std::atan(x);
    case TC_EXP: return std::exp(x);
    case TC_LN: return std::log(x);
    case TC_SINH: return std::sinh(x);
    case TC_COSH: return std::cosh(x);
    case TC_TANH: return std::tanh(x);
    default: return std::sqrt(x);
  }
}

static float orc_load_as(const void *p, int dtype, size_t i) {
  if (dtype == TC_F32) return F32::load(p, i);
  return dtype == TC_BF16 ? BF16::load(p, i) : F16::load(p, i);
}
static void orc_store_as(void *p, int dtype, size_t i, float v) {
  if (dtype == TC_F32) F32::store(p, i, v);
  else if (dtype == TC_BF16) BF16::store(p, i, v);
  else F16::store(p, i, v);
}

int orc_fused(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code, const tc_place *places,
              uint32_t n_places, void *const *outputs, const int *out_dtypes, uint32_t n_outputs) {
  (void)n_places;
  (void)n_outputs;
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < rows * cols; ++i) {
      const size_t row = i / cols, col = i % cols;
      float reg[16] = {0};
      for (uint32_t k = 0; k < n_code; ++k) {
        const tc_instr &in = code[k];
        float v = 0.0f;
        switch (in.code) {
          case TC_I_LOAD: {
            const tc_place &pl = places[in.slot];
            size_t at = pl.offset + col * pl.col_step, rest = row;
            for (int a = int(pl.lead) - 1; a >= 0; --a) {
              at += (rest % pl.dims[a]) * pl.steps[a];
              rest /= pl.dims[a];
            }
            v = T::round(orc_load_as(pl.data, pl.dtype, at));
            break;
          }
          case TC_I_CONST: v = T::round(in.value); break;
          case TC_I_BINARY: v = T::round(binary_value(in.op, reg[in.a], reg[in.b])); break;
          case TC_I_UNARY: v = T::round(orc_analytic(in.op, reg[in.a])); break;
          case TC_I_CMP: v = compare_value(in.op, reg[in.a], reg[in.b]); break;
          default: orc_store_as(outputs[in.slot], out_dtypes[in.slot], i, reg[in.a]); continue;
        }
        reg[in.dst] = v;
      }
    }
    return int(TC_OK);
  });
}

// ---- the other vector methods (kernels.rs:870-891) -------------------------

// Analytic::derivative (kernels.rs:357-387) in T: each operation of the rule
// rounded to T, as the Host's Real arithmetic on T rounds.
template <class T> static float orc_derivative(int op, float x) {
  auto r = [](float v) { return T::round(v); };
  auto recip = [&](float v) { return r(1.0f / v); };
  auto val = [&](int g) { return r(orc_analytic(g, x)); };
  switch (op) {
    case TC_SIN: return val(TC_COS);
    case TC_COS: return -val(TC_SIN);
    case TC_TAN: { float c = val(TC_COS); return recip(r(c * c)); }
    case TC_SEC: { float c = val(TC_COS); return r(val(TC_SIN) / r(c * c)); }
    case TC_CSC: { float s = val(TC_SIN); return r(-val(TC_COS) / r(s * s)); }
    case TC_ARCSIN: return recip(r(std::sqrt(r(1.0f - r(x * x)))));
    case TC_ARCCOS: return -recip(r(std::sqrt(r(1.0f - r(x * x)))));
    case TC_ARCTAN: return recip(r(1.0f + r(x * x)));
    case TC_EXP: return val(TC_EXP);
    case TC_LN: return recip(x);
    case TC_SINH: return val(TC_COSH);
    case TC_COSH: return val(TC_SINH);
    case TC_TANH: { float t = val(TC_TANH); return r(1.0f - r(t * t)); }
    default: return recip(r(2.0f * r(std::sqrt(x))));
  }
}

// vector_unary (kernels.rs:1257-1268): vmath's f32 function rounded once to
// T.  The restatement calls the C library's f32 functions, which agree with
// vmath's within their 2-ulp bound (parity for transcendentals is 2 ulp).
int orc_unary(int dtype, int f, const void *a, void *out, size_t n) {
  if (f < TC_SIN || f > TC_SQRT) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < n; ++i) T::store(out, i, orc_analytic(f, T::load(a, i)));
    return int(TC_OK);
  });
}

// vector_unary_dual (kernels.rs:1284-1304): (f(x), f'(x) * d), the product
// rounded in T.
int orc_unary_dual(int dtype, int f, const void *value, const void *tangent, void *out_value, void *out_tangent,
                   size_t n) {
  if (f < TC_SIN || f > TC_SQRT) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < n; ++i) {
      const float x = T::load(value, i);
      T::store(out_value, i, orc_analytic(f, x));
      T::store(out_tangent, i, orc_derivative<T>(f, x) * T::load(tangent, i));
    }
    return int(TC_OK);
  });
}

// Vector::prefix_sum (vector.rs:578-589) and compact::prefix_sum
// (compact.rs:209-221): a serial f32 running total, each output rounded to T.
int orc_prefix_sum(int dtype, const void *a, void *out, size_t n) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    float running = 0.0f;
    for (size_t i = 0; i < n; ++i) {
      running = running + T::load(a, i);
      T::store(out, i, running);
    }
    return int(TC_OK);
  });
}

// Vector::sorted (vector.rs:874-886): sort_unstable_by the SortOrder
// comparator, total_cmp (kernels.rs:257-269): the values' bits compared as
// signed integers after flipping the magnitude bits of negative values.
template <class U, class I> static I total_key(U bits) {
  const I s = I(bits);
  constexpr int shift = int(sizeof(U) * 8 - 1);
  return I(s ^ I(U(U(s >> shift) >> 1)));
}
int orc_sort(int dtype, int order, const void *a, void *out, size_t n) {
  if (order != TC_ASCENDING && order != TC_DESCENDING) return int(TC_EINVAL);
  auto run = [&](auto unsigned_zero, auto signed_zero) {
    using U = decltype(unsigned_zero);
    using I = decltype(signed_zero);
    const U *in = static_cast<const U *>(a);
    std::vector<U> v(in, in + n);
    auto less = [](U x, U y) { return total_key<U, I>(x) < total_key<U, I>(y); };
    if (order == TC_ASCENDING) std::sort(v.begin(), v.end(), less);
    else std::sort(v.begin(), v.end(), [&](U x, U y) { return less(y, x); });
    std::memcpy(out, v.data(), n * sizeof(U));
    return int(TC_OK);
  };
  if (dtype == TC_F32) return run(uint32_t(0), int32_t(0));
  if (dtype == TC_F16 || dtype == TC_BF16) return run(uint16_t(0), int16_t(0));
  return int(TC_EINVAL);
}

// pow_elementwise / power_scalar (kernels.rs:1270-1282): powf per element,
// f16/bf16 through f32 and rounded once.
int orc_power(int dtype, const void *a, const void *b, void *out, size_t n) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < n; ++i) T::store(out, i, power_value(T::load(a, i), T::load(b, i)));
    return int(TC_OK);
  });
}
int orc_power_scalar(int dtype, const void *a, double scalar, int scalar_left, void *out, size_t n) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const float s = float(scalar);
    for (size_t i = 0; i < n; ++i) {
      const float x = T::load(a, i);
      T::store(out, i, scalar_left ? power_value(s, x) : power_value(x, s));
    }
    return int(TC_OK);
  });
}

// ---- windowed matrix methods (kernels.rs:998-1028) -------------------------

// correlate_values (kernels.rs:1720-1751), through widened() / narrowed()
// for f16/bf16 (kernels.rs:1514-1529): per output, the taps in row-major
// order, sum = sum + x*k with both operations rounded in f32.
int orc_correlate(int dtype, size_t rows, size_t cols, size_t wrows, size_t wcols, int flip, const void *input,
                  const void *window, void *out) {
  if (wrows > rows || wcols > cols || wrows == 0 || wcols == 0) return int(TC_EINVAL);
  const size_t orows = rows - wrows + 1, ocols = cols - wcols + 1;
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t r = 0; r < orows; ++r)
      for (size_t c = 0; c < ocols; ++c) {
        float sum = 0.0f;
        for (size_t a = 0; a < wrows; ++a)
          for (size_t b = 0; b < wcols; ++b) {
            const size_t tr = flip ? wrows - 1 - a : a, tc = flip ? wcols - 1 - b : b;
            const float prod = T::load(input, (r + a) * cols + c + b) * T::load(window, tr * wcols + tc);
            sum = sum + prod;
          }
        T::store(out, r * ocols + c, sum);
      }
    return int(TC_OK);
  });
}

// correlate_input_gradient_values (kernels.rs:1754-1788): the full
// correlation, out-of-range adjoint indices skipped.
int orc_correlate_input_gradient(int dtype, size_t arows, size_t acols, size_t wrows, size_t wcols, int forward_flip,
                                 const void *adjoint, const void *window, void *out) {
  if (wrows == 0 || wcols == 0 || arows == 0 || acols == 0) return int(TC_EINVAL);
  const size_t rows = arows + wrows - 1, cols = acols + wcols - 1;
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t r = 0; r < rows; ++r)
      for (size_t c = 0; c < cols; ++c) {
        float sum = 0.0f;
        for (size_t a = 0; a < wrows; ++a)
          for (size_t b = 0; b < wcols; ++b) {
            if (r < a || c < b) continue;
            const size_t sr = r - a, sc = c - b;
            if (sr >= arows || sc >= acols) continue;
            const size_t tr = forward_flip ? wrows - 1 - a : a, tc = forward_flip ? wcols - 1 - b : b;
            const float prod = T::load(adjoint, sr * acols + sc) * T::load(window, tr * wcols + tc);
            sum = sum + prod;
          }
        T::store(out, r * cols + c, sum);
      }
    return int(TC_OK);
  });
}

// pad (kernels.rs:1575-1601) and flip (kernels.rs:1531-1542): bits moved.
int orc_pad(int dtype, size_t rows, size_t cols, size_t pr, size_t pc, const void *input, void *out) {
  const size_t e = dtype == TC_F32 ? 4 : 2, ocols = cols + 2 * pc, orows = rows + 2 * pr;
  const char *in = static_cast<const char *>(input);
  char *o = static_cast<char *>(out);
  for (size_t r = 0; r < orows; ++r)
    for (size_t c = 0; c < ocols; ++c) {
      const bool inside = r >= pr && r < pr + rows && c >= pc && c < pc + cols;
      if (inside) std::memcpy(o + (r * ocols + c) * e, in + ((r - pr) * cols + c - pc) * e, e);
      else std::memset(o + (r * ocols + c) * e, 0, e);
    }
  return int(TC_OK);
}
int orc_flip(int dtype, size_t rows, size_t cols, const void *input, void *out) {
  const size_t e = dtype == TC_F32 ? 4 : 2;
  const char *in = static_cast<const char *>(input);
  char *o = static_cast<char *>(out);
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < cols; ++c)
      std::memcpy(o + (r * cols + c) * e, in + ((rows - 1 - r) * cols + cols - 1 - c) * e, e);
  return int(TC_OK);
}

// ---- moments and distributions (kernels.rs:1035-1070) -----------------------

// moments_of / axis_moments_of (statistics/mod.rs:419-500): f32 for the
// compact types (widened), the mean as sum / count, then the sum of squared
// deviations from that mean; both rounded to T.  An empty slice gives NaNs.
static void orc_moments_of(const std::vector<float> &v, float &mean, float &dev) {
  if (v.empty()) {
    mean = dev = std::nanf("");
    return;
  }
  float s = 0.0f;
  for (float x : v) s = s + x;
  mean = s / float(v.size());
  float d = 0.0f;
  for (float x : v) {
    const float e = x - mean;
    d = d + e * e;
  }
  dev = d;
}

int orc_moments(int dtype, const void *a, size_t n, void *out) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    std::vector<float> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = T::load(a, i);
    float mean, dev;
    orc_moments_of(v, mean, dev);
    T::store(out, 0, mean);
    T::store(out, 1, dev);
    return int(TC_OK);
  });
}

int orc_axis_moments(int dtype, size_t rows, size_t cols, int axis, const void *a, void *means, void *devs) {
  if (axis != TC_ROWS && axis != TC_COLUMNS) return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const size_t extent = axis == TC_ROWS ? rows : cols, depth = axis == TC_ROWS ? cols : rows;
    for (size_t k = 0; k < extent; ++k) {
      std::vector<float> v(depth);
      for (size_t j = 0; j < depth; ++j) v[j] = T::load(a, axis == TC_ROWS ? k * cols + j : j * cols + k);
      float mean, dev;
      orc_moments_of(v, mean, dev);
      T::store(means, k, mean);
      T::store(devs, k, dev);
    }
    return int(TC_OK);
  });
}

// The special functions of statistics/special.rs, in f64: Cody's rational
// Chebyshev erf/erfc (split at 0.46875 and 4) and Wichura's AS 241 normal
// quantile, with the published coefficients.
namespace special {
const double FRAC_1_SQRT_PI = 0.5641895835477563, SQRT_2PI = 2.5066282746310002;
const double FRAC_1_SQRT_2 = 0.70710678118654752440, LN_2 = 0.69314718055994530942, PI = 3.14159265358979323846;

static double erf_central(double x) {
  static const double A[5] = {3.1611237438705656, 113.864154151050156, 377.485237685302021, 3209.37758913846947,
                              0.185777706184603153};
  static const double B[4] = {23.6012909523441209, 244.024637934444173, 1282.61652607737228, 2844.23683343917062};
  const double z = x * x;
  double num = A[4] * z, den = z;
  for (int i = 0; i < 3; ++i) {
    num = (num + A[i]) * z;
    den = (den + B[i]) * z;
  }
  return x * (num + A[3]) / (den + B[3]);
}
static double erfc_scaled(double x) {
  static const double C[9] = {0.564188496988670089, 8.88314979438837594, 66.1191906371416295, 298.635138197400131,
                              881.95222124176909, 1712.04761263407058, 2051.07837782607147, 1230.33935479799725,
                              2.15311535474403846e-8};
  static const double D[8] = {15.7449261107098347, 117.693950891312499, 537.181101862009858, 1621.38957456669019,
                              3290.79923573345963, 4362.61909014324716, 3439.36767414372164, 1230.33935480374942};
  static const double P[6] = {0.305326634961232344, 0.360344899949804439, 0.125781726111229246,
                              0.0160837851487422766, 0.000658749161529837803, 0.0163153871373020978};
  static const double Q[5] = {2.56852019228982242, 1.87295284992346047, 0.527905102951428412,
                              0.0605183413124413191, 0.00233520497626869185};
  if (x <= 4.0) {
    double num = C[8] * x, den = x;
    for (int i = 0; i < 7; ++i) {
      num = (num + C[i]) * x;
      den = (den + D[i]) * x;
    }
    return (num + C[7]) / (den + D[7]);
  }
  const double z = 1.0 / (x * x);
  double num = P[5] * z, den = z;
  for (int i = 0; i < 4; ++i) {
    num = (num + P[i]) * z;
    den = (den + Q[i]) * z;
  }
  const double correction = z * (num + P[4]) / (den + Q[4]);
  return (FRAC_1_SQRT_PI - correction) / x;
}
static double erfc_positive(double x) {
  if (x > 27.25) return 0.0;
  const double leading = std::trunc(x * 16.0) / 16.0;
  const double correction = (x - leading) * (x + leading);
  return std::exp(-leading * leading) * std::exp(-correction) * erfc_scaled(x);
}
static double erfc(double x) {
  if (std::isnan(x)) return x;
  if (x < -0.46875) return 2.0 - erfc_positive(-x);
  if (x <= 0.46875) return 1.0 - erf_central(x);
  return erfc_positive(x);
}
static double ln_erfc(double x) {
  if (std::isnan(x)) return x;
  if (x <= 0.46875) return std::log(erfc(x));
  return std::log(erfc_scaled(x)) - x * x;
}
static double polynomial(const double *c, int n, double x) {
  double total = 0.0;
  for (int i = n - 1; i >= 0; --i) total = total * x + c[i];
  return total;
}
static double std_pdf(double z) { return std::exp(-0.5 * z * z) / SQRT_2PI; }
static double std_cdf(double z) { return 0.5 * erfc(-z * FRAC_1_SQRT_2); }
static double std_ln_cdf(double z) { return ln_erfc(-z * FRAC_1_SQRT_2) - LN_2; }
static double std_ppf(double p) {
  if (std::isnan(p) || !(p >= 0.0 && p <= 1.0)) return std::nan("");
  if (p == 0.0) return -INFINITY;
  if (p == 1.0) return INFINITY;
  const double q = p - 0.5;
  if (std::fabs(q) <= 0.425) {
    static const double A[8] = {3.3871328727963666080, 133.14166789178437745, 1971.5909503065514427,
                                13731.693765509461125, 45921.953931549871457, 67265.770927008700853,
                                33430.575583588128105, 2509.0809287301226727};
    static const double B[7] = {42.313330701600911252, 687.18700749205790830, 5394.1960214247511077,
                                21213.794301586595867, 39307.895800092710610, 28729.085735721942674,
                                5226.4952788528545610};
    const double r = 0.180625 - q * q;
    return q * polynomial(A, 8, r) / (polynomial(B, 7, r) * r + 1.0);
  }
  const double tail = q < 0.0 ? p : 1.0 - p;
  double r = std::sqrt(-std::log(tail));
  double value;
  if (r <= 5.0) {
    static const double C[8] = {1.42343711074968357734, 4.63033784615654529590, 5.76949722146069140550,
                                3.64784832476320460504, 1.27045825245236838258, 0.241780725177450611770,
                                0.0227238449892691845833, 0.000774545014278341407640};
    static const double D[7] = {2.05319162663775882187, 1.67638483018380384940, 0.689767334985100004550,
                                0.148103976427480074590, 0.0151986665636164571966, 0.000547593808499534494600,
                                1.05075007164441684324e-9};
    r = r - 1.6;
    value = polynomial(C, 8, r) / (polynomial(D, 7, r) * r + 1.0);
  } else {
    static const double E[8] = {6.65790464350110377720, 5.46378491116411436990, 1.78482653991729133580,
                                0.296560571828504891230, 0.0265321895265761230930, 0.00124266094738807843860,
                                0.0000271155556874348757815, 2.01033439929228813265e-7};
    static const double F[7] = {0.599832206555887937690, 0.136929880922735805310, 0.0148753612908506148525,
                                0.000786869131145613259100, 0.0000184631831751005468180,
                                1.42151175831644588870e-7, 2.04426310338993978564e-15};
    r = r - 5.0;
    value = polynomial(E, 8, r) / (polynomial(F, 7, r) * r + 1.0);
  }
  return q < 0.0 ? -value : value;
}
static bool positive(double v) { return v > 0.0; }
static double ig_pdf(double x, double mean, double shape) {
  if (!positive(mean) || !positive(shape)) return std::nan("");
  if (x <= 0.0) return 0.0;
  const double deviation = x - mean;
  const double exponent = -shape * deviation * deviation / (2.0 * mean * mean * x);
  return std::sqrt(shape / (2.0 * PI * x * x * x)) * std::exp(exponent);
}
static double ig_cdf(double x, double mean, double shape) {
  if (!positive(mean) || !positive(shape)) return std::nan("");
  if (x <= 0.0) return 0.0;
  const double scale = std::sqrt(shape / x), ratio = x / mean;
  const double lower = scale * (ratio - 1.0), upper = scale * (ratio + 1.0);
  const double tail = 2.0 * shape / mean + std_ln_cdf(-upper);
  return std::fmin(std_cdf(lower) + std::exp(tail), 1.0);
}
static double ig_ppf(double p, double mean, double shape) {
  if (!positive(mean) || !positive(shape) || std::isnan(p) || !(p >= 0.0 && p <= 1.0)) return std::nan("");
  if (p == 0.0) return 0.0;
  if (p == 1.0) return INFINITY;
  double low = 0.0, high = mean;
  while (ig_cdf(high, mean, shape) < p) {
    low = high;
    high *= 2.0;
    if (std::isinf(high)) return INFINITY;
  }
  double guess = 0.5 * (low + high);
  for (int k = 0; k < 60; ++k) {
    const double error = ig_cdf(guess, mean, shape) - p;
    if (error > 0.0) high = guess;
    else low = guess;
    const double density = ig_pdf(guess, mean, shape);
    const double step = density > 0.0 ? guess - error / density : std::nan("");
    const double next = (std::isfinite(step) && step > low && step < high) ? step : 0.5 * (low + high);
    if (next == guess) break;
    guess = next;
  }
  return guess;
}
// Distribution::evaluate (statistics/mod.rs:285-303).
static double evaluate(int family, int statistic, double x, double first, double second) {
  if (family == TC_NORMAL) {
    if (std::isnan(second) || second <= 0.0) return std::nan("");
    if (statistic == TC_PDF) return std_pdf((x - first) / second) / second;
    if (statistic == TC_CDF) return std_cdf((x - first) / second);
    return first + second * std_ppf(x);
  }
  if (statistic == TC_PDF) return ig_pdf(x, first, second);
  if (statistic == TC_CDF) return ig_cdf(x, first, second);
  return ig_ppf(x, first, second);
}
}  // namespace special

// f64 rounded once to T: the f32 cast, or crate half's direct f64
// conversion (round to odd into f32, then to nearest even into 16 bits,
// which is the correctly rounded result).
template <class T> static void store_f64(void *out, size_t i, double d) {
  float f = float(d);
  if (!std::is_same<T, F32>::value && std::isfinite(d) && double(f) != d) {
    // round toward zero into f32, then make the last bit odd
    float z = float(d);
    if (std::fabs(double(z)) > std::fabs(d)) z = std::nextafter(z, 0.0f);
    uint32_t b;
    std::memcpy(&b, &z, 4);
    b |= 1u;
    std::memcpy(&f, &b, 4);
  }
  T::store(out, i, f);
}

int orc_distribution(int dtype, int family, int statistic, const void *a, size_t n, double first, double second,
                     void *out) {
  if (family < TC_NORMAL || family > TC_INVERSE_GAUSSIAN || statistic < TC_PDF || statistic > TC_PPF)
    return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < n; ++i)
      store_f64<T>(out, i, special::evaluate(family, statistic, double(T::load(a, i)), first, second));
    return int(TC_OK);
  });
}

int orc_axis_distribution(int dtype, size_t rows, size_t cols, int axis, int family, int statistic, const void *a,
                          const void *first, const void *second, void *out) {
  if (family < TC_NORMAL || family > TC_INVERSE_GAUSSIAN || statistic < TC_PDF || statistic > TC_PPF ||
      (axis != TC_ROWS && axis != TC_COLUMNS))
    return int(TC_EINVAL);
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < rows * cols; ++i) {
      const size_t along = axis == TC_ROWS ? i / cols : i % cols;
      store_f64<T>(out, i, special::evaluate(family, statistic, double(T::load(a, i)),
                                             double(T::load(first, along)), double(T::load(second, along))));
    }
    return int(TC_OK);
  });
}

// Distribution::evaluate in f64 before any rounding to the element type,
// for pinning the special functions against published values.
double orc_evaluate_f64(int family, int statistic, double x, double first, double second) {
  return special::evaluate(family, statistic, x, first, second);
}

// ---- fused programs with row statistics and sums (kernels.rs:1090-1135) ----

// host_row_moments (fused/mod.rs:4030-4043): the rows x cols matrix `place`
// reads, converted to T (input_matrix), then axis_moments_of along Rows.
int orc_row_moments(int dtype, const tc_place *place, size_t rows, size_t cols, void *means, void *devs) {
  return with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    std::vector<float> m(rows * cols);
    for (size_t i = 0; i < rows * cols; ++i) {
      const size_t row = i / cols, col = i % cols;
      size_t at = place->offset + col * place->col_step, rest = row;
      for (int a = int(place->lead) - 1; a >= 0; --a) {
        at += (rest % place->dims[a]) * place->steps[a];
        rest /= place->dims[a];
      }
      m[i] = T::round(orc_load_as(place->data, place->dtype, at));
    }
    for (size_t r = 0; r < rows; ++r) {
      std::vector<float> v(m.begin() + r * cols, m.begin() + (r + 1) * cols);
      float mean, dev;
      orc_moments_of(v, mean, dev);
      T::store(means, r, mean);
      T::store(devs, r, dev);
    }
    return int(TC_OK);
  });
}

// Kernels::fused_with_statistics' default (kernels.rs:1103-1117): the
// statistics computed first by row_moments, then passed to the program as
// inputs read one value per row.
int orc_fused_with_statistics(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code,
                              const tc_place *places, uint32_t n_places, const tc_row_statistic *stats,
                              uint32_t n_stats, void *const *outputs, const int *out_dtypes, uint32_t n_outputs) {
  const size_t e = dtype == TC_F32 ? 4 : 2;
  std::vector<tc_place> all(places, places + n_places);
  std::vector<std::vector<char>> vectors;
  for (uint32_t s = 0; s < n_stats; ++s) {
    std::vector<char> means(rows * e), devs(rows * e);
    if (int st = orc_row_moments(dtype, &places[stats[s].of_place], rows, cols, means.data(), devs.data())) return st;
    vectors.push_back(stats[s].statistic == TC_ROW_MEAN ? means : devs);
  }
  for (uint32_t s = 0; s < n_stats; ++s) {
    tc_place q{};
    q.data = vectors[s].data();
    q.dtype = dtype;
    q.lead = 1;
    q.dims[0] = rows;
    q.steps[0] = 1;
    q.col_step = 0;
    all[stats[s].into_place] = q;
  }
  return orc_fused(dtype, rows, cols, code, n_code, all.data(), n_places, outputs, out_dtypes, n_outputs);
}

// Program::run_sum's unfused definition (fused/mod.rs:1081-1084, axis_sum at
// 4045-4052): the program's one output of type T, then matvec with ones
// (Rows) or vecmat (Columns).
int orc_fused_sum(int dtype, size_t rows, size_t cols, const tc_instr *code, uint32_t n_code, const tc_place *places,
                  uint32_t n_places, int axis, void *sums) {
  if (axis != TC_ROWS && axis != TC_COLUMNS) return int(TC_EINVAL);
  const size_t e = dtype == TC_F32 ? 4 : 2;
  std::vector<char> out(rows * cols * e);
  void *outs[1] = {out.data()};
  const int dts[1] = {dtype};
  if (int st = orc_fused(dtype, rows, cols, code, n_code, places, n_places, outs, dts, 1)) return st;
  std::vector<char> ones(std::max(rows, cols) * e);
  with_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    for (size_t i = 0; i < std::max(rows, cols); ++i) T::store(ones.data(), i, 1.0f);
    return 0;
  });
  if (axis == TC_ROWS) return orc_matvec(dtype, rows, cols, out.data(), ones.data(), sums, 0);
  return orc_vecmat(dtype, rows, cols, ones.data(), out.data(), sums);
}

// host_matmul (fused/mod.rs:4754-4764): the product a.matmul(b), rounded to
// T, then the program with it as input 0.
int orc_matmul_program(int dtype, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                       const tc_instr *code, uint32_t n_code, const tc_place *places, uint32_t n_places,
                       void *const *outputs, const int *out_dtypes, uint32_t n_outputs) {
  const size_t e = dtype == TC_F32 ? 4 : 2;
  std::vector<char> product(rows * cols * e);
  if (int st = orc_matmul(dtype, TC_TRANS_NONE, rows, inner, cols, a, b, product.data(), 0)) return st;
  std::vector<tc_place> all(places, places + n_places);
  all[0].data = product.data();
  all[0].dtype = dtype;
  return orc_fused(dtype, rows, cols, code, n_code, all.data(), n_places, outputs, out_dtypes, n_outputs);
}
