// stats.cu — moments and distribution functions of Kernels<T>
// (vector_moments, matrix_moments, matrix_axis_moments,
// vector_distribution, matrix_distribution, matrix_axis_distribution;
// kernels.rs:1035-1070).
//
// Moments are the variance kernels with divisor 1, which is the sum of
// squared deviations from the f32 mean (statistics/mod.rs:419-441); those
// kernels write the mean (f32 sum / count) as well, each rounded once to T.
//
// The distribution functions are evaluated in f64 per element, as the Host
// does (statistics/special.rs), with the products, sums and quotients
// written as explicitly rounded operations so none is contracted into an
// FMA: the same arithmetic as the Host's, step for step, with CUDA's
// double-precision exp/log/sqrt.  The error function is Cody's rational
// Chebyshev approximation (Math. Comp. 23 (1969) 631-637), split at 0.46875
// and 4; the normal quantile is Wichura's AS 241 (PPND16, Appl. Statist. 37
// (1988) 477-484); the inverse Gaussian quantile brackets the root by
// doubling and refines it by safeguarded Newton steps, at most 60.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace tc {
namespace {

// ---------------------------------------------------------------------------
// Moments through the reduction kernels.
// ---------------------------------------------------------------------------
template <class S> __global__ void fill_value(S *out, long long n, S v) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = v;
}

// n quiet NaNs of the element type (what the Host's moments give an empty
// slice, statistics/mod.rs:428-434, 470-476).
int nan_fill(int dtype, void *out, size_t n, cudaStream_t s) {
  if (n == 0) return TC_OK;
  if (dtype == TC_F32)
    fill_value<uint32_t><<<grid_for(n, 256, 4), 256, 0, s>>>(static_cast<uint32_t *>(out), (long long)n, 0x7FC00000u);
  else
    fill_value<uint16_t><<<grid_for(n, 256, 4), 256, 0, s>>>(static_cast<uint16_t *>(out), (long long)n,
                                                             uint16_t(dtype == TC_F16 ? 0x7E00u : 0x7FC0u));
  return check_launch("moments (NaN)");
}

// ---------------------------------------------------------------------------
// f64 special functions.
// ---------------------------------------------------------------------------
__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double quo(double a, double b) { return __ddiv_rn(a, b); }

constexpr double FRAC_1_SQRT_PI = 0.5641895835477563, SQRT_2PI = 2.5066282746310002;
constexpr double FRAC_1_SQRT_2 = 0.70710678118654752440, LN_2 = 0.69314718055994530942;
constexpr double PI = 3.14159265358979323846;
__device__ __forceinline__ double quiet_nan() { return __longlong_as_double(0x7FF8000000000000LL); }
__device__ __forceinline__ double infinity() { return __longlong_as_double(0x7FF0000000000000LL); }

// Cody (1969), Table II: erf on |x| <= 0.5 (numerator A, denominator B).
__constant__ double ERF_A[5] = {3.1611237438705656, 113.864154151050156, 377.485237685302021, 3209.37758913846947,
                                0.185777706184603153};
__constant__ double ERF_B[4] = {23.6012909523441209, 244.024637934444173, 1282.61652607737228, 2844.23683343917062};
// Cody (1969), Table III: exp(x²)·erfc(x) on 0.46875 < x <= 4.
__constant__ double ERFC_C[9] = {0.564188496988670089, 8.88314979438837594, 66.1191906371416295,
                                 298.635138197400131,  881.95222124176909,  1712.04761263407058,
                                 2051.07837782607147,  1230.33935479799725, 2.15311535474403846e-8};
__constant__ double ERFC_D[8] = {15.7449261107098347, 117.693950891312499, 537.181101862009858, 1621.38957456669019,
                                 3290.79923573345963, 4362.61909014324716, 3439.36767414372164, 1230.33935480374942};
// Cody (1969), Table IV: the asymptotic tail x > 4, in 1/x².
__constant__ double ERFC_P[6] = {0.305326634961232344, 0.360344899949804439, 0.125781726111229246,
                                 0.0160837851487422766, 0.000658749161529837803, 0.0163153871373020978};
__constant__ double ERFC_Q[5] = {2.56852019228982242, 1.87295284992346047, 0.527905102951428412,
                                 0.0605183413124413191, 0.00233520497626869185};
// Wichura (1988), PPND16: the central region |q| <= 0.425 (A/B), the
// intermediate tail r <= 5 (C/D) and the far tail (E/F).
__constant__ double PPF_A[8] = {3.3871328727963666080, 133.14166789178437745, 1971.5909503065514427,
                                13731.693765509461125, 45921.953931549871457, 67265.770927008700853,
                                33430.575583588128105, 2509.0809287301226727};
__constant__ double PPF_B[7] = {42.313330701600911252, 687.18700749205790830, 5394.1960214247511077,
                                21213.794301586595867, 39307.895800092710610, 28729.085735721942674,
                                5226.4952788528545610};
__constant__ double PPF_C[8] = {1.42343711074968357734, 4.63033784615654529590, 5.76949722146069140550,
                                3.64784832476320460504, 1.27045825245236838258, 0.241780725177450611770,
                                0.0227238449892691845833, 0.000774545014278341407640};
__constant__ double PPF_D[7] = {2.05319162663775882187, 1.67638483018380384940, 0.689767334985100004550,
                                0.148103976427480074590, 0.0151986665636164571966, 0.000547593808499534494600,
                                1.05075007164441684324e-9};
__constant__ double PPF_E[8] = {6.65790464350110377720, 5.46378491116411436990, 1.78482653991729133580,
                                0.296560571828504891230, 0.0265321895265761230930, 0.00124266094738807843860,
                                0.0000271155556874348757815, 2.01033439929228813265e-7};
__constant__ double PPF_F[7] = {0.599832206555887937690, 0.136929880922735805310, 0.0148753612908506148525,
                                0.000786869131145613259100, 0.0000184631831751005468180,
                                1.42151175831644588870e-7, 2.04426310338993978564e-15};

// Horner's rule, highest coefficient first: c[n-1]·x^(n-1) + ... + c[0].
static __device__ double horner(const double *c, int n, double x) {
  double total = 0.0;
  for (int i = n - 1; i >= 0; --i) total = add(mul(total, x), c[i]);
  return total;
}

// The rational forms of Cody's tables, evaluated as nested products: with
// p = leading coefficient, num = ((p·z + a0)·z + a1)·z ..., den likewise.
static __device__ double erf_central(double x) {
  const double z = mul(x, x);
  double num = mul(ERF_A[4], z), den = z;
  for (int i = 0; i < 3; ++i) {
    num = mul(add(num, ERF_A[i]), z);
    den = mul(add(den, ERF_B[i]), z);
  }
  return quo(mul(x, add(num, ERF_A[3])), add(den, ERF_B[3]));
}

static __device__ double erfc_scaled(double x) {
  if (x <= 4.0) {
    double num = mul(ERFC_C[8], x), den = x;
    for (int i = 0; i < 7; ++i) {
      num = mul(add(num, ERFC_C[i]), x);
      den = mul(add(den, ERFC_D[i]), x);
    }
    return quo(add(num, ERFC_C[7]), add(den, ERFC_D[7]));
  }
  const double z = quo(1.0, mul(x, x));
  double num = mul(ERFC_P[5], z), den = z;
  for (int i = 0; i < 4; ++i) {
    num = mul(add(num, ERFC_P[i]), z);
    den = mul(add(den, ERFC_Q[i]), z);
  }
  const double correction = quo(mul(z, add(num, ERFC_P[4])), add(den, ERFC_Q[4]));
  return quo(sub(FRAC_1_SQRT_PI, correction), x);
}

// erfc for x > 0.46875: exp(-x²) split as exp(-l²)·exp(-(x-l)(x+l)) with l
// = x rounded down to a sixteenth, so the square is exact in the first.
static __device__ double erfc_positive(double x) {
  if (x > 27.25) return 0.0;
  const double leading = quo(trunc(mul(x, 16.0)), 16.0);
  const double correction = mul(sub(x, leading), add(x, leading));
  return mul(mul(exp(mul(-leading, leading)), exp(-correction)), erfc_scaled(x));
}

static __device__ double erfc_any(double x) {
  if (isnan(x)) return x;
  if (x < -0.46875) return sub(2.0, erfc_positive(-x));
  if (x <= 0.46875) return sub(1.0, erf_central(x));
  return erfc_positive(x);
}

static __device__ double ln_erfc(double x) {
  if (isnan(x)) return x;
  if (x <= 0.46875) return log(erfc_any(x));
  return sub(log(erfc_scaled(x)), mul(x, x));
}

static __device__ double std_pdf(double z) { return quo(exp(mul(mul(-0.5, z), z)), SQRT_2PI); }
static __device__ double std_cdf(double z) { return mul(0.5, erfc_any(mul(-z, FRAC_1_SQRT_2))); }
static __device__ double std_ln_cdf(double z) { return sub(ln_erfc(mul(-z, FRAC_1_SQRT_2)), LN_2); }

static __device__ double std_ppf(double p) {
  if (isnan(p) || !(p >= 0.0 && p <= 1.0)) return quiet_nan();
  if (p == 0.0) return -infinity();
  if (p == 1.0) return infinity();
  const double q = sub(p, 0.5);
  if (fabs(q) <= 0.425) {
    const double r = sub(0.180625, mul(q, q));
    return quo(mul(q, horner(PPF_A, 8, r)), add(mul(horner(PPF_B, 7, r), r), 1.0));
  }
  const double tail = q < 0.0 ? p : sub(1.0, p);
  double r = __dsqrt_rn(-log(tail));
  double value;
  if (r <= 5.0) {
    r = sub(r, 1.6);
    value = quo(horner(PPF_C, 8, r), add(mul(horner(PPF_D, 7, r), r), 1.0));
  } else {
    r = sub(r, 5.0);
    value = quo(horner(PPF_E, 8, r), add(mul(horner(PPF_F, 7, r), r), 1.0));
  }
  return q < 0.0 ? -value : value;
}

static __device__ double ig_pdf(double x, double mean, double shape) {
  if (!(mean > 0.0) || !(shape > 0.0)) return quiet_nan();
  if (x <= 0.0) return 0.0;
  const double deviation = sub(x, mean);
  const double exponent = quo(mul(mul(-shape, deviation), deviation), mul(mul(mul(2.0, mean), mean), x));
  return mul(__dsqrt_rn(quo(shape, mul(mul(mul(2.0 * PI, x), x), x))), exp(exponent));
}

static __device__ double ig_cdf(double x, double mean, double shape) {
  if (!(mean > 0.0) || !(shape > 0.0)) return quiet_nan();
  if (x <= 0.0) return 0.0;
  const double scale = __dsqrt_rn(quo(shape, x)), ratio = quo(x, mean);
  const double lower = mul(scale, sub(ratio, 1.0)), upper = mul(scale, add(ratio, 1.0));
  const double tail = add(quo(mul(2.0, shape), mean), std_ln_cdf(-upper));
  return fmin(add(std_cdf(lower), exp(tail)), 1.0);
}

static __device__ double ig_ppf(double p, double mean, double shape) {
  if (!(mean > 0.0) || !(shape > 0.0) || isnan(p) || !(p >= 0.0 && p <= 1.0)) return quiet_nan();
  if (p == 0.0) return 0.0;
  if (p == 1.0) return infinity();
  // Bracket: the doubling ends at the latest when `high` overflows (about
  // 1100 steps from the smallest positive mean).
  double low = 0.0, high = mean;
  while (ig_cdf(high, mean, shape) < p) {
    low = high;
    high = mul(high, 2.0);
    if (isinf(high)) return infinity();
  }
  double guess = mul(0.5, add(low, high));
  for (int k = 0; k < 60; ++k) {
    const double error = sub(ig_cdf(guess, mean, shape), p);
    if (error > 0.0) high = guess;
    else low = guess;
    const double density = ig_pdf(guess, mean, shape);
    const double step = density > 0.0 ? sub(guess, quo(error, density)) : quiet_nan();
    const double next = (isfinite(step) && step > low && step < high) ? step : mul(0.5, add(low, high));
    if (next == guess) break;
    guess = next;
  }
  return guess;
}

static __device__ double evaluate(int family, int statistic, double x, double first, double second) {
  if (family == TC_NORMAL) {
    if (isnan(second) || second <= 0.0) return quiet_nan();
    if (statistic == TC_PDF) return quo(std_pdf(quo(sub(x, first), second)), second);
    if (statistic == TC_CDF) return std_cdf(quo(sub(x, first), second));
    return add(first, mul(second, std_ppf(x)));
  }
  if (statistic == TC_PDF) return ig_pdf(x, first, second);
  if (statistic == TC_CDF) return ig_cdf(x, first, second);
  return ig_ppf(x, first, second);
}

// An f64 rounded once to T: the f32 conversion, or for f16/bf16 rounding to
// odd into f32 first (toward zero, the last bit set when inexact), which
// keeps the following round-to-nearest-even into 16 bits correct.
template <class T> __device__ __forceinline__ typename T::S narrow_f64(double d) {
  if (sizeof(typename T::S) == 4) return T::store(__double2float_rn(d));
  float z = __double2float_rz(d);
  if (isfinite(d) && double(z) != d) z = __uint_as_float(__float_as_uint(z) | 1u);
  return T::store(z);
}

// One thread per element.  axis < 0: one parameter pair for all; otherwise
// the pair of the element's row (TC_ROWS) or column (TC_COLUMNS).
template <class T>
__global__ void __launch_bounds__(256) distribution_kernel(const typename T::S *a, typename T::S *out, long long n,
                                                           int family, int statistic, double first, double second,
                                                           const typename T::S *firsts,
                                                           const typename T::S *seconds, long long cols, int axis) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    double p0 = first, p1 = second;
    if (axis >= 0) {
      const long long along = axis == TC_ROWS ? i / cols : i % cols;
      p0 = T::load(firsts[along]);
      p1 = T::load(seconds[along]);
    }
    out[i] = narrow_f64<T>(evaluate(family, statistic, double(T::load(a[i])), p0, p1));
  }
}

int check_family(int family, int statistic) {
  if (family != TC_NORMAL && family != TC_INVERSE_GAUSSIAN) return fail(TC_EINVAL, "bad Family %d", family);
  if (statistic < TC_PDF || statistic > TC_PPF) return fail(TC_EINVAL, "bad Statistic %d", statistic);
  return TC_OK;
}

int launch_distribution(int dtype, const void *a, void *out, size_t n, int family, int statistic, double first,
                        double second, const void *firsts, const void *seconds, size_t cols, int axis,
                        cudaStream_t s) {
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    // f64 work per element is heavy: 128-thread blocks, several per SM.
    distribution_kernel<T><<<grid_for(n, 128, 16), 128, 0, s>>>(
        static_cast<const S *>(a), static_cast<S *>(out), (long long)n, family, statistic, first, second,
        static_cast<const S *>(firsts), static_cast<const S *>(seconds), (long long)cols, axis);
    return check_launch("distribution");
  });
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_moments(int dtype, const void *a, size_t n, void *out_dev, void *stream) {
  if (!out_dev) return fail(TC_EINVAL, "moments: null output");
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16) return fail(TC_EINVAL, "unknown element type %d", dtype);
  cudaStream_t s = as_stream(stream);
  if (n == 0) return nan_fill(dtype, out_dev, 2, s);
  if (!a) return fail(TC_EINVAL, "moments: null input");
  const size_t shape[1] = {n}, strides[1] = {1};
  const uint32_t axes[1] = {0};
  char *out = static_cast<char *>(out_dev);
  return reduce_moments(dtype, 1, shape, a, 0, strides, 1, axes, out, out + dtype_bytes(dtype), s);
}

int tc_axis_moments(int dtype, size_t rows, size_t cols, int axis, const void *a, void *means, void *deviations,
                    void *stream) {
  if (axis != TC_ROWS && axis != TC_COLUMNS) return fail(TC_EINVAL, "bad Axis %d", axis);
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16) return fail(TC_EINVAL, "unknown element type %d", dtype);
  const size_t extent = axis == TC_ROWS ? rows : cols, depth = axis == TC_ROWS ? cols : rows;
  if (extent == 0) return TC_OK;
  if (!means || !deviations) return fail(TC_EINVAL, "axis_moments: null output");
  cudaStream_t s = as_stream(stream);
  if (depth == 0) {
    if (int st = nan_fill(dtype, means, extent, s)) return st;
    return nan_fill(dtype, deviations, extent, s);
  }
  if (!a) return fail(TC_EINVAL, "axis_moments: null input");
  const size_t shape[2] = {rows, cols}, strides[2] = {cols, 1};
  const uint32_t axes[1] = {axis == TC_ROWS ? 1u : 0u};
  return reduce_moments(dtype, 2, shape, a, 0, strides, 1, axes, means, deviations, s);
}

int tc_distribution(int dtype, int family, int statistic, const void *a, size_t n, double first, double second,
                    void *out, void *stream) {
  if (int st = check_family(family, statistic)) return st;
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "distribution: null pointer");
  return launch_distribution(dtype, a, out, n, family, statistic, first, second, nullptr, nullptr, 1, -1,
                             as_stream(stream));
}

int tc_axis_distribution(int dtype, size_t rows, size_t cols, int axis, int family, int statistic, const void *a,
                         const void *first, const void *second, void *out, void *stream) {
  if (int st = check_family(family, statistic)) return st;
  if (axis != TC_ROWS && axis != TC_COLUMNS) return fail(TC_EINVAL, "bad Axis %d", axis);
  const size_t n = rows * cols;
  if (n == 0) return TC_OK;
  if (!a || !first || !second || !out) return fail(TC_EINVAL, "axis_distribution: null pointer");
  return launch_distribution(dtype, a, out, n, family, statistic, 0.0, 0.0, first, second, cols, axis,
                             as_stream(stream));
}

}  // extern "C"
