// common.cuh — shared pieces of the tensorcrate CUDA backend: element
// traits, status reporting, launch geometry and the host-side layout
// arithmetic (coalescing) that every strided kernel's descriptor is built
// from.  sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <cmath>
#include <cstdio>
#include <string>

#include "../../include/tccuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tensorcrate_b200 targets sm_100a only"
#endif

namespace tc {

// ---------------------------------------------------------------------------
// Status: a thread-local last error, set by fail(); every entry point returns
// the status it set.
// ---------------------------------------------------------------------------
int fail(int status, const char *fmt, ...);
int check_cuda(cudaError_t err, const char *what);
// The launch status of the last kernel (cudaGetLastError) as a tc status.
int check_launch(const char *what);

// SMs on the current device (148 on B200), cached per device.
int sm_count();

// A device scratch buffer of at least `bytes` for partial results, one per
// (device, stream), grown on demand.  Work that uses it is ordered on that
// stream, so calls on other streams never share it.  A stream belongs to one
// host thread at a time: two threads that enqueue multi-kernel calls on the
// same stream could interleave them.
int scratch(size_t bytes, void **out, cudaStream_t stream);
// `n` zeroed device counters per (device, stream), grown on demand.  A
// kernel that takes tickets from them sets each back to zero when it is
// done, so they are zero between launches.
int counters(size_t n, int **out, cudaStream_t stream);
// cudaMalloc, counted (tc_alloc_counts).
int device_malloc(void **ptr, size_t bytes, const char *what);
// One block of a data-parallel step's flat parameter buffers, updated by
// this rank for its shard [first, first + count) (16-byte packs): the
// gradient is the sum, in rank order and in f32, of every rank's gradient
// block (grads[r] is rank r's, mapped over NVLink; grads[rank] this rank's),
// rounded once to the element type; Adam's program then runs on it with
// this rank's moments m, v (indexed like the block), and the new parameters
// go to every rank's copy (params[r]); the summed gradient replaces this
// rank's shard of grads[rank] (optim.cu).
constexpr int MAX_PEER_RANKS = 8;
struct PeerAdam {
  int nranks, rank;
  const void *grads[MAX_PEER_RANKS];
  void *params[MAX_PEER_RANKS];
  void *m, *v;
  size_t first, count;
};
int peer_adam_run(int dtype, const PeerAdam &x, int resumed, double rate, double beta1, double beta2, double eps,
                  double c1, double c2, cudaStream_t stream);

// Rank `rank`'s copy of a peer buffer as this GPU maps it (this rank's own
// when rank is this one), and a host-side barrier of every rank (comm.cu).
void *peer_buffer_remote(tc_peer_buffer *buf, int rank);
int comm_barrier(tc_comm *comm);

// The means and sums of squared deviations (in the element type) of the
// slices of `input` folded over `axes`, in as few passes as the layout
// allows (reduce.cu).
int reduce_moments(int dtype, uint32_t rank, const size_t *shape, const void *input, size_t offset,
                   const size_t *strides, uint32_t n_axes, const uint32_t *axes, void *means, void *deviations,
                   cudaStream_t stream);

// ---------------------------------------------------------------------------
// Element types.  A kernel computes in f32; loads widen exactly and stores
// round once, to nearest even, as crate `half` does (NaN kept quiet with
// the top of its payload), so every elementwise result is the correctly
// rounded one the reference's Host computes (src/compact.rs:5-22).
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t x = __float_as_uint(f);
#else
  uint32_t x; memcpy(&x, &f, 4);
#endif
  if ((x & 0x7fffffffu) > 0x7f800000u) return uint16_t((x >> 16) | 0x0040u);
  // round half to even: add 0x7fff plus the lowest kept bit
  x += 0x7fffu + ((x >> 16) & 1u);
  return uint16_t(x >> 16);
}
__host__ __device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(uint32_t(h) << 16);
#else
  uint32_t x = uint32_t(h) << 16; float f; memcpy(&f, &x, 4); return f;
#endif
}
__host__ __device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t x = __float_as_uint(f);
#else
  uint32_t x; memcpy(&x, &f, 4);
#endif
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) return uint16_t(sign | 0x7c00u | (man ? (0x0200u | (man >> 13)) : 0u));
  int e = int(exp) - 112;  // rebias 127 -> 15
  if (e >= 0x1f) return uint16_t(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    man |= 0x800000u;
    uint32_t shift = uint32_t(14 - e);
    uint32_t h = man >> shift;
    uint32_t round_bit = 1u << (shift - 1);
    if ((man & round_bit) && (man & (3u * round_bit - 1u))) h++;
    return uint16_t(sign | h);
  }
  uint32_t out = sign | (uint32_t(e) << 10) | (man >> 13);
  if ((man & 0x1000u) && (man & 0x2fffu)) out++;
  return uint16_t(out);
}
__host__ __device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0x1fu) x = sign | 0x7f800000u | (man << 13);
  else if (exp == 0) {
    if (man == 0) x = sign;
    else {
      float v = float(man) * 5.9604644775390625e-08f;
      return sign ? -v : v;
    }
  } else x = sign | ((exp + 112u) << 23) | (man << 13);
#ifdef __CUDA_ARCH__
  return __uint_as_float(x);
#else
  float f; memcpy(&f, &x, 4); return f;
#endif
}

// Device code rounds with the hardware conversions (cvt.rn.f16.f32 /
// cvt.rn.bf16.f32: round to nearest even, subnormals kept), which agree with
// the software conversions above on every value but a NaN's payload; host
// code uses the software ones.
struct F32T {
  using S = float;
  static constexpr int code = TC_F32;
  __host__ __device__ __forceinline__ static float load(S s) { return s; }
  __host__ __device__ __forceinline__ static S store(float v) { return v; }
};
struct F16T {
  using S = uint16_t;
  static constexpr int code = TC_F16;
  __host__ __device__ __forceinline__ static float load(S s) {
#ifdef __CUDA_ARCH__
    return __half2float(__ushort_as_half(s));
#else
    return f16_bits_to_f32(s);
#endif
  }
  __host__ __device__ __forceinline__ static S store(float v) {
#ifdef __CUDA_ARCH__
    return __half_as_ushort(__float2half_rn(v));
#else
    return f32_to_f16_bits(v);
#endif
  }
};
struct BF16T {
  using S = uint16_t;
  static constexpr int code = TC_BF16;
  __host__ __device__ __forceinline__ static float load(S s) { return bf16_bits_to_f32(s); }
  __host__ __device__ __forceinline__ static S store(float v) {
#ifdef __CUDA_ARCH__
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
#else
    return f32_to_bf16_bits(v);
#endif
  }
};

// Two values rounded to the element type and packed low-first.
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}
__device__ __forceinline__ uint32_t pack2_f16(float lo, float hi) {
  __half2 p = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}

// Dispatch a functor templated on the element trait.
template <class F> int with_real(int dtype, F &&f) {
  switch (dtype) {
    case TC_F32: return f(F32T{});
    case TC_F16: return f(F16T{});
    case TC_BF16: return f(BF16T{});
    default: return fail(TC_EINVAL, "unknown element type %d", dtype);
  }
}

inline size_t dtype_bytes(int dtype) { return dtype == TC_F32 || dtype == TC_U32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// Scalar semantics of the reference's operation enums (kernels.rs:138-153,
// 195-226, 431-441).  minNum/maxNum: fminf/fmaxf return the number when one
// operand is a NaN.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float compare_value(int op, float a, float b) {
  switch (op) {
    case TC_MIN: return fminf(a, b);
    case TC_MAX: return fmaxf(a, b);
    case TC_MAX_SHARE: return a > b ? 1.0f : (a < b ? 0.0f : 0.5f);
    case TC_LESS: return a < b ? 1.0f : 0.0f;
    case TC_LESS_EQUAL: return a <= b ? 1.0f : 0.0f;
    case TC_GREATER: return a > b ? 1.0f : 0.0f;
    default: return a >= b ? 1.0f : 0.0f;
  }
}
// IEEE add/sub/mul/div with round-to-nearest and no contraction: the
// explicit _rn intrinsics keep the compiler from fusing a*b+c across ops.
__device__ __forceinline__ float binary_value(int op, float a, float b) {
  switch (op) {
    case TC_ADD: return __fadd_rn(a, b);
    case TC_SUB: return __fsub_rn(a, b);
    case TC_MUL: return __fmul_rn(a, b);
    case TC_DIV: return __fdiv_rn(a, b);
    default: return fmodf(a, b);
  }
}

// ---------------------------------------------------------------------------
// Layout descriptors (host): at most TC_MAX_RANK axes, element strides.
// ---------------------------------------------------------------------------
struct Dims {
  uint32_t rank = 0;
  size_t v[TC_MAX_RANK] = {0, 0, 0, 0, 0, 0};
};

// layout.rs:419-446 `coalesce`, for N operands: axes of one element dropped,
// an axis merged into the previous one wherever every operand steps across
// the pair as across one axis.
template <int N>
inline void coalesce(uint32_t rank, const size_t *shape, const size_t *const *strides, Dims &out_shape,
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
      for (int o = 0; o < N; ++o) {
        out[o].v[r] = strides[o][axis];
        out[o].rank++;
      }
    }
  }
}

inline size_t element_count(uint32_t rank, const size_t *shape) {
  size_t n = 1;
  for (uint32_t a = 0; a < rank; ++a) n *= shape[a];
  return n;
}

// layout.rs:136-149 `reach` + backend.rs:226-252 `check_strided`: TC_OK if a
// layout of `shape` from `offset` with `strides` stays inside `len`
// elements.
int check_layout(const char *what, size_t len, uint32_t rank, const size_t *shape, size_t offset,
                 const size_t *strides);

inline void contiguous_strides(uint32_t rank, const size_t *shape, size_t *out) {
  size_t step = 1;
  for (int a = int(rank) - 1; a >= 0; --a) {
    out[a] = step;
    step *= shape[a];
  }
}

// Kernel-side descriptor of up to 6 axes with up to 3 operands' strides, as
// 64-bit values; coordinates are decomposed from a flat row-major index.
struct Walk {
  int rank;
  long long shape[TC_MAX_RANK];
  long long stride[3][TC_MAX_RANK];
  long long offset[3];
};

template <int N>
__device__ __forceinline__ void walk_positions(const Walk &w, long long flat, long long *pos) {
#pragma unroll
  for (int o = 0; o < N; ++o) pos[o] = w.offset[o];
  for (int a = w.rank - 1; a >= 0; --a) {
    long long e = w.shape[a];
    long long c = flat % e;
    flat /= e;
#pragma unroll
    for (int o = 0; o < N; ++o) pos[o] += c * w.stride[o][a];
  }
}

inline unsigned grid_for(size_t work, unsigned block, unsigned max_blocks_per_sm = 8) {
  size_t want = (work + block - 1) / block;
  size_t cap = size_t(sm_count()) * max_blocks_per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return unsigned(want);
}

inline cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

}  // namespace tc
