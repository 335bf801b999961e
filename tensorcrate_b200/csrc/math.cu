// math.cu — the vector methods of Kernels<T> that are neither elementwise
// arithmetic nor reductions: the Analytic functions and their forward-mode
// step (vector_unary / matrix_unary, vector_unary_dual / matrix_unary_dual,
// kernels.rs:876, 891, 941, 950), the inclusive prefix sum
// (vector_prefix_sum, kernels.rs:870) and the total-order sort (vector_sort,
// kernels.rs:873).
//
// All of it is HBM-bound: 16-byte packs per thread, grids sized to the SMs.
#include <algorithm>
#include <climits>

#include "analytic.cuh"

namespace tc {
namespace {

template <class T> struct Pack {
  using S = typename T::S;
  static constexpr int N = 16 / int(sizeof(S));
  union {
    uint4 raw;
    S v[N];
  };
};

bool aligned16(const void *p) { return (uintptr_t(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Analytic functions.  vector_unary: vmath's f32 function, rounded once to T
// (Host kernels.rs:1257-1268; Sqrt is compact::sqrt, the f32 root rounded).
// vector_unary_dual: (f(x), f'(x)·t), the derivative and the product each in
// T (kernels.rs:1284-1304).
// ---------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(256) unary_kernel(const typename T::S *a, typename T::S *out, long long n, int f,
                                                    bool vec) {
  constexpr int N = Pack<T>::N;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const long long packs = n / N;
    for (long long p = i; p < packs; p += stride) {
      Pack<T> x, y;
      x.raw = __ldg(reinterpret_cast<const uint4 *>(a) + p);
#pragma unroll
      for (int j = 0; j < N; ++j) y.v[j] = T::store(analytic(f, T::load(x.v[j])));
      reinterpret_cast<uint4 *>(out)[p] = y.raw;
    }
    i += packs * N;
  }
  for (; i < n; i += stride) out[i] = T::store(analytic(f, T::load(a[i])));
}

template <class T>
__global__ void __launch_bounds__(256) unary_dual_kernel(const typename T::S *value, const typename T::S *tangent,
                                                         typename T::S *out_value, typename T::S *out_tangent,
                                                         long long n, int f, bool vec) {
  constexpr int N = Pack<T>::N;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const long long packs = n / N;
    for (long long p = i; p < packs; p += stride) {
      Pack<T> x, t, y, d;
      x.raw = __ldg(reinterpret_cast<const uint4 *>(value) + p);
      t.raw = __ldg(reinterpret_cast<const uint4 *>(tangent) + p);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float xv = T::load(x.v[j]);
        y.v[j] = T::store(analytic(f, xv));
        d.v[j] = T::store(__fmul_rn(analytic_derivative<T>(f, xv), T::load(t.v[j])));
      }
      reinterpret_cast<uint4 *>(out_value)[p] = y.raw;
      reinterpret_cast<uint4 *>(out_tangent)[p] = d.raw;
    }
    i += packs * N;
  }
  for (; i < n; i += stride) {
    const float xv = T::load(value[i]);
    out_value[i] = T::store(analytic(f, xv));
    out_tangent[i] = T::store(__fmul_rn(analytic_derivative<T>(f, xv), T::load(tangent[i])));
  }
}

// ---------------------------------------------------------------------------
// Inclusive prefix sum, reduce-then-scan (three launches, deterministic):
//   1. each of G blocks sums its chunk of `per` elements (a multiple of the
//      2048-element tile);
//   2. one block turns the G chunk sums into exclusive chunk offsets;
//   3. each block scans its chunk tile by tile from its offset: 8 elements
//      per thread in registers, warp and block scans of the thread totals.
// The running total is f32 and each output is rounded once to T, as the
// Host keeps an f32 running total for every type (vector.rs:578-589,
// compact::prefix_sum).  The association differs from the Host's serial
// chain, so f32 results agree within a sum's rounding, and exactly whenever
// the partial sums are exact (integral values below 2^24).
// ---------------------------------------------------------------------------
constexpr int SCAN_THREADS = 256, SCAN_ITEMS = 8, SCAN_TILE = SCAN_THREADS * SCAN_ITEMS, MAX_CHUNKS = 1024;

template <class T>
__device__ __forceinline__ void load_items(const typename T::S *a, long long at, long long n, bool vec, float v[8]) {
  using S = typename T::S;
  if (vec && at + SCAN_ITEMS <= n) {
    if (sizeof(S) == 2) {
      Pack<T> k;
      k.raw = __ldg(reinterpret_cast<const uint4 *>(a + at));
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = T::load(k.v[j]);
    } else {
      Pack<T> k0, k1;
      k0.raw = __ldg(reinterpret_cast<const uint4 *>(a + at));
      k1.raw = __ldg(reinterpret_cast<const uint4 *>(a + at) + 1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = T::load(k0.v[j]);
        v[4 + j] = T::load(k1.v[j]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = at + j < n ? T::load(a[at + j]) : 0.0f;
  }
}

// Inclusive scan of one value per thread across the block; `total` gets the
// block's sum.  Every thread of the block calls it.
__device__ __forceinline__ float block_inclusive(float x, float *warp_sums, float &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x = __fadd_rn(x, y);
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    float w = lane < warps ? warp_sums[lane] : 0.0f;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w = __fadd_rn(w, y);
    }
    if (lane < warps) warp_sums[lane] = w;
  }
  __syncthreads();
  if (warp > 0) x = __fadd_rn(x, warp_sums[warp - 1]);
  total = warp_sums[warps - 1];
  __syncthreads();
  return x;
}

template <class T>
__global__ void __launch_bounds__(SCAN_THREADS) chunk_sums(const typename T::S *a, long long n, long long per,
                                                           bool vec, float *sums) {
  __shared__ float warp_sums[32];
  const long long begin = (long long)blockIdx.x * per, end = min(n, begin + per);
  float s = 0.0f;
  for (long long t = begin; t < end; t += SCAN_TILE) {
    float v[8];
    load_items<T>(a, t + (long long)threadIdx.x * SCAN_ITEMS, end, vec, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[j]);
  }
  float total;
  block_inclusive(s, warp_sums, total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// offsets[b] = sums[0] + ... + sums[b-1], for b < chunks <= 1024.
__global__ void __launch_bounds__(MAX_CHUNKS) chunk_offsets(float *sums, int chunks) {
  __shared__ float warp_sums[32];
  const int t = threadIdx.x;
  const float x = t > 0 && t <= chunks ? sums[t - 1] : 0.0f;
  float total;
  const float incl = block_inclusive(x, warp_sums, total);
  __syncthreads();
  if (t < chunks) sums[t] = incl;
}

template <class T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_chunks(const typename T::S *a, typename T::S *out, long long n,
                                                            long long per, bool vec, const float *offsets) {
  using S = typename T::S;
  __shared__ float warp_sums[32];
  const long long begin = (long long)blockIdx.x * per, end = min(n, begin + per);
  float carry = offsets[blockIdx.x];
  // The next tile's items are loaded before this tile is scanned, so its
  // reads are in flight during the scan and the stores.
  float nv[8];
  if (begin < end) load_items<T>(a, begin + (long long)threadIdx.x * SCAN_ITEMS, end, vec, nv);
  for (long long t = begin; t < end; t += SCAN_TILE) {
    const long long at = t + (long long)threadIdx.x * SCAN_ITEMS;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = nv[j];
    if (t + SCAN_TILE < end) load_items<T>(a, at + SCAN_TILE, end, vec, nv);
#pragma unroll
    for (int j = 1; j < 8; ++j) v[j] = __fadd_rn(v[j - 1], v[j]);
    float tile_total;
    const float incl = block_inclusive(v[7], warp_sums, tile_total);
    // This thread's exclusive prefix within the tile: the inclusive scan of
    // the thread before it.
    float before = __shfl_up_sync(0xffffffffu, incl, 1);
    if ((threadIdx.x & 31) == 0) before = threadIdx.x == 0 ? 0.0f : warp_sums[(threadIdx.x >> 5) - 1];
    const float base = threadIdx.x == 0 ? carry : __fadd_rn(carry, before);
    S r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = T::store(__fadd_rn(base, v[j]));
    if (vec && at + SCAN_ITEMS <= end) {
      if (sizeof(S) == 2) {
        Pack<T> k;
#pragma unroll
        for (int j = 0; j < 8; ++j) k.v[j] = r[j];
        *reinterpret_cast<uint4 *>(out + at) = k.raw;
      } else {
        Pack<T> k0, k1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          k0.v[j] = r[j];
          k1.v[j] = r[4 + j];
        }
        reinterpret_cast<uint4 *>(out + at)[0] = k0.raw;
        reinterpret_cast<uint4 *>(out + at)[1] = k1.raw;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (at + j < end) out[at + j] = r[j];
    }
    carry = __fadd_rn(carry, tile_total);
    __syncthreads();  // warp_sums is read above and rewritten by the next tile
  }
}

// ---------------------------------------------------------------------------
// Sort in the total order of f32::total_cmp / half's total_cmp (the
// comparator of SortOrder, kernels.rs:252-269; Host vector.rs:874-886):
// -NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN, ordered within the NaNs by
// payload.  Mapping each value's bits to an unsigned key (every bit flipped
// for a negative sign, the sign bit set otherwise) turns that order into
// the keys' unsigned order, so a radix sort of the keys sorts the values;
// equal keys are equal bits, so the result is the unique sorted sequence.
// ---------------------------------------------------------------------------
template <class K> __device__ __forceinline__ K order_key(K bits) {
  constexpr K sign = K(K(1) << (sizeof(K) * 8 - 1));
  return (bits & sign) ? K(~bits) : K(bits | sign);
}
template <class K> __device__ __forceinline__ K key_bits(K key) {
  constexpr K sign = K(K(1) << (sizeof(K) * 8 - 1));
  return (key & sign) ? K(key ^ sign) : K(~key);
}

// What a radix pass does to the words it reads and writes: the first pass
// reads the values and maps them to keys, the last writes the values back
// (a descending sort sorts the keys' complements ascending: `flip`); the
// passes between move keys as they are.
template <class K> struct KeyMap {
  bool map_in, map_out;
  K flip;
  __device__ __forceinline__ K in(K v) const { return map_in ? K(order_key(v) ^ flip) : v; }
  __device__ __forceinline__ K out(K k) const { return map_out ? key_bits(K(k ^ flip)) : k; }
};

// ---------------------------------------------------------------------------
// LSD radix sort of the keys, 8 bits a pass (4 passes for f32's keys, 2 for
// f16/bf16's).  Each pass is stable, so after the last one the keys are in
// unsigned order.  The keys are cut into tiles of RADIX_TILE; a pass
//   1. counts each tile's digits (warp-private histograms in shared memory)
//      into counts[digit][tile];
//   2. turns the counts into each (digit, tile)'s first output position: an
//      exclusive scan along each digit's row of tiles (a block per digit),
//      then of the 256 digit totals;
//   3. moves every key to its position: each warp of a block ranks its own
//      contiguous share of the tile (512 keys, 32 at a time in index order)
//      against warp-private digit counts (a key's rank among the warp's keys
//      of its digit is the count so far plus its rank among the step's lanes
//      with that digit, found by a vote per digit bit), then one pass over
//      the digits turns the warps' counts into each warp's first place per
//      digit in the tile sorted by digit, in warp order, so equal digits keep
//      their input order; the tile is sorted in shared memory and written
//      out in order, each digit's run of keys to consecutive places.
// The first pass maps the values to keys as it reads them and the last maps
// the keys back as it writes them (KeyMap).
// ---------------------------------------------------------------------------
constexpr int RADIX_BINS = 256;
constexpr int RADIX_THREADS = 256;
constexpr int RADIX_ITEMS = 16;
constexpr int RADIX_TILE = RADIX_THREADS * RADIX_ITEMS;
constexpr int RADIX_WARPS = RADIX_THREADS / 32;

template <class K>
__global__ void __launch_bounds__(RADIX_THREADS) radix_histogram(const K *keys, long long n, int shift,
                                                                 uint32_t *counts, int tiles, bool vec, KeyMap<K> m) {
  __shared__ uint32_t h[RADIX_WARPS][RADIX_BINS];
  const int tid = threadIdx.x, warp = tid >> 5;
#pragma unroll
  for (int w = 0; w < RADIX_WARPS; ++w) h[w][tid] = 0;
  __syncthreads();
  const long long base = (long long)blockIdx.x * RADIX_TILE;
  constexpr int P = 16 / int(sizeof(K));  // keys per 16-byte load
  if (vec && base + RADIX_TILE <= n) {
    // a whole tile on 16-byte boundaries: every load in flight at once
    uint4 q[RADIX_ITEMS / P];
#pragma unroll
    for (int j = 0; j < RADIX_ITEMS / P; ++j)
      q[j] = __ldg(reinterpret_cast<const uint4 *>(keys + base) + j * RADIX_THREADS + tid);
#pragma unroll
    for (int j = 0; j < RADIX_ITEMS / P; ++j) {
      const K *k = reinterpret_cast<const K *>(&q[j]);
#pragma unroll
      for (int e = 0; e < P; ++e) atomicAdd(&h[warp][(uint32_t(m.in(k[e])) >> shift) & 255u], 1u);
    }
  } else {
#pragma unroll 4
    for (int i = 0; i < RADIX_ITEMS; ++i) {
      const long long idx = base + (long long)i * RADIX_THREADS + tid;
      if (idx < n) atomicAdd(&h[warp][(uint32_t(m.in(keys[idx])) >> shift) & 255u], 1u);
    }
  }
  __syncthreads();
  uint32_t total = 0;
#pragma unroll
  for (int w = 0; w < RADIX_WARPS; ++w) total += h[w][tid];
  counts[size_t(tid) * size_t(tiles) + blockIdx.x] = total;
}

// Block `digit`: exclusive scan of counts[digit][0..tiles) in place; the
// row's total into totals[digit].
__global__ void __launch_bounds__(RADIX_THREADS) radix_scan_rows(uint32_t *counts, int tiles, uint32_t *totals) {
  __shared__ uint32_t warp_sums[RADIX_WARPS];
  uint32_t *row = counts + size_t(blockIdx.x) * size_t(tiles);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t carry = 0;
  for (int start = 0; start < tiles; start += RADIX_THREADS) {
    const int i = start + tid;
    const uint32_t v = i < tiles ? row[i] : 0u;
    uint32_t x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(~0u, x, d);
      if (lane >= d) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    uint32_t before = 0, chunk = 0;
#pragma unroll
    for (int w = 0; w < RADIX_WARPS; ++w) {
      const uint32_t ws = warp_sums[w];
      if (w < warp) before += ws;
      chunk += ws;
    }
    if (i < tiles) row[i] = carry + before + x - v;
    carry += chunk;
    __syncthreads();
  }
  if (tid == 0) totals[blockIdx.x] = carry;
}

// Exclusive scan of the 256 digit totals: each digit's first output position.
__global__ void __launch_bounds__(RADIX_BINS) radix_scan_totals(const uint32_t *totals, uint32_t *starts) {
  __shared__ uint32_t warp_sums[RADIX_BINS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t v = totals[tid];
  uint32_t x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(~0u, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  uint32_t before = 0;
  for (int w = 0; w < warp; ++w) before += warp_sums[w];
  starts[tid] = before + x - v;
}

template <class K>
__global__ void __launch_bounds__(RADIX_THREADS) radix_scatter(const K *in, K *out, long long n, int shift,
                                                               const uint32_t *counts, const uint32_t *starts,
                                                               int tiles, KeyMap<K> m) {
  // counts[w][d]: how many of warp w's keys so far have digit d; then where
  // warp w's first key with digit d goes in the tile sorted by digit
  __shared__ uint32_t warp_counts[RADIX_WARPS][RADIX_BINS];
  __shared__ uint32_t base_of[RADIX_BINS], warp_sums[RADIX_WARPS];
  __shared__ K sorted[RADIX_TILE];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int w = 0; w < RADIX_WARPS; ++w) warp_counts[w][tid] = 0;
  __syncthreads();
  const unsigned below = (1u << lane) - 1u;
  // Warp w ranks keys [first, first + 32·RADIX_ITEMS) of the tile, 32 at a
  // time in index order: a key's rank among the warp's keys of its digit is
  // the warp's count of that digit so far (read by the digit's first lane
  // in this step, which adds the step's keys of the digit) plus its rank
  // among this step's lanes with the digit.  No block barrier.
  const long long first = (long long)blockIdx.x * RADIX_TILE + (long long)warp * 32 * RADIX_ITEMS;
  K keys[RADIX_ITEMS];
  uint32_t place[RADIX_ITEMS];  // digit << 16 | rank among the warp's keys of the digit
  unsigned peers[RADIX_ITEMS];  // the step's lanes with this lane's digit
#pragma unroll
  for (int i = 0; i < RADIX_ITEMS; ++i) {
    const long long idx = first + (long long)i * 32 + lane;
    keys[i] = idx < n ? m.in(in[idx]) : K(0);
  }
  // Lanes with the same digit, by one vote per digit bit (and one for lanes
  // past the end, whose keys do not exist): independent of the counts, so
  // every step's votes are taken before the counting walk.
#pragma unroll
  for (int i = 0; i < RADIX_ITEMS; ++i) {
    const bool valid = first + (long long)i * 32 + lane < n;
    const uint32_t digit = (uint32_t(keys[i]) >> shift) & 255u;
    const unsigned live = __ballot_sync(~0u, valid);
    unsigned same = valid ? live : ~live;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const unsigned ones = __ballot_sync(~0u, (digit >> b) & 1u);
      same &= ((digit >> b) & 1u) ? ones : ~ones;
    }
    peers[i] = same;
  }
#pragma unroll
  for (int i = 0; i < RADIX_ITEMS; ++i) {
    const long long idx = first + (long long)i * 32 + lane;
    const bool valid = idx < n;
    // Lanes past the end take digit 256, which no key has.
    const uint32_t digit = valid ? (uint32_t(keys[i]) >> shift) & 255u : 256u;
    const int leader = __ffs(peers[i]) - 1;
    uint32_t before = 0;
    if (valid && lane == leader) {
      before = warp_counts[warp][digit];
      warp_counts[warp][digit] = before + uint32_t(__popc(peers[i]));
    }
    before = __shfl_sync(~0u, before, leader);
    place[i] = (digit << 16) | (before + uint32_t(__popc(peers[i] & below)));
    __syncwarp();  // this step's counts are seen by the next step's leaders
  }
  __syncthreads();
  // Digit `tid`: the tile's count of it and, by a scan over the digits, where
  // its keys start in the tile sorted by digit; each warp's keys of it follow
  // in warp order.  base_of[d] + (place in the sorted tile) is the output
  // position (the digit's start plus this tile's scanned count).
  uint32_t tile_count = 0;
#pragma unroll
  for (int w = 0; w < RADIX_WARPS; ++w) tile_count += warp_counts[w][tid];
  uint32_t x = tile_count;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(~0u, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  uint32_t local = x - tile_count;
  for (int w = 0; w < warp; ++w) local += warp_sums[w];
  base_of[tid] = starts[tid] + counts[size_t(tid) * size_t(tiles) + blockIdx.x] - local;
#pragma unroll
  for (int w = 0; w < RADIX_WARPS; ++w) {
    const uint32_t c = warp_counts[w][tid];
    warp_counts[w][tid] = local;
    local += c;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < RADIX_ITEMS; ++i) {
    const uint32_t digit = place[i] >> 16;
    if (digit < RADIX_BINS) sorted[warp_counts[warp][digit] + (place[i] & 0xffffu)] = keys[i];
  }
  __syncthreads();
  // The sorted tile out in order: each digit's keys to consecutive places.
  const int in_tile = int(min((long long)RADIX_TILE, n - (long long)blockIdx.x * RADIX_TILE));
  for (int j = tid; j < in_tile; j += RADIX_THREADS) {
    const K key = sorted[j];
    out[base_of[(uint32_t(key) >> shift) & 255u] + j] = m.out(key);
  }
}

template <class K> int sort_keys(const void *a, void *out, size_t n, bool descending, cudaStream_t s) {
  if (n > size_t(INT_MAX)) return fail(TC_EINVAL, "sort: %zu elements exceed the radix sort's 2^31-1", n);
  // The second key buffer and the counts come from the stream's scratch.
  K *keys = static_cast<K *>(out);
  const int tiles = int((n + RADIX_TILE - 1) / RADIX_TILE);
  const size_t alt_bytes = (n * sizeof(K) + 255) & ~size_t(255);
  const size_t count_bytes = (size_t(RADIX_BINS) * size_t(tiles) * 4 + 255) & ~size_t(255);
  void *block = nullptr;
  if (int st = scratch(alt_bytes + count_bytes + 2 * RADIX_BINS * 4, &block, s)) return st;
  K *alt = static_cast<K *>(block);
  uint32_t *counts = reinterpret_cast<uint32_t *>(static_cast<char *>(block) + alt_bytes);
  uint32_t *totals = reinterpret_cast<uint32_t *>(static_cast<char *>(block) + alt_bytes + count_bytes);
  uint32_t *starts = totals + RADIX_BINS;
  auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  // The first pass reads the values (mapping them to keys as it goes), the
  // last writes values (mapping back); an even number of passes ends in
  // `out`, which the first pass does not write (an in-place sort is safe).
  const K flip = descending ? K(~K(0)) : K(0);
  const K *src = static_cast<const K *>(a);
  K *dst = alt;
  constexpr int passes = int(sizeof(K) * 8) / 8;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    const KeyMap<K> m{pass == 0, pass == passes - 1, flip};
    radix_histogram<K><<<tiles, RADIX_THREADS, 0, s>>>(src, (long long)n, shift, counts, tiles, aligned(src), m);
    radix_scan_rows<<<RADIX_BINS, RADIX_THREADS, 0, s>>>(counts, tiles, totals);
    radix_scan_totals<<<1, RADIX_BINS, 0, s>>>(totals, starts);
    radix_scatter<K><<<tiles, RADIX_THREADS, 0, s>>>(src, dst, (long long)n, shift, counts, starts, tiles, m);
    if (int st = check_launch("sort (radix pass)")) return st;
    src = dst;
    dst = dst == alt ? keys : alt;
  }
  return TC_OK;
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_unary(int dtype, int f, const void *a, void *out, size_t n, void *stream) {
  if (f < TC_SIN || f > TC_SQRT) return fail(TC_EINVAL, "bad Analytic %d", f);
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "unary: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    const bool vec = aligned16(a) && aligned16(out);
    unary_kernel<T><<<grid_for((n + Pack<T>::N - 1) / Pack<T>::N, 256, 8), 256, 0, as_stream(stream)>>>(
        static_cast<const S *>(a), static_cast<S *>(out), (long long)n, f, vec);
    return check_launch("unary");
  });
}

int tc_unary_dual(int dtype, int f, const void *value, const void *tangent, void *out_value, void *out_tangent,
                  size_t n, void *stream) {
  if (f < TC_SIN || f > TC_SQRT) return fail(TC_EINVAL, "bad Analytic %d", f);
  if (n == 0) return TC_OK;
  if (!value || !tangent || !out_value || !out_tangent) return fail(TC_EINVAL, "unary_dual: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    const bool vec = aligned16(value) && aligned16(tangent) && aligned16(out_value) && aligned16(out_tangent);
    unary_dual_kernel<T><<<grid_for((n + Pack<T>::N - 1) / Pack<T>::N, 256, 8), 256, 0, as_stream(stream)>>>(
        static_cast<const S *>(value), static_cast<const S *>(tangent), static_cast<S *>(out_value),
        static_cast<S *>(out_tangent), (long long)n, f, vec);
    return check_launch("unary_dual");
  });
}

int tc_prefix_sum(int dtype, const void *a, void *out, size_t n, void *stream) {
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "prefix_sum: null pointer");
  return with_real(dtype, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    cudaStream_t s = as_stream(stream);
    const long long tiles = ((long long)n + SCAN_TILE - 1) / SCAN_TILE;
    const long long want = std::min<long long>(MAX_CHUNKS, (long long)sm_count() * 4);
    const long long per = ((tiles + want - 1) / want) * SCAN_TILE;
    const int chunks = int(((long long)n + per - 1) / per);
    float *sums = nullptr;
    if (int st = scratch(MAX_CHUNKS * sizeof(float), reinterpret_cast<void **>(&sums), s)) return st;
    const bool vec = aligned16(a) && aligned16(out);
    chunk_sums<T><<<chunks, SCAN_THREADS, 0, s>>>(static_cast<const S *>(a), (long long)n, per, vec, sums);
    if (int st = check_launch("prefix_sum (chunks)")) return st;
    chunk_offsets<<<1, MAX_CHUNKS, 0, s>>>(sums, chunks);
    if (int st = check_launch("prefix_sum (offsets)")) return st;
    scan_chunks<T><<<chunks, SCAN_THREADS, 0, s>>>(static_cast<const S *>(a), static_cast<S *>(out), (long long)n,
                                                   per, vec, sums);
    return check_launch("prefix_sum (scan)");
  });
}

int tc_sort(int dtype, int order, const void *a, void *out, size_t n, void *stream) {
  if (order != TC_ASCENDING && order != TC_DESCENDING) return fail(TC_EINVAL, "bad SortOrder %d", order);
  if (n == 0) return TC_OK;
  if (!a || !out) return fail(TC_EINVAL, "sort: null pointer");
  if (dtype == TC_F32) return sort_keys<uint32_t>(a, out, n, order == TC_DESCENDING, as_stream(stream));
  if (dtype == TC_F16 || dtype == TC_BF16)
    return sort_keys<uint16_t>(a, out, n, order == TC_DESCENDING, as_stream(stream));
  return fail(TC_EINVAL, "unknown element type %d", dtype);
}

}  // extern "C"
