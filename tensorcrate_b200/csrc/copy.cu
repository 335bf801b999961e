// copy.cu — the one strided layout copy behind permute, transpose, slice,
// split, concatenate and stack (Backend::strided_copy / assemble /
// strided_write, src/tensors/backend.rs:141-173).  It moves bits, so it is
// written over element widths (1, 2, 4, 8, 16 bytes), never over a type.
//
// Every region is coalesced on the host first (layout.rs:419-446), then one
// of three kernels runs it:
//  - runs: both sides step by one element along the innermost axis.  The
//    run is copied in the widest unit (16, 8, 4, 2 or 1 bytes) that every
//    base, offset, stride and run length allows; 128-bit loads and stores
//    where the layout permits.
//  - transpose: the target steps by one along the innermost axis and the
//    source along another axis t.  A tile over (t, innermost) is staged in
//    shared memory so both the reads and the writes are coalesced.
//  - gather: anything else (zero strides, scatters), one element per thread.
#include <algorithm>

#include "common.cuh"

namespace tc {
namespace {

// A region as the kernels take it: up to 6 axes, element strides of the
// source (0) and target (1), offsets, base pointers.
struct CopyDesc {
  int rank;
  long long shape[TC_MAX_RANK];
  long long stride[2][TC_MAX_RANK];
  long long offset[2];
  const char *src;
  char *dst;
  long long count;  // units to copy
  // Division by shape[a] as a multiply and shift, for 32-bit indices
  // (n < 2^31): n / d = umulhi(n, mul) >> shift, mul = ceil(2^(31+l) / d),
  // shift = l - 1, l = ceil(log2 d) (Granlund and Montgomery, 1994); d = 1
  // is marked by mul = 0.
  uint32_t mul[TC_MAX_RANK], shift[TC_MAX_RANK];
};

// Fill d.mul / d.shift from d.shape (host).
void prepare_division(CopyDesc &d) {
  for (int a = 0; a < d.rank; ++a) {
    const uint64_t e = uint64_t(d.shape[a]);
    if (e <= 1 || e >= (1ull << 31)) {
      d.mul[a] = 0;
      d.shift[a] = 0;
      continue;
    }
    int l = 0;
    while ((1ull << l) < e) ++l;
    d.mul[a] = uint32_t(((1ull << (31 + l)) + e - 1) / e);
    d.shift[a] = uint32_t(l - 1);
  }
}

template <int W> struct Unit;
template <> struct Unit<1> { using T = uint8_t; };
template <> struct Unit<2> { using T = uint16_t; };
template <> struct Unit<4> { using T = uint32_t; };
template <> struct Unit<8> { using T = uint2; };
template <> struct Unit<16> { using T = uint4; };

// Copy `d.count` units of W bytes: flat row-major index -> both positions.
// Shapes, strides and offsets are in units.  Each thread issues UNROLL
// loads (one per grid stride) before it stores any.
constexpr int UNROLL = 4;

template <typename Index>
__device__ __forceinline__ void unit_positions(const CopyDesc &d, Index i, Index &s, Index &t) {
  const int rank = d.rank;
  Index rest = i;
  s = Index(d.offset[0]);
  t = Index(d.offset[1]);
  for (int a = rank - 1; a >= 0; --a) {
    const Index e = Index(d.shape[a]);
    Index q;
    if (sizeof(Index) == 4)
      q = d.mul[a] ? Index(__umulhi(uint32_t(rest), d.mul[a]) >> d.shift[a]) : (e == 1 ? rest : Index(0));
    else
      q = rest / e;
    const Index ca = rest - q * e;
    rest = q;
    s += ca * Index(d.stride[0][a]);
    t += ca * Index(d.stride[1][a]);
  }
}

template <int W, typename Index>
__global__ void __launch_bounds__(256) copy_units(const CopyDesc d) {
  using U = typename Unit<W>::T;
  const U *src = reinterpret_cast<const U *>(d.src);
  U *dst = reinterpret_cast<U *>(d.dst);
  const Index stride = Index(gridDim.x) * blockDim.x;
  const Index count = Index(d.count);
  for (Index i0 = Index(blockIdx.x) * blockDim.x + threadIdx.x; i0 < count; i0 += stride * UNROLL) {
    U v[UNROLL];
    Index t[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      const Index i = i0 + Index(k) * stride;
      if (i < count) {
        Index s;
        unit_positions(d, i, s, t[k]);
        v[k] = __ldg(src + s);
      }
    }
#pragma unroll
    for (int k = 0; k < UNROLL; ++k)
      if (i0 + Index(k) * stride < count) dst[t[k]] = v[k];
  }
}

// Several regions of one unit width in one launch (an assemble of run
// copies): region k holds flat units [start[k], start[k+1]).
constexpr int MAX_BATCH = 8;
struct MultiDesc {
  int n;
  long long start[MAX_BATCH + 1];
  CopyDesc r[MAX_BATCH];
  // Row form (every region's innermost run contiguous on both sides): work
  // items of ROW_ITEM units along one row; region k holds items
  // [items[k], items[k+1]), `per_row[k]` of them per row (with its
  // multiply-shift division constants).
  long long items[MAX_BATCH + 1];
  uint32_t per_row[MAX_BATCH], per_row_mul[MAX_BATCH], per_row_shift[MAX_BATCH];
};
constexpr int ROW_ITEM = 32 * 4;  // a warp's item: 4 units per lane

template <int W, typename Index>
__global__ void __launch_bounds__(256) copy_units_multi(const __grid_constant__ MultiDesc m) {
  using U = typename Unit<W>::T;
  const Index total = Index(m.start[m.n]);
  const Index stride = Index(gridDim.x) * blockDim.x;
  for (Index i0 = Index(blockIdx.x) * blockDim.x + threadIdx.x; i0 < total; i0 += stride * UNROLL) {
    U v[UNROLL];
    U *to[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      const Index i = i0 + Index(k) * stride;
      if (i < total) {
        int r = 0;
        while (r + 1 < m.n && i >= Index(m.start[r + 1])) ++r;
        const CopyDesc &d = m.r[r];
        Index s, t;
        unit_positions(d, i - Index(m.start[r]), s, t);
        v[k] = __ldg(reinterpret_cast<const U *>(d.src) + s);
        to[k] = reinterpret_cast<U *>(d.dst) + t;
      }
    }
#pragma unroll
    for (int k = 0; k < UNROLL; ++k)
      if (i0 + Index(k) * stride < total) *to[k] = v[k];
  }
}

// Position of the start of row `row` (all axes but the innermost).
template <typename Index>
__device__ __forceinline__ void row_positions(const CopyDesc &d, Index row, Index &s, Index &t) {
  Index rest = row;
  s = Index(d.offset[0]);
  t = Index(d.offset[1]);
  for (int a = d.rank - 2; a >= 0; --a) {
    const Index e = Index(d.shape[a]);
    Index q;
    if (sizeof(Index) == 4)
      q = d.mul[a] ? Index(__umulhi(uint32_t(rest), d.mul[a]) >> d.shift[a]) : (e == 1 ? rest : Index(0));
    else
      q = rest / e;
    const Index ca = rest - q * e;
    rest = q;
    s += ca * Index(d.stride[0][a]);
    t += ca * Index(d.stride[1][a]);
  }
}

// Regions whose innermost run is contiguous on both sides: a warp per item
// of ROW_ITEM units along one row, each lane 4 units 32 apart (loads before
// stores); the row's start costs one division per item, not per unit.
template <int W, typename Index>
__global__ void __launch_bounds__(256) copy_rows_multi(const __grid_constant__ MultiDesc m) {
  using U = typename Unit<W>::T;
  const Index total = Index(m.items[m.n]);
  const int lane = threadIdx.x & 31;
  const Index warps = Index(gridDim.x) * (blockDim.x >> 5);
  for (Index item = Index(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < total; item += warps) {
    int r = 0;
    while (r + 1 < m.n && item >= Index(m.items[r + 1])) ++r;
    const CopyDesc &d = m.r[r];
    const Index local = item - Index(m.items[r]);
    Index row;
    if (sizeof(Index) == 4)
      row = m.per_row_mul[r] ? Index(__umulhi(uint32_t(local), m.per_row_mul[r]) >> m.per_row_shift[r]) : local;
    else
      row = local / Index(m.per_row[r]);
    const Index col0 = (local - row * Index(m.per_row[r])) * ROW_ITEM + lane;
    const Index inner = Index(d.shape[d.rank - 1]);
    Index s, t;
    row_positions(d, row, s, t);
    const U *src = reinterpret_cast<const U *>(d.src) + s;
    U *dst = reinterpret_cast<U *>(d.dst) + t;
    U v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (col0 + 32 * k < inner) v[k] = __ldg(src + col0 + 32 * k);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (col0 + 32 * k < inner) dst[col0 + 32 * k] = v[k];
  }
}

// Tiled transpose: axis `t` (source stride 1) against the innermost axis
// (target stride 1).  Each block moves one TILE x TILE tile for one index of
// the remaining axes (flattened into blockIdx.z and below).
constexpr int TILE = 32;
template <int W>
__global__ void __launch_bounds__(256) copy_transpose(const CopyDesc d, int t_axis, long long others) {
  using U = typename Unit<W>::T;
  __shared__ U tile[TILE][TILE + 1];
  const U *src = reinterpret_cast<const U *>(d.src);
  U *dst = reinterpret_cast<U *>(d.dst);
  const int rank = d.rank;
  const long long n_in = d.shape[rank - 1], n_t = d.shape[t_axis];
  const long long in0 = (long long)blockIdx.x * TILE, t0 = (long long)blockIdx.y * TILE;
  for (long long o = blockIdx.z; o < others; o += gridDim.z) {
    // Positions of the remaining axes (all but t_axis and the innermost).
    long long rest = o, s = d.offset[0], t = d.offset[1];
    for (int a = rank - 2; a >= 0; --a) {
      if (a == t_axis) continue;
      long long e = d.shape[a];
      long long c = rest % e;
      rest /= e;
      s += c * d.stride[0][a];
      t += c * d.stride[1][a];
    }
    // Read: consecutive threads walk axis t (source-contiguous).
    for (int r = threadIdx.y; r < TILE; r += blockDim.y) {
      long long i_in = in0 + r, i_t = t0 + threadIdx.x;
      if (i_in < n_in && i_t < n_t)
        tile[r][threadIdx.x] = __ldg(src + s + i_in * d.stride[0][rank - 1] + i_t);
    }
    __syncthreads();
    // Write: consecutive threads walk the innermost axis (target-contiguous).
    for (int r = threadIdx.y; r < TILE; r += blockDim.y) {
      long long i_t = t0 + r, i_in = in0 + threadIdx.x;
      if (i_in < n_in && i_t < n_t) dst[t + i_t * d.stride[1][t_axis] + i_in] = tile[threadIdx.x][r];
    }
    __syncthreads();
  }
}


// Tiled transpose for 2-byte elements moved as 32-bit pairs: tiles of 64
// target-contiguous (inner) by TT source-contiguous (t) elements, TT = 32 or
// 64 to fit the t extent.  A warp reads whole 2*TT-byte source rows (one
// inner index each) and writes 128-byte target rows (one t index each).  The
// tile sits t-major in shared memory, so the writers read 32-bit pairs
// along the inner axis without bank conflicts.  A block loads BATCH tiles
// before it stores any.  Needs even extents, strides and offsets along both
// tile axes.  A persistent grid walks (other axes, inner tile, t tile).
template <int TT, int BATCH>
__global__ void __launch_bounds__(256) copy_transpose_pairs(const CopyDesc d, int t_axis, long long others) {
  constexpr int ROWS_PER_PASS = 256 / (TT / 2);  // inner rows one pass of the block reads
  constexpr int PASSES = 64 / ROWS_PER_PASS;
  constexpr int PITCH = 64 + 2;                   // u16 per t row: 33 words
  // Two tile buffers and three descriptor slots: while a batch is written
  // out of one buffer, the next batch's loads are in flight into registers
  // and the one after it is being described.
  __shared__ __align__(16) uint16_t tile[2][BATCH][TT][PITCH];
  __shared__ const uint16_t *sb[3][BATCH];
  __shared__ uint16_t *tb[3][BATCH];
  __shared__ int ilim[3][BATCH], tlim[3][BATCH];  // valid inner / t extent of each tile
  const uint16_t *src = reinterpret_cast<const uint16_t *>(d.src);
  uint16_t *dst = reinterpret_cast<uint16_t *>(d.dst);
  const int rank = d.rank;
  const long long n_in = d.shape[rank - 1], n_t = d.shape[t_axis];
  const long long tiles_i = (n_in + 63) / 64, tiles_t = (n_t + TT - 1) / TT;
  const long long total = others * tiles_i * tiles_t;
  const long long s_in = d.stride[0][rank - 1], d_t = d.stride[1][t_axis];
  const long long step = (long long)gridDim.x * BATCH;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rp = threadIdx.x / (TT / 2), pp = threadIdx.x % (TT / 2);  // read: row in pass, pair
  // One thread per tile of a batch decomposes its index into slot `sl`.
  auto describe = [&](long long w0, int sl) {
    if (threadIdx.x >= BATCH) return;
    const long long w = w0 + threadIdx.x;
    if (w >= total) {
      ilim[sl][threadIdx.x] = tlim[sl][threadIdx.x] = 0;
      return;
    }
    long long o = w / (tiles_i * tiles_t);
    const long long rem = w - o * tiles_i * tiles_t;
    long long so = d.offset[0], to = d.offset[1];
    for (int a = rank - 2; a >= 0; --a) {
      if (a == t_axis) continue;
      const long long e = d.shape[a], c = o % e;
      o /= e;
      so += c * d.stride[0][a];
      to += c * d.stride[1][a];
    }
    const long long i0 = (rem / tiles_t) * 64, j0 = (rem % tiles_t) * TT;
    sb[sl][threadIdx.x] = src + so + i0 * s_in + j0;
    tb[sl][threadIdx.x] = dst + to + j0 * d_t + i0;
    ilim[sl][threadIdx.x] = int(min(64LL, n_in - i0));
    tlim[sl][threadIdx.x] = int(min((long long)TT, n_t - j0));
  };
  uint32_t v[BATCH][PASSES];
  auto load = [&](int sl) {
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const uint16_t *base = sb[sl][q] + 2 * pp;
      const bool tok = 2 * pp < tlim[sl][q];
#pragma unroll
      for (int k = 0; k < PASSES; ++k) {
        const int i = rp + ROWS_PER_PASS * k;
        v[q][k] = (tok && i < ilim[sl][q]) ? __ldg(reinterpret_cast<const uint32_t *>(base + (long long)i * s_in)) : 0u;
      }
    }
  };
  long long w0 = (long long)blockIdx.x * BATCH;
  if (w0 >= total) return;
  describe(w0, 0);
  __syncthreads();
  load(0);
  for (int it = 0; w0 < total; w0 += step, ++it) {
    const int buf = it & 1, sl = it % 3, nsl = (it + 1) % 3;
    // stage this batch (already in registers) in shared memory, t-major
#pragma unroll
    for (int q = 0; q < BATCH; ++q)
#pragma unroll
      for (int k = 0; k < PASSES; ++k) {
        const int i = rp + ROWS_PER_PASS * k;
        tile[buf][q][2 * pp][i] = uint16_t(v[q][k] & 0xffffu);
        tile[buf][q][2 * pp + 1][i] = uint16_t(v[q][k] >> 16);
      }
    describe(w0 + step, nsl);
    __syncthreads();
    // the next batch's loads go out before this batch's stores
    if (w0 + step < total) load(nsl);
    // write: warp rows = t indices, lanes = pairs along inner
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const bool iok = 2 * lane < ilim[sl][q];
      uint16_t *out = tb[sl][q] + 2 * lane;
#pragma unroll
      for (int k = 0; k < TT / 8; ++k) {
        const int j = warp + 8 * k;
        if (iok && j < tlim[sl][q])
          *reinterpret_cast<uint32_t *>(out + (long long)j * d_t) = *reinterpret_cast<const uint32_t *>(&tile[buf][q][j][2 * lane]);
      }
    }
  }
}

int largest_unit(size_t elem, const Dims &shape, const Dims *st, const void *src, const void *dst) {
  // The innermost run must be contiguous on both sides to widen.
  uint32_t r = shape.rank;
  if (r == 0 || st[0].v[r - 1] != 1 || st[1].v[r - 1] != 1) return int(elem);
  for (int w = 16; w > int(elem); w >>= 1) {
    if (size_t(w) % elem) continue;
    size_t per = size_t(w) / elem;  // elements per unit
    bool ok = (shape.v[r - 1] % per) == 0 && (uintptr_t(src) % w) == 0 && (uintptr_t(dst) % w) == 0;
    for (uint32_t a = 0; ok && a + 1 < r; ++a) ok = (st[0].v[a] % per) == 0 && (st[1].v[a] % per) == 0;
    if (ok) return w;
  }
  return int(elem);
}

// True when every index a region computes (counts, and the furthest
// position on either side) fits a signed 32-bit integer.
bool fits32(const CopyDesc &d) {
  if (d.count >= (1LL << 31)) return false;
  for (int side = 0; side < 2; ++side) {
    long long reach = d.offset[side];
    for (int a = 0; a < d.rank; ++a) reach += (d.shape[a] - 1) * d.stride[side][a];
    if (reach >= (1LL << 31)) return false;
  }
  return true;
}

// Launch the regions of `m` (one unit width): in row form when every
// region's innermost run is contiguous on both sides, else unit by unit.
template <int W>
int launch_multi(MultiDesc &m, cudaStream_t stream) {
  bool rows = true, narrow = true;
  for (int k = 0; k < m.n; ++k) {
    const CopyDesc &d = m.r[k];
    rows = rows && d.stride[0][d.rank - 1] == 1 && d.stride[1][d.rank - 1] == 1;
    narrow = narrow && fits32(d);
  }
  if (rows) {
    m.items[0] = 0;
    for (int k = 0; k < m.n; ++k) {
      const CopyDesc &d = m.r[k];
      const long long inner = d.shape[d.rank - 1];
      const long long per_row = (inner + ROW_ITEM - 1) / ROW_ITEM;
      m.items[k + 1] = m.items[k] + d.count / inner * per_row;
      m.per_row[k] = uint32_t(per_row);
      m.per_row_mul[k] = m.per_row_shift[k] = 0;
      if (per_row > 1 && per_row < (1LL << 31)) {
        int l = 0;
        while ((1LL << l) < per_row) ++l;
        m.per_row_mul[k] = uint32_t(((1ull << (31 + l)) + uint64_t(per_row) - 1) / uint64_t(per_row));
        m.per_row_shift[k] = uint32_t(l - 1);
      }
    }
    const long long items = m.items[m.n];
    narrow = narrow && items < (1LL << 31);
    const unsigned grid = unsigned(std::max(1LL, std::min((items + 7) / 8, (long long)sm_count() * 8)));
    if (narrow) copy_rows_multi<W, int><<<grid, 256, 0, stream>>>(m);
    else copy_rows_multi<W, long long><<<grid, 256, 0, stream>>>(m);
    return check_launch("strided copy (rows)");
  }
  const long long total = m.start[m.n];
  const unsigned grid = grid_for(size_t(total), 256, 16);
  if (m.n == 1) {
    if (narrow) copy_units<W, int><<<grid, 256, 0, stream>>>(m.r[0]);
    else copy_units<W, long long><<<grid, 256, 0, stream>>>(m.r[0]);
  } else {
    if (narrow && total < (1LL << 31)) copy_units_multi<W, int><<<grid, 256, 0, stream>>>(m);
    else copy_units_multi<W, long long><<<grid, 256, 0, stream>>>(m);
  }
  return check_launch("strided copy");
}

int launch_multi_width(int w, MultiDesc &m, cudaStream_t stream) {
  switch (w) {
    case 1: return launch_multi<1>(m, stream);
    case 2: return launch_multi<2>(m, stream);
    case 4: return launch_multi<4>(m, stream);
    case 8: return launch_multi<8>(m, stream);
    case 16: return launch_multi<16>(m, stream);
  }
  return fail(TC_EINVAL, "strided copy: element width %d", w);
}

int launch_width(int w, const CopyDesc &d, cudaStream_t stream) {
  MultiDesc m{};
  m.n = 1;
  m.r[0] = d;
  m.start[1] = d.count;
  return launch_multi_width(w, m, stream);
}

template <int W>
int launch_transpose(const CopyDesc &d, int t_axis, cudaStream_t stream) {
  long long others = 1;
  for (int a = 0; a + 1 < d.rank; ++a)
    if (a != t_axis) others *= d.shape[a];
  long long gx = (d.shape[d.rank - 1] + TILE - 1) / TILE, gy = (d.shape[t_axis] + TILE - 1) / TILE;
  if (gx > 0x7fffffffll || gy > 65535) return -1;
  long long gz = std::min<long long>(others, 65535);
  dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)gz);
  copy_transpose<W><<<grid, dim3(TILE, 8), 0, stream>>>(d, t_axis, others);
  return check_launch("strided copy (transpose)");
}

// The unit-copy descriptor of a coalesced region: the widest unit, shape
// and strides counted in units.
int units_desc(size_t elem, const Dims &cs, const Dims *cst, const char *s, char *t, CopyDesc &d) {
  const uint32_t r = cs.rank;
  int w = largest_unit(elem, cs, cst, s, t);
  size_t per = size_t(w) / elem;
  for (uint32_t a = 0; a < r; ++a) {
    bool inner = a + 1 == r;
    d.shape[a] = (long long)(inner ? cs.v[a] / per : cs.v[a]);
    d.stride[0][a] = (long long)(inner ? cst[0].v[a] : cst[0].v[a] / per);
    d.stride[1][a] = (long long)(inner ? cst[1].v[a] : cst[1].v[a] / per);
  }
  if (per > 1) {  // contiguous inner run counted in units
    d.stride[0][r - 1] = 1;
    d.stride[1][r - 1] = 1;
  }
  d.count = (long long)(element_count(r, cs.v) / per);
  prepare_division(d);
  return w;
}

// A region that copies as plain units: its width and descriptor.
struct UnitPlan {
  int width;
  CopyDesc desc;
};

// Copy one region: `shape` from (src, from) to (dst, to); both layouts
// already checked.  With `plan`, a region that would run as plain units is
// described there instead of launched (TC_OK); any other region is launched
// and plan->width is set to 0.
int copy_region(size_t elem, uint32_t rank, const size_t *shape, const void *src, size_t from_offset,
                const size_t *from_strides, void *dst, size_t to_offset, const size_t *to_strides,
                cudaStream_t stream, UnitPlan *plan = nullptr) {
  if (plan) plan->width = 0;
  if (element_count(rank, shape) == 0) return TC_OK;
  const size_t *ops[2] = {from_strides, to_strides};
  Dims cs, cst[2];
  coalesce<2>(rank, shape, ops, cs, cst);
  if (cs.rank == 0) {  // one element
    cs.rank = 1;
    cs.v[0] = 1;
    cst[0].rank = cst[1].rank = 1;
    cst[0].v[0] = cst[1].v[0] = 1;
  }
  const char *s = static_cast<const char *>(src) + from_offset * elem;
  char *t = static_cast<char *>(dst) + to_offset * elem;

  CopyDesc d{};
  d.rank = int(cs.rank);
  d.src = s;
  d.dst = t;
  d.offset[0] = d.offset[1] = 0;

  // Transpose path: target inner stride 1, source inner stride not 1, and
  // some outer axis with source stride 1.
  uint32_t r = cs.rank;
  if (r >= 2 && cst[1].v[r - 1] == 1 && cst[0].v[r - 1] != 1 && (elem == 2 || elem == 4 || elem == 8)) {
    int t_axis = -1;
    for (int a = int(r) - 2; a >= 0; --a)
      if (cst[0].v[a] == 1) { t_axis = a; break; }
    if (t_axis >= 0 && cs.v[r - 1] >= 8 && cs.v[t_axis] >= 8) {
      for (uint32_t a = 0; a < r; ++a) {
        d.shape[a] = (long long)cs.v[a];
        d.stride[0][a] = (long long)cst[0].v[a];
        d.stride[1][a] = (long long)cst[1].v[a];
      }
      d.count = (long long)element_count(r, cs.v);
      // 2-byte elements with even extents, strides and base offsets along
      // both tile axes move as 32-bit pairs.
      bool pairs = elem == 2 && cs.v[r - 1] % 2 == 0 && cs.v[t_axis] % 2 == 0 &&
                   cst[0].v[r - 1] % 2 == 0 && cst[1].v[t_axis] % 2 == 0 && (uintptr_t(s) & 3u) == 0 &&
                   (uintptr_t(t) & 3u) == 0;
      for (uint32_t a = 0; pairs && a + 1 < r; ++a)
        if (int(a) != t_axis) pairs = cst[0].v[a] % 2 == 0 && cst[1].v[a] % 2 == 0;
      if (pairs) {
        long long others = 1;
        for (uint32_t a = 0; a + 1 < r; ++a)
          if (int(a) != t_axis) others *= (long long)cs.v[a];
        // 64 x 32 tiles when the t axis is short, else 64 x 64; each
        // block moves 32 KB per batch.
        const bool short_t = cs.v[t_axis] <= 32;
        const long long tt = short_t ? 32 : 64, batch = short_t ? 4 : 2;
        const long long tiles = others * (((long long)cs.v[r - 1] + 63) / 64) * (((long long)cs.v[t_axis] + tt - 1) / tt);
        // One resident wave of persistent blocks.
        static int resident[2] = {0, 0};
        if (!resident[short_t]) {
          int n = 0;
          if (short_t) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, copy_transpose_pairs<32, 4>, 256, 0);
          else cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, copy_transpose_pairs<64, 2>, 256, 0);
          resident[short_t] = std::max(1, n);
        }
        unsigned grid = unsigned(std::max(1LL, std::min<long long>((tiles + batch - 1) / batch,
                                                                   (long long)sm_count() * resident[short_t])));
        if (short_t) copy_transpose_pairs<32, 4><<<grid, 256, 0, stream>>>(d, t_axis, others);
        else copy_transpose_pairs<64, 2><<<grid, 256, 0, stream>>>(d, t_axis, others);
        return check_launch("strided copy (transpose pairs)");
      }
      int st = elem == 2 ? launch_transpose<2>(d, t_axis, stream)
             : elem == 4 ? launch_transpose<4>(d, t_axis, stream)
                         : launch_transpose<8>(d, t_axis, stream);
      if (st >= 0) return st;
    }
  }

  int w = units_desc(elem, cs, cst, s, t, d);
  if (plan) {
    plan->width = w;
    plan->desc = d;
    return TC_OK;
  }
  return launch_width(w, d, stream);
}

bool valid_width(size_t elem) { return elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16; }

// True when every region writes a box of one common target layout and no
// two boxes meet: the same strides, strictly nested (each divides the one
// before), and each region's offset decomposed into coordinates with its
// shape inside every axis's extent.  A concatenation's regions pass.
bool disjoint_boxes(const tc_region *regions, size_t n) {
  const uint32_t rank = regions[0].rank;
  const size_t *st = regions[0].to_strides;
  if (rank == 0) return false;
  for (uint32_t a = 0; a < rank; ++a)
    if (st[a] == 0 || (a && (st[a - 1] <= st[a] || st[a - 1] % st[a]))) return false;
  size_t lo[64][TC_MAX_RANK], hi[64][TC_MAX_RANK];
  for (size_t i = 0; i < n; ++i) {
    const tc_region &r = regions[i];
    if (r.rank != rank) return false;
    for (uint32_t a = 0; a < rank; ++a)
      if (r.to_strides[a] != st[a]) return false;
    size_t off = r.to_offset;
    for (uint32_t a = 0; a < rank; ++a) {
      const size_t c = a ? (off % st[a - 1]) / st[a] : off / st[0];
      if (a && c + r.shape[a] > st[a - 1] / st[a]) return false;  // the box would wrap
      lo[i][a] = c;
      hi[i][a] = c + r.shape[a];
    }
    if (off % st[rank - 1]) return false;
  }
  for (size_t i = 0; i < n; ++i)
    for (size_t j = i + 1; j < n; ++j) {
      bool apart = false;
      for (uint32_t a = 0; a < rank && !apart; ++a) apart = hi[i][a] <= lo[j][a] || hi[j][a] <= lo[i][a];
      if (!apart) return false;
    }
  return true;
}

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" {

int tc_strided_copy(size_t elem, uint32_t rank, const size_t *shape, const void *src, size_t src_len,
                    size_t src_offset, const size_t *src_strides, void *dst, void *stream) {
  if (!valid_width(elem)) return fail(TC_EINVAL, "strided copy: element width %zu", elem);
  if (int st = check_layout("strided copy", src_len, rank, shape, src_offset, src_strides)) return st;
  size_t n = element_count(rank, shape);
  if (n == 0) return TC_OK;
  if (!src || !dst) return fail(TC_EINVAL, "strided copy: null pointer");
  size_t to[TC_MAX_RANK];
  contiguous_strides(rank, shape, to);
  return copy_region(elem, rank, shape, src, src_offset, src_strides, dst, 0, to, as_stream(stream));
}

int tc_strided_write(size_t elem, void *target, size_t target_len, const tc_region *r, void *stream) {
  if (!valid_width(elem)) return fail(TC_EINVAL, "strided write: element width %zu", elem);
  if (!r) return fail(TC_EINVAL, "strided write: null region");
  if (int st = check_layout("strided write source", r->source_len, r->rank, r->shape, r->from_offset,
                            r->from_strides))
    return st;
  if (int st = check_layout("strided write target", target_len, r->rank, r->shape, r->to_offset, r->to_strides))
    return st;
  if (element_count(r->rank, r->shape) == 0) return TC_OK;
  if (!r->source || !target) return fail(TC_EINVAL, "strided write: null pointer");
  return copy_region(elem, r->rank, r->shape, r->source, r->from_offset, r->from_strides, target, r->to_offset,
                     r->to_strides, as_stream(stream));
}

int tc_assemble(size_t elem, void *dst, size_t len, const tc_region *regions, size_t n, void *stream) {
  if (!valid_width(elem)) return fail(TC_EINVAL, "assemble: element width %zu", elem);
  if (n && !regions) return fail(TC_EINVAL, "assemble: null regions");
  for (size_t i = 0; i < n; ++i) {
    const tc_region &r = regions[i];
    if (int st = check_layout("assemble source", r.source_len, r.rank, r.shape, r.from_offset, r.from_strides))
      return st;
    if (int st = check_layout("assemble target", len, r.rank, r.shape, r.to_offset, r.to_strides)) return st;
  }
  // Regions that copy as plain units of one width go out together, up to
  // MAX_BATCH per launch, when their targets are provably disjoint; any
  // other region, and every region when they may overlap, launches on its
  // own in order, so a later region wins where two write one element, as
  // the Host's sequential writes do (backend.rs:303-323).
  const bool batch = n > 1 && n <= 64 && disjoint_boxes(regions, n);
  MultiDesc m{};
  int width = 0;
  auto flush = [&]() -> int {
    if (m.n == 0) return TC_OK;
    const int st = launch_multi_width(width, m, as_stream(stream));
    m.n = 0;
    return st;
  };
  for (size_t i = 0; i < n; ++i) {
    const tc_region &r = regions[i];
    if (element_count(r.rank, r.shape) == 0) continue;
    if (!r.source || !dst) return fail(TC_EINVAL, "assemble: null pointer");
    UnitPlan plan{};
    if (int st = copy_region(elem, r.rank, r.shape, r.source, r.from_offset, r.from_strides, dst, r.to_offset,
                             r.to_strides, as_stream(stream), batch ? &plan : nullptr))
      return st;
    if (!plan.width) continue;  // launched already
    if (m.n == MAX_BATCH || (m.n && plan.width != width))
      if (int st = flush()) return st;
    width = plan.width;
    m.r[m.n] = plan.desc;
    m.start[m.n + 1] = m.start[m.n] + plan.desc.count;
    m.n++;
  }
  return flush();
}

}  // extern "C"
