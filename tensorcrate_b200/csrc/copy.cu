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
};

template <int W> struct Unit;
template <> struct Unit<1> { using T = uint8_t; };
template <> struct Unit<2> { using T = uint16_t; };
template <> struct Unit<4> { using T = uint32_t; };
template <> struct Unit<8> { using T = uint2; };
template <> struct Unit<16> { using T = uint4; };

// Copy `d.count` units of W bytes: flat row-major index -> both positions.
// Shapes, strides and offsets are in units.
template <int W, typename Index>
__global__ void __launch_bounds__(256) copy_units(const CopyDesc d) {
  using U = typename Unit<W>::T;
  const U *src = reinterpret_cast<const U *>(d.src);
  U *dst = reinterpret_cast<U *>(d.dst);
  Index stride = Index(gridDim.x) * blockDim.x;
  const int rank = d.rank;
  Index inner = Index(d.shape[rank - 1]);
  Index s_in = Index(d.stride[0][rank - 1]), t_in = Index(d.stride[1][rank - 1]);
  for (Index i = Index(blockIdx.x) * blockDim.x + threadIdx.x; i < Index(d.count); i += stride) {
    Index rest = i / inner;
    Index c = i - rest * inner;
    Index s = Index(d.offset[0]) + c * s_in, t = Index(d.offset[1]) + c * t_in;
    for (int a = rank - 2; a >= 0; --a) {
      Index e = Index(d.shape[a]);
      Index q = rest / e;
      Index ca = rest - q * e;
      rest = q;
      s += ca * Index(d.stride[0][a]);
      t += ca * Index(d.stride[1][a]);
    }
    dst[t] = __ldg(src + s);
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


// Tiled transpose for 2-byte elements, 64 x 64 tiles moved as 32-bit pairs:
// a warp reads 64 source-contiguous elements (128 bytes) of one inner
// index, and writes 64 target-contiguous elements of one t index.  Needs
// even extents, strides and offsets along both axes.  A persistent grid
// walks (other axes, inner tile, t tile).
__global__ void __launch_bounds__(256) copy_transpose_pairs(const CopyDesc d, int t_axis, long long others) {
  __shared__ uint16_t tile[64][66];  // [inner][t]
  const uint16_t *src = reinterpret_cast<const uint16_t *>(d.src);
  uint16_t *dst = reinterpret_cast<uint16_t *>(d.dst);
  const int rank = d.rank;
  const long long n_in = d.shape[rank - 1], n_t = d.shape[t_axis];
  const long long tiles_i = (n_in + 63) / 64, tiles_t = (n_t + 63) / 64;
  const long long total = others * tiles_i * tiles_t;
  const long long s_in = d.stride[0][rank - 1], d_t = d.stride[1][t_axis];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long w = blockIdx.x; w < total; w += gridDim.x) {
    long long o = w / (tiles_i * tiles_t);
    const long long rem = w - o * tiles_i * tiles_t;
    const long long i0 = (rem / tiles_t) * 64, t0 = (rem % tiles_t) * 64;
    long long s = d.offset[0], t = d.offset[1];
    for (int a = rank - 2; a >= 0; --a) {
      if (a == t_axis) continue;
      const long long e = d.shape[a], c = o % e;
      o /= e;
      s += c * d.stride[0][a];
      t += c * d.stride[1][a];
    }
    // read: warp rows = inner indices, lanes = pairs along t
    const long long tp = t0 + 2 * lane;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = warp + 8 * k;
      if (i0 + i < n_in && tp < n_t) {
        const uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(src + s + (i0 + i) * s_in + tp));
        tile[i][2 * lane] = uint16_t(v & 0xffffu);
        tile[i][2 * lane + 1] = uint16_t(v >> 16);
      }
    }
    __syncthreads();
    // write: warp rows = t indices, lanes = pairs along inner
    const long long ip = i0 + 2 * lane;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = warp + 8 * k;
      if (t0 + j < n_t && ip < n_in) {
        const uint32_t v = uint32_t(tile[2 * lane][j]) | (uint32_t(tile[2 * lane + 1][j]) << 16);
        *reinterpret_cast<uint32_t *>(dst + t + (t0 + j) * d_t + ip) = v;
      }
    }
    __syncthreads();
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

template <int W>
int launch_units(const CopyDesc &d, cudaStream_t stream) {
  unsigned block = 256;
  unsigned grid = grid_for(size_t(d.count), block, 16);
  if (d.count < (1ll << 31)) copy_units<W, int><<<grid, block, 0, stream>>>(d);
  else copy_units<W, long long><<<grid, block, 0, stream>>>(d);
  return check_launch("strided copy");
}

int launch_width(int w, const CopyDesc &d, cudaStream_t stream) {
  switch (w) {
    case 1: return launch_units<1>(d, stream);
    case 2: return launch_units<2>(d, stream);
    case 4: return launch_units<4>(d, stream);
    case 8: return launch_units<8>(d, stream);
    case 16: return launch_units<16>(d, stream);
  }
  return fail(TC_EINVAL, "strided copy: element width %d", w);
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

// Copy one region: `shape` from (src, from) to (dst, to); both layouts
// already checked.
int copy_region(size_t elem, uint32_t rank, const size_t *shape, const void *src, size_t from_offset,
                const size_t *from_strides, void *dst, size_t to_offset, const size_t *to_strides,
                cudaStream_t stream) {
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
        const long long tiles = others * (((long long)cs.v[r - 1] + 63) / 64) * (((long long)cs.v[t_axis] + 63) / 64);
        unsigned grid = unsigned(std::min<long long>(tiles, (long long)sm_count() * 8));
        copy_transpose_pairs<<<std::max(1u, grid), 256, 0, stream>>>(d, t_axis, others);
        return check_launch("strided copy (transpose pairs)");
      }
      int st = elem == 2 ? launch_transpose<2>(d, t_axis, stream)
             : elem == 4 ? launch_transpose<4>(d, t_axis, stream)
                         : launch_transpose<8>(d, t_axis, stream);
      if (st >= 0) return st;
    }
  }

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
  return launch_width(w, d, stream);
}

bool valid_width(size_t elem) { return elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16; }

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
  for (size_t i = 0; i < n; ++i) {
    const tc_region &r = regions[i];
    if (element_count(r.rank, r.shape) == 0) continue;
    if (!r.source || !dst) return fail(TC_EINVAL, "assemble: null pointer");
    if (int st = copy_region(elem, r.rank, r.shape, r.source, r.from_offset, r.from_strides, dst, r.to_offset,
                             r.to_strides, as_stream(stream)))
      return st;
  }
  return TC_OK;
}

}  // extern "C"
