// runtime.cu — status reporting, devices, the caching device pool, pinned
// host staging and the copy entry points of the C ABI.
#include <cstdarg>
#include <cstdlib>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace tc {

namespace {
thread_local int t_status = TC_OK;
thread_local char t_message[512] = "";
}  // namespace

int fail(int status, const char *fmt, ...) {
  t_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_message, sizeof t_message, fmt, ap);
  va_end(ap);
  return status;
}

int check_cuda(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return TC_OK;
  int status = err == cudaErrorMemoryAllocation ? TC_ENOMEM : TC_ECUDA;
  return fail(status, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

int check_launch(const char *what) { return check_cuda(cudaGetLastError(), what); }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int check_layout(const char *what, size_t len, uint32_t rank, const size_t *shape, size_t offset,
                 const size_t *strides) {
  if (rank > TC_MAX_RANK) return fail(TC_EINVAL, "%s: %u axes, more than %d", what, rank, TC_MAX_RANK);
  if (rank && (!shape || !strides)) return fail(TC_EINVAL, "%s: null shape or strides", what);
  for (uint32_t a = 0; a < rank; ++a)
    if (shape[a] == 0) return TC_OK;
  size_t end = offset;
  for (uint32_t a = 0; a < rank; ++a) {
    size_t span;
    if (__builtin_mul_overflow(shape[a] - 1, strides[a], &span) || __builtin_add_overflow(end, span, &end))
      return fail(TC_ERANGE, "%s: layout arithmetic overflows", what);
  }
  if (end >= len)
    return fail(TC_ERANGE, "%s: layout from offset %zu reaches element %zu, past %zu elements", what, offset,
                end, len);
  return TC_OK;
}

namespace {
struct Scratch {
  std::mutex mu;
  void *ptr[64] = {nullptr};
  size_t bytes[64] = {0};
};
Scratch &scratch_state() {
  static Scratch *s = new Scratch;  // never destroyed
  return *s;
}
}  // namespace

int scratch(size_t bytes, void **out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(TC_EINVAL, "device %d", dev);
  Scratch &s = scratch_state();
  std::lock_guard<std::mutex> g(s.mu);
  if (s.bytes[dev] < bytes) {
    if (s.ptr[dev]) {
      // Queued work may still read the old block: free it once the device
      // is idle.
      cudaDeviceSynchronize();
      cudaFree(s.ptr[dev]);
      s.ptr[dev] = nullptr;
      s.bytes[dev] = 0;
    }
    size_t want = bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes;
    if (int st = check_cuda(cudaMalloc(&s.ptr[dev], want), "cudaMalloc (scratch)")) return st;
    s.bytes[dev] = want;
  }
  *out = s.ptr[dev];
  return TC_OK;
}

namespace {
struct Counters {
  std::mutex mu;
  int *ptr[64] = {nullptr};
  size_t n[64] = {0};
};
Counters &counter_state() {
  static Counters *c = new Counters;  // never destroyed
  return *c;
}
}  // namespace

int counters(size_t n, int **out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(TC_EINVAL, "device %d", dev);
  Counters &c = counter_state();
  std::lock_guard<std::mutex> g(c.mu);
  if (c.n[dev] < n) {
    if (c.ptr[dev]) {
      cudaDeviceSynchronize();
      cudaFree(c.ptr[dev]);
      c.ptr[dev] = nullptr;
      c.n[dev] = 0;
    }
    size_t want = n < 65536 ? 65536 : n;
    if (int st = check_cuda(cudaMalloc(&c.ptr[dev], want * sizeof(int)), "cudaMalloc (counters)")) return st;
    if (int st = check_cuda(cudaMemset(c.ptr[dev], 0, want * sizeof(int)), "cudaMemset (counters)")) return st;
    c.n[dev] = want;
  }
  *out = c.ptr[dev];
  return TC_OK;
}

// ---------------------------------------------------------------------------
// Device pool: freed blocks are kept per (device, size class) and handed to
// the next request of that class, as Metal's buffer pool does
// (src/metal/pool.rs).  Blocks are not stream-ordered: a block freed while a
// kernel on another stream still uses it must not be freed until that work
// is ordered before the next user.
// ---------------------------------------------------------------------------
namespace {
struct Pool {
  std::mutex mu;
  std::map<std::pair<int, size_t>, std::vector<void *>> free_blocks;
  std::unordered_map<void *, std::pair<int, size_t>> live;
};
Pool &pool() {
  static Pool *p = new Pool;  // never destroyed: outlives static destructors
  return *p;
}
size_t size_class(size_t bytes) {
  if (bytes <= 512) return 512;
  if (bytes <= (size_t(1) << 20)) {
    size_t c = 512;
    while (c < bytes) c <<= 1;
    return c;
  }
  const size_t two_mib = size_t(2) << 20;
  return (bytes + two_mib - 1) / two_mib * two_mib;
}
}  // namespace

}  // namespace tc

using namespace tc;

extern "C" {

int tc_last_error(char *buf, size_t len) {
  if (buf && len) {
    strncpy(buf, t_message, len - 1);
    buf[len - 1] = 0;
  }
  return t_status;
}

const char *tc_build_info(void) {
  return "tensorcrate_b200 0.1 sm_100a: strided copy/assemble/write, elementwise, strided binary, "
         "axis reduce, arg reduce, tcgen05 bf16/f16 GEMM and 3xTF32 f32 GEMM with epilogues, gemv, "
         "Adam/SGD, fused programs (statistics, sums, GEMM epilogues), analytic unary and dual, power, "
         "prefix sum, sort, correlation, pad, flip, moments, distributions, NCCL and NVLink peer stores";
}

int tc_set_device(int device) { return check_cuda(cudaSetDevice(device), "cudaSetDevice"); }

int tc_device_count(int *count) {
  if (!count) return fail(TC_EINVAL, "tc_device_count: null");
  return check_cuda(cudaGetDeviceCount(count), "cudaGetDeviceCount");
}

int tc_malloc(void **out, size_t bytes) {
  if (!out) return fail(TC_EINVAL, "tc_malloc: null out");
  *out = nullptr;
  if (bytes == 0) bytes = 1;
  int dev = 0;
  cudaGetDevice(&dev);
  size_t cls = size_class(bytes);
  Pool &p = pool();
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.free_blocks.find({dev, cls});
    if (it != p.free_blocks.end() && !it->second.empty()) {
      *out = it->second.back();
      it->second.pop_back();
      p.live[*out] = {dev, cls};
      return TC_OK;
    }
  }
  void *ptr = nullptr;
  cudaError_t err = cudaMalloc(&ptr, cls);
  if (err == cudaErrorMemoryAllocation) {
    // Give the cached blocks back and try once more.
    cudaGetLastError();
    tc_pool_trim();
    err = cudaMalloc(&ptr, cls);
  }
  if (err != cudaSuccess) return check_cuda(err, "cudaMalloc");
  std::lock_guard<std::mutex> g(p.mu);
  p.live[ptr] = {dev, cls};
  *out = ptr;
  return TC_OK;
}

int tc_free(void *dev_ptr) {
  if (!dev_ptr) return TC_OK;
  Pool &p = pool();
  std::lock_guard<std::mutex> g(p.mu);
  auto it = p.live.find(dev_ptr);
  if (it == p.live.end()) return fail(TC_EINVAL, "tc_free: %p was not allocated by tc_malloc", dev_ptr);
  p.free_blocks[it->second].push_back(dev_ptr);
  p.live.erase(it);
  return TC_OK;
}

int tc_pool_trim(void) {
  Pool &p = pool();
  std::vector<std::pair<int, void *>> blocks;
  {
    std::lock_guard<std::mutex> g(p.mu);
    for (auto &kv : p.free_blocks)
      for (void *b : kv.second) blocks.push_back({kv.first.first, b});
    p.free_blocks.clear();
  }
  int cur = 0;
  cudaGetDevice(&cur);
  for (auto &b : blocks) {
    cudaSetDevice(b.first);
    cudaFree(b.second);
  }
  cudaSetDevice(cur);
  return TC_OK;
}

int tc_host_alloc(void **out, size_t bytes) {
  if (!out) return fail(TC_EINVAL, "tc_host_alloc: null out");
  return check_cuda(cudaMallocHost(out, bytes ? bytes : 1), "cudaMallocHost");
}

int tc_host_free(void *host) { return host ? check_cuda(cudaFreeHost(host), "cudaFreeHost") : TC_OK; }

static int copy(void *dst, const void *src, size_t bytes, cudaMemcpyKind kind, void *stream, bool wait) {
  if (bytes == 0) return TC_OK;
  if (!dst || !src) return fail(TC_EINVAL, "copy: null pointer");
  int st = check_cuda(cudaMemcpyAsync(dst, src, bytes, kind, as_stream(stream)), "cudaMemcpyAsync");
  if (st) return st;
  if (wait) return check_cuda(cudaStreamSynchronize(as_stream(stream)), "cudaStreamSynchronize");
  return TC_OK;
}

int tc_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream) {
  return copy(dst, src, bytes, cudaMemcpyHostToDevice, stream, stream == nullptr);
}
int tc_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream) {
  return copy(dst, src, bytes, cudaMemcpyDeviceToHost, stream, stream == nullptr);
}
int tc_memcpy_d2d(void *dst, const void *src, size_t bytes, void *stream) {
  return copy(dst, src, bytes, cudaMemcpyDeviceToDevice, stream, false);
}
int tc_memset(void *dst, int value, size_t bytes, void *stream) {
  if (bytes == 0) return TC_OK;
  return check_cuda(cudaMemsetAsync(dst, value, bytes, as_stream(stream)), "cudaMemsetAsync");
}
int tc_stream_sync(void *stream) {
  return check_cuda(cudaStreamSynchronize(as_stream(stream)), "cudaStreamSynchronize");
}

int tc_coalesce(uint32_t rank, const size_t *shape, uint32_t n_ops, const size_t *strides,
                uint32_t *out_rank, size_t *out_shape, size_t *out_strides) {
  if (rank > TC_MAX_RANK || n_ops < 1 || n_ops > 3 || !out_rank || !out_shape || !out_strides)
    return fail(TC_EINVAL, "tc_coalesce: bad arguments");
  const size_t *ops[3] = {strides, strides + rank, strides + 2 * rank};
  Dims cs, cst[3];
  if (n_ops == 1) coalesce<1>(rank, shape, ops, cs, cst);
  else if (n_ops == 2) coalesce<2>(rank, shape, ops, cs, cst);
  else coalesce<3>(rank, shape, ops, cs, cst);
  *out_rank = cs.rank;
  for (uint32_t a = 0; a < cs.rank; ++a) out_shape[a] = cs.v[a];
  for (uint32_t o = 0; o < n_ops; ++o)
    for (uint32_t a = 0; a < cs.rank; ++a) out_strides[o * cs.rank + a] = cst[o].v[a];
  return TC_OK;
}

}  // extern "C"
