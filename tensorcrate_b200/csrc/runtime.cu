// runtime.cu — status reporting, devices, the caching device pool, pinned
// host staging and the copy entry points of the C ABI.
#include <algorithm>
#include <atomic>
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

// ---------------------------------------------------------------------------
// Per-stream scratch and ticket counters.  Every stream (or context) gets
// its own blocks, so calls on different streams of one device, from any
// threads, never share partial results.  A block that has to grow is not
// freed: queued work on its stream, or a caller on another thread that has
// the pointer but has not launched yet, may still use it.  It is retired to
// its stream's list and freed when the stream's context is destroyed
// (tc_ctx_destroy), after the stream is idle.  Growth at least doubles, so
// the retired blocks of a stream add up to less than its current block.
// ---------------------------------------------------------------------------
namespace {
std::atomic<uint64_t> g_device_allocations{0};
std::atomic<uint64_t> g_scratch_requests{0};

struct StreamBlocks {
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  int *counters = nullptr;
  size_t counter_n = 0;
  std::vector<void *> retired;
};
struct StreamState {
  std::mutex mu;
  std::map<std::pair<int, uintptr_t>, StreamBlocks> by_stream;
};
StreamState &stream_state() {
  static StreamState *s = new StreamState;  // never destroyed
  return *s;
}
int current_device(int *dev) {
  if (int st = check_cuda(cudaGetDevice(dev), "cudaGetDevice")) return st;
  if (*dev < 0 || *dev >= 64) return fail(TC_EINVAL, "device %d", *dev);
  return TC_OK;
}
}  // namespace

int device_malloc(void **ptr, size_t bytes, const char *what) {
  g_device_allocations.fetch_add(1, std::memory_order_relaxed);
  return check_cuda(cudaMalloc(ptr, bytes), what);
}

int scratch(size_t bytes, void **out, cudaStream_t stream) {
  g_scratch_requests.fetch_add(1, std::memory_order_relaxed);
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  StreamState &s = stream_state();
  std::lock_guard<std::mutex> g(s.mu);
  StreamBlocks &b = s.by_stream[{dev, reinterpret_cast<uintptr_t>(stream)}];
  if (b.scratch_bytes < bytes) {
    size_t want = std::max(bytes, std::max(size_t(1) << 20, 2 * b.scratch_bytes));
    void *fresh = nullptr;
    if (int st = device_malloc(&fresh, want, "cudaMalloc (scratch)")) return st;
    if (b.scratch) b.retired.push_back(b.scratch);
    b.scratch = fresh;
    b.scratch_bytes = want;
  }
  *out = b.scratch;
  return TC_OK;
}

int counters(size_t n, int **out, cudaStream_t stream) {
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  StreamState &s = stream_state();
  std::lock_guard<std::mutex> g(s.mu);
  StreamBlocks &b = s.by_stream[{dev, reinterpret_cast<uintptr_t>(stream)}];
  if (b.counter_n < n) {
    size_t want = std::max(n, std::max(size_t(65536), 2 * b.counter_n));
    void *fresh = nullptr;
    if (int st = device_malloc(&fresh, want * sizeof(int), "cudaMalloc (counters)")) return st;
    // Zero before any kernel of this stream takes a ticket from them.
    if (int st = check_cuda(cudaMemsetAsync(fresh, 0, want * sizeof(int), stream), "cudaMemsetAsync (counters)")) {
      cudaFree(fresh);
      return st;
    }
    if (b.counters) b.retired.push_back(b.counters);
    b.counters = static_cast<int *>(fresh);
    b.counter_n = want;
  }
  *out = b.counters;
  return TC_OK;
}

namespace {
// Free a stream's blocks; the caller has made the stream idle.
void release_stream_blocks(int dev, cudaStream_t stream) {
  StreamState &s = stream_state();
  StreamBlocks b;
  {
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.by_stream.find({dev, reinterpret_cast<uintptr_t>(stream)});
    if (it == s.by_stream.end()) return;
    b = std::move(it->second);
    s.by_stream.erase(it);
  }
  if (b.scratch) cudaFree(b.scratch);
  if (b.counters) cudaFree(b.counters);
  for (void *p : b.retired) cudaFree(p);
}

// ---------------------------------------------------------------------------
// Device pool: freed blocks are kept per (device, size class) and handed to
// the next request of that class, as Metal's buffer pool does
// (src/metal/pool.rs).  tc_free makes a block reusable at once (the caller
// says no queued work uses it); tc_free_async records an event on the
// stream whose work last uses the block, and the block goes to a request
// only in that stream's order: at once to a request on the same stream,
// after the event has completed to tc_malloc, and to tc_malloc_async on
// another stream with that stream made to wait for the event.
// ---------------------------------------------------------------------------
struct FreeBlock {
  void *ptr;
  uintptr_t stream;  // the stream it was freed on (tc_free_async)
  cudaEvent_t done;  // recorded there; null: no queued work uses the block
};
struct Pool {
  std::mutex mu;
  std::map<std::pair<int, size_t>, std::vector<FreeBlock>> free_blocks;
  std::unordered_map<void *, std::pair<int, size_t>> live;
  std::vector<cudaEvent_t> spare_events;
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

// A cached block of class `cls` on `dev` that a request may take (with the
// pool's lock held).  `stream` is the requesting stream, or has_stream false
// for tc_malloc.  On success the block is live and, when it was freed on
// another stream with work still queued, `stream` waits for that work.
bool take_cached(Pool &p, int dev, size_t cls, bool has_stream, cudaStream_t stream, void **out) {
  auto it = p.free_blocks.find({dev, cls});
  if (it == p.free_blocks.end() || it->second.empty()) return false;
  auto &v = it->second;
  const uintptr_t key = reinterpret_cast<uintptr_t>(stream);
  int pick = -1;
  bool wait = false;
  for (int pass = 0; pass < 3 && pick < 0; ++pass) {
    for (int i = int(v.size()) - 1; i >= 0 && pick < 0; --i) {
      const FreeBlock &f = v[size_t(i)];
      if (pass == 0) {
        if (!f.done || (has_stream && f.stream == key)) pick = i;
      } else if (pass == 1) {
        if (cudaEventQuery(f.done) == cudaSuccess) pick = i;
        else cudaGetLastError();  // cudaErrorNotReady is not a failure
      } else if (has_stream) {
        pick = i;
        wait = true;
      }
    }
  }
  if (pick < 0) return false;
  FreeBlock f = v[size_t(pick)];
  v.erase(v.begin() + pick);
  if (wait && cudaStreamWaitEvent(stream, f.done, 0) != cudaSuccess) {
    cudaGetLastError();
    cudaEventSynchronize(f.done);
  }
  if (f.done) p.spare_events.push_back(f.done);
  p.live[f.ptr] = {dev, cls};
  *out = f.ptr;
  return true;
}

int pool_malloc(void **out, size_t bytes, bool has_stream, cudaStream_t stream) {
  if (!out) return fail(TC_EINVAL, "tc_malloc: null out");
  *out = nullptr;
  if (bytes == 0) bytes = 1;
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  size_t cls = size_class(bytes);
  Pool &p = pool();
  {
    std::lock_guard<std::mutex> g(p.mu);
    if (take_cached(p, dev, cls, has_stream, stream, out)) return TC_OK;
  }
  void *ptr = nullptr;
  g_device_allocations.fetch_add(1, std::memory_order_relaxed);
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

int pool_free(void *dev_ptr, bool has_stream, cudaStream_t stream) {
  if (!dev_ptr) return TC_OK;
  Pool &p = pool();
  std::lock_guard<std::mutex> g(p.mu);
  auto it = p.live.find(dev_ptr);
  if (it == p.live.end()) return fail(TC_EINVAL, "tc_free: %p was not allocated by tc_malloc", dev_ptr);
  FreeBlock f{dev_ptr, reinterpret_cast<uintptr_t>(stream), nullptr};
  if (has_stream) {
    if (!p.spare_events.empty()) {
      f.done = p.spare_events.back();
      p.spare_events.pop_back();
    } else if (int st = check_cuda(cudaEventCreateWithFlags(&f.done, cudaEventDisableTiming), "cudaEventCreate")) {
      return st;
    }
    if (int st = check_cuda(cudaEventRecord(f.done, stream), "cudaEventRecord")) {
      p.spare_events.push_back(f.done);
      return st;
    }
  }
  p.free_blocks[it->second].push_back(f);
  p.live.erase(it);
  return TC_OK;
}

// After `stream` is idle: its freed blocks need no more ordering.
void settle_stream_blocks(int dev, cudaStream_t stream) {
  Pool &p = pool();
  std::lock_guard<std::mutex> g(p.mu);
  const uintptr_t key = reinterpret_cast<uintptr_t>(stream);
  for (auto &kv : p.free_blocks) {
    if (kv.first.first != dev) continue;
    for (FreeBlock &f : kv.second)
      if (f.done && f.stream == key) {
        p.spare_events.push_back(f.done);
        f.done = nullptr;
      }
  }
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

int tc_sm_count(int *count) {
  if (!count) return fail(TC_EINVAL, "tc_sm_count: null");
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  *count = sm_count();
  return TC_OK;
}

int tc_malloc(void **out, size_t bytes) { return pool_malloc(out, bytes, false, nullptr); }
int tc_malloc_async(void **out, size_t bytes, void *stream) { return pool_malloc(out, bytes, true, as_stream(stream)); }
int tc_free(void *dev_ptr) { return pool_free(dev_ptr, false, nullptr); }
int tc_free_async(void *dev_ptr, void *stream) { return pool_free(dev_ptr, true, as_stream(stream)); }

int tc_pool_trim(void) {
  Pool &p = pool();
  std::vector<std::pair<int, FreeBlock>> blocks;
  {
    std::lock_guard<std::mutex> g(p.mu);
    for (auto &kv : p.free_blocks)
      for (FreeBlock &b : kv.second) blocks.push_back({kv.first.first, b});
    p.free_blocks.clear();
  }
  int cur = 0;
  cudaGetDevice(&cur);
  for (auto &b : blocks) {
    cudaSetDevice(b.first);
    if (b.second.done) {
      cudaEventSynchronize(b.second.done);
      cudaEventDestroy(b.second.done);
    }
    cudaFree(b.second.ptr);
  }
  cudaSetDevice(cur);
  return TC_OK;
}

int tc_alloc_counts(uint64_t *device_allocations, uint64_t *scratch_requests) {
  if (device_allocations) *device_allocations = g_device_allocations.load();
  if (scratch_requests) *scratch_requests = g_scratch_requests.load();
  return TC_OK;
}

}  // extern "C"

// A device and a stream of its own, owned by one thread at a time: the
// CUDA counterpart of Metal's per-thread device and command queue.  Its
// stream keys its scratch, ticket counters and stream-ordered pool frees.
struct tc_ctx {
  int device;
  cudaStream_t stream;
};

extern "C" {

int tc_ctx_create(int device, tc_ctx **out) {
  if (!out) return fail(TC_EINVAL, "tc_ctx_create: null out");
  *out = nullptr;
  if (int st = check_cuda(cudaSetDevice(device), "cudaSetDevice")) return st;
  cudaStream_t s = nullptr;
  if (int st = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return st;
  *out = new tc_ctx{device, s};
  return TC_OK;
}

int tc_ctx_stream(tc_ctx *ctx, void **stream) {
  if (!ctx || !stream) return fail(TC_EINVAL, "tc_ctx_stream: null");
  *stream = ctx->stream;
  return TC_OK;
}

int tc_ctx_device(tc_ctx *ctx, int *device) {
  if (!ctx || !device) return fail(TC_EINVAL, "tc_ctx_device: null");
  *device = ctx->device;
  return TC_OK;
}

int tc_ctx_destroy(tc_ctx *ctx) {
  if (!ctx) return TC_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(ctx->device);
  int st = check_cuda(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  settle_stream_blocks(ctx->device, ctx->stream);
  release_stream_blocks(ctx->device, ctx->stream);
  if (!st) st = check_cuda(cudaStreamDestroy(ctx->stream), "cudaStreamDestroy");
  cudaSetDevice(cur);
  delete ctx;
  return st;
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
