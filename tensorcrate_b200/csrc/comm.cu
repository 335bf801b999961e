// comm.cu — NCCL over NVLink/NVSwitch for the sharded paths: the all-gather
// of row panels of a product, the all-gather / all-reduce that finish a
// reduction split over the leading axis, and the data-parallel gradient
// all-reduce.  The reference is single-device and has no collectives.
//
// NCCL is loaded at first use with dlopen, so the library carries no link
// dependency on a particular libnccl and shares the copy the process (for
// example torch) already loaded.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace tc {
namespace {

struct Nccl {
  bool ok = false;
  const char *(*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
};

Nccl &nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.error_string = (const char *(*)(ncclResult_t))dlsym(h, "ncclGetErrorString");
    n.get_unique_id = (ncclResult_t(*)(ncclUniqueId *))dlsym(h, "ncclGetUniqueId");
    n.init_rank = (ncclResult_t(*)(ncclComm_t *, int, ncclUniqueId, int))dlsym(h, "ncclCommInitRank");
    n.destroy = (ncclResult_t(*)(ncclComm_t))dlsym(h, "ncclCommDestroy");
    n.abort = (ncclResult_t(*)(ncclComm_t))dlsym(h, "ncclCommAbort");
    n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
    n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
    n.reduce_scatter = (decltype(n.reduce_scatter))dlsym(h, "ncclReduceScatter");
    n.ok = n.error_string && n.get_unique_id && n.init_rank && n.destroy && n.abort && n.all_gather && n.all_reduce &&
           n.reduce_scatter;
  });
  return n;
}

int check_nccl(ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return TC_OK;
  return fail(TC_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

int nccl_type(int dtype, ncclDataType_t *out) {
  switch (dtype) {
    case TC_F32: *out = ncclFloat32; return TC_OK;
    case TC_F16: *out = ncclFloat16; return TC_OK;
    case TC_BF16: *out = ncclBfloat16; return TC_OK;
    case TC_U32: *out = ncclUint32; return TC_OK;
  }
  return fail(TC_EINVAL, "collective: element type %d", dtype);
}

}  // namespace
}  // namespace tc

struct tc_comm {
  ncclComm_t comm;
  int rank, nranks;
};

// One device buffer per rank, every rank holding a mapping of every other
// rank's (CUDA IPC handles exchanged over the communicator), so a kernel can
// store straight into the peers' copies over NVLink.
struct tc_peer_buffer {
  tc_comm *comm;
  size_t bytes;
  void *local;
  void *remote[64];  // remote[r] = rank r's buffer (local for this rank)
  int *token;        // one int on this device: the completion collective's operand
};

namespace tc {
void *peer_buffer_remote(tc_peer_buffer *buf, int rank) {
  return buf && rank >= 0 && rank < buf->comm->nranks ? buf->remote[rank] : nullptr;
}

// Every rank meets: an all-reduce of one int on a private stream, waited for.
int comm_barrier(tc_comm *comm) {
  cudaStream_t s = nullptr;
  if (int st = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return st;
  void *token = nullptr;
  int st = device_malloc(&token, sizeof(int), "cudaMalloc (barrier)");
  if (!st) st = check_cuda(cudaMemsetAsync(token, 0, sizeof(int), s), "cudaMemsetAsync");
  if (!st)
    st = check_nccl(nccl().all_reduce(token, token, 1, ncclInt32, ncclSum, comm->comm, s), "ncclAllReduce (barrier)");
  if (!st) st = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (token) cudaFree(token);
  cudaStreamDestroy(s);
  return st;
}
}  // namespace tc

using namespace tc;

extern "C" {

int tc_comm_unique_id(uint8_t id[128]) {
  if (!nccl().ok) return fail(TC_ENCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  if (int st = check_nccl(nccl().get_unique_id(&u), "ncclGetUniqueId")) return st;
  memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return TC_OK;
}

int tc_comm_init(int rank, int nranks, const uint8_t id[128], tc_comm **out) {
  if (!out || !id || rank < 0 || rank >= nranks) return fail(TC_EINVAL, "tc_comm_init: bad arguments");
  if (!nccl().ok) return fail(TC_ENCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t c;
  if (int st = check_nccl(nccl().init_rank(&c, nranks, u, rank), "ncclCommInitRank")) return st;
  *out = new tc_comm{c, rank, nranks};
  return TC_OK;
}

int tc_comm_destroy(tc_comm *comm) {
  if (!comm) return TC_OK;
  int st = check_nccl(nccl().destroy(comm->comm), "ncclCommDestroy");
  delete comm;
  return st;
}

int tc_allgather(tc_comm *comm, int dtype, const void *send, void *recv, size_t count, void *stream) {
  if (!comm) return fail(TC_EINVAL, "allgather: null communicator");
  ncclDataType_t t = ncclFloat32;
  if (int st = nccl_type(dtype, &t)) return st;
  return check_nccl(nccl().all_gather(send, recv, count, t, comm->comm, as_stream(stream)), "ncclAllGather");
}

int tc_comm_rank(tc_comm *comm, int *rank, int *nranks) {
  if (!comm || !rank || !nranks) return fail(TC_EINVAL, "tc_comm_rank: null");
  *rank = comm->rank;
  *nranks = comm->nranks;
  return TC_OK;
}

int tc_reducescatter(tc_comm *comm, int dtype, const void *send, void *recv, size_t count, int op, void *stream) {
  if (!comm) return fail(TC_EINVAL, "reducescatter: null communicator");
  ncclDataType_t t = ncclFloat32;
  if (int st = nccl_type(dtype, &t)) return st;
  ncclRedOp_t r = op == TC_SUM ? ncclSum : op == TC_RMIN ? ncclMin : op == TC_RMAX ? ncclMax : ncclNumOps;
  if (r == ncclNumOps) return fail(TC_EINVAL, "reducescatter: bad Reduce %d", op);
  return check_nccl(nccl().reduce_scatter(send, recv, count, t, r, comm->comm, as_stream(stream)),
                    "ncclReduceScatter");
}

int tc_allreduce(tc_comm *comm, int dtype, void *buf, size_t count, int op, void *stream) {
  if (!comm) return fail(TC_EINVAL, "allreduce: null communicator");
  ncclDataType_t t = ncclFloat32;
  if (int st = nccl_type(dtype, &t)) return st;
  ncclRedOp_t r = op == TC_SUM ? ncclSum : op == TC_RMIN ? ncclMin : op == TC_RMAX ? ncclMax : ncclNumOps;
  if (r == ncclNumOps) return fail(TC_EINVAL, "allreduce: bad Reduce %d", op);
  return check_nccl(nccl().all_reduce(buf, buf, count, t, r, comm->comm, as_stream(stream)), "ncclAllReduce");
}

// Every rank's `bytes` of scratch meet in `all` (nranks * bytes), in rank
// order, through an all-gather on a private stream.
static int exchange(tc_comm *comm, const void *mine, size_t bytes, void *all) {
  cudaStream_t s = nullptr;
  if (int st = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return st;
  void *dev = nullptr;
  int st = device_malloc(&dev, bytes * size_t(comm->nranks), "cudaMalloc (handle exchange)");
  if (!st) st = check_cuda(cudaMemcpyAsync(static_cast<uint8_t *>(dev) + bytes * comm->rank, mine, bytes,
                                           cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
  if (!st) st = check_nccl(nccl().all_gather(static_cast<uint8_t *>(dev) + bytes * comm->rank, dev, bytes, ncclUint8,
                                             comm->comm, s), "ncclAllGather (handles)");
  if (!st) st = check_cuda(cudaMemcpyAsync(all, dev, bytes * size_t(comm->nranks), cudaMemcpyDeviceToHost, s),
                           "cudaMemcpyAsync");
  if (!st) st = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (dev) cudaFree(dev);
  cudaStreamDestroy(s);
  return st;
}

// A collective that returns on each rank's stream once every rank has
// reached it: an all-reduce of one int.
static int rendezvous(tc_peer_buffer *buf, cudaStream_t stream) {
  return check_nccl(nccl().all_reduce(buf->token, buf->token, 1, ncclInt32, ncclSum, buf->comm->comm, stream),
                    "ncclAllReduce (rendezvous)");
}

int tc_peer_buffer_create(tc_comm *comm, size_t bytes, tc_peer_buffer **out) {
  if (!comm || !out || bytes == 0) return fail(TC_EINVAL, "tc_peer_buffer_create: bad arguments");
  if (comm->nranks > 64) return fail(TC_EINVAL, "tc_peer_buffer_create: %d ranks, at most 64", comm->nranks);
  *out = nullptr;
  auto *buf = new tc_peer_buffer{};
  buf->comm = comm;
  buf->bytes = bytes;
  int st = device_malloc(&buf->local, bytes, "cudaMalloc (peer buffer)");
  if (!st) st = device_malloc(reinterpret_cast<void **>(&buf->token), sizeof(int), "cudaMalloc (peer buffer token)");
  if (!st) st = check_cuda(cudaMemset(buf->token, 0, sizeof(int)), "cudaMemset");
  std::vector<cudaIpcMemHandle_t> handles(size_t(comm->nranks));
  cudaIpcMemHandle_t mine;
  if (!st) st = check_cuda(cudaIpcGetMemHandle(&mine, buf->local), "cudaIpcGetMemHandle");
  if (!st) st = exchange(comm, &mine, sizeof mine, handles.data());
  for (int r = 0; !st && r < comm->nranks; ++r) {
    if (r == comm->rank) {
      buf->remote[r] = buf->local;
      continue;
    }
    st = check_cuda(cudaIpcOpenMemHandle(&buf->remote[r], handles[size_t(r)], cudaIpcMemLazyEnablePeerAccess),
                    "cudaIpcOpenMemHandle");
  }
  if (st) {
    for (int r = 0; r < comm->nranks; ++r)
      if (r != comm->rank && buf->remote[r]) cudaIpcCloseMemHandle(buf->remote[r]);
    if (buf->local) cudaFree(buf->local);
    if (buf->token) cudaFree(buf->token);
    delete buf;
    return st;
  }
  *out = buf;
  return TC_OK;
}

int tc_peer_buffer_pointer(tc_peer_buffer *buf, void **local) {
  if (!buf || !local) return fail(TC_EINVAL, "tc_peer_buffer_pointer: null");
  *local = buf->local;
  return TC_OK;
}

int tc_peer_buffer_destroy(tc_peer_buffer *buf) {
  if (!buf) return TC_OK;
  // No rank may still write into another's buffer, nor hold a mapping of
  // it when it is freed: meet before unmapping and again before freeing.
  int st = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (!st) st = rendezvous(buf, nullptr);
  if (!st) st = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  for (int r = 0; r < buf->comm->nranks; ++r)
    if (r != buf->comm->rank && buf->remote[r]) cudaIpcCloseMemHandle(buf->remote[r]);
  if (!st) st = rendezvous(buf, nullptr);
  if (!st) st = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  cudaFree(buf->local);
  cudaFree(buf->token);
  delete buf;
  return st;
}

int tc_matmul_allgather(tc_comm *comm, int dtype, size_t rows, size_t inner, size_t cols, const void *a,
                        const void *b, tc_peer_buffer *c, void *stream) {
  if (!comm || !c || c->comm != comm) return fail(TC_EINVAL, "matmul_allgather: communicator and buffer differ");
  if (dtype != TC_BF16 && dtype != TC_F16)
    return fail(TC_ENOTSUP, "matmul_allgather: tensor-core element types only (f16, bf16)");
  if (comm->nranks - 1 > 7) return fail(TC_ENOTSUP, "matmul_allgather: at most 8 ranks");
  const size_t need = size_t(comm->nranks) * rows * cols * 2;
  if (need > c->bytes)
    return fail(TC_ERANGE, "matmul_allgather: C needs %zu bytes, the buffer has %zu", need, c->bytes);
  if (rows == 0 || cols == 0) return TC_OK;
  if (!a || !b) return fail(TC_EINVAL, "matmul_allgather: null operand");
  const size_t at = size_t(comm->rank) * rows * cols;  // this rank's panel, in elements
  void *peers[7];
  int n = 0;
  for (int r = 0; r < comm->nranks; ++r)
    if (r != comm->rank) peers[n++] = static_cast<uint16_t *>(c->remote[r]) + at;
  cudaStream_t s = as_stream(stream);
  int st = gemm_tc_run_peers(dtype, TC_TRANS_NONE, rows, inner, cols, a, b, static_cast<uint16_t *>(c->local) + at,
                             false, peers, n, s);
  if (st == TC_ENOTSUP) return fail(TC_ENOTSUP, "matmul_allgather: shape or alignment the tensor-core tiles refuse");
  if (st) return st;
  return rendezvous(c, s);
}

}  // extern "C"
