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

#include "common.cuh"

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
    n.ok = n.error_string && n.get_unique_id && n.init_rank && n.destroy && n.abort && n.all_gather && n.all_reduce;
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

int tc_allreduce(tc_comm *comm, int dtype, void *buf, size_t count, int op, void *stream) {
  if (!comm) return fail(TC_EINVAL, "allreduce: null communicator");
  ncclDataType_t t = ncclFloat32;
  if (int st = nccl_type(dtype, &t)) return st;
  ncclRedOp_t r = op == TC_SUM ? ncclSum : op == TC_RMIN ? ncclMin : op == TC_RMAX ? ncclMax : ncclNumOps;
  if (r == ncclNumOps) return fail(TC_EINVAL, "allreduce: bad Reduce %d", op);
  return check_nccl(nccl().all_reduce(buf, buf, count, t, r, comm->comm, as_stream(stream)), "ncclAllReduce");
}

}  // extern "C"
