// mlp.cu — one training step of a dense ReLU network as tensorcrate's
// reverse-mode tape runs it, replayed through this backend's kernels, and
// the Adam rule's update of every parameter (config 4 of the benchmark).
//
// The network is the one benches/nn_ops.rs:877-921 builds, with any number
// of layers: for each layer l
//     Z = W_l · IN            (MatrixVar::matmul, tape/mod.rs:1195)
//     O = b_l ⊗ ones          (VectorVar::outer, tape/mod.rs:979-988)
//     A = Z + O               (MatrixVar binary Add, tape/mod.rs:1026-1033)
//     H = relu(A)             (select_scalar Max, tape/mod.rs:1110-1130)
// the last layer without the ReLU, then R = P - Y, S = R * R and the loss
// sum(S) · 1/(outputs·batch) (frobenius_dot + scale, tape/mod.rs:1299,
// 1174).  The backward pass visits the nodes in reverse order of creation
// and applies each node's rule with the same Kernels<T> calls and operand
// order the tape uses; copies the tape makes (`duplicate`) are elided where
// a buffer can be shared, which cannot change a value.  Every leaf's adjoint
// is computed, as the tape computes it, including the inputs', targets' and
// the ones vector's.
//
// Under data parallelism each rank runs the step on its own batch with the
// loss scaled by the global batch, so the sum of the ranks' gradients is the
// gradient of the whole batch.  Each layer's gradients are exchanged on a
// second stream as soon as the backward pass has produced them.  With 2-8
// ranks the optimizer is sharded (ZeRO stage 1 style): the layer's
// gradient block is reduce-scattered, each rank runs Adam on its 1/P of the
// block, and the updated parameters are all-gathered, so the Adam pass
// shrinks with P and the collectives move the same bytes an all-reduce
// would.  With more ranks the gradients are all-reduced and every rank runs
// the whole Adam pass.
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

struct tc_comm;

namespace tc {
namespace {

struct Buf {
  void *p = nullptr;
  size_t n = 0;
};

// Matrix::filled: every element `value` (rounded to the element type on
// the host).
template <class T>
__global__ void fill_kernel(typename T::S *out, size_t n, typename T::S value) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = value;
}

// The loss and its first backward steps, one pass over the outputs:
//   R = P - Y, S = R * R                       (binary Sub, Mul)
//   S̄ = filled(factor); R̄ = S̄ * R + S̄ * R      (Mul's rule, both operands R)
//   Ȳ = R̄ * -1                                 (Sub's rule for the right side)
// each operation rounded to T as the separate kernels round it.  S is
// written only when the loss is wanted, Ȳ only when not pruned.
template <class T>
__global__ void __launch_bounds__(256) mse_backward(const typename T::S *pred, const typename T::S *y, float factor,
                                                   typename T::S *s_out, typename T::S *rbar, typename T::S *ybar,
                                                   size_t n) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const float r = T::load(T::store(__fsub_rn(T::load(pred[i]), T::load(y[i]))));
    if (s_out) s_out[i] = T::store(__fmul_rn(r, r));
    const float t = T::load(T::store(__fmul_rn(factor, r)));
    const typename T::S rb = T::store(__fadd_rn(t, t));
    rbar[i] = rb;
    if (ybar) ybar[i] = T::store(__fmul_rn(T::load(rb), -1.0f));
  }
}

// ---------------------------------------------------------------------------
// Flags between the ranks of a data-parallel step over NVLink peer memory.
// Each rank holds, in memory every rank maps, one u32 per (rank, layer) for
// "ready" (that rank's gradients of the layer are final and it reads the
// layer's parameters no more this step) and one for "written" (that rank
// has stored its shard of the layer's updated parameters into every rank's
// copy).  A flag holds the number of the last step it announced.  Waits are
// bounded: on expiry the kernel records the fault (tc_device_status) and
// returns.
// ---------------------------------------------------------------------------
__device__ int g_peer_fault = 0;
constexpr unsigned long long PEER_WAIT_NS = 5000000000ull;  // 5 s by default
std::atomic<unsigned long long> g_peer_wait_ns{PEER_WAIT_NS};

struct FlagSlots {
  uint32_t *slot[8];
  int n;
};

// Announce `value` in every slot (one per rank), ordered after everything
// this stream did before (the exchange kernel's stores to the ranks among
// it).
__global__ void signal_slots(FlagSlots s, uint32_t value) {
  const int i = threadIdx.x;
  __threadfence_system();
  if (i < s.n) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(s.slot[i]), "r"(value) : "memory");
}

// Wait until flags[first + k*stride] >= value for k = 0..count-1, lane k of
// the warp watching flag k (count <= 32 * blocks).
__global__ void wait_slots(const uint32_t *flags, int first, int stride, int count, uint32_t value,
                           unsigned long long limit_ns) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= count) return;
  const uint32_t *f = flags + first + size_t(k) * size_t(stride);
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t i = 0; i < (1u << 30); ++i) {
    uint32_t seen;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(f) : "memory");
    if (seen >= value) return;
    if ((i & 255u) == 255u) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > limit_ns) break;
      __nanosleep(200);
    }
  }
  atomicExch(&g_peer_fault, 1);
}

// Round a host value to the element type, as Real::from_f64 does (one
// rounding from f64; round-to-odd into f32 first keeps it single).
float round_to(int dtype, double d) {
  float f = float(d);
  if (dtype == TC_F32) return f;
  if (std::isfinite(d) && double(f) != d && std::isfinite(f)) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if (std::fabs(double(f)) > std::fabs(d)) u -= 1;
    u |= 1u;
    memcpy(&f, &u, 4);
  }
  return dtype == TC_BF16 ? bf16_bits_to_f32(f32_to_bf16_bits(f)) : f16_bits_to_f32(f32_to_f16_bits(f));
}
float round_f32(int dtype, float f) {
  if (dtype == TC_F32) return f;
  return dtype == TC_BF16 ? bf16_bits_to_f32(f32_to_bf16_bits(f)) : f16_bits_to_f32(f32_to_f16_bits(f));
}
// f32 powi by square-and-multiply, the loop compiler-rt's __powisf2 runs
// (what Rust's f32::powi lowers to); f16/bf16 powi is f32 powi, rounded.
float powi(float a, int b) {
  bool recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

}  // namespace
}  // namespace tc

using namespace tc;

struct tc_mlp {
  int dtype = TC_BF16;
  size_t esz = 2;
  int layers = 0;
  std::vector<size_t> dims;  // dims[0] inputs ... dims[layers] outputs
  size_t batch = 0, global_batch = 0;
  float rate = 0, beta1 = 0, beta2 = 0, eps = 0;  // element-type values
  uint32_t steps = 0;
  std::vector<Buf> W, b, gW, gb, mW, vW, mb, vb;
  std::vector<Buf> A, H;
  Buf ones, S, Rbar, Ybar, Xbar, abar, inbar, onesbar, ovec, loss_sum;
  // Parameters, their gradients and Adam's two moments each in one flat
  // allocation with the same layout: layer l's block starts at element
  // block_at[l] and holds [W_l | b_l] (b_l 16-byte aligned, gaps zero),
  // padded to block_len[l], a multiple of SHARD_UNIT elements.  W[l], b[l],
  // gW[l], ... point into them.  One collective moves a layer's block, and
  // every rank count P <= 8 cuts a block into P equal, 16-byte-aligned
  // shards.
  Buf params, grads, mom1, mom2;
  std::vector<size_t> block_at, block_len;
  size_t total = 0;
  cudaStream_t comm_stream = nullptr;
  // After tc_mlp_attach: the communicator whose steps exchange over NVLink
  // peer memory, and the buffers every rank maps: the flat parameters and
  // gradients, and the flags.
  tc_comm *attached = nullptr;
  int rank = 0, nranks = 1;
  tc_peer_buffer *peer_params = nullptr, *peer_grads = nullptr, *peer_flags = nullptr;
  std::vector<cudaEvent_t> grad_ready, params_free;
  cudaEvent_t reduced = nullptr;
  // The bias adjoints (matvec, vecmat: memory-bound) run on a side stream,
  // beside each layer's products.
  cudaStream_t side = nullptr;
  std::vector<cudaEvent_t> abar_ready, side_done;
  bool prune = false;
};

namespace {

int alloc(Buf &b, size_t n, size_t esz) {
  b.n = n;
  return tc_malloc(&b.p, std::max<size_t>(n * esz, 16));
}

// 840 = lcm(1, ..., 8): a block of a multiple of 840 16-byte groups splits
// into P equal shards of whole groups for every P <= 8.
constexpr size_t SHARD_UNIT_GROUPS = 840;
constexpr int MAX_SHARDS = 8;

// Adam::update's host arithmetic (optim.rs:1106-1124) in the element type.
void adam_coefficients(const tc_mlp &m, uint32_t step, float &c1, float &c2) {
  const int d = m.dtype;
  float f1 = round_f32(d, 1.0f - round_f32(d, powi(m.beta1, int(step))));
  float f2 = round_f32(d, 1.0f - round_f32(d, powi(m.beta2, int(step))));
  c1 = round_f32(d, 1.0f / f1);
  c2 = round_f32(d, 1.0f / f2);
}

}  // namespace

extern "C" {

int tc_mlp_create(int dtype, uint32_t layers, const uint32_t *dims, uint32_t batch, uint32_t global_batch,
                  double rate, double beta1, double beta2, double eps, tc_mlp **out) {
  if (!out || !dims || layers == 0 || batch == 0) return fail(TC_EINVAL, "mlp_create: bad arguments");
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16) return fail(TC_EINVAL, "mlp_create: dtype");
  tc_mlp *m = new tc_mlp;
  m->dtype = dtype;
  m->esz = dtype_bytes(dtype);
  m->layers = int(layers);
  m->dims.assign(dims, dims + layers + 1);
  m->batch = batch;
  m->global_batch = global_batch ? global_batch : batch;
  m->rate = round_to(dtype, rate);
  m->beta1 = round_to(dtype, beta1);
  m->beta2 = round_to(dtype, beta2);
  m->eps = round_to(dtype, eps);
  const size_t B = batch, e = m->esz;
  int st = TC_OK;
  auto need = [&](Buf &x, size_t n) {
    if (!st) st = alloc(x, n, e);
  };
  for (int l = 0; l < m->layers; ++l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    m->W.emplace_back(); m->b.emplace_back(); m->gW.emplace_back(); m->gb.emplace_back();
    m->mW.emplace_back(); m->vW.emplace_back(); m->mb.emplace_back(); m->vb.emplace_back();
    m->A.emplace_back(); m->H.emplace_back();
    need(m->A[l], outd * B);
    if (l + 1 < m->layers) need(m->H[l], outd * B);
  }
  {
    const size_t group = 16 / e;  // elements per 16 bytes
    const size_t unit = SHARD_UNIT_GROUPS * group;
    auto up = [](size_t n, size_t to) { return (n + to - 1) / to * to; };
    size_t total = 0;
    std::vector<size_t> at_b(layers);
    m->block_at.resize(layers);
    m->block_len.resize(layers);
    for (uint32_t l = 0; l < layers; ++l) {
      const size_t nw = size_t(m->dims[l + 1]) * m->dims[l], nb = m->dims[l + 1];
      m->block_at[l] = total;
      at_b[l] = total + up(nw, group);
      m->block_len[l] = up(up(nw, group) + nb, unit);
      total += m->block_len[l];
    }
    m->total = total;
    need(m->params, total); need(m->grads, total); need(m->mom1, total); need(m->mom2, total);
    for (Buf *f : {&m->params, &m->grads, &m->mom1, &m->mom2})
      if (!st) st = check_cuda(cudaMemset(f->p, 0, total * e), "cudaMemset");
    for (uint32_t l = 0; l < layers && !st; ++l) {
      const size_t nw = size_t(m->dims[l + 1]) * m->dims[l], nb = m->dims[l + 1];
      auto at = [&](Buf &f, size_t off, size_t n) {
        Buf v;
        v.p = static_cast<char *>(f.p) + off * e;
        v.n = n;
        return v;
      };
      m->W[l] = at(m->params, m->block_at[l], nw); m->b[l] = at(m->params, at_b[l], nb);
      m->gW[l] = at(m->grads, m->block_at[l], nw); m->gb[l] = at(m->grads, at_b[l], nb);
      m->mW[l] = at(m->mom1, m->block_at[l], nw); m->mb[l] = at(m->mom1, at_b[l], nb);
      m->vW[l] = at(m->mom2, m->block_at[l], nw); m->vb[l] = at(m->mom2, at_b[l], nb);
    }
  }
  size_t widest = 0;
  for (size_t d : m->dims) widest = std::max(widest, d);
  const size_t last = m->dims[m->layers];
  need(m->ones, B); need(m->S, last * B);
  need(m->Rbar, last * B); need(m->Ybar, last * B); need(m->Xbar, m->dims[0] * B);
  need(m->abar, widest * B); need(m->inbar, widest * B);
  need(m->onesbar, B); need(m->ovec, B); need(m->loss_sum, 1);
  if (st) {
    tc_mlp_destroy(m);
    return st;
  }
  // ones: the tape's constant vector of the batch's length
  int rc = with_real(dtype, [&](auto t) {
    using T = decltype(t);
    fill_kernel<T><<<grid_for(B, 256), 256>>>(static_cast<typename T::S *>(m->ones.p), B, T::store(1.0f));
    return check_launch("mlp ones");
  });
  if (rc || (rc = check_cuda(cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking), "stream")) ||
      (rc = check_cuda(cudaEventCreateWithFlags(&m->reduced, cudaEventDisableTiming), "event"))) {
    tc_mlp_destroy(m);
    return rc;
  }
  if ((rc = check_cuda(cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking), "stream"))) {
    tc_mlp_destroy(m);
    return rc;
  }
  m->grad_ready.resize(m->layers);
  m->params_free.resize(m->layers);
  m->abar_ready.resize(m->layers);
  m->side_done.resize(m->layers);
  for (auto *evs : {&m->grad_ready, &m->params_free, &m->abar_ready, &m->side_done})
    for (auto &ev : *evs)
      if ((rc = check_cuda(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event"))) {
        tc_mlp_destroy(m);
        return rc;
      }
  *out = m;
  return TC_OK;
}

int tc_mlp_destroy(tc_mlp *m) {
  if (!m) return TC_OK;
  cudaDeviceSynchronize();
  auto drop = [](Buf &b) {
    if (b.p) tc_free(b.p);
    b.p = nullptr;
  };
  for (auto *v : {&m->A, &m->H})
    for (auto &b : *v) drop(b);
  // W, b, their gradients and moments point into these (the parameters and
  // gradients into peer buffers once attached: collective to free)
  if (m->attached) {
    m->params.p = m->grads.p = nullptr;
    for (tc_peer_buffer *pb : {m->peer_params, m->peer_grads, m->peer_flags}) tc_peer_buffer_destroy(pb);
  }
  for (Buf *f : {&m->params, &m->grads, &m->mom1, &m->mom2}) drop(*f);
  for (Buf *b : {&m->ones, &m->S, &m->Rbar, &m->Ybar, &m->Xbar, &m->abar,
                 &m->inbar, &m->onesbar, &m->ovec, &m->loss_sum})
    drop(*b);
  for (auto *evs : {&m->grad_ready, &m->params_free, &m->abar_ready, &m->side_done})
    for (auto ev : *evs)
      if (ev) cudaEventDestroy(ev);
  if (m->reduced) cudaEventDestroy(m->reduced);
  if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
  if (m->side) cudaStreamDestroy(m->side);
  delete m;
  return TC_OK;
}

// Move the flat parameters and gradients into buffers every rank of `comm`
// maps (CUDA IPC over NVLink), so that data-parallel steps over `comm`
// exchange them with peer loads and stores (see tc_mlp_step).  Collective.
int tc_mlp_attach(tc_mlp *m, tc_comm *comm) {
  if (!m || !comm) return fail(TC_EINVAL, "mlp_attach: null argument");
  if (m->attached) return fail(TC_EINVAL, "mlp_attach: already attached");
  int rank = 0, nranks = 1;
  if (int st = tc_comm_rank(comm, &rank, &nranks)) return st;
  if (nranks > MAX_SHARDS) return fail(TC_ENOTSUP, "mlp_attach: %d ranks, at most %d", nranks, MAX_SHARDS);
  const size_t bytes = m->total * m->esz, flag_bytes = size_t(2) * size_t(nranks) * size_t(m->layers) * 4;
  tc_peer_buffer *pp = nullptr, *pg = nullptr, *pf = nullptr;
  int st = tc_peer_buffer_create(comm, bytes, &pp);
  if (!st) st = tc_peer_buffer_create(comm, bytes, &pg);
  if (!st) st = tc_peer_buffer_create(comm, flag_bytes, &pf);
  void *np = peer_buffer_remote(pp, rank), *ng = peer_buffer_remote(pg, rank), *nf = peer_buffer_remote(pf, rank);
  if (!st) st = check_cuda(cudaMemcpy(np, m->params.p, bytes, cudaMemcpyDeviceToDevice), "cudaMemcpy");
  if (!st) st = check_cuda(cudaMemset(ng, 0, bytes), "cudaMemset");
  if (!st) st = check_cuda(cudaMemset(nf, 0, flag_bytes), "cudaMemset");
  if (!st) st = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  // No rank signals into another's flags before every rank has zeroed them.
  if (!st) st = comm_barrier(comm);
  if (st) {
    for (tc_peer_buffer *b : {pp, pg, pf}) tc_peer_buffer_destroy(b);
    return st;
  }
  auto move = [&](Buf &flat, void *to, std::vector<Buf> &w, std::vector<Buf> &b) {
    for (int l = 0; l < m->layers; ++l) {
      w[l].p = static_cast<char *>(to) + (static_cast<char *>(w[l].p) - static_cast<char *>(flat.p));
      b[l].p = static_cast<char *>(to) + (static_cast<char *>(b[l].p) - static_cast<char *>(flat.p));
    }
    tc_free(flat.p);
    flat.p = to;
  };
  move(m->params, np, m->W, m->b);
  move(m->grads, ng, m->gW, m->gb);
  m->attached = comm;
  m->rank = rank;
  m->nranks = nranks;
  m->peer_params = pp;
  m->peer_grads = pg;
  m->peer_flags = pf;
  return TC_OK;
}

// Upload (dir = 0) or download (dir = 1) layer `l`'s weight [dims[l+1] x
// dims[l]] and bias [dims[l+1]], in the element type's storage form.
int tc_mlp_params(tc_mlp *m, uint32_t l, void *w_host, void *b_host, int dir) {
  if (!m || int(l) >= m->layers) return fail(TC_EINVAL, "mlp_params: layer %u", l);
  const size_t wb = m->W[l].n * m->esz, bb = m->b[l].n * m->esz;
  if (dir == 0) {
    if (w_host) if (int st = tc_memcpy_h2d(m->W[l].p, w_host, wb, nullptr)) return st;
    if (b_host) if (int st = tc_memcpy_h2d(m->b[l].p, b_host, bb, nullptr)) return st;
    return TC_OK;
  }
  if (w_host) if (int st = tc_memcpy_d2h(w_host, m->W[l].p, wb, nullptr)) return st;
  if (b_host) if (int st = tc_memcpy_d2h(b_host, m->b[l].p, bb, nullptr)) return st;
  return TC_OK;
}

// Download layer `l`'s gradients (after a step): dW and db.
int tc_mlp_grads(tc_mlp *m, uint32_t l, void *gw_host, void *gb_host) {
  if (!m || int(l) >= m->layers) return fail(TC_EINVAL, "mlp_grads: layer %u", l);
  if (gw_host) if (int st = tc_memcpy_d2h(gw_host, m->gW[l].p, m->gW[l].n * m->esz, nullptr)) return st;
  if (gb_host) if (int st = tc_memcpy_d2h(gb_host, m->gb[l].p, m->gb[l].n * m->esz, nullptr)) return st;
  return TC_OK;
}

// Where layer `l`'s parameters sit in its block of the flat buffers: the
// block's length in elements (a multiple of every rank count up to 8 times
// 16 bytes) and the element at which b_l starts (W_l starts at 0).  Rank r
// of P owns elements [r*len/P, (r+1)*len/P) of every block in a sharded
// step.
int tc_mlp_block(tc_mlp *m, uint32_t l, size_t *len, size_t *bias_at) {
  if (!m || int(l) >= m->layers || !len || !bias_at) return fail(TC_EINVAL, "mlp_block: layer %u", l);
  *len = m->block_len[l];
  *bias_at = size_t(static_cast<char *>(m->b[l].p) - static_cast<char *>(m->W[l].p)) / m->esz;
  return TC_OK;
}

// Skip the adjoints nothing reads (inputs', targets', the ones vector's).
// Off by default: the tape computes them.
int tc_mlp_prune_leaves(tc_mlp *m, int prune) {
  if (!m) return fail(TC_EINVAL, "mlp: null");
  m->prune = prune != 0;
  return TC_OK;
}

int tc_allreduce(tc_comm *comm, int dtype, void *buf, size_t count, int op, void *stream);
int tc_allgather(tc_comm *comm, int dtype, const void *send, void *recv, size_t count, void *stream);
int tc_reducescatter(tc_comm *comm, int dtype, const void *send, void *recv, size_t count, int op, void *stream);
int tc_comm_rank(tc_comm *comm, int *rank, int *nranks);

// One step: forward, loss (into loss_out, one element, if not null),
// backward, optional gradient exchange over `comm`, Adam.  x: [dims[0] x
// batch], y: [dims[L] x batch], both device buffers, column per sample.
int tc_mlp_step(tc_mlp *m, const void *x, const void *y, tc_comm *comm, void *loss_out, void *stream_v) {
  if (!m || !x || !y) return fail(TC_EINVAL, "mlp_step: null argument");
  cudaStream_t s = as_stream(stream_v);
  const int d = m->dtype, L = m->layers;
  const size_t B = m->batch, e = m->esz;
  void *st = stream_v;
#define TRY(call)                   \
  do {                              \
    if (int rc_ = (call)) return rc_; \
  } while (0)
  int rank = 0, nranks = 1;
  if (comm) TRY(tc_comm_rank(comm, &rank, &nranks));
  if (nranks == 1) comm = nullptr;
  // With 2-8 ranks the optimizer is sharded: every rank updates its own
  // shard of each layer's block with the gradient summed over the ranks, and
  // every rank receives every shard's new parameters.  Attached to `comm`
  // (tc_mlp_attach), one kernel per layer does all of it over NVLink peer
  // memory; otherwise NCCL reduce-scatters the gradients and all-gathers the
  // parameters around a local Adam.  More ranks all-reduce the gradients and
  // run Adam on everything.
  const bool sharded = comm && nranks <= MAX_SHARDS;
  const bool peers = sharded && comm == m->attached;
  // On one GPU each layer's Adam runs on the second stream as soon as the
  // backward pass is done with the layer, beside the products of the layers
  // below it (Adam is bound by memory, the products by the tensor cores).
  const bool layered = !comm;
  // Adam's coefficients for this step (Adam::update, optim.rs:1106-1124).
  m->steps += 1;
  float c1, c2;
  adam_coefficients(*m, m->steps, c1, c2);
  const int resumed = m->steps > 1;
  auto adam_range = [&](size_t at, size_t n, cudaStream_t on) {
    char *p = static_cast<char *>(m->params.p), *g = static_cast<char *>(m->grads.p);
    char *m1 = static_cast<char *>(m->mom1.p), *m2 = static_cast<char *>(m->mom2.p);
    return tc_adam(d, n, p + at * e, g + at * e, m1 + at * e, m2 + at * e, resumed, m->rate, m->beta1, m->beta2,
                   m->eps, c1, c2, on);
  };
  // ---- forward ----
  for (int l = 0; l < L; ++l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    const void *input = l == 0 ? x : m->H[l - 1].p;
    // Z = W·IN, O = b ⊗ ones, A = Z + O, H = max(A, 0): one product whose
    // epilogue adds the bias row and applies the ReLU, rounding as the
    // separate operations do (b ⊗ ones is b exactly).
    TRY(tc_matmul_epilogue(d, TC_TRANS_NONE, outd, in, B, m->W[l].p, input, nullptr, m->b[l].p, m->A[l].p,
                           l + 1 < L ? m->H[l].p : nullptr, st));
  }
  const size_t last = m->dims[L];
  const float factor = round_to(d, 1.0 / (double(last) * double(m->global_batch)));
  // The second stream's work (collectives, exchanges, Adam) runs beside
  // the backward products: leave it SMs (the products' CTAs fill an SM's
  // shared memory).
  struct Reserve {
    explicit Reserve(bool on) { gemm_reserve_sms(on ? 16 : 0); }
    ~Reserve() { gemm_reserve_sms(0); }
  } reserve(comm != nullptr || layered);
  // Loss and the top of the backward pass (frobenius_dot, scale, sum's and
  // Mul's and Sub's rules) in one pass.
  TRY(with_real(d, [&](auto t) {
    using T = decltype(t);
    using S = typename T::S;
    mse_backward<T><<<grid_for(last * B, 256), 256, 0, s>>>(
        static_cast<const S *>(m->A[L - 1].p), static_cast<const S *>(y), factor,
        loss_out ? static_cast<S *>(m->S.p) : nullptr, static_cast<S *>(m->Rbar.p),
        m->prune ? nullptr : static_cast<S *>(m->Ybar.p), last * B);
    return check_launch("mlp loss");
  }));
  if (loss_out) {
    // The lazy scalar, forced: sum of S (f32, rounded once), then `scale`.
    TRY(tc_vector_reduce(d, TC_SUM, m->S.p, last * B, m->loss_sum.p, st));
    TRY(tc_broadcast_scalar(d, TC_MUL, m->loss_sum.p, factor, 0, loss_out, 1, st));
  }
  // The exchange of layer l over peer memory.
  auto exchange_layer = [&](int l) -> int {
    // This rank's gradients of the layer are final and nothing of this
    // step reads W_l or b_l any more (params_free[l]; the side stream's
    // vecmat read b_l before side_done[l]): say so to every rank, wait until
    // every rank has, then one kernel sums this rank's shard of the layer's
    // block over the ranks (peer loads), updates it and stores it into every
    // rank's parameters (peer stores); then say that.
    cudaStream_t c = m->comm_stream;
    TRY(check_cuda(cudaStreamWaitEvent(c, m->params_free[l], 0), "wait"));
    TRY(check_cuda(cudaStreamWaitEvent(c, m->side_done[l], 0), "wait"));
    const size_t count = m->block_len[l] / size_t(nranks);
    FlagSlots ready{}, written{};
    ready.n = written.n = nranks;
    PeerAdam x{};
    x.nranks = nranks;
    x.rank = rank;
    for (int q = 0; q < nranks; ++q) {
      uint32_t *fl = static_cast<uint32_t *>(peer_buffer_remote(m->peer_flags, q));
      ready.slot[q] = fl + size_t(rank) * L + l;
      written.slot[q] = fl + size_t(nranks) * L + size_t(rank) * L + l;
      x.grads[q] = static_cast<char *>(peer_buffer_remote(m->peer_grads, q)) + m->block_at[l] * e;
      x.params[q] = static_cast<char *>(peer_buffer_remote(m->peer_params, q)) + m->block_at[l] * e;
    }
    const uint32_t *mine = static_cast<const uint32_t *>(peer_buffer_remote(m->peer_flags, rank));
    signal_slots<<<1, 32, 0, c>>>(ready, m->steps);
    wait_slots<<<1, 32, 0, c>>>(mine, l, L, nranks, m->steps, g_peer_wait_ns.load());
    TRY(check_launch("mlp flags"));
    x.m = static_cast<char *>(m->mom1.p) + m->block_at[l] * e;
    x.v = static_cast<char *>(m->mom2.p) + m->block_at[l] * e;
    x.first = size_t(rank) * count;
    x.count = count;
    TRY(peer_adam_run(d, x, resumed, m->rate, m->beta1, m->beta2, m->eps, c1, c2, c));
    signal_slots<<<1, 32, 0, c>>>(written, m->steps);
    TRY(check_launch("mlp flags"));
    return TC_OK;
  };
  const void *abar = m->Rbar.p;  // Ā of the top layer = P̄
  for (int l = L - 1; l >= 0; --l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    const void *input = l == 0 ? x : m->H[l - 1].p;
    // A = Z + O: Z̄ = Ō = Ā (shared).  O = b ⊗ ones: b̄ += Ō·ones,
    // ones̄ += bᵀ·Ō (vecmat), accumulated in node order.  These read Ā
    // only, so they run on the side stream while the products below run
    // here; the side stream's calls keep their partial sums in that
    // stream's own scratch.
    TRY(check_cuda(cudaEventRecord(m->abar_ready[l], s), "event"));
    TRY(check_cuda(cudaStreamWaitEvent(m->side, m->abar_ready[l], 0), "wait"));
    TRY(tc_matvec(d, outd, B, abar, m->ones.p, m->gb[l].p, 0, m->side));
    if (!m->prune) {
      void *dst = l == L - 1 ? m->onesbar.p : m->ovec.p;
      TRY(tc_vecmat(d, outd, B, m->b[l].p, abar, dst, m->side));
      if (l != L - 1) TRY(tc_elementwise(d, TC_ADD, m->onesbar.p, m->ovec.p, m->onesbar.p, B, m->side));
    }
    TRY(check_cuda(cudaEventRecord(m->side_done[l], m->side), "event"));
    // Z = W·IN: W̄ += Z̄·INᵀ, ĪN += Wᵀ·Z̄ (matmul_transposed_add, both
    // adjoints starting from zero).
    TRY(tc_matmul(d, TC_TRANS_RIGHT, outd, B, in, abar, input, m->gW[l].p, 0, st));
    if (comm && !peers) {
      TRY(check_cuda(cudaEventRecord(m->grad_ready[l], s), "event"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->grad_ready[l], 0), "wait"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->side_done[l], 0), "wait"));
      char *block = static_cast<char *>(m->grads.p) + m->block_at[l] * e;
      if (sharded) {
        // The layer's summed gradient, rank r's shard only.
        const size_t count = m->block_len[l] / size_t(nranks);
        TRY(tc_reducescatter(comm, d, block, block + size_t(rank) * count * e, count, TC_SUM, m->comm_stream));
      } else {
        TRY(tc_allreduce(comm, d, block, m->block_len[l], TC_SUM, m->comm_stream));
      }
    }
    if (l > 0) {
      // H̄ = Wᵀ·Z̄, then H = relu(A): Ā += H̄ · MaxShare(A, 0).  Ā of the
      // layer below goes to the buffer this layer's Ā does not use, which
      // the layer above's side work read: wait for that first.
      void *next = abar == m->abar.p ? m->inbar.p : m->abar.p;
      if (l + 1 < L) TRY(check_cuda(cudaStreamWaitEvent(s, m->side_done[l + 1], 0), "wait"));
      TRY(tc_matmul_epilogue(d, TC_TRANS_LEFT, in, outd, B, m->W[l].p, abar, m->A[l - 1].p, nullptr, next,
                             nullptr, st));
      abar = next;
    } else if (!m->prune) {
      TRY(tc_matmul(d, TC_TRANS_LEFT, in, outd, B, m->W[l].p, abar, m->Xbar.p, 0, st));
    }
    if (peers) {
      TRY(check_cuda(cudaEventRecord(m->params_free[l], s), "event"));
      TRY(exchange_layer(l));
    } else if (sharded) {
      // Nothing of this step reads W_l or b_l any more (the side stream's
      // vecmat read b_l before side_done[l]): update this rank's shard of
      // the layer and gather every rank's.
      TRY(check_cuda(cudaEventRecord(m->params_free[l], s), "event"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->params_free[l], 0), "wait"));
      const size_t count = m->block_len[l] / size_t(nranks);
      const size_t mine = m->block_at[l] + size_t(rank) * count;
      TRY(adam_range(mine, count, m->comm_stream));
      char *block = static_cast<char *>(m->params.p) + m->block_at[l] * e;
      TRY(tc_allgather(comm, d, block + size_t(rank) * count * e, block, count, m->comm_stream));
    } else if (layered) {
      TRY(check_cuda(cudaEventRecord(m->params_free[l], s), "event"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->params_free[l], 0), "wait"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->side_done[l], 0), "wait"));
      TRY(adam_range(m->block_at[l], m->block_len[l], m->comm_stream));
    }
  }
  // Every side-stream result (b̄, ones̄) is complete before Adam and the
  // caller see them.
  TRY(check_cuda(cudaStreamWaitEvent(s, m->side_done[0], 0), "wait"));
  if (comm || layered) {
    TRY(check_cuda(cudaEventRecord(m->reduced, m->comm_stream), "event"));
    TRY(check_cuda(cudaStreamWaitEvent(s, m->reduced, 0), "wait"));
  }
  if (peers) {
    // Every rank has stored its shards of every layer into this rank's
    // parameters (and read this rank's gradients) before anything after
    // the step on this stream runs.
    const uint32_t *mine_flags = static_cast<const uint32_t *>(peer_buffer_remote(m->peer_flags, rank));
    const int count = nranks * L;
    wait_slots<<<(count + 31) / 32, 32, 0, s>>>(mine_flags, nranks * L, 1, count, m->steps, g_peer_wait_ns.load());
    TRY(check_launch("mlp flags"));
  }
  // ---- Adam over every parameter (one launch over the flat blocks; the
  // padding between tensors is zero and is read by nothing) ----
  if (!sharded && !layered) TRY(adam_range(0, m->total, s));
#undef TRY
  return TC_OK;
}

}  // extern "C"

namespace tc {
// Whether a wait between ranks gave up since the library loaded (or the
// last reset).
int peer_wait_fault() {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, g_peer_fault, sizeof(int)) != cudaSuccess) return 0;
  return h;
}
void set_peer_wait_limit(unsigned long long ns) { g_peer_wait_ns.store(ns ? ns : PEER_WAIT_NS); }
int peer_wait_fault_reset() {
  const int zero = 0;
  return check_cuda(cudaMemcpyToSymbol(g_peer_fault, &zero, sizeof(int)), "cudaMemcpyToSymbol");
}
}  // namespace tc
