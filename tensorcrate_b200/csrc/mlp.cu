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
// loss scaled by the global batch, and the parameter gradients are summed
// with NCCL before Adam.  The reduction of each layer's gradients starts, on
// a second stream, as soon as the backward pass has produced them.
#include <cmath>
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
  // Every layer's gradients in one allocation, [gW_l | gb_l] side by side
  // (each 16-byte aligned, the gap zeroed), so that one all-reduce moves a
  // layer's gradients: gW[l].p and gb[l].p point into it.
  Buf grads;
  std::vector<size_t> layer_span;  // elements from gW[l].p to the end of gb[l]
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> grad_ready;
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
    need(m->W[l], outd * in); need(m->mW[l], outd * in); need(m->vW[l], outd * in);
    need(m->b[l], outd); need(m->mb[l], outd); need(m->vb[l], outd);
    need(m->A[l], outd * B);
    if (l + 1 < m->layers) need(m->H[l], outd * B);
  }
  {
    const size_t align = 16 / e;  // elements per 16 bytes
    auto up = [&](size_t n) { return (n + align - 1) / align * align; };
    size_t total = 0;
    std::vector<size_t> at_w(layers), at_b(layers);
    for (uint32_t l = 0; l < layers; ++l) {
      at_w[l] = total;
      total += up(m->dims[l + 1] * m->dims[l]);
      at_b[l] = total;
      total += up(m->dims[l + 1]);
    }
    need(m->grads, total);
    if (!st) st = check_cuda(cudaMemset(m->grads.p, 0, total * e), "cudaMemset");
    m->layer_span.resize(layers);
    for (uint32_t l = 0; l < layers && !st; ++l) {
      m->gW[l].p = static_cast<char *>(m->grads.p) + at_w[l] * e;
      m->gW[l].n = m->dims[l + 1] * m->dims[l];
      m->gb[l].p = static_cast<char *>(m->grads.p) + at_b[l] * e;
      m->gb[l].n = m->dims[l + 1];
      m->layer_span[l] = at_b[l] + m->dims[l + 1] - at_w[l];
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
  m->abar_ready.resize(m->layers);
  m->side_done.resize(m->layers);
  for (auto *evs : {&m->grad_ready, &m->abar_ready, &m->side_done})
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
  for (auto *v : {&m->W, &m->b, &m->mW, &m->vW, &m->mb, &m->vb, &m->A, &m->H})
    for (auto &b : *v) drop(b);
  drop(m->grads);  // gW and gb point into it
  for (Buf *b : {&m->ones, &m->S, &m->Rbar, &m->Ybar, &m->Xbar, &m->abar,
                 &m->inbar, &m->onesbar, &m->ovec, &m->loss_sum})
    drop(*b);
  for (auto *evs : {&m->grad_ready, &m->abar_ready, &m->side_done})
    for (auto ev : *evs)
      if (ev) cudaEventDestroy(ev);
  if (m->reduced) cudaEventDestroy(m->reduced);
  if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
  if (m->side) cudaStreamDestroy(m->side);
  delete m;
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

// Skip the adjoints nothing reads (inputs', targets', the ones vector's).
// Off by default: the tape computes them.
int tc_mlp_prune_leaves(tc_mlp *m, int prune) {
  if (!m) return fail(TC_EINVAL, "mlp: null");
  m->prune = prune != 0;
  return TC_OK;
}

int tc_allreduce(tc_comm *comm, int dtype, void *buf, size_t count, int op, void *stream);

// One step: forward, loss (into loss_out, one element, if not null),
// backward, optional gradient all-reduce over `comm`, Adam.  x: [dims[0] x
// batch], y: [dims[L] x batch], both device buffers, column per sample.
int tc_mlp_step(tc_mlp *m, const void *x, const void *y, tc_comm *comm, void *loss_out, void *stream_v) {
  if (!m || !x || !y) return fail(TC_EINVAL, "mlp_step: null argument");
  cudaStream_t s = as_stream(stream_v);
  const int d = m->dtype, L = m->layers;
  const size_t B = m->batch;
  void *st = stream_v;
#define TRY(call)                   \
  do {                              \
    if (int rc_ = (call)) return rc_; \
  } while (0)
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
  // With a communicator, the gradient all-reduces run beside the backward
  // products: leave them SMs (the products' CTAs fill an SM's shared memory).
  struct Reserve {
    explicit Reserve(bool on) { gemm_reserve_sms(on ? 16 : 0); }
    ~Reserve() { gemm_reserve_sms(0); }
  } reserve(comm != nullptr);
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
  const void *abar = m->Rbar.p;  // Ā of the top layer = P̄
  for (int l = L - 1; l >= 0; --l) {
    const size_t in = m->dims[l], outd = m->dims[l + 1];
    const void *input = l == 0 ? x : m->H[l - 1].p;
    // A = Z + O: Z̄ = Ō = Ā (shared).  O = b ⊗ ones: b̄ += Ō·ones,
    // ones̄ += bᵀ·Ō (vecmat), accumulated in node order.  These read Ā
    // only, so they run on the side stream while the products below run
    // here; the side stream's vecmat keeps its partial sums in the static
    // array of tc_vecmat_noalloc (the per-device scratch belongs to this
    // stream's split-K products), and a shape too large for it runs here.
    TRY(check_cuda(cudaEventRecord(m->abar_ready[l], s), "event"));
    TRY(check_cuda(cudaStreamWaitEvent(m->side, m->abar_ready[l], 0), "wait"));
    TRY(tc_matvec(d, outd, B, abar, m->ones.p, m->gb[l].p, 0, m->side));
    if (!m->prune) {
      void *dst = l == L - 1 ? m->onesbar.p : m->ovec.p;
      int vst = tc_vecmat_noalloc(d, outd, B, m->b[l].p, abar, dst, m->side);
      if (vst == TC_ERANGE) {
        // Too large for the static array: join, and run it on this stream.
        TRY(check_cuda(cudaEventRecord(m->side_done[l], m->side), "event"));
        TRY(check_cuda(cudaStreamWaitEvent(s, m->side_done[l], 0), "wait"));
        TRY(tc_vecmat(d, outd, B, m->b[l].p, abar, dst, st));
        TRY(check_cuda(cudaEventRecord(m->abar_ready[l], s), "event"));
        TRY(check_cuda(cudaStreamWaitEvent(m->side, m->abar_ready[l], 0), "wait"));
      } else if (vst) {
        return vst;
      }
      if (l != L - 1) TRY(tc_elementwise(d, TC_ADD, m->onesbar.p, m->ovec.p, m->onesbar.p, B, m->side));
    }
    TRY(check_cuda(cudaEventRecord(m->side_done[l], m->side), "event"));
    // Z = W·IN: W̄ += Z̄·INᵀ, ĪN += Wᵀ·Z̄ (matmul_transposed_add, both
    // adjoints starting from zero).
    TRY(tc_matmul(d, TC_TRANS_RIGHT, outd, B, in, abar, input, m->gW[l].p, 0, st));
    if (comm) {
      TRY(check_cuda(cudaEventRecord(m->grad_ready[l], s), "event"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->grad_ready[l], 0), "wait"));
      TRY(check_cuda(cudaStreamWaitEvent(m->comm_stream, m->side_done[l], 0), "wait"));
      // the layer's weight and bias gradients in one call
      TRY(tc_allreduce(comm, d, m->gW[l].p, m->layer_span[l], TC_SUM, m->comm_stream));
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
  }
  // Every side-stream result (b̄, ones̄) is complete before Adam and the
  // caller see them.
  TRY(check_cuda(cudaStreamWaitEvent(s, m->side_done[0], 0), "wait"));
  if (comm) {
    TRY(check_cuda(cudaEventRecord(m->reduced, m->comm_stream), "event"));
    TRY(check_cuda(cudaStreamWaitEvent(s, m->reduced, 0), "wait"));
  }
  // ---- Adam, per parameter in the order the driver updates them ----
  m->steps += 1;
  float c1, c2;
  adam_coefficients(*m, m->steps, c1, c2);
  const int resumed = m->steps > 1;
  std::vector<tc_adam_tensor> params;
  for (int l = 0; l < L; ++l) {
    params.push_back({m->W[l].p, m->gW[l].p, m->mW[l].p, m->vW[l].p, m->W[l].n});
    params.push_back({m->b[l].p, m->gb[l].p, m->mb[l].p, m->vb[l].p, m->b[l].n});
  }
  TRY(tc_adam_multi(d, params.data(), params.size(), resumed, m->rate, m->beta1, m->beta2, m->eps, c1, c2, st));
#undef TRY
  return TC_OK;
}

}  // extern "C"
