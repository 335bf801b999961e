// tape.cu — a reverse-mode tape over device tensors, run natively: the
// tensor-level rules of tensorcrate's tape (src/tensors/tape/tensor.rs and
// the MatrixVar rules of src/tensors/tape/mod.rs) recorded in creation order
// and replayed backwards through this backend's kernels.  The reference
// drives these rules from Rust above the Kernels<T> boundary; this is the
// same walk for callers with no Rust toolchain (and the general runner
// behind config 4's fixed network, whose tc_mlp_* replays one shape).
//
// Semantics kept from the reference:
//   - a backward pass first clears every adjoint, seeds the output with one,
//     and visits the nodes up to the output in reverse order of creation
//     (backward_with, tape/mod.rs:507-521); a node no contribution reached
//     has no adjoint (None) and propagates nothing;
//   - `accumulate` keeps the first contribution as the adjoint and adds
//     later ones elementwise (tape/mod.rs:316-322);
//   - binary Add/Sub/Mul/Div broadcast their operands and sum each
//     contribution to its operand's shape (sum_to_shape, tape/tensor.rs:23-37,
//     128-160); relu is select_scalar(Max, 0) with the MaxShare weight
//     (tape/tensor.rs:272-300); scale, sum_axes and mean_axes as
//     tape/tensor.rs:317-323, 581-620; matmul as MatrixVar::matmul
//     (tape/mod.rs:1190-1216: Ā += C̄·Bᵀ, B̄ += Aᵀ·C̄, accumulated into the
//     current adjoint or zeros); sum as MatrixVar::sum (tape/mod.rs:1286-1296,
//     the adjoint filled with the output's adjoint).
#include <vector>

#include "common.cuh"

namespace {

enum Kind { LEAF, BINARY, RELU, SCALE, SUM_AXES, MATMUL, SUM };

struct Node {
  Kind kind = LEAF;
  std::vector<size_t> shape;
  void *value = nullptr;
  bool owned = false;
  void *adjoint = nullptr;  // owned; null: no contribution reached the node
  int op = 0;
  uint32_t a = 0, b = 0;
  std::vector<uint32_t> axes;
  bool mean = false;
  double factor = 0;  // scale's factor, mean's share (values of the element type)
};

size_t count_of(const std::vector<size_t> &shape) {
  size_t n = 1;
  for (size_t e : shape) n *= e;
  return n;
}

}  // namespace

struct tc_tape {
  int dtype = TC_F32;
  size_t esz = 4;
  cudaStream_t stream = nullptr;
  std::vector<Node> nodes;
};

using namespace tc;

namespace {

#define TRY(call)                     \
  do {                                \
    if (int rc_ = (call)) return rc_; \
  } while (0)

int alloc(tc_tape *t, size_t n, void **out) { return tc_malloc_async(out, std::max<size_t>(n * t->esz, 16), t->stream); }
void release(tc_tape *t, void *p) {
  if (p) tc_free_async(p, t->stream);
}

int push(tc_tape *t, Node &&n, uint32_t *out) {
  if (!out) return fail(TC_EINVAL, "tape: null output var");
  *out = uint32_t(t->nodes.size());
  t->nodes.push_back(std::move(n));
  return TC_OK;
}

int check_var(tc_tape *t, uint32_t v) {
  if (!t) return fail(TC_EINVAL, "tape: null tape");
  if (v >= t->nodes.size()) return fail(TC_EINVAL, "tape: no var %u", v);
  return TC_OK;
}

// layout.rs:330-345 broadcast_shape: right-aligned, extents equal or one.
bool broadcast_shape(const std::vector<size_t> &x, const std::vector<size_t> &y, std::vector<size_t> &out) {
  const size_t r = std::max(x.size(), y.size());
  out.assign(r, 1);
  for (size_t i = 0; i < r; ++i) {
    const size_t ex = i < r - x.size() ? 1 : x[i - (r - x.size())];
    const size_t ey = i < r - y.size() ? 1 : y[i - (r - y.size())];
    if (ex != ey && ex != 1 && ey != 1) return false;
    out[i] = std::max(ex, ey);
  }
  return true;
}

// The strides of a row-major `shape` read as `target` (right-aligned): zero
// along broadcast and added axes (layout.rs:347-363 broadcast_strides).
std::vector<size_t> broadcast_strides(const std::vector<size_t> &shape, const std::vector<size_t> &target) {
  std::vector<size_t> own(shape.size());
  contiguous_strides(uint32_t(shape.size()), shape.data(), own.data());
  std::vector<size_t> out(target.size(), 0);
  const size_t added = target.size() - shape.size();
  for (size_t i = added; i < target.size(); ++i)
    out[i] = shape[i - added] == 1 && target[i] != 1 ? 0 : own[i - added];
  return out;
}

// out (shape `to`, fresh) = x op y, each read broadcast to `to`.
int binary_into(tc_tape *t, int op, const void *x, const std::vector<size_t> &xs, const void *y,
                const std::vector<size_t> &ys, const std::vector<size_t> &to, void *out) {
  const auto xst = broadcast_strides(xs, to), yst = broadcast_strides(ys, to);
  return tc_strided_binary(t->dtype, TC_PAIR_ARITHMETIC, op, uint32_t(to.size()), to.data(), x, count_of(xs), 0,
                           xst.data(), y, count_of(ys), 0, yst.data(), out, t->stream);
}

// A fresh contiguous copy of x (shape `xs`) read broadcast to `to`.
int spread(tc_tape *t, const void *x, const std::vector<size_t> &xs, const std::vector<size_t> &to, void **out) {
  TRY(alloc(t, count_of(to), out));
  const auto st = broadcast_strides(xs, to);
  return tc_strided_copy(t->esz, uint32_t(to.size()), to.data(), x, count_of(xs), 0, st.data(), *out, t->stream);
}

// tape/tensor.rs:23-37 sum_to_shape: g (shape gs) summed over the axes that
// `shape` adds or holds at one, kept, then read as `shape`; a fresh buffer.
int sum_to_shape(tc_tape *t, const void *g, const std::vector<size_t> &gs, const std::vector<size_t> &shape,
                 void **out) {
  TRY(alloc(t, count_of(shape), out));
  if (gs == shape) return tc_memcpy_d2d(*out, g, count_of(gs) * t->esz, t->stream);
  const size_t added = gs.size() - shape.size();
  std::vector<uint32_t> axes;
  for (size_t a = 0; a < gs.size(); ++a)
    if (a < added || (shape[a - added] == 1 && gs[a] != 1)) axes.push_back(uint32_t(a));
  std::vector<size_t> st(gs.size());
  contiguous_strides(uint32_t(gs.size()), gs.data(), st.data());
  if (axes.empty()) return tc_memcpy_d2d(*out, g, count_of(gs) * t->esz, t->stream);
  return tc_reduce_axes(t->dtype, uint32_t(gs.size()), gs.data(), g, count_of(gs), 0, st.data(), uint32_t(axes.size()),
                        axes.data(), TC_AXIS_FOLD, TC_SUM, 0, *out, t->stream);
}

// tape/mod.rs:316-322: the first contribution becomes the adjoint, later
// ones are added to it.  Takes ownership of `delta`.
int accumulate(tc_tape *t, Node &n, void *delta) {
  if (!n.adjoint) {
    n.adjoint = delta;
    return TC_OK;
  }
  int st = tc_elementwise(t->dtype, TC_ADD, n.adjoint, delta, n.adjoint, count_of(n.shape), t->stream);
  release(t, delta);
  return st;
}

int scaled(tc_tape *t, const void *x, size_t n, double factor, void **out) {
  TRY(alloc(t, n, out));
  return tc_broadcast_scalar(t->dtype, TC_MUL, x, factor, 0, *out, n, t->stream);
}

// The adjoint to accumulate into by an accumulating product: the current
// one, or zeros (current_or_zeros, tape/mod.rs:326-331).
int current_or_zeros(tc_tape *t, Node &n) {
  if (n.adjoint) return TC_OK;
  TRY(alloc(t, count_of(n.shape), &n.adjoint));
  return tc_memset(n.adjoint, 0, count_of(n.shape) * t->esz, t->stream);
}

int propagate(tc_tape *t, uint32_t i) {
  Node &n = t->nodes[i];
  if (!n.adjoint || n.kind == LEAF) return TC_OK;
  const void *g = n.adjoint;
  switch (n.kind) {
    case BINARY: {
      Node &left = t->nodes[n.a];
      Node &right = t->nodes[n.b];
      void *da = nullptr, *db = nullptr;
      if (n.op == TC_ADD || n.op == TC_SUB) {
        TRY(sum_to_shape(t, g, n.shape, left.shape, &da));
        TRY(accumulate(t, left, da));
        TRY(sum_to_shape(t, g, n.shape, right.shape, &db));
        if (n.op == TC_SUB) {
          void *neg = nullptr;
          TRY(scaled(t, db, count_of(right.shape), -1.0, &neg));
          release(t, db);
          db = neg;
        }
        return accumulate(t, right, db);
      }
      if (n.op == TC_MUL) {
        void *tmp = nullptr;
        TRY(alloc(t, count_of(n.shape), &tmp));
        TRY(binary_into(t, TC_MUL, g, n.shape, right.value, right.shape, n.shape, tmp));
        TRY(sum_to_shape(t, tmp, n.shape, left.shape, &da));
        TRY(accumulate(t, left, da));
        TRY(binary_into(t, TC_MUL, g, n.shape, left.value, left.shape, n.shape, tmp));
        TRY(sum_to_shape(t, tmp, n.shape, right.shape, &db));
        release(t, tmp);
        return accumulate(t, right, db);
      }
      // Div: over = c̄/b, ā += over, b̄ −= (over·a)/b
      void *over = nullptr, *prod = nullptr;
      TRY(alloc(t, count_of(n.shape), &over));
      TRY(alloc(t, count_of(n.shape), &prod));
      TRY(binary_into(t, TC_DIV, g, n.shape, right.value, right.shape, n.shape, over));
      TRY(binary_into(t, TC_MUL, over, n.shape, left.value, left.shape, n.shape, prod));
      TRY(binary_into(t, TC_DIV, prod, n.shape, right.value, right.shape, n.shape, prod));
      TRY(sum_to_shape(t, over, n.shape, left.shape, &da));
      TRY(accumulate(t, left, da));
      TRY(sum_to_shape(t, prod, n.shape, right.shape, &db));
      void *neg = nullptr;
      TRY(scaled(t, db, count_of(right.shape), -1.0, &neg));
      release(t, db);
      release(t, over);
      release(t, prod);
      return accumulate(t, right, neg);
    }
    case RELU: {
      Node &p = t->nodes[n.a];
      const size_t cnt = count_of(p.shape);
      void *weight = nullptr, *d = nullptr;
      TRY(alloc(t, cnt, &weight));
      TRY(tc_compare_scalar(t->dtype, TC_MAX_SHARE, p.value, 0.0, 0, weight, cnt, t->stream));
      TRY(alloc(t, cnt, &d));
      TRY(tc_elementwise(t->dtype, TC_MUL, g, weight, d, cnt, t->stream));
      release(t, weight);
      return accumulate(t, p, d);
    }
    case SCALE: {
      Node &p = t->nodes[n.a];
      void *d = nullptr;
      TRY(scaled(t, g, count_of(p.shape), n.factor, &d));
      return accumulate(t, p, d);
    }
    case SUM_AXES: {
      Node &p = t->nodes[n.a];
      // The adjoint read with the folded axes kept at one, spread back.
      std::vector<size_t> kept = p.shape;
      for (uint32_t ax : n.axes) kept[ax] = 1;
      const void *src = g;
      void *share = nullptr, *d = nullptr;
      if (n.mean) {
        TRY(scaled(t, g, count_of(kept), n.factor, &share));
        src = share;
      }
      TRY(spread(t, src, kept, p.shape, &d));
      release(t, share);
      return accumulate(t, p, d);
    }
    case MATMUL: {
      Node &left = t->nodes[n.a];
      Node &right = t->nodes[n.b];
      const size_t m = left.shape[0], k = left.shape[1], cols = right.shape[1];
      TRY(current_or_zeros(t, left));
      TRY(tc_matmul(t->dtype, TC_TRANS_RIGHT, m, cols, k, g, right.value, left.adjoint, 1, t->stream));
      TRY(current_or_zeros(t, right));
      return tc_matmul(t->dtype, TC_TRANS_LEFT, k, m, cols, left.value, g, right.adjoint, 1, t->stream);
    }
    case SUM: {
      Node &p = t->nodes[n.a];
      void *d = nullptr;
      TRY(spread(t, g, std::vector<size_t>(p.shape.size(), 1), p.shape, &d));
      return accumulate(t, p, d);
    }
    default:
      return TC_OK;
  }
}

}  // namespace

extern "C" {

int tc_tape_create(int dtype, void *stream, tc_tape **out) {
  if (!out) return fail(TC_EINVAL, "tape_create: null out");
  if (dtype != TC_F32 && dtype != TC_F16 && dtype != TC_BF16) return fail(TC_EINVAL, "tape_create: dtype %d", dtype);
  tc_tape *t = new tc_tape;
  t->dtype = dtype;
  t->esz = dtype_bytes(dtype);
  t->stream = as_stream(stream);
  *out = t;
  return TC_OK;
}

int tc_tape_destroy(tc_tape *t) {
  if (!t) return TC_OK;
  for (Node &n : t->nodes) {
    if (n.owned) release(t, n.value);
    release(t, n.adjoint);
  }
  delete t;
  return TC_OK;
}

int tc_tape_leaf(tc_tape *t, const void *dev, uint32_t rank, const size_t *shape, uint32_t *var) {
  if (!t) return fail(TC_EINVAL, "tape: null tape");
  if (rank > TC_MAX_RANK || (rank && !shape)) return fail(TC_EINVAL, "tape_leaf: rank %u", rank);
  Node n;
  n.kind = LEAF;
  n.shape.assign(shape, shape + rank);
  if (count_of(n.shape) && !dev) return fail(TC_EINVAL, "tape_leaf: null storage");
  n.value = const_cast<void *>(dev);
  return push(t, std::move(n), var);
}

int tc_tape_binary(tc_tape *t, int op, uint32_t a, uint32_t b, uint32_t *out) {
  TRY(check_var(t, a));
  TRY(check_var(t, b));
  if (op != TC_ADD && op != TC_SUB && op != TC_MUL && op != TC_DIV)
    return fail(TC_EINVAL, "tape_binary: op %d (add, sub, mul or div)", op);
  Node n;
  n.kind = BINARY;
  n.op = op;
  n.a = a;
  n.b = b;
  if (!broadcast_shape(t->nodes[a].shape, t->nodes[b].shape, n.shape))
    return fail(TC_EINVAL, "tape_binary: shapes do not broadcast");
  if (n.shape.size() > TC_MAX_RANK) return fail(TC_EINVAL, "tape_binary: rank");
  TRY(alloc(t, count_of(n.shape), &n.value));
  n.owned = true;
  TRY(binary_into(t, op, t->nodes[a].value, t->nodes[a].shape, t->nodes[b].value, t->nodes[b].shape, n.shape,
                  n.value));
  return push(t, std::move(n), out);
}

int tc_tape_relu(tc_tape *t, uint32_t a, uint32_t *out) {
  TRY(check_var(t, a));
  Node n;
  n.kind = RELU;
  n.a = a;
  n.shape = t->nodes[a].shape;
  TRY(alloc(t, count_of(n.shape), &n.value));
  n.owned = true;
  TRY(tc_compare_scalar(t->dtype, TC_MAX, t->nodes[a].value, 0.0, 0, n.value, count_of(n.shape), t->stream));
  return push(t, std::move(n), out);
}

int tc_tape_scale(tc_tape *t, uint32_t a, double factor, uint32_t *out) {
  TRY(check_var(t, a));
  Node n;
  n.kind = SCALE;
  n.a = a;
  n.factor = factor;
  n.shape = t->nodes[a].shape;
  TRY(alloc(t, count_of(n.shape), &n.value));
  n.owned = true;
  TRY(tc_broadcast_scalar(t->dtype, TC_MUL, t->nodes[a].value, factor, 0, n.value, count_of(n.shape), t->stream));
  return push(t, std::move(n), out);
}

int tc_tape_sum_axes(tc_tape *t, uint32_t a, uint32_t n_axes, const uint32_t *axes, int mean, int keep_dims,
                     double share, uint32_t *out) {
  TRY(check_var(t, a));
  const std::vector<size_t> &in = t->nodes[a].shape;
  if (n_axes == 0 || !axes) return fail(TC_EINVAL, "tape_sum_axes: no axes");
  std::vector<bool> folded(in.size(), false);
  for (uint32_t i = 0; i < n_axes; ++i) {
    if (axes[i] >= in.size() || folded[axes[i]] || (i && axes[i] <= axes[i - 1]))
      return fail(TC_EINVAL, "tape_sum_axes: axes must be distinct, ascending and in range");
    folded[axes[i]] = true;
  }
  Node n;
  n.kind = SUM_AXES;
  n.a = a;
  n.axes.assign(axes, axes + n_axes);
  n.mean = mean != 0;
  n.factor = share;
  for (size_t d = 0; d < in.size(); ++d)
    if (!folded[d]) n.shape.push_back(in[d]);
    else if (keep_dims) n.shape.push_back(1);
  std::vector<size_t> st(in.size());
  contiguous_strides(uint32_t(in.size()), in.data(), st.data());
  TRY(alloc(t, count_of(n.shape), &n.value));
  n.owned = true;
  TRY(tc_reduce_axes(t->dtype, uint32_t(in.size()), in.data(), t->nodes[a].value, count_of(in), 0, st.data(), n_axes,
                     axes, mean ? TC_AXIS_MEAN : TC_AXIS_FOLD, TC_SUM, 0, n.value, t->stream));
  return push(t, std::move(n), out);
}

int tc_tape_matmul(tc_tape *t, uint32_t a, uint32_t b, uint32_t *out) {
  TRY(check_var(t, a));
  TRY(check_var(t, b));
  const auto &as = t->nodes[a].shape, &bs = t->nodes[b].shape;
  if (as.size() != 2 || bs.size() != 2 || as[1] != bs[0]) return fail(TC_EINVAL, "tape_matmul: shapes");
  Node n;
  n.kind = MATMUL;
  n.a = a;
  n.b = b;
  n.shape = {as[0], bs[1]};
  TRY(alloc(t, count_of(n.shape), &n.value));
  n.owned = true;
  TRY(tc_matmul(t->dtype, TC_TRANS_NONE, as[0], as[1], bs[1], t->nodes[a].value, t->nodes[b].value, n.value, 0,
                t->stream));
  return push(t, std::move(n), out);
}

int tc_tape_sum(tc_tape *t, uint32_t a, uint32_t *out) {
  TRY(check_var(t, a));
  Node n;
  n.kind = SUM;
  n.a = a;
  n.shape = {1};
  TRY(alloc(t, 1, &n.value));
  n.owned = true;
  TRY(tc_vector_reduce(t->dtype, TC_SUM, t->nodes[a].value, count_of(t->nodes[a].shape), n.value, t->stream));
  return push(t, std::move(n), out);
}

int tc_tape_value(tc_tape *t, uint32_t var, const void **dev, uint32_t *rank, size_t *shape) {
  TRY(check_var(t, var));
  const Node &n = t->nodes[var];
  if (dev) *dev = n.value;
  if (rank) *rank = uint32_t(n.shape.size());
  if (shape)
    for (size_t i = 0; i < n.shape.size(); ++i) shape[i] = n.shape[i];
  return TC_OK;
}

int tc_tape_backward(tc_tape *t, uint32_t var) {
  TRY(check_var(t, var));
  if (count_of(t->nodes[var].shape) != 1) return fail(TC_EINVAL, "tape_backward: the output is not one element");
  for (Node &n : t->nodes) {
    release(t, n.adjoint);
    n.adjoint = nullptr;
  }
  // The seed: one, in the element type's bits.
  Node &o = t->nodes[var];
  static const uint32_t one_f32 = 0x3F800000u;
  static const uint16_t one_f16 = 0x3C00u, one_bf16 = 0x3F80u;
  const void *one = t->dtype == TC_F32 ? static_cast<const void *>(&one_f32)
                                       : t->dtype == TC_F16 ? static_cast<const void *>(&one_f16) : &one_bf16;
  TRY(alloc(t, 1, &o.adjoint));
  TRY(tc_memcpy_h2d(o.adjoint, one, t->esz, t->stream));
  for (int64_t i = int64_t(var); i >= 0; --i) TRY(propagate(t, uint32_t(i)));
  return TC_OK;
}

int tc_tape_adjoint(tc_tape *t, uint32_t var, const void **dev) {
  TRY(check_var(t, var));
  if (!dev) return fail(TC_EINVAL, "tape_adjoint: null out");
  *dev = t->nodes[var].adjoint;
  return TC_OK;
}

}  // extern "C"
