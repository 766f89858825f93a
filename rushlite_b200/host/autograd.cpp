// Autograd: Variable, the recorded backward functions and backward().
//
// The backward formulas are the reference's, op for op and in the same
// operand order (csrc/src/autograd/functions/{expand,unary,reduct,matrix}_ops.cpp),
// so each gradient term rounds exactly as the reference's eager evaluation
// does.  What differs is when they run: backward() evaluates the formulas
// under lazy capture and then realizes every leaf gradient in one batch, so
// the chain of per-op kernels, fills and add_inplace calls of the reference
// becomes a few fused passes (intermediate gradients are never materialised
// unless read).
#include <algorithm>
#include <unordered_set>

#include "lamp.hpp"

namespace lmp {
namespace autograd {

using tensor::ImplPtr;
using tensor::LazyNode;
using tensor::TensorImpl;
namespace tops = tensor::ops;

namespace {
thread_local bool t_grad_enabled = true;

Tensor sum_broadcast_axis(const Tensor& g, const std::vector<size_t>& shape) {
  // csrc/src/autograd/utils/grad_utils.cpp:10-36: sum the broadcast axes of
  // the gradient back to the operand's shape.
  if (g.shape() == shape) return g;
  return tops::sum_to_shape(g, shape);
}

Tensor smul(Scalar s, const Tensor& t) {
  return tops::mul(tensor::scalar_tensor(s, t.device(), t.type()), t);
}
Tensor ssub(const Tensor& t, Scalar s) {
  return tops::sub(t, tensor::scalar_tensor(s, t.device(), t.type()));
}

template <typename F>
struct Fn : Function {
  F f;
  explicit Fn(F ff) : f(std::move(ff)) {}
  void apply(const Variable& out) override { f(out, *saved_inputs); }
};

template <typename F>
std::shared_ptr<Function> make_fn(F f, variable_list inputs) {
  auto fn = std::make_shared<Fn<F>>(std::move(f));
  fn->saved_inputs = std::make_shared<variable_list>(std::move(inputs));
  return fn;
}

bool any_requires_grad(const variable_list& v) {
  for (const auto& x : v)
    if (x.requires_grad()) return true;
  return false;
}

// ForwardFunction::apply (csrc/include/lamp3/autograd/forward_function.hpp:26-39)
template <typename B>
Variable record(const Tensor& result, variable_list inputs, B backward) {
  const bool rg = is_grad_enabled() && any_requires_grad(inputs);
  Variable out(result, rg);
  if (rg) out.set_grad_fn(make_fn(std::move(backward), std::move(inputs)));
  return out;
}

// dA += G · op(B) on the tensor-core GEMM, accumulating straight into the
// gradient buffer (beta = 1), or writing it (beta = 0) when the gradient is
// still the untouched zero; other dtypes take the reference's
// matmul-then-accumulate route.
void gemm_accumulate(Variable& v, const Tensor& A, bool ta, const Tensor& B, bool tb) {
  if (v.impl()->grad_shared) {  // the GEMM accumulates in place: give v a gradient of its own first
    v.impl()->grad_shared = false;
    v.grad_slot() = tops::add(v.grad_slot(), tensor::zeros_like(v.grad_slot()));
  }
  Tensor& G = v.grad_slot();
  const bool fp32 = A.type() == DataType::Float32 && B.type() == DataType::Float32 &&
                    G.type() == DataType::Float32 && G.device() == DeviceType::CUDA;
  if (!fp32) {
    Tensor a = ta ? tops::transpose(A) : A;
    Tensor b = tb ? tops::transpose(B) : B;
    v.incr_grad(tops::matmul(a, b));
    return;
  }
  const int64_t m = (int64_t)(ta ? A.shape()[1] : A.shape()[0]);
  const int64_t k = (int64_t)(ta ? A.shape()[0] : A.shape()[1]);
  const int64_t n = (int64_t)(tb ? B.shape()[0] : B.shape()[1]);
  LMP_CHECK((size_t)m * (size_t)n == G.numel(), "matmul backward: gradient shape mismatch");
  const ImplPtr& gi = G.impl();
  float beta = 1.f;
  if (gi->lazy && gi->lazy->kind == LazyNode::kConst && gi->lazy->p0 == 0.0) {
    if (!gi->storage || gi->storage->bytes < gi->nbytes())
      gi->storage = tensor::make_storage(gi->nbytes(), DeviceType::CUDA);
    gi->lazy = nullptr;
    beta = 0.f;
  } else {
    gi->data();  // materialise any pending accumulation first
  }
  const void* pa = A.impl()->data();
  const void* pb = B.impl()->data();
  LMPB_OK_OR_THROW(lmpb_gemm_f32(ta, tb, static_cast<const float*>(pa), static_cast<const float*>(pb),
                                 static_cast<float*>(gi->storage->ptr), m, n, k, beta, tensor::current_stream()));
  if (v.impl()->grad_hook) v.impl()->grad_hook();
}

}  // namespace

void set_grad_enabled(bool enabled) { t_grad_enabled = enabled; }
bool is_grad_enabled() { return t_grad_enabled; }

// ------------------------------------------------------------ Variable

Variable::Variable(const Tensor& data, bool requires_grad) : impl_(std::make_shared<VariableImpl>()) {
  impl_->data = data;
  impl_->requires_grad = requires_grad;
  if (requires_grad) impl_->grad = tensor::zeros_like(data);
}

Variable::Variable(const Tensor& data, const Tensor& grad, bool requires_grad, std::shared_ptr<Function> fn)
    : impl_(std::make_shared<VariableImpl>()) {
  impl_->data = data;
  impl_->grad = grad;
  impl_->requires_grad = requires_grad;
  impl_->grad_fn = std::move(fn);
}

const Tensor& Variable::grad() const {
  LMP_CHECK(impl_->requires_grad, "Cannot access grad() if requires_grad = false");
  return impl_->grad;
}

void Variable::zero_grad() {
  LMP_CHECK(requires_grad(), "Cannot access grad() if requires_grad = false");
  impl_->grad_shared = false;
  impl_->grad = tensor::zeros_like(impl_->grad);
  impl_->grad_fn = nullptr;
}

// Variable::incr_grad (csrc/src/autograd/variable.cpp:30-35).  On CUDA the
// accumulation is recorded lazily as old + g and later written into the
// gradient's existing storage, so the buffer keeps its address.
void Variable::incr_grad(const Tensor& g) {
  LMP_CHECK(requires_grad(), "Cannot access grad() if requires_grad = false");
  Tensor& G = impl_->grad;
  LMP_CHECK(g.shape() == G.shape(), "There should be no broadcasting in incr_grad");
  if (G.device() != DeviceType::CUDA) {
    tops::add_inplace(G, g);
    return;
  }
  const ImplPtr& gi = G.impl();
  if (impl_->grad_fn && !impl_->grad_shared && gi->lazy && gi->lazy->kind == LazyNode::kConst &&
      gi->lazy->p0 == 0.0 && !gi->storage && g.type() == G.type() && g.defined()) {
    // An intermediate's first gradient term: keep g itself rather than 0 + g,
    // so the kernel that materialises g (for a GEMM operand, say) also serves
    // every other reader of this gradient (the bias gradient's row sum).
    G = g;
    impl_->grad_shared = true;
    return;
  }
  if (impl_->grad_shared) {  // copy on write: a new pending sum, the shared tensor untouched
    auto n = std::make_shared<LazyNode>();
    n->kind = LazyNode::kBinary;
    n->op = LMPB_ADD;
    n->inputs = {gi, g.impl()};
    auto t = std::make_shared<TensorImpl>();
    t->shape = gi->shape;
    t->dtype = gi->dtype;
    t->device = gi->device;
    t->lazy = n;
    G = Tensor(t);
    impl_->grad_shared = false;
    return;
  }
  auto old = std::make_shared<TensorImpl>();
  old->shape = gi->shape;
  old->dtype = gi->dtype;
  old->device = gi->device;
  if (gi->lazy) old->lazy = gi->lazy;  // the pending value (it already reads the storage if it has one)
  else old->storage = gi->storage;     // the realized value
  auto n = std::make_shared<LazyNode>();
  n->kind = LazyNode::kBinary;
  n->op = LMPB_ADD;
  n->inputs = {old, g.impl()};
  gi->lazy = n;
}

void Variable::set_grad_fn(std::shared_ptr<Function> fn) {
  LMP_CHECK(requires_grad(), "Cannot access grad() if requires_grad = false");
  impl_->grad_fn = std::move(fn);
}

void Variable::copy(const Variable& other) { impl_->data.copy(other.data()); }
void Variable::fill(Scalar item) { impl_->data.fill(item); }
void Variable::realize() { impl_->data.realize(); }

static void dfs(const Variable& v, std::unordered_set<void*>& seen, std::vector<Variable>& topo) {
  if (!seen.insert(v.impl().get()).second) return;
  if (v.grad_fn())
    for (const auto& c : *v.grad_fn()->saved_inputs) dfs(c, seen, topo);
  topo.push_back(v);
}

// Variable::backward (csrc/src/autograd/variable.cpp:46-55): seed ones, apply
// every recorded function in reverse topological order.
void Variable::backward() {
  LMP_CHECK(requires_grad(), "Must be declared with requires_grad");
  std::vector<Variable> topo;
  std::unordered_set<void*> seen;
  dfs(*this, seen, topo);
  std::reverse(topo.begin(), topo.end());
  // A repeated backward over the same graph accumulates into every node's
  // gradient, intermediates included, as the reference's eager sweep does.
  // Intermediate gradients left pending by the previous sweep are read by
  // other pending gradients of that sweep, so they are materialised before
  // this sweep updates them in place.  A first sweep finds only untouched
  // constant gradients (zeros; the seed is replaced, not updated) and skips this.
  std::vector<ImplPtr> stale;
  for (Variable& node : topo) {
    if (!node.grad_fn() || !node.requires_grad() || !node.impl()->grad.defined()) continue;
    const ImplPtr& gi = node.impl()->grad.impl();
    if (gi->lazy && gi->lazy->kind != LazyNode::kConst) stale.push_back(gi);
  }
  if (!stale.empty()) tensor::realize_all(stale);
  // A gradient shared with another tensor (an intermediate's first term, kept
  // as is) gets a private copy now, before this sweep updates either in place.
  std::vector<ImplPtr> copies;
  for (Variable& node : topo) {
    if (!node.impl()->grad_shared) continue;
    node.impl()->grad_shared = false;
    node.grad_slot() = tops::add(node.grad_slot(), tensor::zeros_like(node.grad_slot()));
    copies.push_back(node.grad_slot().impl());
  }
  if (!copies.empty()) tensor::realize_all(copies);
  impl_->grad = tensor::ones_like(impl_->grad);
  {
    tensor::lazy::CaptureGuard cap(true);
    for (Variable& node : topo)
      if (node.grad_fn()) node.grad_fn()->apply(node);
  }
  std::vector<ImplPtr> leaves;
  for (Variable& node : topo)
    if (!node.grad_fn() && node.requires_grad() && node.impl()->grad.defined())
      leaves.push_back(node.impl()->grad.impl());
  tensor::realize_all(leaves);
}

// ----------------------------------------------------------------- ops

namespace ops {

#define LMP_BIN(NAME, OPC, SELF_GRAD, OTHER_GRAD)                                                      \
  Variable NAME(const Variable& a, const Variable& b) {                                              \
    Tensor r = tops::binary(OPC, a.data(), b.data());                                                \
    return record(r, {a, b}, [](const Variable& out, variable_list& in) {                            \
      Variable& self = in[0];                                                                        \
      Variable& other = in[1];                                                                       \
      const Tensor& g = out.grad();                                                                  \
      (void)g;                                                                                       \
      if (self.requires_grad()) self.incr_grad(SELF_GRAD);                                           \
      if (other.requires_grad()) other.incr_grad(OTHER_GRAD);                                        \
    });                                                                                              \
  }

LMP_BIN(add, LMPB_ADD, sum_broadcast_axis(g, self.data().shape()), sum_broadcast_axis(g, other.data().shape()))
LMP_BIN(sub, LMPB_SUB, sum_broadcast_axis(g, self.data().shape()),
        sum_broadcast_axis(tops::neg(g), other.data().shape()))
LMP_BIN(mul, LMPB_MUL, sum_broadcast_axis(tops::mul(other.data(), g), self.data().shape()),
        sum_broadcast_axis(tops::mul(self.data(), g), other.data().shape()))
LMP_BIN(div, LMPB_DIV, sum_broadcast_axis(tops::div(g, other.data()), self.data().shape()),
        sum_broadcast_axis(smul(-1.0, tops::div(tops::mul(out.data(), g), other.data())), other.data().shape()))
LMP_BIN(pow, LMPB_POW,
        sum_broadcast_axis(tops::mul(tops::mul(g, other.data()), tops::pow(self.data(), ssub(other.data(), 1.0))),
                           self.data().shape()),
        sum_broadcast_axis(tops::mul(tops::mul(g, out.data()), tops::log(self.data())), other.data().shape()))

#define LMP_CMP(NAME, OPC)                                                                  \
  Variable NAME(const Variable& a, const Variable& b) {                                   \
    Tensor r = tops::binary(OPC, a.data(), b.data());                                     \
    return record(r, {a, b}, [](const Variable&, variable_list&) {                        \
      throw std::runtime_error("Not implemented: comparison ops have no gradient");       \
    });                                                                                   \
  }
LMP_CMP(eq, LMPB_EQ)
LMP_CMP(ne, LMPB_NE)
LMP_CMP(ge, LMPB_GE)
LMP_CMP(le, LMPB_LE)
LMP_CMP(gt, LMPB_GT)
LMP_CMP(lt, LMPB_LT)

Variable binary(int op, const Variable& a, const Variable& b) {
  switch (op) {
    case LMPB_ADD: return add(a, b);
    case LMPB_SUB: return sub(a, b);
    case LMPB_MUL: return mul(a, b);
    case LMPB_DIV: return div(a, b);
    case LMPB_POW: return pow(a, b);
    case LMPB_EQ: return eq(a, b);
    case LMPB_NE: return ne(a, b);
    case LMPB_GE: return ge(a, b);
    case LMPB_LE: return le(a, b);
    case LMPB_GT: return gt(a, b);
    case LMPB_LT: return lt(a, b);
    default: throw std::runtime_error("unknown binary op");
  }
}

// binary_op(Variable, Scalar) (csrc/include/lamp3/autograd/functions/overloads.hpp:16-29):
// the scalar becomes a {1}-shaped tensor of the Variable's dtype.
Variable binary_scalar(int op, const Variable& v, Scalar s, bool scalar_left) {
  Variable sv(tensor::scalar_tensor(s, v.data().device(), v.data().type()), false);
  return scalar_left ? binary(op, sv, v) : binary(op, v, sv);
}

#define LMP_UN(NAME, FWD, GRAD)                                                          \
  Variable NAME(const Variable& a) {                                                   \
    Tensor r = FWD;                                                                    \
    return record(r, {a}, [](const Variable& out, variable_list& in) {                 \
      Variable& self = in[0];                                                          \
      const Tensor& g = out.grad();                                                    \
      (void)g;                                                                         \
      if (self.requires_grad()) self.incr_grad(GRAD);                                  \
    });                                                                                \
  }

LMP_UN(neg, tops::neg(a.data()), tops::neg(g))
LMP_UN(exp, tops::exp(a.data()), tops::mul(out.data(), g))
LMP_UN(log, tops::log(a.data()), tops::div(g, self.data()))
LMP_UN(sqrt, tops::sqrt(a.data()), tops::div(g, tops::add(out.data(), out.data())))
LMP_UN(abs, tops::abs(a.data()), tops::abs_backward(self.data(), g))
LMP_UN(sin, tops::sin(a.data()), tops::mul(g, tops::cos(self.data())))
LMP_UN(cos, tops::cos(a.data()), tops::mul(tops::neg(tops::sin(self.data())), g))
LMP_UN(tan, tops::tan(a.data()), tops::add(g, tops::mul(tops::mul(g, out.data()), out.data())))

// ClampBackward (csrc/src/autograd/functions/unary_ops.cpp): g where
// lo < x < hi.  It is evaluated on the output instead of the input: clamp
// and its backward both compare in the tensor's dtype against the same cast
// bounds, and the output is lo, hi or x, so lo < out < hi exactly when
// lo < x < hi (NaN and lo > hi included).  The input then need not stay
// materialised: a fused Linear+ReLU never writes its pre-activation.
Variable clamp(const Variable& a, Scalar lo, Scalar hi) {
  Tensor r = tops::clamp(a.data(), lo, hi);
  return record(r, {a}, [lo, hi](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::clamp_backward(out.data(), out.grad(), lo, hi));
  });
}

Variable sum(const Variable& a, size_t axis) {
  Tensor r = tops::sum(a.data(), axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::mul(tensor::ones_like(self.data()), out.grad()));
  });
}

Variable max(const Variable& a, size_t axis) {
  Tensor r = tops::max(a.data(), axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::mul(out.grad(), tops::eq(self.data(), out.data())));
  });
}

Variable min(const Variable& a, size_t axis) {
  Tensor r = tops::min(a.data(), axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::mul(out.grad(), tops::eq(self.data(), out.data())));
  });
}

Variable prod(const Variable& a, size_t axis) {
  Tensor r = tops::prod(a.data(), axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::mul(out.grad(), tops::div(out.data(), self.data())));
  });
}

// MatrixMultiplicationBackward (csrc/src/autograd/functions/matrix_ops.cpp:8-24):
// dA = G·Bᵀ, dB = Aᵀ·G, only for inputs that require grad.
Variable matmul(const Variable& a, const Variable& b) {
  Tensor r = tops::matmul(a.data(), b.data());
  return record(r, {a, b}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    Variable& other = in[1];
    const Tensor& g = out.grad();
    if (self.requires_grad()) gemm_accumulate(self, g, false, other.data(), true);
    if (other.requires_grad()) gemm_accumulate(other, self.data(), true, g, false);
  });
}

Variable transpose(const Variable& a) {
  Tensor r = tops::transpose(a.data());
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(tops::transpose(out.grad()));
  });
}

// View ops: the gradient is the output gradient viewed in the input's shape.
Variable reshape(const Variable& a, const std::vector<size_t>& shape) {
  Tensor r = a.data().reshape(shape);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(out.grad().reshape(self.data().shape()));
  });
}
Variable squeeze(const Variable& a, size_t axis) {
  Tensor r = a.data().squeeze(axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(out.grad().reshape(self.data().shape()));
  });
}
Variable expand_dims(const Variable& a, size_t axis) {
  Tensor r = a.data().expand_dims(axis);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(out.grad().reshape(self.data().shape()));
  });
}
Variable to(const Variable& a, DeviceType device) {
  Tensor r = a.data().to(device);
  return record(r, {a}, [](const Variable& out, variable_list& in) {
    Variable& self = in[0];
    if (self.requires_grad()) self.incr_grad(out.grad().to(self.data().device()));
  });
}

}  // namespace ops

Variable full(const std::vector<size_t>& shape, Scalar v, bool requires_grad, DeviceType device, DataType dtype) {
  size_t n = 1;
  for (size_t s : shape) n *= s;
  Tensor t(std::vector<double>(n, v), shape, device, dtype);
  return Variable(t, requires_grad);
}
Variable zeros(const std::vector<size_t>& shape, bool rg, DeviceType d, DataType dt) { return full(shape, 0.0, rg, d, dt); }
Variable ones(const std::vector<size_t>& shape, bool rg, DeviceType d, DataType dt) { return full(shape, 1.0, rg, d, dt); }

}  // namespace autograd
}  // namespace lmp
