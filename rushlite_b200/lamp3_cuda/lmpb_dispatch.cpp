// lmpb_dispatch.cpp — Lamp3's CUDA device, served by liblmpb (include/lmpb.h).
//
// This is the registration unit a Lamp3 build links in place of the
// reference's own CUDA sources.  It fills every DeviceType::CUDA slot of the
// dispatch table and registers the CUDA lazy backend, so the unchanged
// front-end — lmp::tensor::Tensor, lmp::autograd::Variable, the capture flag,
// the pybind11 module — runs on the sm_100a kernels of liblmpb.so.
//
// It replaces, one for one:
//   * the op registrations of csrc/src/tensor/cuda/kernels.cu:124-156
//     (add..lt, neg..tan, clamp, abs_backward, clamp_backward, matmul,
//     transpose, sum/max/min/prod);
//   * the memory registrations of csrc/src/tensor/cuda/memory.cu:97-101,218
//     (empty, fill, resize, add_inplace, copy) and the host-to-device copy
//     vecCopyHostToDevice that csrc/src/tensor/cpu/memory.cpp:67-73 calls in a
//     CUDA build (declared in csrc/include/lamp3/tensor/cuda/memory.cuh:31);
//   * the NVRTC lazy backend, LMP_REGISTER_LAZY_BACKEND at
//     csrc/src/inductor/nvrtc/nvrtc_backend.cpp:192.
//
// Build: compile with the reference's include tree and -DLMP_ENABLE_CUDA
// (the Makefile beside this file does, together with the reference's
// tensor/autograd core), link with liblmpb.so and cudart.
//
// Semantics kept from the reference:
//   * every op allocates its output through the Storage of the CUDA device
//     (the stub contract, csrc/src/tensor/cpu/meta_handler.cpp:9-73) and
//     returns the TensorImpl by value;
//   * user errors throw std::runtime_error through LMP_CHECK
//     (csrc/include/lamp3/common/assert.hpp:89-90); a failed lmpb call is
//     reported the same way with lmpb_last_error()'s message;
//   * kernels run in order on the legacy default stream, and every copy to
//     host memory synchronises that stream before it returns, so a host read
//     (to_vector, index, print) sees finished results without the reference's
//     cudaDeviceSynchronize after every kernel.
// The lazy backend differs on purpose: besides same-shape chains it fuses
// broadcast binaries (their smaller operands become broadcast leaves of the
// one kernel), where the reference realizes every broadcast op eagerly.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "lamp3/common/assert.hpp"
#include "lamp3/tensor/cuda/memory.cuh"
#include "lamp3/tensor/data_ptr.hpp"
#include "lamp3/tensor/data_type.hpp"
#include "lamp3/tensor/device_type.hpp"
#include "lamp3/tensor/dispatch_stub.hpp"
#include "lamp3/tensor/infer_meta.hpp"
#include "lamp3/tensor/lazy/functions/elementwise_binary.hpp"
#include "lamp3/tensor/lazy/functions/elementwise_unary.hpp"
#include "lamp3/tensor/lazy/lazy_backend.hpp"
#include "lamp3/tensor/lazy/realize.hpp"
#include "lamp3/tensor/native/expand_ops.hpp"
#include "lamp3/tensor/native/matrix_ops.hpp"
#include "lamp3/tensor/native/memory_ops.hpp"
#include "lamp3/tensor/native/reduct_ops.hpp"
#include "lamp3/tensor/native/unary_ops.hpp"
#include "lamp3/tensor/storage.hpp"
#include "lamp3/tensor/tensor_impl.hpp"
#include "lmpb.h"

namespace lmp::tensor::detail::lmpb_cuda {

namespace {

void ok(lmpb_status s, const char* what) {
  LMP_CHECK(s == LMPB_OK) << what << ": " << lmpb_last_error();
}

int dt(DataType t) { return static_cast<int>(t); }

size_t elem_size(DataType t) {
  switch (t) {
    case DataType::Bool: return 1;
    case DataType::Int16: return 2;
    case DataType::Int32: return 4;
    case DataType::Int64: return 8;
    case DataType::Float32: return 4;
    case DataType::Float64: return 8;
  }
  return 0;
}

std::vector<int64_t> dims(const TensorImpl& t) {
  return std::vector<int64_t>(t.shape().begin(), t.shape().end());
}

void* ptr(const TensorImpl& t) { return const_cast<TensorImpl&>(t).data(); }

TensorImpl make_out(const OpMeta& m) {
  Storage st(m.size * elem_size(m.dtype), DeviceType::CUDA);
  return TensorImpl(st, m.shape, m.dtype);
}

// ------------------------------------------------------------- elementwise

TensorImpl binary_op(int op, const TensorImpl& a, const TensorImpl& b, Scalar p0 = 0, Scalar p1 = 0) {
  LMP_CHECK(a.device() == DeviceType::CUDA && b.device() == DeviceType::CUDA)
      << "CUDA op given a tensor on another device";
  OpMeta m = infer_binary(&a, &b);
  TensorImpl out = make_out(m);
  if (m.size == 0) return out;
  auto as = dims(a), bs = dims(b);
  ok(lmpb_binary(op, dt(m.dtype), ptr(a), dt(a.type()), as.data(), (int)as.size(), ptr(b), dt(b.type()),
                 bs.data(), (int)bs.size(), ptr(out), p0, p1, nullptr),
     "lmpb_binary");
  return out;
}

template <int OP>
TensorImpl binary(const TensorImpl& a, const TensorImpl& b) {
  return binary_op(OP, a, b);
}

TensorImpl unary_op(int op, const TensorImpl& a, Scalar p0 = 0, Scalar p1 = 0) {
  LMP_CHECK(a.device() == DeviceType::CUDA) << "CUDA op given a tensor on another device";
  OpMeta m = infer_unary(&a);
  TensorImpl out = make_out(m);
  if (m.size == 0) return out;
  ok(lmpb_unary(op, dt(a.type()), ptr(a), ptr(out), (int64_t)m.size, p0, p1, nullptr), "lmpb_unary");
  return out;
}

template <int OP>
TensorImpl unary(const TensorImpl& a) {
  return unary_op(OP, a);
}

TensorImpl clamp(const TensorImpl& a, Scalar lo, Scalar hi) { return unary_op(LMPB_CLAMP, a, lo, hi); }

TensorImpl abs_backward(const TensorImpl& input, const TensorImpl& grad) {
  LMP_CHECK(input.shape() == grad.shape()) << "abs_backward: input and gradient shapes differ";
  return binary_op(LMPB_ABS_BACKWARD, input, grad);
}

TensorImpl clamp_backward(const TensorImpl& input, const TensorImpl& grad, Scalar lo, Scalar hi) {
  LMP_CHECK(input.shape() == grad.shape()) << "clamp_backward: input and gradient shapes differ";
  return binary_op(LMPB_CLAMP_BACKWARD, input, grad, lo, hi);
}

// -------------------------------------------------------------- reductions

template <int OP>
TensorImpl reduce(const TensorImpl& a, size_t axis) {
  LMP_CHECK(axis < a.shape().size()) << "reduction axis " << axis << " out of range for a "
                                     << a.shape().size() << "-d tensor";
  OpMeta m = infer_reduct(&a, axis);
  TensorImpl out = make_out(m);
  if (m.size == 0 || a.numel() == 0) return out;
  auto s = dims(a);
  ok(lmpb_reduce(OP, dt(a.type()), ptr(a), s.data(), (int)s.size(), (int)axis, ptr(out), nullptr),
     "lmpb_reduce");
  return out;
}

// ------------------------------------------------------------------ matrix

TensorImpl matmul(const TensorImpl& a, const TensorImpl& b) {
  LMP_CHECK(a.shape().size() == 2 && b.shape().size() == 2) << "Both matrices must be 2D.";
  LMP_CHECK(a.shape()[1] == b.shape()[0]) << "Incompatible matrix dimensions for multiplication.";
  const size_t m = a.shape()[0], k = a.shape()[1], n = b.shape()[1];
  OpMeta meta{type_upcast(a.type(), b.type()), m * n, {m, n}, false};
  TensorImpl out = make_out(meta);
  if (m * n == 0) return out;
  if (k == 0) {
    ok(lmpb_fill(dt(meta.dtype), ptr(out), (int64_t)(m * n), 0.0, nullptr), "lmpb_fill");
    return out;
  }
  ok(lmpb_matmul(dt(meta.dtype), ptr(a), dt(a.type()), ptr(b), dt(b.type()), ptr(out), (int64_t)m,
                 (int64_t)k, (int64_t)n, nullptr),
     "lmpb_matmul");
  return out;
}

TensorImpl transpose(const TensorImpl& a) {
  LMP_CHECK(a.shape().size() == 2) << "Invalid argument, transpose can only be performed on matrices of dim 2";
  const size_t m = a.shape()[0], n = a.shape()[1];
  OpMeta meta{a.type(), m * n, {n, m}, false};
  TensorImpl out = make_out(meta);
  if (m * n == 0) return out;
  ok(lmpb_transpose(dt(a.type()), ptr(a), ptr(out), (int64_t)m, (int64_t)n, nullptr), "lmpb_transpose");
  return out;
}

// ------------------------------------------------------------------ memory

DataPtr empty(size_t bytes) {
  if (bytes == 0) return {};
  void* p = nullptr;
  ok(lmpb_malloc(&p, bytes, nullptr), "lmpb_malloc");
  return DataPtr(p, [](void* q) { lmpb_free(q, nullptr); });
}

void fill(void* p, size_t n, Scalar v, DataType t) {
  if (n == 0) return;
  ok(lmpb_fill(dt(t), p, (int64_t)n, v, nullptr), "lmpb_fill");
}

void add_inplace(void* dst, const void* src, size_t n, DataType t) {
  if (n == 0) return;
  ok(lmpb_add_inplace(dt(t), dst, src, (int64_t)n, nullptr), "lmpb_add_inplace");
}

// The stub receives the DataPtr by value, so a new allocation cannot be
// handed back to the Storage (the reference's own CUDA and CPU versions have
// the same limitation and drop the copy they make).  Shrinking keeps the
// existing block, which is large enough; growing is refused instead of
// leaving a Storage whose size exceeds its allocation.
void resize(DataPtr, size_t old_bytes, size_t new_bytes) {
  LMP_CHECK(new_bytes <= old_bytes) << "resize: a CUDA storage cannot grow through resize_stub, which "
                                       "receives its DataPtr by value";
}

void copy(DeviceType to, const void* src, void* dst, size_t n, DataType s, DataType d) {
  if (n == 0) return;
  if (to == DeviceType::CPU) {
    ok(lmpb_copy(LMPB_D2H, src, dt(s), dst, dt(d), (int64_t)n, nullptr), "lmpb_copy(D2H)");
    // the host reads right after this returns
    const cudaError_t e = cudaStreamSynchronize(nullptr);
    LMP_CHECK(e == cudaSuccess) << "copy to host: " << cudaGetErrorString(e);
  } else {
    ok(lmpb_copy(LMPB_D2D, src, dt(s), dst, dt(d), (int64_t)n, nullptr), "lmpb_copy(D2D)");
  }
}

// ------------------------------------------------------------ lazy backend

// Op code of a recorded elementwise function; -1 for anything else.
struct NodeOp {
  int kind = -1;  // LMPB_FN_BINARY / LMPB_FN_UNARY
  int sub = 0;
  double p0 = 0, p1 = 0;
};

// ClampFn keeps its bounds private; its generated expression prints both
// with max_digits10 digits (csrc/src/tensor/lazy/functions/elementwise_unary.cpp:10-14,47-54),
// which reads back to the same doubles.
bool clamp_bounds(const std::string& expr, double& lo, double& hi) {
  const std::string a = "({0}) < (", b = "({0}) > (";
  size_t i = expr.find(a), j = expr.find(b);
  if (i == std::string::npos || j == std::string::npos) return false;
  lo = std::strtod(expr.c_str() + i + a.size(), nullptr);
  hi = std::strtod(expr.c_str() + j + b.size(), nullptr);
  return true;
}

NodeOp classify(lazy::LazyFunction* f) {
  using namespace lazy;
  NodeOp r;
  auto bin = [&](int op) { r.kind = LMPB_FN_BINARY; r.sub = op; };
  auto un = [&](int op) { r.kind = LMPB_FN_UNARY; r.sub = op; };
  if (dynamic_cast<AddFn*>(f)) bin(LMPB_ADD);
  else if (dynamic_cast<SubFn*>(f)) bin(LMPB_SUB);
  else if (dynamic_cast<MulFn*>(f)) bin(LMPB_MUL);
  else if (dynamic_cast<DivFn*>(f)) bin(LMPB_DIV);
  else if (dynamic_cast<PowFn*>(f)) bin(LMPB_POW);
  else if (dynamic_cast<EqFn*>(f)) bin(LMPB_EQ);
  else if (dynamic_cast<NeFn*>(f)) bin(LMPB_NE);
  else if (dynamic_cast<GeFn*>(f)) bin(LMPB_GE);
  else if (dynamic_cast<LeFn*>(f)) bin(LMPB_LE);
  else if (dynamic_cast<GtFn*>(f)) bin(LMPB_GT);
  else if (dynamic_cast<LtFn*>(f)) bin(LMPB_LT);
  else if (dynamic_cast<NegFn*>(f)) un(LMPB_NEG);
  else if (dynamic_cast<ExpFn*>(f)) un(LMPB_EXP);
  else if (dynamic_cast<LogFn*>(f)) un(LMPB_LOG);
  else if (dynamic_cast<SqrtFn*>(f)) un(LMPB_SQRT);
  else if (dynamic_cast<AbsFn*>(f)) un(LMPB_ABS);
  else if (dynamic_cast<SinFn*>(f)) un(LMPB_SIN);
  else if (dynamic_cast<CosFn*>(f)) un(LMPB_COS);
  else if (dynamic_cast<TanFn*>(f)) un(LMPB_TAN);
  else if (dynamic_cast<ClampFn*>(f)) {
    if (clamp_bounds(f->codegen_expr(), r.p0, r.p1)) un(LMPB_CLAMP);
  }
  return r;
}

// One fused program: the root's pending elementwise DAG over the root's
// shape.  A pending input of another shape (a broadcast operand such as
// log(b + 1) of shape [rows, 1]) and every realized tensor become leaves.
class Program {
 public:
  explicit Program(TensorImpl* root) : root_(root) {
    for (size_t d : root->shape()) iter_.push_back((int64_t)d);
    out_node_ = visit(root, true);
  }

  void launch() {
    lmpb_fout o{};
    o.node = out_node_;
    o.mode = LMPB_OUT_STORE;
    o.dtype = dt(root_->type());
    o.addend = -1;
    o.ndim = (int)iter_.size();
    for (size_t i = 0; i < iter_.size(); ++i) o.shape[i] = iter_[i];
    lmpb_fused h = handle(o);
    Storage out(root_->numel() * elem_size(root_->type()), DeviceType::CUDA);
    std::vector<const void*> lp;
    for (TensorImpl* t : leaf_impls_) lp.push_back(t->storage().data());
    void* op = out.data();
    ok(lmpb_fused_launch(h, lp.data(), &op, nullptr), "lmpb_fused_launch");
    root_->set_realized(out);
  }

 private:
  int visit(TensorImpl* t, bool is_root = false) {
    auto it = memo_.find(t);
    if (it != memo_.end()) return it->second;
    NodeOp op;
    if (t->is_deferred() && (is_root || t->shape() == root_->shape())) op = classify(t->lazy_op().get());
    int idx;
    if (op.kind < 0) {
      if (is_root) {  // not an elementwise op: let it compute itself
        for (const auto& in : t->lazy_op()->inputs) lazy::realize(in.get());
        t->lazy_op()->run_eager(*t);
        return -1;
      }
      lazy::realize(t);  // fused or eager on its own, then read as a leaf
      LMP_CHECK(t->shape().size() <= LMPB_MAX_DIMS) << "fusion: more than " << LMPB_MAX_DIMS << " dims";
      lmpb_fleaf lf{};
      lf.dtype = dt(t->type());
      lf.ndim = (int)t->shape().size();
      for (size_t i = 0; i < t->shape().size(); ++i) lf.shape[i] = (int64_t)t->shape()[i];
      leaves_.push_back(lf);
      leaf_impls_.push_back(t);
      lmpb_fnode n{};
      n.kind = LMPB_FN_LEAF;
      n.dtype = lf.dtype;
      n.a = (int)leaves_.size() - 1;
      nodes_.push_back(n);
      idx = (int)nodes_.size() - 1;
    } else {
      const auto& ins = t->lazy_op()->inputs;
      lmpb_fnode n{};
      n.kind = op.kind;
      n.sub = op.sub;
      n.dtype = dt(t->type());
      n.p0 = op.p0;
      n.p1 = op.p1;
      n.a = visit(ins[0].get());
      n.b = op.kind == LMPB_FN_BINARY ? visit(ins[1].get()) : 0;
      nodes_.push_back(n);
      idx = (int)nodes_.size() - 1;
    }
    memo_[t] = idx;
    return idx;
  }

  // Built programs are kept for the life of the process, keyed by their bytes.
  lmpb_fused handle(const lmpb_fout& o) {
    std::string key;
    auto put = [&](const void* p, size_t n) { key.append(static_cast<const char*>(p), n); };
    put(nodes_.data(), nodes_.size() * sizeof(lmpb_fnode));
    key.push_back('|');
    put(leaves_.data(), leaves_.size() * sizeof(lmpb_fleaf));
    key.push_back('|');
    put(&o, sizeof(o));
    static std::mutex mu;
    static std::unordered_map<std::string, lmpb_fused> cache;
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    lmpb_fused h = nullptr;
    ok(lmpb_fused_build(nodes_.data(), (int)nodes_.size(), leaves_.data(), (int)leaves_.size(), &o, 1,
                        iter_.data(), (int)iter_.size(), &h),
       "lmpb_fused_build");
    cache.emplace(std::move(key), h);
    return h;
  }

  TensorImpl* root_;
  std::vector<int64_t> iter_;
  std::vector<lmpb_fnode> nodes_;
  std::vector<lmpb_fleaf> leaves_;
  std::vector<TensorImpl*> leaf_impls_;
  std::unordered_map<TensorImpl*, int> memo_;
  int out_node_ = -1;
};

struct LmpbLazyBackend : lazy::LazyBackend {
  void realize(TensorImpl* impl) override {
    if (!impl->is_deferred()) return;
    if (impl->numel() == 0) {
      for (const auto& in : impl->lazy_op()->inputs) lazy::realize(in.get());
      impl->set_realized(Storage(0, DeviceType::CUDA));
      return;
    }
    Program p(impl);
    if (impl->is_deferred()) p.launch();
  }
};

}  // namespace

// Memory registrations: csrc/src/tensor/cuda/memory.cu:97-101,218
LMP_REGISTER_DISPATCH(ops::empty_stub, DeviceType::CUDA, empty);
LMP_REGISTER_DISPATCH(ops::fill_stub, DeviceType::CUDA, fill);
LMP_REGISTER_DISPATCH(ops::resize_stub, DeviceType::CUDA, resize);
LMP_REGISTER_DISPATCH(ops::add_inplace_stub, DeviceType::CUDA, add_inplace);
LMP_REGISTER_DISPATCH(ops::copy_stub, DeviceType::CUDA, copy);

// Op registrations: csrc/src/tensor/cuda/kernels.cu:124-156
#define LMPB_REG_BIN(stub, op)                     \
  namespace {                                      \
  TensorImpl stub##_lmpb(const TensorImpl& a, const TensorImpl& b) { return binary<op>(a, b); } \
  }                                                \
  LMP_REGISTER_DISPATCH(ops::stub##_stub, DeviceType::CUDA, stub##_lmpb)
#define LMPB_REG_UN(stub, op)                                                 \
  namespace {                                                                 \
  TensorImpl stub##_lmpb(const TensorImpl& a) { return unary<op>(a); }        \
  }                                                                           \
  LMP_REGISTER_DISPATCH(ops::stub##_stub, DeviceType::CUDA, stub##_lmpb)
#define LMPB_REG_RED(stub, op)                                                          \
  namespace {                                                                           \
  TensorImpl stub##_lmpb(const TensorImpl& a, size_t axis) { return reduce<op>(a, axis); } \
  }                                                                                     \
  LMP_REGISTER_DISPATCH(ops::stub##_stub, DeviceType::CUDA, stub##_lmpb)

LMPB_REG_BIN(add, LMPB_ADD);
LMPB_REG_BIN(sub, LMPB_SUB);
LMPB_REG_BIN(mul, LMPB_MUL);
LMPB_REG_BIN(div, LMPB_DIV);
LMPB_REG_BIN(pow, LMPB_POW);
LMPB_REG_BIN(eq, LMPB_EQ);
LMPB_REG_BIN(ne, LMPB_NE);
LMPB_REG_BIN(le, LMPB_LE);
LMPB_REG_BIN(lt, LMPB_LT);
LMPB_REG_BIN(ge, LMPB_GE);
LMPB_REG_BIN(gt, LMPB_GT);
LMPB_REG_UN(neg, LMPB_NEG);
LMPB_REG_UN(log, LMPB_LOG);
LMPB_REG_UN(exp, LMPB_EXP);
LMPB_REG_UN(sqrt, LMPB_SQRT);
LMPB_REG_UN(abs, LMPB_ABS);
LMPB_REG_UN(sin, LMPB_SIN);
LMPB_REG_UN(cos, LMPB_COS);
LMPB_REG_UN(tan, LMPB_TAN);
LMP_REGISTER_DISPATCH(ops::clamp_stub, DeviceType::CUDA, clamp);
LMP_REGISTER_DISPATCH(ops::abs_backward_stub, DeviceType::CUDA, abs_backward);
LMP_REGISTER_DISPATCH(ops::clamp_backward_stub, DeviceType::CUDA, clamp_backward);
LMP_REGISTER_DISPATCH(ops::matmul_stub, DeviceType::CUDA, matmul);
LMP_REGISTER_DISPATCH(ops::transpose_stub, DeviceType::CUDA, transpose);
LMPB_REG_RED(sum, LMPB_SUM);
LMPB_REG_RED(max, LMPB_MAX);
LMPB_REG_RED(min, LMPB_MIN);
LMPB_REG_RED(prod, LMPB_PROD);

// Lazy backend: csrc/src/inductor/nvrtc/nvrtc_backend.cpp:192
using LmpbLazy = LmpbLazyBackend;
LMP_REGISTER_LAZY_BACKEND(DeviceType::CUDA, LmpbLazy)

}  // namespace lmp::tensor::detail::lmpb_cuda

// The host-to-device copy a CUDA build of csrc/src/tensor/cpu/memory.cpp:67-73
// calls (declared in csrc/include/lamp3/tensor/cuda/memory.cuh:31).
namespace lmp::tensor::detail::cuda {
void vecCopyHostToDevice(const void* src, void* dst, size_t n, DataType s, DataType d) {
  if (n == 0) return;
  lmpb_status st = lmpb_copy(LMPB_H2D, src, static_cast<int>(s), dst, static_cast<int>(d), (int64_t)n, nullptr);
  LMP_CHECK(st == LMPB_OK) << "lmpb_copy(H2D): " << lmpb_last_error();
}
}  // namespace lmp::tensor::detail::cuda
