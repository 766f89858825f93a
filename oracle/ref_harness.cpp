// ref_harness.cpp — TEST INFRASTRUCTURE ONLY.
//
// A small C ABI over the reference's own public C++ API (lmp::tensor,
// lmp::autograd), linked with the reference CPU core that oracle/Makefile
// compiles from the reference sources into _ref/liblamp3_ref.so.  Tests and
// bench.py's reference arm drive it through ctypes (oracle/ref.py).  Handles
// are heap-allocated lmp::autograd::Variable objects.
#include <cstdint>
#include <cstring>
#include <type_traits>
#include <vector>

#include <omp.h>

#include "lamp3/lamp3.hpp"

using lmp::autograd::Variable;
using lmp::tensor::DataType;
using lmp::tensor::DeviceType;
using lmp::tensor::Tensor;
namespace aops = lmp::autograd::ops;
namespace tops = lmp::tensor::ops;

namespace {

template <typename F>
void with_type(int dt, F&& f) {
  switch (dt) {
    case 0: f(bool{}); break;
    case 1: f(int16_t{}); break;
    case 2: f(int32_t{}); break;
    case 3: f(int64_t{}); break;
    case 4: f(float{}); break;
    default: f(double{}); break;
  }
}

// Device of the tensors lref_tensor creates.  The CPU build of the reference
// (_ref/liblamp3_ref.so) only has the CPU device; the harness linked with the
// reference core whose CUDA device is served by lmpb
// (_ref/liblamp3_cuda_harness.so) creates CUDA tensors after lref_set_device(1).
DeviceType g_device = DeviceType::CPU;

Variable* wrap(const Variable& v) { return new Variable(v); }
Variable* wrap_t(const Tensor& t) { return new Variable(t, false); }

}  // namespace

extern "C" {

void* lref_tensor(int dt, const void* data, const int64_t* shape, int ndim, int requires_grad) {
  std::vector<size_t> sh(shape, shape + ndim);
  size_t n = 1;
  for (size_t s : sh) n *= s;
  Variable* out = nullptr;
  with_type(dt, [&](auto tag) {
    using T = decltype(tag);
    // the reference cannot build from std::vector<bool>; bool data travels as int16
    using H = std::conditional_t<std::is_same_v<T, bool>, int16_t, T>;
    std::vector<H> v(n);
    const T* src = static_cast<const T*>(data);
    for (size_t i = 0; i < n; ++i) v[i] = static_cast<H>(src[i]);
    Tensor t(v, sh, g_device, static_cast<DataType>(dt));
    out = new Variable(t, requires_grad != 0);
  });
  return out;
}

void lref_free(void* h) { delete static_cast<Variable*>(h); }
int lref_ndim(void* h) { return (int)static_cast<Variable*>(h)->data().shape().size(); }
int lref_dtype(void* h) { return (int)static_cast<Variable*>(h)->data().type(); }
void lref_shape(void* h, int64_t* out) {
  const auto& s = static_cast<Variable*>(h)->data().shape();
  for (size_t i = 0; i < s.size(); ++i) out[i] = (int64_t)s[i];
}

static void read_tensor(const Tensor& t, void* dst) {
  with_type((int)t.type(), [&](auto tag) {
    using T = decltype(tag);
    using H = std::conditional_t<std::is_same_v<T, bool>, int16_t, T>;
    std::vector<H> v = t.to_vector<H>();
    T* out = static_cast<T*>(dst);
    for (size_t i = 0; i < v.size(); ++i) out[i] = static_cast<T>(v[i]);
  });
}

void lref_data(void* h, void* dst) { read_tensor(static_cast<Variable*>(h)->data(), dst); }
void lref_grad(void* h, void* dst) { read_tensor(static_cast<Variable*>(h)->grad(), dst); }

void* lref_binary(int op, void* a, void* b) {
  const Variable& x = *static_cast<Variable*>(a);
  const Variable& y = *static_cast<Variable*>(b);
  switch (op) {
    case 0: return wrap(aops::add(x, y));
    case 1: return wrap(aops::sub(x, y));
    case 2: return wrap(aops::mul(x, y));
    case 3: return wrap(aops::div(x, y));
    case 4: return wrap(aops::pow(x, y));
    case 5: return wrap(aops::eq(x, y));
    case 6: return wrap(aops::ne(x, y));
    case 7: return wrap(aops::ge(x, y));
    case 8: return wrap(aops::le(x, y));
    case 9: return wrap(aops::gt(x, y));
    case 10: return wrap(aops::lt(x, y));
    default: return nullptr;
  }
}

void* lref_binary_backward(int op, void* input, void* grad, double p0, double p1) {
  const Tensor& x = static_cast<Variable*>(input)->data();
  const Tensor& g = static_cast<Variable*>(grad)->data();
  if (op == 11) return wrap_t(tops::abs_backward(x, g));
  return wrap_t(tops::clamp_backward(x, g, p0, p1));
}

void* lref_unary(int op, void* a, double p0, double p1) {
  const Variable& x = *static_cast<Variable*>(a);
  switch (op) {
    case 0: return wrap(aops::neg(x));
    case 1: return wrap(aops::exp(x));
    case 2: return wrap(aops::log(x));
    case 3: return wrap(aops::sqrt(x));
    case 4: return wrap(aops::abs(x));
    case 5: return wrap(aops::sin(x));
    case 6: return wrap(aops::cos(x));
    case 7: return wrap(aops::tan(x));
    case 8: return wrap(aops::clamp(x, p0, p1));
    default: return nullptr;
  }
}

void* lref_reduce(int op, void* a, int axis) {
  const Variable& x = *static_cast<Variable*>(a);
  switch (op) {
    case 0: return wrap(aops::sum(x, (size_t)axis));
    case 1: return wrap(aops::max(x, (size_t)axis));
    case 2: return wrap(aops::min(x, (size_t)axis));
    default: return wrap(aops::prod(x, (size_t)axis));
  }
}

void* lref_matmul(void* a, void* b) {
  return wrap(aops::matmul(*static_cast<Variable*>(a), *static_cast<Variable*>(b)));
}
void* lref_transpose(void* a) { return wrap(aops::transpose(*static_cast<Variable*>(a))); }

void lref_backward(void* h) { static_cast<Variable*>(h)->backward(); }

// OpenMP thread count of the reference's parallel loops.  A launcher such as
// torchrun exports OMP_NUM_THREADS=1 into every rank; the CPU baseline sets
// the count explicitly to the cores the process may run on.
void lref_set_threads(int n) { omp_set_num_threads(n); }
int lref_get_threads(void) { return omp_get_max_threads(); }

void lref_set_device(int cuda) { g_device = cuda ? DeviceType::CUDA : DeviceType::CPU; }
int lref_device(void* h) { return (int)static_cast<Variable*>(h)->data().device(); }
// The thread's capture flag (lmp::tensor::lazy::set_capture_enabled): while
// set, elementwise ops on a device with a lazy backend are recorded and
// realized on first read.
void lref_set_capture(int on) { lmp::tensor::lazy::set_capture_enabled(on != 0); }

}  // extern "C"
