// Host side of the Lamp3 B200 backend: the tensor / lazy-capture / autograd
// API that the reference exposes (namespace lmp), re-implemented over the lmpb
// C ABI.  Names, argument meanings and error behaviour follow the reference's
// public interface:
//   lmp::tensor::Tensor       csrc/include/lamp3/tensor/tensor.hpp:29-102
//   lmp::tensor::ops::*       csrc/include/lamp3/tensor/native/*.hpp
//   lmp::tensor::lazy capture csrc/src/tensor/lazy/capture_mode.cpp:7-22
//   lmp::autograd::Variable   csrc/include/lamp3/autograd/variable.hpp:18-67
//   lmp::autograd::ops::*     csrc/include/lamp3/autograd/functions/*.hpp
// User errors throw std::runtime_error (LMP_CHECK, common/assert.hpp:89-90);
// CUDA/kernel failures reported by lmpb throw too, with lmpb's message.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "lmpb.h"

namespace lmp {

#define LMP_CHECK(cond, msg)                                   \
  do {                                                         \
    if (!(cond)) {                                             \
      std::ostringstream os_;                                  \
      os_ << msg;                                              \
      throw std::runtime_error(os_.str());                     \
    }                                                          \
  } while (0)

void lmpb_throw(lmpb_status st, const char* what);
#define LMPB_OK_OR_THROW(expr)                          \
  do {                                                  \
    lmpb_status st_ = (expr);                           \
    if (st_ != LMPB_OK) ::lmp::lmpb_throw(st_, #expr);  \
  } while (0)

namespace tensor {

using Scalar = double;

enum class DataType : uint8_t { Bool = 0, Int16 = 1, Int32 = 2, Int64 = 3, Float32 = 4, Float64 = 5 };
enum class DeviceType : size_t { CPU = 0, CUDA = 1 };

inline DataType type_upcast(DataType a, DataType b) {
  return static_cast<DataType>(std::max(static_cast<uint8_t>(a), static_cast<uint8_t>(b)));
}
size_t dtype_size(DataType dt);
const char* dtype_name(DataType dt);

// Raw bytes on one device.  CUDA storage comes from the stream-ordered pool
// (lmpb_malloc) and goes back to it when the last owner drops it.
struct StorageImpl {
  void* ptr = nullptr;
  size_t bytes = 0;
  DeviceType device = DeviceType::CPU;
  // set when allocated while a Graph was capturing (graph memory): false
  // once that capture was aborted, when the address was never backed
  std::shared_ptr<const bool> graph_live;
  ~StorageImpl();
};
using Storage = std::shared_ptr<StorageImpl>;
Storage make_storage(size_t bytes, DeviceType device);

struct LazyNode;

// One tensor value: realized (storage) and/or pending (lazy).  When both are
// set, the pending expression is written into the existing storage on
// realization, so a gradient buffer keeps its address across accumulation
// (csrc/tests/autograd_tests.cpp:487-499 of the reference).
struct TensorImpl {
  Storage storage;
  std::vector<size_t> shape;
  DataType dtype = DataType::Float32;
  DeviceType device = DeviceType::CPU;
  std::shared_ptr<LazyNode> lazy;

  size_t numel() const;
  bool is_deferred() const { return lazy != nullptr; }
  void* data();  // realizes if deferred
  size_t nbytes() const { return numel() * dtype_size(dtype); }
};
using ImplPtr = std::shared_ptr<TensorImpl>;

// Pending computation recorded under capture (csrc/include/lamp3/tensor/lazy/
// lazy_function.hpp:11-22).  Elementwise nodes fuse through broadcasts;
// ReduceSum (sum over the axes where the target shape is 1) fuses into the
// kernel that produces its input, as an epilogue.  Matmul (fp32) is pending
// too, so that clamp(matmul + bias) and matmul + bias realize as one GEMM
// with the bias and clamp in its epilogue; read any other way it realizes as
// a plain GEMM.
struct LazyNode {
  enum Kind { kBinary, kUnary, kConst, kReduceSum, kMatmul, kReduceMax };
  Kind kind;
  int op = 0;
  double p0 = 0.0, p1 = 0.0;  // clamp bounds / constant value
  std::vector<ImplPtr> inputs;
};

class Tensor {
 public:
  Tensor() = default;
  explicit Tensor(ImplPtr p) : impl_(std::move(p)) {}
  // Host data (converted to dtype) on `device`.
  Tensor(const std::vector<double>& data, const std::vector<size_t>& shape, DeviceType device,
         DataType dtype);
  // Raw host bytes of `src_dtype`.
  static Tensor from_host(const void* data, DataType src_dtype, const std::vector<size_t>& shape,
                          DeviceType device, DataType dtype);

  void* data();
  DataType type() const { return impl_->dtype; }
  DeviceType device() const { return impl_->device; }
  const std::vector<size_t>& shape() const { return impl_->shape; }
  std::vector<int64_t> strides() const;
  size_t numel() const { return impl_->numel(); }
  bool defined() const { return impl_ != nullptr; }

  // Copies to host memory in `dtype` (synchronises the stream).
  void read(void* dst, DataType dtype) const;
  std::vector<double> to_vector() const;
  Scalar index(const std::vector<size_t>& idx) const;

  Tensor reshape(std::vector<size_t> new_shape) const;
  Tensor squeeze(size_t dim) const;
  Tensor expand_dims(size_t dim) const;
  Tensor to(DeviceType device) const;
  void copy(const Tensor& other);
  void fill(Scalar item);
  void realize();

  const ImplPtr& impl() const { return impl_; }

 private:
  ImplPtr impl_;
};

std::ostream& operator<<(std::ostream& os, const Tensor& t);

// ---------------------------------------------------- asynchronous host I/O
//
// Host transfers on two per-device copy streams (one per direction), ordered
// against the compute stream with events, so an upload or download overlaps
// compute already queued and a download of one step overlaps the upload of
// the next (PCIe is full duplex).  Host buffers should be pinned for the
// copies to be asynchronous, and must stay valid until the copy completes.

// A pending device-to-host copy; wait() blocks until the bytes are on the
// host.  It keeps the source storage alive until then.
struct HostCopy {
  Storage keep;
  void* done = nullptr;  // cudaEvent_t
  void wait();
  ~HostCopy();
};

// New CUDA tensor filled from `data` (same dtype, contiguous) on the upload
// stream; compute queued after this call waits for the copy.
Tensor upload_async(const void* data, const std::vector<size_t>& shape, DataType dtype);
// Queue a copy of `t` (realized first) into `dst` (t's dtype, numel elements).
std::shared_ptr<HostCopy> download_async(const Tensor& t, void* dst);

// ------------------------------------------------------------ lazy capture
namespace lazy {
void set_capture_enabled(bool enabled);
bool is_capture_enabled();
bool should_capture(DeviceType device);
// RAII: capture on (or off) for a scope.
struct CaptureGuard {
  bool prev;
  explicit CaptureGuard(bool on);
  ~CaptureGuard();
};
}  // namespace lazy

// Realizes every pending tensor in `ts`, grouping those that share an
// iteration space into one multi-output kernel.
void realize_all(const std::vector<ImplPtr>& ts);

// Stream the backend launches on (default: legacy default stream).
void set_stream(void* stream);
void* current_stream();
void synchronize();

// CUDA-graph capture and replay of a repeated step (no counterpart in the
// reference, which launches and synchronises every op).  Between
// capture_begin() and capture_end() every kernel, copy, allocation and free
// the host layer issues is recorded on a private stream instead of running;
// replay() runs the recorded step again with one launch.  The recorded
// addresses are fixed, so a replayable step updates its state in place
// (Tensor::copy into the parameters, zero_grad) and reads no values on the
// host.  Memory:
//   * allocated during capture: graph memory at a fixed address, rewritten
//     by each replay (a tensor created by the captured step shows the latest
//     replay's values); freed inside the step, it is freed inside the graph;
//   * allocated before and released during capture: kept until the Graph is
//     destroyed, since every replay still reads it.
// Build every fused program once before capturing (run the step once).
class Graph {
 public:
  Graph() = default;
  ~Graph();
  Graph(const Graph&) = delete;
  Graph& operator=(const Graph&) = delete;
  void capture_begin();
  void capture_end();
  void capture_abort();  // ends a capture and discards it
  void replay();
  size_t kernels() const { return kernels_; }  // kernel nodes in the graph
  void defer_free(void* p) { deferred_.push_back(p); }
  const std::shared_ptr<bool>& live() const { return live_; }

 private:
  void* stream_ = nullptr;  // capture stream
  void* prev_ = nullptr;    // the host layer's stream before capture; replays run on it
  void* graph_ = nullptr;
  void* exec_ = nullptr;
  bool capturing_ = false;
  size_t kernels_ = 0;
  std::vector<void*> deferred_;
  std::shared_ptr<bool> live_;
};
Graph* capturing_graph();

namespace ops {
Tensor add(const Tensor& a, const Tensor& b);
Tensor sub(const Tensor& a, const Tensor& b);
Tensor mul(const Tensor& a, const Tensor& b);
Tensor div(const Tensor& a, const Tensor& b);
Tensor pow(const Tensor& a, const Tensor& b);
Tensor eq(const Tensor& a, const Tensor& b);
Tensor ne(const Tensor& a, const Tensor& b);
Tensor ge(const Tensor& a, const Tensor& b);
Tensor le(const Tensor& a, const Tensor& b);
Tensor gt(const Tensor& a, const Tensor& b);
Tensor lt(const Tensor& a, const Tensor& b);
Tensor binary(int op, const Tensor& a, const Tensor& b);

Tensor neg(const Tensor& a);
Tensor exp(const Tensor& a);
Tensor log(const Tensor& a);
Tensor sqrt(const Tensor& a);
Tensor abs(const Tensor& a);
Tensor sin(const Tensor& a);
Tensor cos(const Tensor& a);
Tensor tan(const Tensor& a);
Tensor clamp(const Tensor& a, Scalar min_val, Scalar max_val);
Tensor unary(int op, const Tensor& a, Scalar p0 = 0, Scalar p1 = 0);
Tensor abs_backward(const Tensor& input, const Tensor& grad_output);
Tensor clamp_backward(const Tensor& input, const Tensor& grad_output, Scalar min_val, Scalar max_val);

Tensor sum(const Tensor& a, size_t axis);
Tensor max(const Tensor& a, size_t axis);
Tensor min(const Tensor& a, size_t axis);
Tensor prod(const Tensor& a, size_t axis);
// Sum over the axes where `shape` is 1 (a broadcast undone); lazy under
// capture so it fuses into the producer.
Tensor sum_to_shape(const Tensor& a, const std::vector<size_t>& shape);

Tensor matmul(const Tensor& a, const Tensor& b);
Tensor transpose(const Tensor& a);

void add_inplace(Tensor& dst, const Tensor& src);
}  // namespace ops

Tensor full_like(const Tensor& t, Scalar v);
Tensor zeros_like(const Tensor& t);
Tensor ones_like(const Tensor& t);
Tensor scalar_tensor(Scalar v, DeviceType device, DataType dtype);

}  // namespace tensor

// ================================================================ autograd
namespace autograd {

using tensor::DataType;
using tensor::DeviceType;
using tensor::Scalar;
using tensor::Tensor;

void set_grad_enabled(bool enabled);
bool is_grad_enabled();

class Variable;
using variable_list = std::vector<Variable>;

// A backward function: computes the input gradients of one recorded op and
// accumulates them (csrc/include/lamp3/autograd/function.hpp).
struct Function {
  std::shared_ptr<variable_list> saved_inputs;
  virtual ~Function() = default;
  virtual void apply(const Variable& out) = 0;
};

struct VariableImpl {
  Tensor data;
  Tensor grad;
  bool requires_grad = false;
  std::shared_ptr<Function> grad_fn;
  // Called during backward() right after a kernel that accumulates directly
  // into this gradient's buffer (the matmul-gradient GEMM) has been queued on
  // the backend stream; lets a data-parallel caller start that gradient's
  // all-reduce while the rest of the backward is still running.
  std::function<void()> grad_hook;
  // The gradient is the very tensor another gradient expression produced (an
  // intermediate's first contribution is taken as is, not as 0 + g), so
  // realizing either materialises both; it must be copied before it is
  // updated in place.
  bool grad_shared = false;
};

class Variable {
 public:
  Variable() = default;
  explicit Variable(const Tensor& data, bool requires_grad = false);
  Variable(const Tensor& data, const Tensor& grad, bool requires_grad, std::shared_ptr<Function> fn);

  const Tensor& grad() const;
  const Tensor& data() const { return impl_->data; }
  std::shared_ptr<Function> grad_fn() const { return impl_->grad_fn; }
  bool requires_grad() const { return impl_->requires_grad; }
  void zero_grad();
  void incr_grad(const Tensor& g);
  void set_grad_fn(std::shared_ptr<Function> fn);
  void copy(const Variable& other);
  void fill(Scalar item);
  void realize();
  void backward();
  bool defined() const { return impl_ != nullptr; }
  const std::shared_ptr<VariableImpl>& impl() const { return impl_; }
  // raw gradient slot (for the optimizer / gemm accumulation)
  Tensor& grad_slot() { return impl_->grad; }

 private:
  std::shared_ptr<VariableImpl> impl_;
};

namespace ops {
Variable add(const Variable& a, const Variable& b);
Variable sub(const Variable& a, const Variable& b);
Variable mul(const Variable& a, const Variable& b);
Variable div(const Variable& a, const Variable& b);
Variable pow(const Variable& a, const Variable& b);
Variable eq(const Variable& a, const Variable& b);
Variable ne(const Variable& a, const Variable& b);
Variable ge(const Variable& a, const Variable& b);
Variable le(const Variable& a, const Variable& b);
Variable gt(const Variable& a, const Variable& b);
Variable lt(const Variable& a, const Variable& b);
Variable binary(int op, const Variable& a, const Variable& b);
Variable binary_scalar(int op, const Variable& a, Scalar s, bool scalar_left);

Variable neg(const Variable& a);
Variable exp(const Variable& a);
Variable log(const Variable& a);
Variable sqrt(const Variable& a);
Variable abs(const Variable& a);
Variable sin(const Variable& a);
Variable cos(const Variable& a);
Variable tan(const Variable& a);
Variable clamp(const Variable& a, Scalar min_val, Scalar max_val);

Variable sum(const Variable& a, size_t axis);
Variable max(const Variable& a, size_t axis);
Variable min(const Variable& a, size_t axis);
Variable prod(const Variable& a, size_t axis);

Variable matmul(const Variable& a, const Variable& b);
Variable transpose(const Variable& a);

Variable reshape(const Variable& a, const std::vector<size_t>& shape);
Variable squeeze(const Variable& a, size_t axis);
Variable expand_dims(const Variable& a, size_t axis);
Variable to(const Variable& a, DeviceType device);
}  // namespace ops

Variable zeros(const std::vector<size_t>& shape, bool requires_grad, DeviceType device, DataType dtype);
Variable ones(const std::vector<size_t>& shape, bool requires_grad, DeviceType device, DataType dtype);
Variable full(const std::vector<size_t>& shape, Scalar v, bool requires_grad, DeviceType device, DataType dtype);

}  // namespace autograd
}  // namespace lmp
