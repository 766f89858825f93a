// Tensor values, eager ops, lazy capture and the realization engine that
// turns captured graphs into lmpb fused programs.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <iomanip>
#include <map>
#include <mutex>
#include <unordered_map>
#include <unordered_set>

#include "lamp.hpp"

namespace lmp {

void lmpb_throw(lmpb_status st, const char* what) {
  std::ostringstream os;
  os << "lmpb error " << static_cast<int>(st) << " in " << what << ": " << lmpb_last_error();
  throw std::runtime_error(os.str());
}

namespace tensor {

namespace {
void* g_stream = nullptr;
thread_local bool t_capture = false;

int as_dt(DataType d) { return static_cast<int>(d); }

bool same_shape(const std::vector<size_t>& a, const std::vector<size_t>& b) { return a == b; }

std::vector<int64_t> to_i64(const std::vector<size_t>& s) { return std::vector<int64_t>(s.begin(), s.end()); }

void require_cuda(const Tensor& t, const char* op) {
  LMP_CHECK(t.defined(), op << ": undefined tensor");
  LMP_CHECK(t.device() == DeviceType::CUDA,
            op << ": this backend computes on CUDA tensors; move the tensor with .to(device.cuda)");
}
}  // namespace

void set_stream(void* s) { g_stream = s; }
void* current_stream() { return g_stream; }
void synchronize() {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(g_stream));
  if (e != cudaSuccess) cudaGetLastError();  // reported here, not again by the next launch
  LMP_CHECK(e == cudaSuccess, "CUDA error: " << cudaGetErrorString(e));
}

size_t dtype_size(DataType dt) {
  static const size_t s[] = {1, 2, 4, 8, 4, 8};
  return s[static_cast<int>(dt)];
}

const char* dtype_name(DataType dt) {
  static const char* n[] = {"Bool", "Int16", "Int32", "Int64", "Float32", "Float64"};
  return n[static_cast<int>(dt)];
}

StorageImpl::~StorageImpl() {
  if (!ptr) return;
  if (device != DeviceType::CUDA) {
    std::free(ptr);
    return;
  }
  if (graph_live && !*graph_live) return;  // its capture was aborted: nothing to free
  Graph* g = capturing_graph();
  if (g) {
    // a capture already invalidated (an operation that cannot be recorded
    // failed) accepts no further calls; its graph memory was never backed
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(g_stream), &cs) != cudaSuccess ||
        cs == cudaStreamCaptureStatusInvalidated) {
      cudaGetLastError();
      if (!graph_live) g->defer_free(ptr);
      return;
    }
  }
  if (g && !graph_live) {
    g->defer_free(ptr);  // captured kernels still read it on every replay
    return;
  }
  if (lmpb_free(ptr, g_stream) != LMPB_OK) cudaGetLastError();  // no stale error for the next launch check
}

Storage make_storage(size_t bytes, DeviceType device) {
  auto s = std::make_shared<StorageImpl>();
  s->bytes = bytes;
  s->device = device;
  if (bytes == 0) return s;
  if (device == DeviceType::CUDA) {
    if (Graph* g = capturing_graph()) s->graph_live = g->live();
    LMPB_OK_OR_THROW(lmpb_malloc(&s->ptr, bytes, g_stream));
  } else {
    s->ptr = std::aligned_alloc(64, (bytes + 63) / 64 * 64);
    LMP_CHECK(s->ptr, "host allocation of " << bytes << " bytes failed");
  }
  return s;
}

size_t TensorImpl::numel() const {
  size_t n = 1;
  for (size_t s : shape) n *= s;
  return n;
}

void realize_one(TensorImpl* t);

void* TensorImpl::data() {
  if (lazy) realize_one(this);
  return storage ? storage->ptr : nullptr;
}

// ------------------------------------------------------------------ Tensor

static ImplPtr new_impl(const std::vector<size_t>& shape, DataType dt, DeviceType dev, bool alloc) {
  auto p = std::make_shared<TensorImpl>();
  p->shape = shape;
  p->dtype = dt;
  p->device = dev;
  if (alloc) p->storage = make_storage(p->numel() * dtype_size(dt), dev);
  return p;
}

template <typename T>
static void host_convert(const void* src, DataType sdt, T* dst, size_t n) {
  switch (sdt) {
    case DataType::Bool: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const bool*>(src)[i]); break;
    case DataType::Int16: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const int16_t*>(src)[i]); break;
    case DataType::Int32: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const int32_t*>(src)[i]); break;
    case DataType::Int64: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const int64_t*>(src)[i]); break;
    case DataType::Float32: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const float*>(src)[i]); break;
    case DataType::Float64: for (size_t i = 0; i < n; ++i) dst[i] = static_cast<T>(static_cast<const double*>(src)[i]); break;
  }
}

static void host_cast(const void* src, DataType sdt, void* dst, DataType ddt, size_t n) {
  if (sdt == ddt) {
    std::memcpy(dst, src, n * dtype_size(sdt));
    return;
  }
  switch (ddt) {
    case DataType::Bool: host_convert(src, sdt, static_cast<bool*>(dst), n); break;
    case DataType::Int16: host_convert(src, sdt, static_cast<int16_t*>(dst), n); break;
    case DataType::Int32: host_convert(src, sdt, static_cast<int32_t*>(dst), n); break;
    case DataType::Int64: host_convert(src, sdt, static_cast<int64_t*>(dst), n); break;
    case DataType::Float32: host_convert(src, sdt, static_cast<float*>(dst), n); break;
    case DataType::Float64: host_convert(src, sdt, static_cast<double*>(dst), n); break;
  }
}

Tensor Tensor::from_host(const void* data, DataType sdt, const std::vector<size_t>& shape,
                         DeviceType device, DataType dtype) {
  ImplPtr p = new_impl(shape, dtype, device, true);
  const size_t n = p->numel();
  if (n == 0) return Tensor(p);
  if (device == DeviceType::CUDA) {
    LMPB_OK_OR_THROW(lmpb_copy(LMPB_H2D, data, as_dt(sdt), p->storage->ptr, as_dt(dtype), (int64_t)n, g_stream));
  } else {
    host_cast(data, sdt, p->storage->ptr, dtype, n);
  }
  return Tensor(p);
}

Tensor::Tensor(const std::vector<double>& data, const std::vector<size_t>& shape, DeviceType device,
               DataType dtype) {
  size_t n = 1;
  for (size_t s : shape) n *= s;
  LMP_CHECK(data.size() == n, "Tensor: data has " << data.size() << " elements, shape needs " << n);
  *this = from_host(data.data(), DataType::Float64, shape, device, dtype);
}

void* Tensor::data() { return impl_->data(); }

std::vector<int64_t> Tensor::strides() const {
  std::vector<int64_t> s(impl_->shape.size());
  int64_t acc = 1;
  for (int i = (int)s.size() - 1; i >= 0; --i) {
    s[i] = acc;
    acc *= impl_->shape[i];
  }
  return s;
}

void Tensor::read(void* dst, DataType dtype) const {
  const size_t n = numel();
  if (n == 0) return;
  void* src = impl_->data();
  if (device() == DeviceType::CUDA) {
    LMPB_OK_OR_THROW(lmpb_copy(LMPB_D2H, src, as_dt(type()), dst, as_dt(dtype), (int64_t)n, g_stream));
    synchronize();
  } else {
    host_cast(src, type(), dst, dtype, n);
  }
}

std::vector<double> Tensor::to_vector() const {
  std::vector<double> v(numel());
  read(v.data(), DataType::Float64);
  return v;
}

Scalar Tensor::index(const std::vector<size_t>& idx) const {
  LMP_CHECK(idx.size() == shape().size(), "index: expected " << shape().size() << " indices");
  size_t off = 0;
  auto st = strides();
  for (size_t i = 0; i < idx.size(); ++i) {
    LMP_CHECK(idx[i] < shape()[i], "index out of bounds");
    off += idx[i] * st[i];
  }
  double v = 0;
  char* base = static_cast<char*>(impl_->data()) + off * dtype_size(type());
  if (device() == DeviceType::CUDA) {
    LMPB_OK_OR_THROW(lmpb_copy(LMPB_D2H, base, as_dt(type()), &v, LMPB_FLOAT64, 1, g_stream));
    synchronize();
  } else {
    host_cast(base, type(), &v, DataType::Float64, 1);
  }
  return v;
}

static Tensor view_with_shape(const Tensor& t, std::vector<size_t> shape) {
  ImplPtr src = t.impl();
  src->data();  // views share realized storage
  auto p = std::make_shared<TensorImpl>();
  p->storage = src->storage;
  p->shape = std::move(shape);
  p->dtype = src->dtype;
  p->device = src->device;
  return Tensor(p);
}

Tensor Tensor::reshape(std::vector<size_t> new_shape) const {
  size_t n = 1;
  for (size_t s : new_shape) n *= s;
  LMP_CHECK(n == numel(), "Cannot reshape tensor of " << numel() << " elements into " << n);
  return view_with_shape(*this, std::move(new_shape));
}

Tensor Tensor::squeeze(size_t dim) const {
  LMP_CHECK(dim < shape().size(), "squeeze: dim out of range");
  LMP_CHECK(shape()[dim] == 1, "squeeze: dim must have size 1");
  std::vector<size_t> s = shape();
  s.erase(s.begin() + dim);
  return view_with_shape(*this, s);
}

Tensor Tensor::expand_dims(size_t dim) const {
  LMP_CHECK(dim <= shape().size(), "expand_dims: dim out of range");
  std::vector<size_t> s = shape();
  s.insert(s.begin() + dim, 1);
  return view_with_shape(*this, s);
}

Tensor Tensor::to(DeviceType device) const {
  ImplPtr out = new_impl(shape(), type(), device, true);
  const size_t n = numel();
  if (n == 0) return Tensor(out);
  void* src = impl_->data();
  int kind = this->device() == DeviceType::CPU ? (device == DeviceType::CPU ? LMPB_H2H : LMPB_H2D)
                                              : (device == DeviceType::CPU ? LMPB_D2H : LMPB_D2D);
  if (kind == LMPB_H2H) {
    std::memcpy(out->storage->ptr, src, n * dtype_size(type()));
  } else {
    LMPB_OK_OR_THROW(lmpb_copy(kind, src, as_dt(type()), out->storage->ptr, as_dt(type()), (int64_t)n, g_stream));
    if (kind == LMPB_D2H) synchronize();
  }
  return Tensor(out);
}

// True when realizing `t` straight into storage `dst` (of shape `shape`) is
// safe: every read of dst in the expression is at the index being written
// (same shape, no broadcast) and dst carries no pending value of its own.
// Below a matmul or a reduction the operands are read at other indices than
// the one written, so dst must not appear there at all.
static bool in_place_safe(const TensorImpl* t, const StorageImpl* dst, const std::vector<size_t>& shape,
                          std::unordered_set<const TensorImpl*>& seen, bool elementwise = true) {
  // a node is checked once per context (elementwise or below a matmul/reduction)
  const auto key = reinterpret_cast<const TensorImpl*>(reinterpret_cast<uintptr_t>(t) | (elementwise ? 0u : 1u));
  if (!seen.insert(key).second) return true;
  if (t->storage.get() == dst) return elementwise && !t->lazy && t->shape == shape;
  if (!t->lazy) return true;
  const bool ew = elementwise && t->lazy->kind != LazyNode::kMatmul && t->lazy->kind != LazyNode::kReduceSum &&
                  t->lazy->kind != LazyNode::kReduceMax;
  for (const auto& in : t->lazy->inputs)
    if (!in_place_safe(in.get(), dst, shape, seen, ew)) return false;
  return true;
}

void Tensor::copy(const Tensor& other) {
  LMP_CHECK(other.numel() == numel(), "copy: size mismatch");
  const ImplPtr& o = other.impl();
  if (device() == DeviceType::CUDA && other.device() == DeviceType::CUDA && o->lazy && !impl_->lazy &&
      impl_->storage && other.type() == type() && other.shape() == shape() &&
      (o->lazy->kind == LazyNode::kBinary || o->lazy->kind == LazyNode::kUnary)) {
    std::unordered_set<const TensorImpl*> seen;
    if (in_place_safe(o.get(), impl_->storage.get(), shape(), seen)) {
      // one fused kernel writes the pending elementwise value into this
      // storage (e.g. an in-place SGD update p.copy(p - lr * g))
      auto t = std::make_shared<TensorImpl>();
      t->shape = shape();
      t->dtype = type();
      t->device = DeviceType::CUDA;
      t->storage = impl_->storage;
      t->lazy = o->lazy;
      realize_all({t});
      return;
    }
  }
  void* dst = impl_->data();
  const void* src = other.impl()->data();
  const size_t n = numel();
  if (n == 0) return;
  const bool sc = other.device() == DeviceType::CUDA, dc = device() == DeviceType::CUDA;
  if (!sc && !dc) {
    host_cast(src, other.type(), dst, type(), n);
    return;
  }
  int kind = sc ? (dc ? LMPB_D2D : LMPB_D2H) : LMPB_H2D;
  LMPB_OK_OR_THROW(lmpb_copy(kind, src, as_dt(other.type()), dst, as_dt(type()), (int64_t)n, g_stream));
  if (kind == LMPB_D2H) synchronize();
}

void Tensor::fill(Scalar item) {
  void* p = impl_->data();
  if (!impl_->storage) impl_->storage = make_storage(impl_->nbytes(), device()), p = impl_->storage->ptr;
  const size_t n = numel();
  if (device() == DeviceType::CUDA) {
    LMPB_OK_OR_THROW(lmpb_fill(as_dt(type()), p, (int64_t)n, item, g_stream));
  } else {
    std::vector<double> v(n, item);
    host_cast(v.data(), DataType::Float64, p, type(), n);
  }
}

void Tensor::realize() { impl_->data(); }

// ------------------------------------------------------- CUDA graphs

namespace {
thread_local Graph* t_graph = nullptr;

void graph_check(cudaError_t e, const char* what) {
  LMP_CHECK(e == cudaSuccess, "CUDA graph " << what << ": " << cudaGetErrorString(e));
}
}  // namespace

Graph* capturing_graph() { return t_graph; }

void Graph::capture_begin() {
  LMP_CHECK(!t_graph, "a CUDA graph is already capturing on this thread");
  LMP_CHECK(!exec_, "this Graph already holds a captured step");
  cudaStream_t s = nullptr;
  graph_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
  stream_ = s;
  prev_ = g_stream;
  // the capture starts after everything already queued on the host layer's stream
  cudaEvent_t ev = nullptr;
  graph_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
  graph_check(cudaEventRecord(ev, static_cast<cudaStream_t>(prev_)), "event record");
  graph_check(cudaStreamWaitEvent(s, ev, 0), "stream wait");
  cudaEventDestroy(ev);
  graph_check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
  live_ = std::make_shared<bool>(true);
  g_stream = s;
  t_graph = this;
  capturing_ = true;
}

void Graph::capture_abort() {
  if (!capturing_) return;
  *live_ = false;
  cudaGraph_t g = nullptr;
  cudaStreamEndCapture(static_cast<cudaStream_t>(stream_), &g);
  if (g) cudaGraphDestroy(g);
  cudaGetLastError();
  g_stream = prev_;
  t_graph = nullptr;
  capturing_ = false;
}

void Graph::capture_end() {
  LMP_CHECK(capturing_ && t_graph == this, "capture_end without capture_begin");
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream_), &g);
  g_stream = prev_;
  t_graph = nullptr;
  capturing_ = false;
  if (e != cudaSuccess || !g) {
    *live_ = false;
    cudaGetLastError();
    LMP_CHECK(false, "CUDA graph capture failed (" << cudaGetErrorString(e)
                                                   << "): the step read a value on the host or used an "
                                                      "operation that cannot be captured");
  }
  graph_ = g;
  size_t n = 0;
  graph_check(cudaGraphGetNodes(g, nullptr, &n), "nodes");
  std::vector<cudaGraphNode_t> nodes(n);
  if (n) graph_check(cudaGraphGetNodes(g, nodes.data(), &n), "nodes");
  kernels_ = 0;
  for (auto& nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels_;
  }
  cudaGraphExec_t x = nullptr;
  graph_check(cudaGraphInstantiateWithFlags(&x, g, cudaGraphInstantiateFlagAutoFreeOnLaunch), "instantiate");
  exec_ = x;
}

void Graph::replay() {
  LMP_CHECK(exec_, "replay before a completed capture");
  LMP_CHECK(!t_graph, "replay while a CUDA graph is capturing");
  graph_check(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec_), static_cast<cudaStream_t>(g_stream)), "launch");
}

Graph::~Graph() {
  if (capturing_ && t_graph == this) capture_abort();
  cudaStream_t s = static_cast<cudaStream_t>(prev_);
  if (exec_) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec_));
  if (graph_) cudaGraphDestroy(static_cast<cudaGraph_t>(graph_));
  for (void* p : deferred_) cudaFreeAsync(p, s);  // after the last replay on that stream
  if (stream_) cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
}

// ---------------------------------------------------- asynchronous host I/O

namespace {
struct CopyStreams {
  cudaStream_t h2d = nullptr, d2h = nullptr;
};

CopyStreams& copy_streams() {
  static std::mutex mu;
  static std::vector<CopyStreams> per_dev;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1);
  CopyStreams& c = per_dev[dev];
  if (!c.h2d) {
    // non-blocking: no implicit ordering with the legacy default stream
    LMP_CHECK(cudaStreamCreateWithFlags(&c.h2d, cudaStreamNonBlocking) == cudaSuccess, "copy stream creation failed");
    LMP_CHECK(cudaStreamCreateWithFlags(&c.d2h, cudaStreamNonBlocking) == cudaSuccess, "copy stream creation failed");
  }
  return c;
}

cudaEvent_t new_event() {
  cudaEvent_t e;
  LMP_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess, "cudaEventCreate failed");
  return e;
}

void check_cuda(cudaError_t e, const char* what) { LMP_CHECK(e == cudaSuccess, what << ": " << cudaGetErrorString(e)); }
}  // namespace

void HostCopy::wait() {
  if (!done) return;
  check_cuda(cudaEventSynchronize(static_cast<cudaEvent_t>(done)), "download wait");
  cudaEventDestroy(static_cast<cudaEvent_t>(done));
  done = nullptr;
  keep.reset();
}

HostCopy::~HostCopy() {
  if (done) {
    cudaEventSynchronize(static_cast<cudaEvent_t>(done));
    cudaEventDestroy(static_cast<cudaEvent_t>(done));
  }
}

Tensor upload_async(const void* data, const std::vector<size_t>& shape, DataType dtype) {
  ImplPtr p = new_impl(shape, dtype, DeviceType::CUDA, true);
  const size_t bytes = p->nbytes();
  if (bytes == 0) return Tensor(p);
  CopyStreams& cs = copy_streams();
  cudaStream_t compute = static_cast<cudaStream_t>(g_stream);
  cudaEvent_t ready = new_event(), copied = new_event();
  // the allocation was ordered on the compute stream: let the copy start after it
  check_cuda(cudaEventRecord(ready, compute), "upload: record");
  check_cuda(cudaStreamWaitEvent(cs.h2d, ready, 0), "upload: wait");
  check_cuda(cudaMemcpyAsync(p->storage->ptr, data, bytes, cudaMemcpyHostToDevice, cs.h2d), "upload: copy");
  check_cuda(cudaEventRecord(copied, cs.h2d), "upload: record");
  check_cuda(cudaStreamWaitEvent(compute, copied, 0), "upload: order");
  cudaEventDestroy(ready);
  cudaEventDestroy(copied);
  return Tensor(p);
}

std::shared_ptr<HostCopy> download_async(const Tensor& t, void* dst) {
  LMP_CHECK(t.device() == DeviceType::CUDA, "download_async: CUDA tensors only");
  auto h = std::make_shared<HostCopy>();
  const size_t bytes = t.impl()->nbytes();
  void* src = t.impl()->data();
  if (bytes == 0) return h;
  CopyStreams& cs = copy_streams();
  cudaEvent_t ready = new_event();
  check_cuda(cudaEventRecord(ready, static_cast<cudaStream_t>(g_stream)), "download: record");
  check_cuda(cudaStreamWaitEvent(cs.d2h, ready, 0), "download: wait");
  check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, cs.d2h), "download: copy");
  cudaEventDestroy(ready);
  cudaEvent_t done = new_event();
  check_cuda(cudaEventRecord(done, cs.d2h), "download: record");
  h->done = done;
  h->keep = t.impl()->storage;
  return h;
}

std::ostream& operator<<(std::ostream& os, const Tensor& t) {
  os << "Tensor(dtype=" << dtype_name(t.type()) << ", device=" << (t.device() == DeviceType::CUDA ? "CUDA" : "CPU")
     << ", shape=[";
  for (size_t i = 0; i < t.shape().size(); ++i) os << (i ? ", " : "") << t.shape()[i];
  os << "], data=[";
  std::vector<double> v = t.to_vector();
  const size_t show = std::min<size_t>(v.size(), 16);
  for (size_t i = 0; i < show; ++i) os << (i ? ", " : "") << v[i];
  if (v.size() > show) os << ", ...";
  os << "])";
  return os;
}

// ------------------------------------------------------------ lazy capture

namespace lazy {
void set_capture_enabled(bool enabled) { t_capture = enabled; }
bool is_capture_enabled() { return t_capture; }
// Capture is live only where a lazy backend exists: this backend serves CUDA
// (capture_mode.cpp:20-22 of the reference).
bool should_capture(DeviceType device) { return t_capture && device == DeviceType::CUDA; }
CaptureGuard::CaptureGuard(bool on) : prev(t_capture) { t_capture = on; }
CaptureGuard::~CaptureGuard() { t_capture = prev; }
}  // namespace lazy

static ImplPtr record(LazyNode::Kind kind, int op, std::vector<ImplPtr> inputs, const std::vector<size_t>& shape,
                      DataType dt, double p0 = 0, double p1 = 0) {
  auto n = std::make_shared<LazyNode>();
  n->kind = kind;
  n->op = op;
  n->p0 = p0;
  n->p1 = p1;
  n->inputs = std::move(inputs);
  ImplPtr t = new_impl(shape, dt, DeviceType::CUDA, false);
  t->lazy = std::move(n);
  return t;
}

// --------------------------------------------------------- realization

namespace {

bool gemm_epilogue_root(const TensorImpl* t);

// Size of the pending graph under `t`, counted up to `cap`.
size_t pending_size(const TensorImpl* t, size_t cap, std::unordered_set<const TensorImpl*>& seen) {
  if (!t->lazy || !seen.insert(t).second) return 0;
  size_t n = 1;
  for (const auto& in : t->lazy->inputs) {
    if (n >= cap) break;
    n += pending_size(in.get(), cap - n, seen);
  }
  return n;
}

struct ProgramBuilder {
  std::vector<lmpb_fnode> nodes;
  std::vector<lmpb_fleaf> leaves;
  std::vector<const void*> leaf_ptrs;
  std::vector<lmpb_fout> outs;
  std::vector<void*> out_ptrs;
  std::unordered_map<const TensorImpl*, int> memo;
  std::map<std::tuple<const void*, int, std::vector<size_t>>, int> leaf_memo;
  std::string sig;  // compact binary signature of the program (cache key)
  size_t budget = 480;
  std::vector<size_t> iter;  // iteration space (when known): enables in-kernel row reductions

  template <typename T>
  void put(const T& v) {
    sig.append(reinterpret_cast<const char*>(&v), sizeof(T));
  }
  void put_shape(const std::vector<size_t>& s) {
    put((uint32_t)s.size());
    for (size_t x : s) put((uint64_t)x);
  }  // node cap per kernel; deeper graphs materialise sub-results

  int add_node(const lmpb_fnode& n) {
    nodes.push_back(n);
    sig.push_back('n');
    put(n.kind);
    put(n.sub);
    put(n.dtype);
    put(n.a);
    put(n.b);
    put(n.p0);
    put(n.p1);
    return (int)nodes.size() - 1;
  }

  int leaf(TensorImpl* t) {
    void* p = t->data();
    auto key = std::make_tuple((const void*)p, (int)t->dtype, t->shape);
    auto it = leaf_memo.find(key);
    int slot;
    if (it != leaf_memo.end()) {
      slot = it->second;
    } else {
      lmpb_fleaf lf{};
      lf.dtype = (int)t->dtype;
      lf.ndim = (int)t->shape.size();
      for (size_t i = 0; i < t->shape.size(); ++i) lf.shape[i] = (int64_t)t->shape[i];
      leaves.push_back(lf);
      leaf_ptrs.push_back(p);
      slot = (int)leaves.size() - 1;
      leaf_memo[key] = slot;
      sig.push_back('L');
      put(lf.dtype);
      put_shape(t->shape);
      sig.push_back(((uintptr_t)p & 15u) == 0 ? 'a' : 'u');
    }
    lmpb_fnode n{};
    n.kind = LMPB_FN_LEAF;
    n.dtype = (int)t->dtype;
    n.a = slot;
    return add_node(n);
  }

  // True when no realized leaf under `t` has extent > 1 on the axes that a
  // sum from shape `full` down to shape `target` reduces.
  static bool invariant_along(TensorImpl* t, const std::vector<size_t>& full, const std::vector<size_t>& target,
                              std::unordered_set<TensorImpl*>& seen) {
    if (!seen.insert(t).second) return true;
    if (!t->lazy || t->lazy->kind == LazyNode::kReduceSum || t->lazy->kind == LazyNode::kMatmul ||
        t->lazy->kind == LazyNode::kReduceMax) {
      const size_t nd = full.size();
      for (size_t k = 0; k < nd; ++k) {
        const size_t d = nd - 1 - k;
        const bool reduced = full[d] != 1 && (k >= target.size() || target[target.size() - 1 - k] == 1);
        if (!reduced) continue;
        if (k < t->shape.size() && t->shape[t->shape.size() - 1 - k] != 1) return false;
      }
      return true;
    }
    for (const auto& in : t->lazy->inputs)
      if (!invariant_along(in.get(), full, target, seen)) return false;
    return true;
  }

  // True when pending reduction `t` reduces only the last axis of this
  // program's iteration space (its input has the iteration shape).
  bool row_reduction(const TensorImpl* t) const {
    const TensorImpl* x = t->lazy->inputs[0].get();
    const size_t nd = iter.size();
    if (nd == 0 || x->shape != iter || iter[nd - 1] <= 1 || t->shape.size() != nd || t->dtype != x->dtype)
      return false;
    for (size_t d = 0; d + 1 < nd; ++d)
      if (t->shape[d] != iter[d]) return false;
    return t->shape[nd - 1] == 1;
  }

  int visit(TensorImpl* t) {
    auto it = memo.find(t);
    if (it != memo.end()) return it->second;
    int id;
    if (t->lazy && t->lazy->kind == LazyNode::kReduceSum && nodes.size() <= budget) {
      // A sum over axes its input does not vary along is that value times the
      // number of summed elements: no reduction kernel needed.
      TensorImpl* x = t->lazy->inputs[0].get();
      std::unordered_set<TensorImpl*> seen;
      if (invariant_along(x, x->shape, t->shape, seen)) {
        size_t count = 1;
        const size_t nd = x->shape.size();
        for (size_t k = 0; k < nd; ++k) {
          const size_t d = nd - 1 - k;
          if (x->shape[d] != 1 && (k >= t->shape.size() || t->shape[t->shape.size() - 1 - k] == 1)) count *= x->shape[d];
        }
        lmpb_fnode c{};
        c.kind = LMPB_FN_CONST;
        c.dtype = (int)t->dtype;
        c.p0 = (double)count;
        const int cn = add_node(c);
        lmpb_fnode m{};
        m.kind = LMPB_FN_BINARY;
        m.sub = LMPB_MUL;
        m.dtype = (int)t->dtype;
        m.a = visit(x);
        m.b = cn;
        id = add_node(m);
        memo[t] = id;
        return id;
      }
    }
    if (t->lazy && (t->lazy->kind == LazyNode::kReduceSum || t->lazy->kind == LazyNode::kReduceMax) &&
        nodes.size() <= budget && row_reduction(t)) {
      // a keep-dim sum / max over the last axis of this program's own space
      // (a softmax's max and sum): computed inside the kernel, per row
      lmpb_fnode n{};
      n.kind = LMPB_FN_ROWRED;
      n.sub = t->lazy->kind == LazyNode::kReduceMax ? LMPB_MAX : LMPB_SUM;
      n.dtype = (int)t->dtype;
      n.a = visit(t->lazy->inputs[0].get());
      id = add_node(n);
      memo[t] = id;
      return id;
    }
    // Realized first, then read as a leaf: barriers (reductions the kernel
    // cannot place, matmuls); a Linear (matmul + bias [+ clamp]), which runs
    // as one GEMM with the bias and clamp in its epilogue; an operand smaller
    // than the iteration space with a long pending history (e.g. a parameter
    // updated lazily step after step), which inlined would be recomputed for
    // every element and grow the program every step; oversize graphs.
    bool materialise = !t->lazy || t->lazy->kind == LazyNode::kReduceSum || t->lazy->kind == LazyNode::kMatmul ||
                       t->lazy->kind == LazyNode::kReduceMax || nodes.size() > budget || gemm_epilogue_root(t);
    if (!materialise && !iter.empty() && t->shape != iter) {
      std::unordered_set<const TensorImpl*> seen;
      materialise = pending_size(t, 17, seen) > 16;
    }
    if (materialise) {
      id = leaf(t);  // realizes barriers / oversize sub-graphs first
    } else {
      LazyNode& L = *t->lazy;
      lmpb_fnode n{};
      n.dtype = (int)t->dtype;
      n.p0 = L.p0;
      n.p1 = L.p1;
      if (L.kind == LazyNode::kConst) {
        n.kind = LMPB_FN_CONST;
      } else if (L.kind == LazyNode::kBinary) {
        n.kind = LMPB_FN_BINARY;
        n.sub = L.op;
        n.a = visit(L.inputs[0].get());
        n.b = visit(L.inputs[1].get());
      } else {
        n.kind = LMPB_FN_UNARY;
        n.sub = L.op;
        n.a = visit(L.inputs[0].get());
      }
      id = add_node(n);
    }
    memo[t] = id;
    return id;
  }

  // Left-to-right ADD chain over `terms` in dtype dt.
  int chain(const std::vector<ImplPtr>& terms, DataType dt) {
    int node = visit(terms[0].get());
    for (size_t i = 1; i < terms.size(); ++i) {
      lmpb_fnode n{};
      n.kind = LMPB_FN_BINARY;
      n.sub = LMPB_ADD;
      n.dtype = (int)dt;
      n.a = node;
      n.b = visit(terms[i].get());
      node = add_node(n);
    }
    return node;
  }

  void output(int node, int mode, DataType dt, const std::vector<size_t>& shape, void* ptr, int addend = -1) {
    lmpb_fout o{};
    o.node = node;
    o.mode = mode;
    o.addend = addend;
    o.dtype = (int)dt;
    o.ndim = (int)shape.size();
    for (size_t i = 0; i < shape.size(); ++i) o.shape[i] = (int64_t)shape[i];
    outs.push_back(o);
    out_ptrs.push_back(ptr);
    sig.push_back('O');
    put(node);
    put(mode);
    put(addend);
    put(o.dtype);
    put_shape(shape);
    sig.push_back(((uintptr_t)ptr & 15u) == 0 ? 'a' : 'u');
  }
};

std::mutex g_prog_mu;
std::unordered_map<std::string, lmpb_fused>& prog_cache() {
  static auto* m = new std::unordered_map<std::string, lmpb_fused>();
  return *m;
}

// Compiles (cached by program signature) and launches.  Returns the status
// of building so callers can fall back on LMPB_ERR_UNSUPPORTED.
lmpb_status run_program(ProgramBuilder& pb, const std::vector<size_t>& iter) {
  pb.sig.push_back('I');
  pb.put_shape(iter);
  const std::string& key = pb.sig;
  lmpb_fused h = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_prog_mu);
    auto it = prog_cache().find(key);
    if (it != prog_cache().end()) h = it->second;
  }
  if (!h) {
    static const bool log = getenv("LMPB_FUSED_LOG") != nullptr;
    if (log) fprintf(stderr, "[lmpb fused] new program: %zu nodes, %zu leaves, %zu outputs\n", pb.nodes.size(),
                     pb.leaves.size(), pb.outs.size());
    std::vector<int64_t> it64 = to_i64(iter);
    lmpb_status st = lmpb_fused_build(pb.nodes.data(), (int)pb.nodes.size(), pb.leaves.data(), (int)pb.leaves.size(),
                                      pb.outs.data(), (int)pb.outs.size(), it64.data(), (int)it64.size(), &h);
    if (st != LMPB_OK) return st;
    std::lock_guard<std::mutex> lk(g_prog_mu);
    prog_cache()[key] = h;
  }
  LMPB_OK_OR_THROW(lmpb_fused_launch(h, pb.leaf_ptrs.data(), pb.out_ptrs.data(), g_stream));
  return LMPB_OK;
}

// Flattens a same-dtype chain of ADDs into its terms, left to right.
void add_terms(const ImplPtr& t, DataType dt, std::vector<ImplPtr>& terms) {
  if (t->lazy && t->lazy->kind == LazyNode::kBinary && t->lazy->op == LMPB_ADD && t->dtype == dt &&
      !t->storage) {
    add_terms(t->lazy->inputs[0], dt, terms);
    add_terms(t->lazy->inputs[1], dt, terms);
  } else {
    terms.push_back(t);
  }
}

bool is_reduce_term(const ImplPtr& t) {
  return t->lazy && t->lazy->kind == LazyNode::kReduceSum && !t->storage;
}

// One output of a realization batch.
struct Request {
  std::vector<size_t> iter;
  int mode;
  ImplPtr expr;                  // expression root (for STORE / ACCUM) or reduce input
  std::vector<ImplPtr> chain;    // ADD chain of these terms instead of expr (if non-empty)
  TensorImpl* target;
  std::vector<ImplPtr> addend;   // REDUCE: elementwise terms added to the sum
};

// Sum over axes by successive keep-dim lmpb_reduce calls (the fallback of a
// reduction the fused compiler cannot place in one kernel).
ImplPtr reduce_to_shape_eager(const ImplPtr& in, const std::vector<size_t>& shape) {
  ImplPtr cur = in;
  cur->data();
  const size_t nd = cur->shape.size();
  std::vector<size_t> tgt(nd, 1);
  for (size_t k = 0; k < shape.size(); ++k) tgt[nd - 1 - k] = shape[shape.size() - 1 - k];
  for (size_t ax = 0; ax < nd; ++ax) {
    if (tgt[ax] == 1 && cur->shape[ax] != 1) {
      std::vector<size_t> os = cur->shape;
      os[ax] = 1;
      ImplPtr o = new_impl(os, cur->dtype, DeviceType::CUDA, true);
      std::vector<int64_t> s64 = to_i64(cur->shape);
      LMPB_OK_OR_THROW(lmpb_reduce(LMPB_SUM, (int)cur->dtype, cur->storage->ptr, s64.data(), (int)nd, (int)ax,
                                   o->storage->ptr, g_stream));
      cur = o;
    }
  }
  auto v = std::make_shared<TensorImpl>(*cur);
  v->shape = shape;
  return v;
}

void run_requests(std::vector<Request>& reqs) {
  // group by iteration shape, preserving first-seen order
  std::vector<std::vector<size_t>> order;
  std::map<std::vector<size_t>, std::vector<Request*>> groups;
  for (auto& r : reqs) {
    if (!groups.count(r.iter)) order.push_back(r.iter);
    groups[r.iter].push_back(&r);
  }
  for (const auto& iter : order) {
    auto& g = groups[iter];
    ProgramBuilder pb;
    pb.iter = iter;
    for (Request* r : g) {
      const int node = r->chain.empty() ? pb.visit(r->expr.get()) : pb.chain(r->chain, r->target->dtype);
      const int addend = r->addend.empty() ? -1 : pb.chain(r->addend, r->target->dtype);
      const std::vector<size_t>& oshape = (r->mode >= LMPB_OUT_REDUCE_SUM) ? r->target->shape : iter;
      pb.output(node, r->mode, r->target->dtype, oshape, r->target->storage->ptr, addend);
    }
    lmpb_status st = run_program(pb, iter);
    if (st == LMPB_ERR_UNSUPPORTED) {
      // one request at a time; reductions through materialise + lmpb_reduce
      for (Request* r : g) {
        if (r->mode < LMPB_OUT_REDUCE_SUM) {
          ProgramBuilder p1;
          p1.iter = iter;
          int node = r->chain.empty() ? p1.visit(r->expr.get()) : -1;
          if (node < 0) {
            node = p1.visit(r->chain[0].get());
            for (size_t i = 1; i < r->chain.size(); ++i) {
              lmpb_fnode n{};
              n.kind = LMPB_FN_BINARY;
              n.sub = LMPB_ADD;
              n.dtype = (int)r->target->dtype;
              n.a = node;
              n.b = p1.visit(r->chain[i].get());
              node = p1.add_node(n);
            }
          }
          p1.output(node, r->mode, r->target->dtype, iter, r->target->storage->ptr);
          LMPB_OK_OR_THROW(run_program(p1, iter));
        } else {
          if (!r->addend.empty()) {  // the elementwise part first, then accumulate the reduction
            ProgramBuilder p0;
            p0.output(p0.chain(r->addend, r->target->dtype), LMPB_OUT_STORE, r->target->dtype, r->target->shape,
                      r->target->storage->ptr);
            LMPB_OK_OR_THROW(run_program(p0, r->target->shape));
            r->mode = LMPB_OUT_REDUCE_SUM_ACCUM;
          }
          ImplPtr full = new_impl(iter, r->target->dtype, DeviceType::CUDA, true);
          ProgramBuilder p1;
          p1.iter = iter;
          const int rn = r->chain.empty() ? p1.visit(r->expr.get()) : p1.chain(r->chain, r->target->dtype);
          p1.output(rn, LMPB_OUT_STORE, full->dtype, iter, full->storage->ptr);
          LMPB_OK_OR_THROW(run_program(p1, iter));
          ImplPtr red = reduce_to_shape_eager(full, r->target->shape);
          void* dst = r->target->storage->ptr;
          const int64_t n = (int64_t)r->target->numel();
          if (r->mode == LMPB_OUT_REDUCE_SUM_ACCUM)
            LMPB_OK_OR_THROW(lmpb_add_inplace((int)r->target->dtype, dst, red->storage->ptr, n, g_stream));
          else
            LMPB_OK_OR_THROW(lmpb_copy(LMPB_D2D, red->storage->ptr, (int)red->dtype, dst, (int)r->target->dtype, n, g_stream));
        }
      }
    } else if (st != LMPB_OK) {
      lmpb_throw(st, "lmpb_fused_build");
    }
  }
}

// Writes the product of pending matmul node M (inputs A [m,k], B [k,n], fp32)
// into `dst`'s storage; with `ep_of` (the target of a matched pattern) the
// bias row and clamp of that pattern run in the GEMM's epilogue.
struct EpilogueSpec {
  TensorImpl* bias = nullptr;
  bool clamp = false;
  double lo = 0.0, hi = 0.0;
};

void run_matmul(TensorImpl* dst, TensorImpl* M, const EpilogueSpec* ep) {
  if (!M) M = dst;
  LazyNode& L = *M->lazy;
  TensorImpl* A = L.inputs[0].get();
  TensorImpl* B = L.inputs[1].get();
  const int64_t m = (int64_t)A->shape[0], k = (int64_t)A->shape[1], n = (int64_t)B->shape[1];
  const void* pa = A->data();
  const void* pb = B->data();
  const void* pbias = ep && ep->bias ? ep->bias->data() : nullptr;
  if (!dst->storage || dst->storage->bytes < dst->nbytes()) dst->storage = make_storage(dst->nbytes(), dst->device);
  float* pc = static_cast<float*>(dst->storage->ptr);
  if (ep)
    LMPB_OK_OR_THROW(lmpb_gemm_f32_bias_act(0, 0, static_cast<const float*>(pa), static_cast<const float*>(pb), pc,
                                            m, n, k, static_cast<const float*>(pbias), ep->clamp ? 1 : 0, ep->lo,
                                            ep->hi, g_stream));
  else
    LMPB_OK_OR_THROW(lmpb_matmul(LMPB_FLOAT32, pa, LMPB_FLOAT32, pb, LMPB_FLOAT32, pc, m, k, n, g_stream));
  dst->lazy = nullptr;
}

// t = clamp(M + bias, lo, hi) or t = M + bias, with M a pending fp32 matmul
// [m,n] and bias an fp32 row of n ([n] or [1,n]): one GEMM with the epilogue.
// M itself stays pending (it realizes as a plain GEMM if it is ever read).
// True when pending `t` is one of the GEMM-epilogue patterns gemm_epilogue
// realizes as one GEMM: matmul + bias row, or clamp(matmul + bias row).
bool gemm_epilogue_root(const TensorImpl* t) {
  if (!t->lazy || t->dtype != DataType::Float32 || t->shape.size() != 2 || t->storage) return false;
  const TensorImpl* add = t;
  if (t->lazy->kind == LazyNode::kUnary && t->lazy->op == LMPB_CLAMP) add = t->lazy->inputs[0].get();
  if (!add->lazy || add->storage || add->lazy->kind != LazyNode::kBinary || add->lazy->op != LMPB_ADD ||
      add->dtype != DataType::Float32 || add->shape != t->shape)
    return false;
  const size_t n = t->shape[1];
  for (int s = 0; s < 2; ++s) {
    const TensorImpl* M = add->lazy->inputs[s].get();
    const TensorImpl* b = add->lazy->inputs[1 - s].get();
    const bool row = b->shape == std::vector<size_t>{n} || b->shape == std::vector<size_t>{1, n};
    if (M->lazy && M->lazy->kind == LazyNode::kMatmul && !M->storage && M->shape == t->shape &&
        b->dtype == DataType::Float32 && row)
      return true;
  }
  return false;
}

bool gemm_epilogue(const ImplPtr& t) {
  if (t->dtype != DataType::Float32 || t->shape.size() != 2 || t->storage) return false;
  const size_t n = t->shape[1];
  EpilogueSpec ep;
  TensorImpl* add = t.get();
  if (t->lazy->kind == LazyNode::kUnary && t->lazy->op == LMPB_CLAMP) {
    ep.clamp = true;
    ep.lo = t->lazy->p0;
    ep.hi = t->lazy->p1;
    add = t->lazy->inputs[0].get();
  }
  if (!add->lazy || add->storage || add->lazy->kind != LazyNode::kBinary || add->lazy->op != LMPB_ADD ||
      add->dtype != DataType::Float32 || add->shape != t->shape)
    return false;
  for (int s = 0; s < 2; ++s) {
    TensorImpl* M = add->lazy->inputs[s].get();
    TensorImpl* b = add->lazy->inputs[1 - s].get();
    const bool row = b->shape == std::vector<size_t>{n} || b->shape == std::vector<size_t>{1, n};
    if (M->lazy && M->lazy->kind == LazyNode::kMatmul && !M->storage && M->shape == t->shape &&
        b->dtype == DataType::Float32 && row) {
      ep.bias = b;
      run_matmul(t.get(), M, &ep);
      return true;
    }
  }
  return false;
}

}  // namespace

// Realizes a batch of pending tensors.  A pending tensor whose expression is
// an ADD chain containing ReduceSum terms (a gradient receiving contributions
// through broadcast ops) is split: the elementwise terms are stored in one
// pass, each reduction is accumulated as the epilogue of the kernel that
// walks its (larger) iteration space — which is usually the same kernel that
// produces another gradient, so every input is read once.
void realize_all(const std::vector<ImplPtr>& ts) {
  std::vector<ImplPtr> pending;
  std::unordered_set<TensorImpl*> seen;
  for (const auto& t : ts)
    if (t && t->lazy && seen.insert(t.get()).second) pending.push_back(t);
  if (pending.empty()) return;
  std::vector<Request> reqs;
  std::vector<ImplPtr> done;  // keep lazy graphs alive until the kernels are queued
  for (const ImplPtr& t : pending) {
    const size_t n = t->numel();
    std::shared_ptr<LazyNode> L = t->lazy;
    // (before storage is attached: a target that already has storage is a
    // pending accumulation, which the fused GEMM must not overwrite)
    if (n > 0 && gemm_epilogue(t)) continue;
    if (!t->storage || t->storage->bytes < t->nbytes()) t->storage = make_storage(t->nbytes(), t->device);
    if (n == 0) {
      t->lazy = nullptr;
      continue;
    }
    if (L->kind == LazyNode::kConst) {
      LMPB_OK_OR_THROW(lmpb_fill((int)t->dtype, t->storage->ptr, (int64_t)n, L->p0, g_stream));
      t->lazy = nullptr;
      continue;
    }
    if (L->kind == LazyNode::kMatmul) {
      run_matmul(t.get(), nullptr, nullptr);
      continue;
    }
    if (L->kind == LazyNode::kReduceMax) {  // read on its own: the eager kernel
      TensorImpl* x = L->inputs[0].get();
      const void* px = x->data();
      std::vector<int64_t> s64 = to_i64(x->shape);
      LMPB_OK_OR_THROW(lmpb_reduce(LMPB_MAX, (int)x->dtype, px, s64.data(), (int)s64.size(), (int)s64.size() - 1,
                                   t->storage->ptr, g_stream));
      t->lazy = nullptr;
      continue;
    }
    if (L->kind == LazyNode::kReduceSum) {
      reqs.push_back({L->inputs[0]->shape, LMPB_OUT_REDUCE_SUM, L->inputs[0], {}, t.get()});
      done.push_back(t);
      continue;
    }
    std::vector<ImplPtr> terms;
    if (L->kind == LazyNode::kBinary && L->op == LMPB_ADD) {
      add_terms(L->inputs[0], t->dtype, terms);
      add_terms(L->inputs[1], t->dtype, terms);
    }
    bool has_reduce = false;
    for (auto& x : terms) has_reduce |= is_reduce_term(x);
    if (!has_reduce) {
      reqs.push_back({t->shape, LMPB_OUT_STORE, t, {}, t.get()});
      done.push_back(t);
      continue;
    }
    std::vector<ImplPtr> elem, red;
    for (auto& x : terms) (is_reduce_term(x) ? red : elem).push_back(x);
    bool one_space = true;
    for (auto& x : red) one_space &= x->lazy->inputs[0]->shape == red[0]->lazy->inputs[0]->shape;
    if (one_space) {
      // target = (elementwise terms) + sum(reduce inputs): one output of the
      // kernel that walks the reduce inputs' iteration space
      std::vector<ImplPtr> ins;
      for (auto& x : red) ins.push_back(x->lazy->inputs[0]);
      Request rq{ins[0]->shape, LMPB_OUT_REDUCE_SUM, nullptr, ins, t.get(), elem};
      reqs.push_back(rq);
      done.push_back(t);
      continue;
    }
    // The elementwise part must not be ordered after the reductions when it
    // overwrites the target: give the target its elementwise value first
    // (zero-filled when there is none), then accumulate every reduction.
    if (elem.empty()) {
      LMPB_OK_OR_THROW(lmpb_fill((int)t->dtype, t->storage->ptr, (int64_t)n, 0.0, g_stream));
    } else {
      std::vector<Request> first{{t->shape, LMPB_OUT_STORE, nullptr, elem, t.get()}};
      bool reads_target = false;
      for (auto& x : elem) reads_target |= (!x->lazy && x->storage == t->storage);
      if (reads_target) {
        reqs.push_back(first[0]);  // order-free: it reads the target it rewrites
      } else {
        run_requests(first);
      }
    }
    for (auto& x : red)
      reqs.push_back({x->lazy->inputs[0]->shape, LMPB_OUT_REDUCE_SUM_ACCUM, x->lazy->inputs[0], {}, t.get()});
    done.push_back(t);
  }
  run_requests(reqs);
  for (const ImplPtr& t : done) t->lazy = nullptr;
}

void realize_one(TensorImpl* t) {
  // wrap without ownership: t is alive for the duration of the call
  ImplPtr p(t, [](TensorImpl*) {});
  realize_all({p});
}

// ------------------------------------------------------------------- ops

namespace ops {

static std::vector<size_t> bcast(const Tensor& a, const Tensor& b) {
  std::vector<int64_t> as = to_i64(a.shape()), bs = to_i64(b.shape());
  int64_t out[LMPB_MAX_DIMS];
  int nd = 0;
  lmpb_status st = lmpb_broadcast_shape(as.data(), (int)as.size(), bs.data(), (int)bs.size(), out, &nd);
  LMP_CHECK(st == LMPB_OK, lmpb_last_error());
  return std::vector<size_t>(out, out + nd);
}

Tensor binary(int op, const Tensor& a, const Tensor& b) {
  LMP_CHECK(a.device() == b.device(), "Tensors are on different devices");
  require_cuda(a, "binary op");
  const std::vector<size_t> shape = bcast(a, b);
  const DataType dt = type_upcast(a.type(), b.type());
  if (lazy::should_capture(a.device())) return Tensor(record(LazyNode::kBinary, op, {a.impl(), b.impl()}, shape, dt));
  ImplPtr out = new_impl(shape, dt, DeviceType::CUDA, true);
  std::vector<int64_t> as = to_i64(a.shape()), bs = to_i64(b.shape());
  const void* pa = a.impl()->data();
  const void* pb = b.impl()->data();
  LMPB_OK_OR_THROW(lmpb_binary(op, (int)dt, pa, (int)a.type(), as.data(), (int)as.size(), pb, (int)b.type(),
                               bs.data(), (int)bs.size(), out->storage->ptr, 0.0, 0.0, g_stream));
  return Tensor(out);
}

Tensor add(const Tensor& a, const Tensor& b) { return binary(LMPB_ADD, a, b); }
Tensor sub(const Tensor& a, const Tensor& b) { return binary(LMPB_SUB, a, b); }
Tensor mul(const Tensor& a, const Tensor& b) { return binary(LMPB_MUL, a, b); }
Tensor div(const Tensor& a, const Tensor& b) { return binary(LMPB_DIV, a, b); }
Tensor pow(const Tensor& a, const Tensor& b) { return binary(LMPB_POW, a, b); }
Tensor eq(const Tensor& a, const Tensor& b) { return binary(LMPB_EQ, a, b); }
Tensor ne(const Tensor& a, const Tensor& b) { return binary(LMPB_NE, a, b); }
Tensor ge(const Tensor& a, const Tensor& b) { return binary(LMPB_GE, a, b); }
Tensor le(const Tensor& a, const Tensor& b) { return binary(LMPB_LE, a, b); }
Tensor gt(const Tensor& a, const Tensor& b) { return binary(LMPB_GT, a, b); }
Tensor lt(const Tensor& a, const Tensor& b) { return binary(LMPB_LT, a, b); }

Tensor unary(int op, const Tensor& a, Scalar p0, Scalar p1) {
  require_cuda(a, "unary op");
  if (lazy::should_capture(a.device()))
    return Tensor(record(LazyNode::kUnary, op, {a.impl()}, a.shape(), a.type(), p0, p1));
  ImplPtr out = new_impl(a.shape(), a.type(), DeviceType::CUDA, true);
  const void* pa = a.impl()->data();
  LMPB_OK_OR_THROW(lmpb_unary(op, (int)a.type(), pa, out->storage->ptr, (int64_t)a.numel(), p0, p1, g_stream));
  return Tensor(out);
}

Tensor neg(const Tensor& a) { return unary(LMPB_NEG, a); }
Tensor exp(const Tensor& a) { return unary(LMPB_EXP, a); }
Tensor log(const Tensor& a) { return unary(LMPB_LOG, a); }
Tensor sqrt(const Tensor& a) { return unary(LMPB_SQRT, a); }
Tensor abs(const Tensor& a) { return unary(LMPB_ABS, a); }
Tensor sin(const Tensor& a) { return unary(LMPB_SIN, a); }
Tensor cos(const Tensor& a) { return unary(LMPB_COS, a); }
Tensor tan(const Tensor& a) { return unary(LMPB_TAN, a); }
Tensor clamp(const Tensor& a, Scalar lo, Scalar hi) { return unary(LMPB_CLAMP, a, lo, hi); }

static Tensor backward_kernel(int op, const Tensor& x, const Tensor& g, Scalar lo, Scalar hi, const char* name) {
  LMP_CHECK(x.device() == g.device(), name << " requires tensors on the same device");
  LMP_CHECK(x.shape() == g.shape(), name << " requires tensors with identical shapes");
  LMP_CHECK(x.type() == g.type(), name << " requires tensors with identical dtypes");
  require_cuda(x, name);
  if (lazy::should_capture(x.device()))
    return Tensor(record(LazyNode::kBinary, op, {x.impl(), g.impl()}, x.shape(), x.type(), lo, hi));
  ImplPtr out = new_impl(x.shape(), x.type(), DeviceType::CUDA, true);
  std::vector<int64_t> s = to_i64(x.shape());
  const void* px = x.impl()->data();
  const void* pg = g.impl()->data();
  LMPB_OK_OR_THROW(lmpb_binary(op, (int)x.type(), px, (int)x.type(), s.data(), (int)s.size(), pg, (int)g.type(),
                               s.data(), (int)s.size(), out->storage->ptr, lo, hi, g_stream));
  return Tensor(out);
}

Tensor abs_backward(const Tensor& x, const Tensor& g) { return backward_kernel(LMPB_ABS_BACKWARD, x, g, 0, 0, "abs_backward"); }
Tensor clamp_backward(const Tensor& x, const Tensor& g, Scalar lo, Scalar hi) {
  return backward_kernel(LMPB_CLAMP_BACKWARD, x, g, lo, hi, "clamp_backward");
}

static Tensor reduce(int op, const Tensor& a, size_t axis) {
  require_cuda(a, "reduction");
  LMP_CHECK(axis < a.shape().size(), "reduction axis " << axis << " out of range for " << a.shape().size() << " dims");
  std::vector<size_t> os = a.shape();
  os[axis] = 1;
  ImplPtr out = new_impl(os, a.type(), DeviceType::CUDA, true);
  std::vector<int64_t> s = to_i64(a.shape());
  const void* pa = a.impl()->data();
  LMPB_OK_OR_THROW(lmpb_reduce(op, (int)a.type(), pa, s.data(), (int)s.size(), (int)axis, out->storage->ptr, g_stream));
  return Tensor(out);
}

// Under capture a float sum or max over the last axis stays pending, so that
// the kernel reading it computes it per row (softmax: max, exp, sum, divide
// and what follows in one pass); read on its own it runs the same row walk
// and tree as the eager kernel (equal bit for bit).
static bool lazy_row_reduction(const Tensor& a, size_t axis) {
  return a.device() == DeviceType::CUDA && lazy::should_capture(a.device()) && axis + 1 == a.shape().size() &&
         a.shape()[axis] > 1 && (a.type() == DataType::Float32 || a.type() == DataType::Float64);
}

Tensor sum(const Tensor& a, size_t axis) {
  if (lazy_row_reduction(a, axis)) {
    std::vector<size_t> os = a.shape();
    os[axis] = 1;
    return Tensor(record(LazyNode::kReduceSum, LMPB_SUM, {a.impl()}, os, a.type()));
  }
  return reduce(LMPB_SUM, a, axis);
}
Tensor max(const Tensor& a, size_t axis) {
  if (lazy_row_reduction(a, axis)) {
    std::vector<size_t> os = a.shape();
    os[axis] = 1;
    return Tensor(record(LazyNode::kReduceMax, LMPB_MAX, {a.impl()}, os, a.type()));
  }
  return reduce(LMPB_MAX, a, axis);
}
Tensor min(const Tensor& a, size_t axis) { return reduce(LMPB_MIN, a, axis); }
Tensor prod(const Tensor& a, size_t axis) { return reduce(LMPB_PROD, a, axis); }

Tensor sum_to_shape(const Tensor& a, const std::vector<size_t>& shape) {
  if (a.shape() == shape) return a;
  require_cuda(a, "sum_to_shape");
  ImplPtr t = record(LazyNode::kReduceSum, LMPB_SUM, {a.impl()}, shape, a.type());
  if (!lazy::should_capture(a.device())) t->data();
  return Tensor(t);
}

Tensor matmul(const Tensor& a, const Tensor& b) {
  LMP_CHECK(a.device() == b.device(), "Tensors must be on the same device");
  require_cuda(a, "matmul");
  LMP_CHECK(a.shape().size() == 2 && b.shape().size() == 2, "matmul expects 2-D tensors");
  LMP_CHECK(a.shape()[1] == b.shape()[0], "matmul: inner dimensions " << a.shape()[1] << " and " << b.shape()[0] << " differ");
  const size_t m = a.shape()[0], k = a.shape()[1], n = b.shape()[1];
  const DataType dt = type_upcast(a.type(), b.type());
  if (lazy::should_capture(a.device()) && a.type() == DataType::Float32 && b.type() == DataType::Float32)
    return Tensor(record(LazyNode::kMatmul, 0, {a.impl(), b.impl()}, {m, n}, dt));
  ImplPtr out = new_impl({m, n}, dt, DeviceType::CUDA, true);
  const void* pa = a.impl()->data();
  const void* pb = b.impl()->data();
  LMPB_OK_OR_THROW(lmpb_matmul((int)dt, pa, (int)a.type(), pb, (int)b.type(), out->storage->ptr, (int64_t)m,
                               (int64_t)k, (int64_t)n, g_stream));
  return Tensor(out);
}

Tensor transpose(const Tensor& a) {
  require_cuda(a, "transpose");
  LMP_CHECK(a.shape().size() == 2, "transpose expects a 2-D tensor");
  const size_t m = a.shape()[0], n = a.shape()[1];
  ImplPtr out = new_impl({n, m}, a.type(), DeviceType::CUDA, true);
  const void* pa = a.impl()->data();
  LMPB_OK_OR_THROW(lmpb_transpose((int)a.type(), pa, out->storage->ptr, (int64_t)m, (int64_t)n, g_stream));
  return Tensor(out);
}

void add_inplace(Tensor& dst, const Tensor& src) {
  LMP_CHECK(dst.shape() == src.shape() && dst.type() == src.type(), "add_inplace: shape/dtype mismatch");
  require_cuda(dst, "add_inplace");
  void* d = dst.impl()->data();
  const void* s = src.impl()->data();
  LMPB_OK_OR_THROW(lmpb_add_inplace((int)dst.type(), d, s, (int64_t)dst.numel(), g_stream));
}

}  // namespace ops

Tensor full_like(const Tensor& t, Scalar v) {
  if (t.device() == DeviceType::CUDA) return Tensor(record(LazyNode::kConst, 0, {}, t.shape(), t.type(), v));
  Tensor out(new_impl(t.shape(), t.type(), DeviceType::CPU, true));
  out.fill(v);
  return out;
}
Tensor zeros_like(const Tensor& t) { return full_like(t, 0.0); }
Tensor ones_like(const Tensor& t) { return full_like(t, 1.0); }

Tensor scalar_tensor(Scalar v, DeviceType device, DataType dtype) {
  if (device == DeviceType::CUDA) return Tensor(record(LazyNode::kConst, 0, {}, {1}, dtype, v));
  return Tensor(std::vector<double>{v}, {1}, device, dtype);
}

}  // namespace tensor
}  // namespace lmp
