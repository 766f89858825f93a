// pybind11 module rushlite_b200._C — the same names as the reference's
// rushlite._C (csrc/bindings/core.cpp:21-36): dtype/device enums, _Tensor,
// Variable with operator overloads, op functions, constructors, capture and
// grad-mode flags and the cuda submodule.  Additive: Variable/_Tensor accept
// NumPy arrays (buffer protocol) and expose .numpy(); a cuda.set_stream hook
// lets the backend share a stream with other CUDA libraries.
#include <cuda_runtime.h>
#include <pybind11/numpy.h>
#include <pybind11/operators.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <random>

#include "lamp.hpp"

namespace py = pybind11;
using lmp::autograd::Variable;
using lmp::tensor::DataType;
using lmp::tensor::DeviceType;
using lmp::tensor::Scalar;
using lmp::tensor::Tensor;
namespace aops = lmp::autograd::ops;
namespace tops = lmp::tensor::ops;

namespace {

constexpr DeviceType kDefaultDevice = DeviceType::CUDA;
constexpr DataType kDefaultDtype = DataType::Float32;

DataType np_dtype(const py::dtype& d) {
  switch (d.kind()) {
    case 'b': return DataType::Bool;
    case 'i':
    case 'u':
      if (d.itemsize() == 2) return DataType::Int16;
      if (d.itemsize() == 4) return DataType::Int32;
      if (d.itemsize() == 8) return DataType::Int64;
      break;
    case 'f':
      if (d.itemsize() == 4) return DataType::Float32;
      if (d.itemsize() == 8) return DataType::Float64;
      break;
  }
  throw py::value_error("Rushlite: unsupported array dtype");
}

py::dtype to_np(DataType d) {
  switch (d) {
    case DataType::Bool: return py::dtype::of<bool>();
    case DataType::Int16: return py::dtype::of<int16_t>();
    case DataType::Int32: return py::dtype::of<int32_t>();
    case DataType::Int64: return py::dtype::of<int64_t>();
    case DataType::Float32: return py::dtype::of<float>();
    default: return py::dtype::of<double>();
  }
}

// flatten_sequence (csrc/bindings/variable.hpp:21-48)
void flatten(const py::handle& node, std::vector<Scalar>& data, std::vector<size_t>& shape, size_t depth) {
  if (py::isinstance<py::sequence>(node) && !py::isinstance<py::str>(node) && !py::isinstance<py::bytes>(node)) {
    auto seq = py::reinterpret_borrow<py::sequence>(node);
    const size_t n = seq.size();
    if (depth == shape.size()) {
      if (!data.empty()) throw py::value_error("Rushlite: array must be uniform");
      shape.push_back(n);
    } else if (shape[depth] != n) {
      throw py::value_error("Rushlite: array must be uniform");
    }
    for (const auto& item : seq) flatten(item, data, shape, depth + 1);
  } else {
    if (depth != shape.size()) throw py::value_error("Rushlite: array must be uniform");
    try {
      data.push_back(node.cast<Scalar>());
    } catch (const py::cast_error&) {
      throw py::value_error("Rushlite: invalid input type");
    }
  }
}

Tensor tensor_from_py(const py::object& data, DeviceType device, DataType dtype) {
  if (py::isinstance<py::array>(data)) {
    py::array arr = py::array::ensure(data, py::array::c_style);
    DataType sdt = np_dtype(arr.dtype());
    std::vector<size_t> shape(arr.shape(), arr.shape() + arr.ndim());
    return Tensor::from_host(arr.data(), sdt, shape, device, dtype);
  }
  std::vector<Scalar> flat;
  std::vector<size_t> shape;
  flatten(data, flat, shape, 0);
  return Tensor(flat, shape, device, dtype);
}

// Copies to host; with `out` (a C-contiguous array of the tensor's size,
// e.g. a view of pinned memory) the copy lands there without a new buffer.
py::array to_numpy(const Tensor& t, py::object out_obj = py::none()) {
  if (!out_obj.is_none()) {
    py::array out = py::reinterpret_borrow<py::array>(out_obj);
    if (!(out.flags() & py::array::c_style) || (size_t)out.size() != t.numel())
      throw py::value_error("numpy(out=...): need a C-contiguous array with the tensor's element count");
    t.read(out.mutable_data(), np_dtype(out.dtype()));
    return out;
  }
  std::vector<py::ssize_t> shape(t.shape().begin(), t.shape().end());
  py::array out(to_np(t.type()), shape);
  t.read(out.mutable_data(), t.type());
  return out;
}

std::mt19937_64& rng() {
  static std::mt19937_64 g{std::random_device{}()};
  return g;
}

size_t count(const std::vector<size_t>& shape) {
  size_t n = shape.empty() ? 0 : 1;
  for (size_t s : shape) n *= s;
  return n;
}

Variable bin_vs(int op, const Variable& a, Scalar s) { return aops::binary_scalar(op, a, s, false); }
Variable bin_sv(int op, Scalar s, const Variable& a) { return aops::binary_scalar(op, a, s, true); }
Tensor tbin_ts(int op, const Tensor& a, Scalar s) { return tops::binary(op, a, lmp::tensor::scalar_tensor(s, a.device(), a.type())); }
Tensor tbin_st(int op, Scalar s, const Tensor& a) { return tops::binary(op, lmp::tensor::scalar_tensor(s, a.device(), a.type()), a); }

std::string repr_var(const Variable& v) {
  std::ostringstream os;
  os << "Variable(requires_grad=" << v.requires_grad() << ", data=" << v.data();
  if (v.requires_grad()) os << ", grad=" << v.grad();
  os << ")";
  return os.str();
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "Lamp3 API on the B200 (sm_100a) backend";

  py::enum_<DataType>(m, "dtype")
      .value("float32", DataType::Float32)
      .value("float64", DataType::Float64)
      .value("bool", DataType::Bool)
      .value("int16", DataType::Int16)
      .value("int32", DataType::Int32)
      .value("int64", DataType::Int64)
      .export_values();
  py::enum_<DeviceType>(m, "device").value("cpu", DeviceType::CPU).value("cuda", DeviceType::CUDA);

  auto cuda = m.def_submodule("cuda");
  cuda.def("sync", []() { cudaDeviceSynchronize(); });
  cuda.def("is_available", []() {
    int n = 0;
    return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
  });
  cuda.def("device_name", []() {
    cudaDeviceProp p{};
    int d = 0;
    cudaGetDevice(&d);
    cudaGetDeviceProperties(&p, d);
    return std::string(p.name);
  });
  cuda.def("set_device", [](int d) {
    cudaError_t e = cudaSetDevice(d);
    if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
  });
  cuda.def("set_stream", [](uintptr_t s) { lmp::tensor::set_stream(reinterpret_cast<void*>(s)); },
           "Launch on this cudaStream_t (an integer handle, 0 = legacy default stream).");
  cuda.def("current_stream", []() { return reinterpret_cast<uintptr_t>(lmp::tensor::current_stream()); });
  cuda.def("synchronize", []() { lmp::tensor::synchronize(); });
  cuda.def("kernel_launches", []() { return lmpb_kernel_launches(); },
           "Kernels launched by the backend library so far in this process.");
  py::class_<lmp::tensor::Graph>(cuda, "Graph",
                                 "CUDA-graph capture of a step: `with g:` records it (nothing runs), "
                                 "g.replay() runs it again with one launch.  The step must update state in "
                                 "place and read no values on the host; run it once before capturing.")
      .def(py::init<>())
      .def("capture_begin", &lmp::tensor::Graph::capture_begin)
      .def("capture_end", &lmp::tensor::Graph::capture_end)
      .def("replay", &lmp::tensor::Graph::replay, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("kernels", &lmp::tensor::Graph::kernels)
      .def("__enter__", [](lmp::tensor::Graph& g) -> lmp::tensor::Graph& {
             g.capture_begin();
             return g;
           }, py::return_value_policy::reference)
      .def("capture_abort", &lmp::tensor::Graph::capture_abort)
      .def("__exit__", [](lmp::tensor::Graph& g, py::object exc_type, py::object, py::object) {
        if (exc_type.is_none()) g.capture_end();
        else g.capture_abort();  // let the step's own exception propagate
        return false;
      });

  py::class_<lmp::tensor::HostCopy, std::shared_ptr<lmp::tensor::HostCopy>>(m, "_HostCopy")
      .def("wait", &lmp::tensor::HostCopy::wait, py::call_guard<py::gil_scoped_release>(),
           "Block until the download has landed in host memory.");

  // Asynchronous host I/O (additive): overlap PCIe transfers with compute.
  m.def("upload", [](py::array arr, bool requires_grad) {
        py::array a = py::array::ensure(arr, py::array::c_style);
        std::vector<size_t> shape(a.shape(), a.shape() + a.ndim());
        return Variable(lmp::tensor::upload_async(a.data(), shape, np_dtype(a.dtype())), requires_grad);
      }, py::arg("array"), py::arg("requires_grad") = false,
      "CUDA Variable with the array's dtype, copied on the upload stream; later ops wait for it. "
      "Pass pinned memory for an asynchronous copy; keep the array alive and unchanged until then.");

  // ----------------------------------------------------------- _Tensor
  auto tcls = py::class_<Tensor>(m, "_Tensor")
      .def(py::init<const std::vector<double>&, const std::vector<size_t>&, DeviceType, DataType>(),
           py::arg("data"), py::arg("shape"), py::arg("device"), py::arg("dtype"))
      .def(py::init([](py::array a, DeviceType device, DataType dtype) { return tensor_from_py(a, device, dtype); }),
           py::arg("array"), py::arg("device") = kDefaultDevice, py::arg("dtype") = kDefaultDtype)
      .def_property_readonly("shape", &Tensor::shape)
      .def_property_readonly("device", &Tensor::device)
      .def_property_readonly("dtype", &Tensor::type)
      .def("index", &Tensor::index, py::arg("idx"))
      .def("reshape", &Tensor::reshape, py::arg("new_shape"))
      .def("squeeze", &Tensor::squeeze, py::arg("dim"))
      .def("expand_dims", &Tensor::expand_dims, py::arg("dim"))
      .def("to", &Tensor::to, py::arg("device"))
      .def("copy", &Tensor::copy, py::arg("other"))
      .def("fill", &Tensor::fill, py::arg("item"))
      .def("realize", &Tensor::realize)
      .def("tolist", [](const Tensor& t) { return t.to_vector(); })
      .def("numpy", [](const Tensor& t, py::object out) { return to_numpy(t, out); }, py::arg("out") = py::none())
      .def("download_async", [](const Tensor& t, py::array out) {
             if (!(out.flags() & py::array::c_style) || (size_t)out.size() != t.numel() || np_dtype(out.dtype()) != t.type())
               throw py::value_error("download_async: need a C-contiguous array of the tensor's dtype and size");
             return lmp::tensor::download_async(t, out.mutable_data());
           }, py::arg("out"), py::keep_alive<0, 2>(),
           "Queue a copy into `out` on the download stream; returns a handle whose wait() blocks until it lands.")
      .def("data_ptr", [](Tensor& t) { return reinterpret_cast<uintptr_t>(t.data()); })
      // zero-copy view for other CUDA libraries (torch.as_tensor, NCCL through torch.distributed);
      // realizes the tensor; work on it is ordered on the backend's stream
      .def_property_readonly("__cuda_array_interface__", [](Tensor& t) {
        if (t.device() != DeviceType::CUDA) throw py::attribute_error("not a CUDA tensor");
        static const char* ts[] = {"|b1", "<i2", "<i4", "<i8", "<f4", "<f8"};
        py::tuple shape(t.shape().size());
        for (size_t i = 0; i < t.shape().size(); ++i) shape[i] = t.shape()[i];
        py::dict d;
        d["shape"] = shape;
        d["typestr"] = ts[static_cast<int>(t.type())];
        d["data"] = py::make_tuple(reinterpret_cast<uintptr_t>(t.data()), false);
        d["version"] = 3;
        d["strides"] = py::none();
        uintptr_t s = reinterpret_cast<uintptr_t>(lmp::tensor::current_stream());
        d["stream"] = s == 0 ? py::object(py::int_(1)) : py::object(py::int_(s));  // 1 = legacy default stream
        return d;
      })
      .def("__repr__", [](const Tensor& t) {
        std::ostringstream os;
        os << t;
        return os.str();
      })
      .def("__neg__", [](const Tensor& a) { return tops::neg(a); });
#define LMP_T_OP(PY, OPC)                                                                    \
  tcls.def(PY, [](const Tensor& a, const Tensor& b) { return tops::binary(OPC, a, b); })     \
      .def(PY, [](const Tensor& a, Scalar s) { return tbin_ts(OPC, a, s); });
#define LMP_T_ROP(PY, OPC) tcls.def(PY, [](const Tensor& a, Scalar s) { return tbin_st(OPC, s, a); });
  LMP_T_OP("__add__", LMPB_ADD) LMP_T_ROP("__radd__", LMPB_ADD)
  LMP_T_OP("__sub__", LMPB_SUB) LMP_T_ROP("__rsub__", LMPB_SUB)
  LMP_T_OP("__mul__", LMPB_MUL) LMP_T_ROP("__rmul__", LMPB_MUL)
  LMP_T_OP("__truediv__", LMPB_DIV) LMP_T_ROP("__rtruediv__", LMPB_DIV)
  LMP_T_OP("__eq__", LMPB_EQ) LMP_T_OP("__ne__", LMPB_NE) LMP_T_OP("__lt__", LMPB_LT)
  LMP_T_OP("__le__", LMPB_LE) LMP_T_OP("__gt__", LMPB_GT) LMP_T_OP("__ge__", LMPB_GE)

  // ---------------------------------------------------------- Variable
  auto vcls = py::class_<Variable>(m, "Variable")
      .def(py::init<Tensor, bool>(), py::arg("data"), py::arg("requires_grad") = false)
      .def(py::init([](const py::object& data, bool rg, DeviceType device, DataType dtype) {
             return Variable(tensor_from_py(data, device, dtype), rg);
           }),
           py::arg("data"), py::arg("requires_grad") = false, py::arg("device") = kDefaultDevice,
           py::arg("dtype") = kDefaultDtype)
      .def_property_readonly("data", &Variable::data)
      .def_property_readonly("grad", &Variable::grad)
      .def_property_readonly("grad_fn", [](const Variable& v) -> py::object {
        return v.grad_fn() ? py::cast(std::string("<backward>")) : py::none();
      })
      .def_property_readonly("requires_grad", &Variable::requires_grad)
      .def_property_readonly("shape", [](const Variable& v) { return v.data().shape(); })
      .def_property_readonly("device", [](const Variable& v) { return v.data().device(); })
      .def_property_readonly("dtype", [](const Variable& v) { return v.data().type(); })
      .def_property_readonly("ndim", [](const Variable& v) { return v.data().shape().size(); })
      .def("backward", &Variable::backward, py::call_guard<py::gil_scoped_release>())
      .def("tolist", [](const Variable& v) { return v.data().to_vector(); })
      .def("numpy", [](const Variable& v, py::object out) { return to_numpy(v.data(), out); }, py::arg("out") = py::none())
      .def("zero_grad", &Variable::zero_grad)
      .def("realize", &Variable::realize)
      .def("set_grad_hook", [](Variable& v, py::object fn) {
             if (fn.is_none()) {
               v.impl()->grad_hook = nullptr;
               return;
             }
             auto f = std::make_shared<py::object>(fn);
             v.impl()->grad_hook = [f]() {
               py::gil_scoped_acquire gil;
               (*f)();
             };
           }, py::arg("fn"),
           "fn() runs during backward() as soon as a kernel writing this Variable's gradient "
           "(the matmul-gradient GEMM) is queued; None removes it.")
      .def("__repr__", &repr_var)
      .def("__neg__", [](const Variable& a) { return aops::neg(a); })
      .def("__abs__", [](const Variable& a) { return aops::abs(a); })
      .def("__matmul__", [](const Variable& a, const Variable& b) { return aops::matmul(a, b); })
      .def("__pow__", [](const Variable& a, const Variable& b) { return aops::pow(a, b); })
      .def("__pow__", [](const Variable& a, Scalar s) { return bin_vs(LMPB_POW, a, s); })
      .def("__rpow__", [](const Variable& a, Scalar s) { return bin_sv(LMPB_POW, s, a); })
      .def("exp", &aops::exp)
      .def("log", &aops::log)
      .def("sqrt", &aops::sqrt)
      .def("abs", &aops::abs)
      .def("sin", &aops::sin)
      .def("cos", &aops::cos)
      .def("tan", &aops::tan)
      .def("to", &aops::to, py::arg("device"))
      .def("reshape", &aops::reshape, py::arg("shape"))
      .def("squeeze", &aops::squeeze, py::arg("axis"))
      .def("expand_dims", &aops::expand_dims, py::arg("axis"))
      .def("clamp", &aops::clamp, py::arg("min"), py::arg("max"))
      .def("sum", &aops::sum, py::arg("axis"))
      .def("max", &aops::max, py::arg("axis"))
      .def("min", &aops::min, py::arg("axis"))
      .def("prod", &aops::prod, py::arg("axis"))
      .def("matmul", &aops::matmul, py::arg("other"))
      .def("transpose", &aops::transpose)
      .def_property_readonly("T", &aops::transpose);
#define LMP_V_OP(PY, OPC)                                                                            \
  vcls.def(PY, [](const Variable& a, const Variable& b) { return aops::binary(OPC, a, b); })         \
      .def(PY, [](const Variable& a, Scalar s) { return bin_vs(OPC, a, s); });
#define LMP_V_ROP(PY, OPC) vcls.def(PY, [](const Variable& a, Scalar s) { return bin_sv(OPC, s, a); });
  LMP_V_OP("__add__", LMPB_ADD) LMP_V_ROP("__radd__", LMPB_ADD)
  LMP_V_OP("__sub__", LMPB_SUB) LMP_V_ROP("__rsub__", LMPB_SUB)
  LMP_V_OP("__mul__", LMPB_MUL) LMP_V_ROP("__rmul__", LMPB_MUL)
  LMP_V_OP("__truediv__", LMPB_DIV) LMP_V_ROP("__rtruediv__", LMPB_DIV)
  LMP_V_OP("__eq__", LMPB_EQ) LMP_V_OP("__ne__", LMPB_NE) LMP_V_OP("__lt__", LMPB_LT)
  LMP_V_OP("__le__", LMPB_LE) LMP_V_OP("__gt__", LMPB_GT) LMP_V_OP("__ge__", LMPB_GE)
  // reflected comparisons: s < v  ==  v > s with the scalar on the left
  vcls.def("__rlt__", [](const Variable& a, Scalar s) { return bin_sv(LMPB_LT, s, a); });

  // ------------------------------------------------------- functions
#define LMP_F_BIN(NAME, OPC)                                                                             \
  m.def(NAME, [](const Variable& a, const Variable& b) { return aops::binary(OPC, a, b); }, py::arg("a"), py::arg("b")); \
  m.def(NAME, [](const Variable& a, Scalar s) { return bin_vs(OPC, a, s); }, py::arg("a"), py::arg("b"));             \
  m.def(NAME, [](Scalar s, const Variable& a) { return bin_sv(OPC, s, a); }, py::arg("a"), py::arg("b"));
  LMP_F_BIN("add", LMPB_ADD)
  LMP_F_BIN("sub", LMPB_SUB)
  LMP_F_BIN("mul", LMPB_MUL)
  LMP_F_BIN("div", LMPB_DIV)
  LMP_F_BIN("pow", LMPB_POW)
  LMP_F_BIN("eq", LMPB_EQ)
  LMP_F_BIN("ne", LMPB_NE)
  LMP_F_BIN("ge", LMPB_GE)
  LMP_F_BIN("le", LMPB_LE)
  LMP_F_BIN("gt", LMPB_GT)
  LMP_F_BIN("lt", LMPB_LT)
  m.def("neg", &aops::neg, py::arg("a"));
  m.def("exp", &aops::exp, py::arg("a"));
  m.def("log", &aops::log, py::arg("a"));
  m.def("sqrt", &aops::sqrt, py::arg("a"));
  m.def("abs", &aops::abs, py::arg("a"));
  m.def("sin", &aops::sin, py::arg("a"));
  m.def("cos", &aops::cos, py::arg("a"));
  m.def("tan", &aops::tan, py::arg("a"));
  m.def("clamp", &aops::clamp, py::arg("a"), py::arg("min"), py::arg("max"));
  m.def("sum", &aops::sum, py::arg("a"), py::arg("axis"));
  m.def("max", &aops::max, py::arg("a"), py::arg("axis"));
  m.def("min", &aops::min, py::arg("a"), py::arg("axis"));
  m.def("prod", &aops::prod, py::arg("a"), py::arg("axis"));
  m.def("matmul", &aops::matmul, py::arg("a"), py::arg("b"));
  m.def("transpose", &aops::transpose, py::arg("a"));
  m.def("reshape", &aops::reshape, py::arg("a"), py::arg("shape"));
  m.def("squeeze", &aops::squeeze, py::arg("a"), py::arg("axis"));
  m.def("expand_dims", &aops::expand_dims, py::arg("a"), py::arg("axis"));
  m.def("to", &aops::to, py::arg("a"), py::arg("device"));

  // tensor-level kernels without autograd (the stub-level API)
  m.def("abs_backward", &tops::abs_backward, py::arg("input"), py::arg("grad"));
  m.def("clamp_backward", &tops::clamp_backward, py::arg("input"), py::arg("grad"), py::arg("min"), py::arg("max"));
  m.def("add_inplace", [](Tensor& dst, const Tensor& src) { tops::add_inplace(dst, src); });

  // ------------------------------------------------------ constructors
  m.def("zeros", &lmp::autograd::zeros, py::arg("shape"), py::arg("requires_grad") = false,
        py::arg("device") = kDefaultDevice, py::arg("dtype") = kDefaultDtype);
  m.def("ones", &lmp::autograd::ones, py::arg("shape"), py::arg("requires_grad") = false,
        py::arg("device") = kDefaultDevice, py::arg("dtype") = kDefaultDtype);
  m.def("rand", [](const std::vector<size_t>& shape, bool rg, DeviceType d, DataType dt) {
        std::uniform_real_distribution<> u(0.0, 1.0);
        std::vector<double> v(count(shape));
        for (auto& x : v) x = u(rng());
        return Variable(Tensor(v, shape, d, dt), rg);
      }, py::arg("shape"), py::arg("requires_grad") = false, py::arg("device") = kDefaultDevice,
      py::arg("dtype") = kDefaultDtype);
  // randn(mean, var, ...): std::normal_distribution(mean, var) like the reference
  // (csrc/src/autograd/utils/constructor.cpp:44-57)
  m.def("randn", [](Scalar mean, Scalar var, const std::vector<size_t>& shape, bool rg, DeviceType d, DataType dt) {
        std::normal_distribution<> g(mean, var);
        std::vector<double> v(count(shape));
        for (auto& x : v) x = g(rng());
        return Variable(Tensor(v, shape, d, dt), rg);
      }, py::arg("mean"), py::arg("var"), py::arg("shape"), py::arg("requires_grad") = false,
      py::arg("device") = kDefaultDevice, py::arg("dtype") = kDefaultDtype);
  m.def("manual_seed", [](uint64_t s) { rng().seed(s); }, py::arg("seed"));

  // ----------------------------------------------------------- flags
  m.def("set_capture_enabled", &lmp::tensor::lazy::set_capture_enabled);
  m.def("is_capture_enabled", &lmp::tensor::lazy::is_capture_enabled);
  m.def("set_grad_enabled", &lmp::autograd::set_grad_enabled);
  m.def("is_grad_enabled", &lmp::autograd::is_grad_enabled);

  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const std::runtime_error& e) {
      PyErr_SetString(PyExc_RuntimeError, e.what());
    }
  });
}
