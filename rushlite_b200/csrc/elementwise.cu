// Eager elementwise kernels: broadcast binary ops, unary ops and the two
// same-shape backward kernels (abs_backward, clamp_backward).
//
// Design for B200 (HBM3e-bound streaming):
//  * same-shape, same-dtype operands take a 16-byte vector path (one uint4 per
//    operand per vector, two vectors in flight per thread) over a grid-stride
//    loop sized to the SM count, so each SM keeps ~64 KB of loads in flight;
//  * broadcasts are collapsed on the host to the fewest dims (adjacent dims
//    merge when every operand is contiguous across them, size-1 dims drop),
//    then indexed with 32-bit multiply-shift division held in __grid_constant__
//    parameters — no per-call H2D copies of stride tables as in
//    csrc/src/tensor/cuda/offset_util.cu:20-29;
//  * when the innermost collapsed dim is a multiple of the vector width, the
//    broadcast path loads 16-byte vectors too (a broadcast operand is read
//    once per vector and splatted);
//  * mixed dtypes convert each operand to the output dtype at load
//    (csrc/include/lamp3/tensor/cuda/ptr_pack.cuh:12-17).
#include <vector>

#include "common.cuh"

namespace lmpb {
namespace {

constexpr int kThreads = 256;

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T v[N];
  };
};

// ------------------------------------------------------------ contiguous

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads)
    binary_contig_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out,
                         int64_t n, T lo, T hi) {
  constexpr int N = Vec<T>::N;
  const int64_t nvec = n / N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4* a4 = reinterpret_cast<const uint4*>(a);
  const uint4* b4 = reinterpret_cast<const uint4*>(b);
  uint4* o4 = reinterpret_cast<uint4*>(out);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    Vec<T> x0, y0, x1, y1, r0, r1;
    x0.raw = __ldg(a4 + i);
    y0.raw = __ldg(b4 + i);
    x1.raw = __ldg(a4 + i + stride);
    y1.raw = __ldg(b4 + i + stride);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      r0.v[j] = binary_apply<OP, T>(x0.v[j], y0.v[j], lo, hi);
      r1.v[j] = binary_apply<OP, T>(x1.v[j], y1.v[j], lo, hi);
    }
    o4[i] = r0.raw;
    o4[i + stride] = r1.raw;
  }
  for (; i < nvec; i += stride) {
    Vec<T> x, y, r;
    x.raw = __ldg(a4 + i);
    y.raw = __ldg(b4 + i);
#pragma unroll
    for (int j = 0; j < N; ++j) r.v[j] = binary_apply<OP, T>(x.v[j], y.v[j], lo, hi);
    o4[i] = r.raw;
  }
  // scalar tail
  const int64_t t = nvec * N + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) out[t] = binary_apply<OP, T>(a[t], b[t], lo, hi);
}

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads)
    unary_contig_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t n, T lo, T hi) {
  constexpr int N = Vec<T>::N;
  const int64_t nvec = n / N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4* i4 = reinterpret_cast<const uint4*>(in);
  uint4* o4 = reinterpret_cast<uint4*>(out);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    Vec<T> x0, x1, r0, r1;
    x0.raw = __ldg(i4 + i);
    x1.raw = __ldg(i4 + i + stride);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      r0.v[j] = unary_apply<OP, T>(x0.v[j], lo, hi);
      r1.v[j] = unary_apply<OP, T>(x1.v[j], lo, hi);
    }
    o4[i] = r0.raw;
    o4[i + stride] = r1.raw;
  }
  for (; i < nvec; i += stride) {
    Vec<T> x, r;
    x.raw = __ldg(i4 + i);
#pragma unroll
    for (int j = 0; j < N; ++j) r.v[j] = unary_apply<OP, T>(x.v[j], lo, hi);
    o4[i] = r.raw;
  }
  const int64_t t = nvec * N + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) out[t] = unary_apply<OP, T>(in[t], lo, hi);
}

// ------------------------------------------------------------- broadcast

struct BcastGeom {
  int ndim;                     // collapsed dims, >= 1
  int64_t size[LMPB_MAX_DIMS];  // output extent per dim
  int64_t sa[LMPB_MAX_DIMS];    // element stride of a per dim (0 = broadcast)
  int64_t sb[LMPB_MAX_DIMS];
  FastDiv fd[LMPB_MAX_DIMS];  // divisors for the 32-bit path
};

struct BcastArgs {
  const void* a;
  const void* b;
  void* out;
  int a_dt, b_dt;
  int64_t n;  // output elements
  BcastGeom g;
};

template <typename IDX>
__device__ __forceinline__ void bcast_offsets(const BcastGeom& g, IDX e, IDX& oa, IDX& ob) {
  oa = 0;
  ob = 0;
  for (int d = g.ndim - 1; d > 0; --d) {
    IDX q;
    if constexpr (sizeof(IDX) == 4) q = g.fd[d].div(e);
    else q = e / (IDX)g.size[d];
    IDX r = e - q * (IDX)g.size[d];
    oa += r * (IDX)g.sa[d];
    ob += r * (IDX)g.sb[d];
    e = q;
  }
  oa += e * (IDX)g.sa[0];
  ob += e * (IDX)g.sb[0];
}

// One thread computes VEC consecutive outputs of the innermost dim.  VEC > 1
// only when a, b and out share dtype T, the innermost extent is a multiple of
// VEC and every pointer is 16-byte aligned; each operand's innermost stride
// is then 1 (vector load) or 0 (scalar load, splatted).
template <int OP, typename T, int VEC, typename IDX>
__global__ void __launch_bounds__(kThreads) binary_bcast_kernel(const __grid_constant__ BcastArgs p,
                                                                T lo, T hi) {
  const IDX nv = (IDX)(p.n / VEC);
  const IDX stride = (IDX)gridDim.x * blockDim.x;
  const int inner = p.g.ndim - 1;
  for (IDX v = (IDX)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    IDX oa, ob;
    bcast_offsets<IDX>(p.g, v * VEC, oa, ob);
    if constexpr (VEC == 1) {
      T x = load_as<T>(p.a, p.a_dt, oa);
      T y = load_as<T>(p.b, p.b_dt, ob);
      static_cast<T*>(p.out)[v] = binary_apply<OP, T>(x, y, lo, hi);
    } else {
      Vec<T> x, y, r;
      const T* a = static_cast<const T*>(p.a);
      const T* b = static_cast<const T*>(p.b);
      if (p.g.sa[inner] == 1) {
        x.raw = __ldg(reinterpret_cast<const uint4*>(a + oa));
      } else {
        T s = a[oa];
#pragma unroll
        for (int j = 0; j < VEC; ++j) x.v[j] = s;
      }
      if (p.g.sb[inner] == 1) {
        y.raw = __ldg(reinterpret_cast<const uint4*>(b + ob));
      } else {
        T s = b[ob];
#pragma unroll
        for (int j = 0; j < VEC; ++j) y.v[j] = s;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) r.v[j] = binary_apply<OP, T>(x.v[j], y.v[j], lo, hi);
      reinterpret_cast<uint4*>(p.out)[v] = r.raw;
    }
  }
}

// ---------------------------------------------------------------- host

int grid_for(int64_t work_items) {
  int64_t blocks = (work_items + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)sm_count() * 8;  // 8 x 256 threads = full occupancy per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Row-major contiguous strides of `shape` right-aligned into `nd` dims,
// with 0 where the operand has extent 1 (init_padded_strides,
// csrc/src/tensor/cpu/offset_util.cpp:7-28).
void padded_strides(const int64_t* shape, int ndim, int nd, int64_t* out) {
  for (int i = 0; i < nd; ++i) out[i] = 0;
  int64_t s = 1;
  for (int k = 0; k < ndim; ++k) {
    int src = ndim - 1 - k, dst = nd - 1 - k;
    out[dst] = shape[src] == 1 ? 0 : s;
    s *= shape[src];
  }
}

// Drops size-1 dims and merges adjacent dims that every operand walks
// contiguously.  Returns the collapsed dim count (>= 1).
int collapse(int nd, const int64_t* size, const int64_t* sa, const int64_t* sb, BcastGeom& g) {
  int m = 0;
  for (int d = 0; d < nd; ++d) {
    if (size[d] == 1) continue;
    if (m > 0) {
      int p = m - 1;
      if (g.sa[p] == sa[d] * size[d] && g.sb[p] == sb[d] * size[d]) {
        g.size[p] *= size[d];
        g.sa[p] = sa[d];
        g.sb[p] = sb[d];
        continue;
      }
    }
    g.size[m] = size[d];
    g.sa[m] = sa[d];
    g.sb[m] = sb[d];
    ++m;
  }
  if (m == 0) {
    g.size[0] = 1;
    g.sa[0] = 0;
    g.sb[0] = 0;
    m = 1;
  }
  g.ndim = m;
  for (int d = 0; d < m; ++d)
    g.fd[d] = FastDiv(static_cast<uint32_t>(g.size[d] < (1ll << 31) ? g.size[d] : 1));
  return m;
}

template <int OP, typename T>
lmpb_status launch_binary(const void* a, int a_dt, const void* b, int b_dt, void* out, int64_t n,
                          bool same_shape, const BcastGeom& g, double p0, double p1,
                          cudaStream_t st) {
  const T lo = scalar_to<T>(p0), hi = scalar_to<T>(p1);
  constexpr int N = Vec<T>::N;
  constexpr int kOutDt = std::is_same<T, bool>::value      ? LMPB_BOOL
                         : std::is_same<T, int16_t>::value ? LMPB_INT16
                         : std::is_same<T, int32_t>::value ? LMPB_INT32
                         : std::is_same<T, int64_t>::value ? LMPB_INT64
                         : std::is_same<T, float>::value   ? LMPB_FLOAT32
                                                           : LMPB_FLOAT64;
  const bool same_dt = a_dt == kOutDt && b_dt == kOutDt;
  const bool al = aligned16(a) && aligned16(b) && aligned16(out);
  if (same_shape && same_dt && al) {
    binary_contig_kernel<OP, T><<<grid_for((n / N + 1) / 2 + 1), kThreads, 0, st>>>(
        static_cast<const T*>(a), static_cast<const T*>(b), static_cast<T*>(out), n, lo, hi);
    return launch_status("binary_contig_kernel");
  }
  if constexpr (OP == LMPB_ABS_BACKWARD || OP == LMPB_CLAMP_BACKWARD) {
    return set_error(LMPB_ERR_INVALID, "backward kernels need equal shapes and dtypes");
  } else {
    BcastArgs args;
    args.a = a;
    args.b = b;
    args.out = out;
    args.a_dt = a_dt;
    args.b_dt = b_dt;
    args.n = n;
    args.g = g;
    const int inner = g.ndim - 1;
    const bool vec = same_dt && al && g.size[inner] % N == 0;
    const bool small = n < (1ll << 31);
    if (vec && small)
      binary_bcast_kernel<OP, T, N, uint32_t><<<grid_for(n / N), kThreads, 0, st>>>(args, lo, hi);
    else if (vec)
      binary_bcast_kernel<OP, T, N, uint64_t><<<grid_for(n / N), kThreads, 0, st>>>(args, lo, hi);
    else if (small)
      binary_bcast_kernel<OP, T, 1, uint32_t><<<grid_for(n), kThreads, 0, st>>>(args, lo, hi);
    else
      binary_bcast_kernel<OP, T, 1, uint64_t><<<grid_for(n), kThreads, 0, st>>>(args, lo, hi);
    return launch_status("binary_bcast_kernel");
  }
}

template <typename T>
lmpb_status binary_op_switch(int op, const void* a, int a_dt, const void* b, int b_dt, void* out,
                             int64_t n, bool same_shape, const BcastGeom& g, double p0, double p1,
                             cudaStream_t st) {
#define LMPB_BIN_CASE(OPC) \
  case OPC: return launch_binary<OPC, T>(a, a_dt, b, b_dt, out, n, same_shape, g, p0, p1, st);
  switch (op) {
    LMPB_BIN_CASE(LMPB_ADD)
    LMPB_BIN_CASE(LMPB_SUB)
    LMPB_BIN_CASE(LMPB_MUL)
    LMPB_BIN_CASE(LMPB_DIV)
    LMPB_BIN_CASE(LMPB_POW)
    LMPB_BIN_CASE(LMPB_EQ)
    LMPB_BIN_CASE(LMPB_NE)
    LMPB_BIN_CASE(LMPB_GE)
    LMPB_BIN_CASE(LMPB_LE)
    LMPB_BIN_CASE(LMPB_GT)
    LMPB_BIN_CASE(LMPB_LT)
    LMPB_BIN_CASE(LMPB_ABS_BACKWARD)
    LMPB_BIN_CASE(LMPB_CLAMP_BACKWARD)
    default: return set_error(LMPB_ERR_INVALID, "lmpb_binary: unknown op");
  }
#undef LMPB_BIN_CASE
}

template <typename T>
lmpb_status unary_op_switch(int op, const void* in, void* out, int64_t n, double p0, double p1,
                            cudaStream_t st) {
  const T lo = scalar_to<T>(p0), hi = scalar_to<T>(p1);
  const int N = Vec<T>::N;
  if (!aligned16(in) || !aligned16(out))
    return set_error(LMPB_ERR_INVALID, "lmpb_unary: buffers must be 16-byte aligned");
  const int grid = grid_for((n / N + 1) / 2 + 1);
#define LMPB_UN_CASE(OPC)                                                                         \
  case OPC:                                                                                       \
    unary_contig_kernel<OPC, T><<<grid, kThreads, 0, st>>>(static_cast<const T*>(in),             \
                                                           static_cast<T*>(out), n, lo, hi);      \
    return launch_status("unary_contig_kernel");
  switch (op) {
    LMPB_UN_CASE(LMPB_NEG)
    LMPB_UN_CASE(LMPB_EXP)
    LMPB_UN_CASE(LMPB_LOG)
    LMPB_UN_CASE(LMPB_SQRT)
    LMPB_UN_CASE(LMPB_ABS)
    LMPB_UN_CASE(LMPB_SIN)
    LMPB_UN_CASE(LMPB_COS)
    LMPB_UN_CASE(LMPB_TAN)
    LMPB_UN_CASE(LMPB_CLAMP)
    default: return set_error(LMPB_ERR_INVALID, "lmpb_unary: unknown op");
  }
#undef LMPB_UN_CASE
}

}  // namespace
}  // namespace lmpb

using namespace lmpb;

extern "C" lmpb_status lmpb_binary(int op, int out_dtype, const void* a, int a_dtype,
                                   const int64_t* a_shape, int a_ndim, const void* b, int b_dtype,
                                   const int64_t* b_shape, int b_ndim, void* out, double p0,
                                   double p1, void* stream) {
  LMPB_CHECK_ARG(valid_dtype(out_dtype) && valid_dtype(a_dtype) && valid_dtype(b_dtype),
                 "lmpb_binary: invalid dtype");
  LMPB_CHECK_ARG(a_ndim >= 0 && a_ndim <= LMPB_MAX_DIMS && b_ndim >= 0 && b_ndim <= LMPB_MAX_DIMS,
                 "lmpb_binary: too many dims");
  int64_t oshape[LMPB_MAX_DIMS];
  int ond = 0;
  lmpb_status s = lmpb_broadcast_shape(a_shape, a_ndim, b_shape, b_ndim, oshape, &ond);
  if (s != LMPB_OK) return s;
  int64_t n = 1;
  for (int i = 0; i < ond; ++i) n *= oshape[i];
  if (n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(a && b && out, "lmpb_binary: null pointer");
  bool same_shape = a_ndim == b_ndim;
  for (int i = 0; same_shape && i < a_ndim; ++i) same_shape = a_shape[i] == b_shape[i];
  if (op == LMPB_ABS_BACKWARD || op == LMPB_CLAMP_BACKWARD)
    LMPB_CHECK_ARG(same_shape && a_dtype == b_dtype && a_dtype == out_dtype,
                   "lmpb_binary: backward kernels need identical shapes and dtypes");
  BcastGeom g;
  {
    int64_t sa[LMPB_MAX_DIMS], sb[LMPB_MAX_DIMS];
    padded_strides(a_shape, a_ndim, ond, sa);
    padded_strides(b_shape, b_ndim, ond, sb);
    if (ond == 0) {
      oshape[0] = 1;
      sa[0] = sb[0] = 0;
      ond = 1;
    }
    collapse(ond, oshape, sa, sb, g);
  }
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(out_dtype, T,
                      return binary_op_switch<T>(op, a, a_dtype, b, b_dtype, out, n, same_shape,
                                                 g, p0, p1, st));
  return set_error(LMPB_ERR_INVALID, "lmpb_binary: invalid dtype");
}

extern "C" lmpb_status lmpb_unary(int op, int dtype, const void* in, void* out, int64_t n,
                                  double p0, double p1, void* stream) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_unary: invalid dtype");
  LMPB_CHECK_ARG(n >= 0, "lmpb_unary: negative size");
  if (n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(in && out, "lmpb_unary: null pointer");
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(dtype, T, return unary_op_switch<T>(op, in, out, n, p0, p1, st));
  return set_error(LMPB_ERR_INVALID, "lmpb_unary: invalid dtype");
}
