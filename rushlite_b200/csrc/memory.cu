// Memory substrate: stream-ordered allocation, fill, casting copy,
// add_inplace (gradient accumulation) and the 2-D transpose.
#include <string>

#include "common.cuh"

namespace lmpb {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t items) {
  int64_t b = (items + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)sm_count() * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_kernel(T* __restrict__ p, int64_t n, T v) {
  constexpr int N = 16 / sizeof(T);
  union U {
    uint4 raw;
    T v[N];
  } u;
#pragma unroll
  for (int j = 0; j < N; ++j) u.v[j] = v;
  const int64_t nv = n / N;
  uint4* p4 = reinterpret_cast<uint4*>(p);
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i < nv; i += stride) p4[i] = u.raw;
  const int64_t t = nv * N + (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t < n) p[t] = v;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_scalar_kernel(T* __restrict__ p, int64_t n, T v) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    p[i] = v;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    add_inplace_kernel(T* __restrict__ dst, const T* __restrict__ src, int64_t n) {
  constexpr int N = 16 / sizeof(T);
  union U {
    uint4 raw;
    T v[N];
  };
  const int64_t nv = n / N;
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + stride < nv; i += 2 * stride) {
    U a0, b0, a1, b1;
    a0.raw = d4[i];
    b0.raw = __ldg(s4 + i);
    a1.raw = d4[i + stride];
    b1.raw = __ldg(s4 + i + stride);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      a0.v[j] = static_cast<T>(r_add(a0.v[j], b0.v[j]));
      a1.v[j] = static_cast<T>(r_add(a1.v[j], b1.v[j]));
    }
    d4[i] = a0.raw;
    d4[i + stride] = a1.raw;
  }
  for (; i < nv; i += stride) {
    U a, b;
    a.raw = d4[i];
    b.raw = __ldg(s4 + i);
#pragma unroll
    for (int j = 0; j < N; ++j) a.v[j] = static_cast<T>(r_add(a.v[j], b.v[j]));
    d4[i] = a.raw;
  }
  const int64_t t = nv * N + (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t < n) dst[t] = static_cast<T>(r_add(dst[t], src[t]));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    add_inplace_scalar_kernel(T* __restrict__ dst, const T* __restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    dst[i] = static_cast<T>(r_add(dst[i], src[i]));
}

template <typename D>
__global__ void __launch_bounds__(kThreads)
    cast_kernel(const void* __restrict__ src, int src_dt, D* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    dst[i] = load_as<D>(src, src_dt, i);
}

// 32x32 tiles through shared memory (padded against bank conflicts): both
// the read of `in` rows and the write of `out` rows are coalesced.
template <typename T>
__global__ void __launch_bounds__(256)
    transpose_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t m, int64_t n) {
  __shared__ T tile[32][33];
  const int64_t bx = (int64_t)blockIdx.x * 32, by = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int j = ty; j < 32; j += 8) {
    int64_t r = by + j, c = bx + tx;
    if (r < m && c < n) tile[j][tx] = in[r * n + c];
  }
  __syncthreads();
  for (int j = ty; j < 32; j += 8) {
    int64_t r = bx + j, c = by + tx;  // out is [n, m]
    if (r < n && c < m) out[r * m + c] = tile[tx][j];
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

lmpb_status cast_on_device(const void* src, int sdt, void* dst, int ddt, int64_t n,
                           cudaStream_t st) {
  LMPB_DISPATCH_DTYPE(ddt, D, {
    cast_kernel<D><<<grid_for(n), kThreads, 0, st>>>(src, sdt, static_cast<D*>(dst), n);
    return launch_status("cast_kernel");
  });
  return set_error(LMPB_ERR_INVALID, "cast: invalid dtype");
}

}  // namespace
}  // namespace lmpb

using namespace lmpb;

extern "C" lmpb_status lmpb_malloc(void** ptr, size_t bytes, void* stream) {
  LMPB_CHECK_ARG(ptr != nullptr, "lmpb_malloc: null out pointer");
  *ptr = nullptr;
  if (bytes == 0) return LMPB_OK;
  LMPB_CUDA_TRY(stream_alloc((void**)ptr, bytes, as_stream(stream)));
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_free(void* ptr, void* stream) {
  if (ptr == nullptr) return LMPB_OK;
  LMPB_CUDA_TRY(cudaFreeAsync(ptr, as_stream(stream)));
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_fill(int dtype, void* ptr, int64_t n, double value, void* stream) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_fill: invalid dtype");
  LMPB_CHECK_ARG(n >= 0, "lmpb_fill: negative size");
  if (n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(ptr != nullptr, "lmpb_fill: null pointer");
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(dtype, T, {
    // fill_cpu casts with static_cast<T>(value) (csrc/src/tensor/cpu/memory.cpp:16-21)
    T v = static_cast<T>(value);
    if (aligned16(ptr))
      fill_kernel<T><<<grid_for(n / (16 / sizeof(T)) + 1), kThreads, 0, st>>>((T*)ptr, n, v);
    else
      fill_scalar_kernel<T><<<grid_for(n), kThreads, 0, st>>>((T*)ptr, n, v);
    return launch_status("fill_kernel");
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_fill: invalid dtype");
}

extern "C" lmpb_status lmpb_add_inplace(int dtype, void* dst, const void* src, int64_t n,
                                        void* stream) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_add_inplace: invalid dtype");
  LMPB_CHECK_ARG(n >= 0, "lmpb_add_inplace: negative size");
  if (n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(dst && src, "lmpb_add_inplace: null pointer");
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(dtype, T, {
    if (aligned16(dst) && aligned16(src))
      add_inplace_kernel<T><<<grid_for((n / (16 / sizeof(T)) + 1) / 2 + 1), kThreads, 0, st>>>(
          (T*)dst, (const T*)src, n);
    else
      add_inplace_scalar_kernel<T><<<grid_for(n), kThreads, 0, st>>>((T*)dst, (const T*)src, n);
    return launch_status("add_inplace_kernel");
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_add_inplace: invalid dtype");
}

extern "C" lmpb_status lmpb_copy(int kind, const void* src, int src_dtype, void* dst,
                                 int dst_dtype, int64_t n, void* stream) {
  LMPB_CHECK_ARG(valid_dtype(src_dtype) && valid_dtype(dst_dtype), "lmpb_copy: invalid dtype");
  LMPB_CHECK_ARG(kind >= LMPB_H2D && kind <= LMPB_H2H, "lmpb_copy: invalid kind");
  LMPB_CHECK_ARG(n >= 0, "lmpb_copy: negative size");
  if (n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(src && dst, "lmpb_copy: null pointer");
  cudaStream_t st = as_stream(stream);
  const size_t sbytes = (size_t)n * dtype_size(src_dtype);
  const size_t dbytes = (size_t)n * dtype_size(dst_dtype);
  static const cudaMemcpyKind kinds[] = {cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost,
                                         cudaMemcpyDeviceToDevice, cudaMemcpyHostToHost};
  if (src_dtype == dst_dtype) {
    LMPB_CUDA_TRY(cudaMemcpyAsync(dst, src, sbytes, kinds[kind], st));
    return LMPB_OK;
  }
  switch (kind) {
    case LMPB_D2D:
      return cast_on_device(src, src_dtype, dst, dst_dtype, n, st);
    case LMPB_H2D: {  // raw bytes up, cast on the device
      void* tmp = nullptr;
      LMPB_CUDA_TRY(stream_alloc((void**)&tmp, sbytes, st));
      LMPB_CUDA_TRY(cudaMemcpyAsync(tmp, src, sbytes, cudaMemcpyHostToDevice, st));
      lmpb_status s = cast_on_device(tmp, src_dtype, dst, dst_dtype, n, st);
      LMPB_CUDA_TRY(cudaFreeAsync(tmp, st));
      return s;
    }
    case LMPB_D2H: {  // cast on the device, bytes down
      void* tmp = nullptr;
      LMPB_CUDA_TRY(stream_alloc((void**)&tmp, dbytes, st));
      lmpb_status s = cast_on_device(src, src_dtype, tmp, dst_dtype, n, st);
      if (s != LMPB_OK) return s;
      LMPB_CUDA_TRY(cudaMemcpyAsync(dst, tmp, dbytes, cudaMemcpyDeviceToHost, st));
      LMPB_CUDA_TRY(cudaFreeAsync(tmp, st));
      return LMPB_OK;
    }
    default:
      return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_copy: host-to-host casts are done on the host");
  }
}

extern "C" lmpb_status lmpb_transpose(int dtype, const void* in, void* out, int64_t m, int64_t n,
                                      void* stream) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_transpose: invalid dtype");
  LMPB_CHECK_ARG(m >= 0 && n >= 0, "lmpb_transpose: negative size");
  if (m == 0 || n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(in && out, "lmpb_transpose: null pointer");
  LMPB_CHECK_ARG((m + 31) / 32 <= 65535, "lmpb_transpose: too many rows");
  dim3 grid((unsigned)((n + 31) / 32), (unsigned)((m + 31) / 32));
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(dtype, T, {
    transpose_kernel<T><<<grid, 256, 0, st>>>((const T*)in, (T*)out, m, n);
    return launch_status("transpose_kernel");
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_transpose: invalid dtype");
}
