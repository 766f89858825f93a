// Shared helpers for the lmpb kernels: status plumbing, dtype dispatch, the
// per-element op semantics of Lamp3, and 32-bit fast division.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <string>
#include <type_traits>

#include "lmpb.h"
#include "ops_device.cuh"
#include <limits>

namespace lmpb {

// ------------------------------------------------------------------ errors

// Records `msg` as the calling thread's last error and returns `st`.
lmpb_status set_error(lmpb_status st, const std::string& msg);

#define LMPB_CHECK_ARG(cond, msg)                                 \
  do {                                                            \
    if (!(cond)) return ::lmpb::set_error(LMPB_ERR_INVALID, msg); \
  } while (0)

#define LMPB_CUDA_TRY(expr)                                                                   \
  do {                                                                                        \
    cudaError_t e_ = (expr);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return ::lmpb::set_error(LMPB_ERR_CUDA, std::string(#expr " failed: ") +              \
                                                  cudaGetErrorString(e_));                    \
  } while (0)

// Checks the launch that was just issued.
lmpb_status launch_status(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

bool valid_dtype(int dt);
size_t dtype_size(int dt);

// cudaMallocAsync from the device's default pool, kept warm (capi.cpp).
cudaError_t stream_alloc(void** p, size_t bytes, cudaStream_t st);

// Number of SMs of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------- dtype dispatch

template <int DT> struct dtype_of;
template <> struct dtype_of<LMPB_BOOL> { using type = bool; };
template <> struct dtype_of<LMPB_INT16> { using type = int16_t; };
template <> struct dtype_of<LMPB_INT32> { using type = int32_t; };
template <> struct dtype_of<LMPB_INT64> { using type = int64_t; };
template <> struct dtype_of<LMPB_FLOAT32> { using type = float; };
template <> struct dtype_of<LMPB_FLOAT64> { using type = double; };

#define LMPB_DISPATCH_DTYPE(dt, T, ...)                  \
  switch (dt) {                                          \
    case LMPB_BOOL: { using T = bool; __VA_ARGS__; } break;      \
    case LMPB_INT16: { using T = int16_t; __VA_ARGS__; } break;  \
    case LMPB_INT32: { using T = int32_t; __VA_ARGS__; } break;  \
    case LMPB_INT64: { using T = int64_t; __VA_ARGS__; } break;  \
    case LMPB_FLOAT32: { using T = float; __VA_ARGS__; } break;  \
    case LMPB_FLOAT64: { using T = double; __VA_ARGS__; } break; \
    default: break;                                      \
  }

// Loads element i of an array of runtime dtype `dt`, converted to T.
template <typename T>
__device__ __forceinline__ T load_as(const void* p, int dt, int64_t i) {
  switch (dt) {
    case LMPB_BOOL: return static_cast<T>(static_cast<const bool*>(p)[i]);
    case LMPB_INT16: return static_cast<T>(static_cast<const int16_t*>(p)[i]);
    case LMPB_INT32: return static_cast<T>(static_cast<const int32_t*>(p)[i]);
    case LMPB_INT64: return static_cast<T>(static_cast<const int64_t*>(p)[i]);
    case LMPB_FLOAT32: return static_cast<T>(static_cast<const float*>(p)[i]);
    default: return static_cast<T>(static_cast<const double*>(p)[i]);
  }
}

// ------------------------------------------------------------- op semantics

using lmpb_dev::binary_apply;
using lmpb_dev::r_add;
using lmpb_dev::r_mul;
using lmpb_dev::r_sub;
using lmpb_dev::unary_apply;

// Host-side conversion of a clamp bound to T.  The reference does a plain
// static_cast (ClampFunctor, kernels.hpp:134-136); for an integral T a bound
// outside T's range (ReLU's DBL_MAX) saturates here instead of being UB.
template <typename T>
inline T scalar_to(double v) {
  if constexpr (std::is_same<T, bool>::value) {
    return v != 0.0;
  } else if constexpr (std::is_integral<T>::value) {
    if (std::isnan(v)) return T(0);
    if (v >= static_cast<double>(std::numeric_limits<T>::max())) return std::numeric_limits<T>::max();
    if (v <= static_cast<double>(std::numeric_limits<T>::lowest())) return std::numeric_limits<T>::lowest();
    return static_cast<T>(v);
  } else {
    return static_cast<T>(v);
  }
}

// --------------------------------------------------------- fast division
//
// Division of 32-bit unsigned n by an invariant d with one multiply-high and
// a shift: m = ceil(2^(32+s) / d) with s = ceil(log2 d), q = (umulhi(n, m') + n) >> s
// where m' = m - 2^32 (Granlund & Montgomery, "Division by Invariant Integers
// using Multiplication", PLDI 1994, section 4).  Valid for n, d < 2^31.
struct FastDiv {
  uint32_t d;
  uint32_t mul;
  uint32_t shift;
  FastDiv() : d(1), mul(0), shift(0) {}
  explicit FastDiv(uint32_t div) : d(div) {
    shift = 0;
    while ((1ull << shift) < div) ++shift;
    uint64_t m = ((1ull << (32 + shift)) + div - 1) / div;  // ceil(2^(32+s)/d)
    mul = static_cast<uint32_t>(m - (1ull << 32));
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    uint32_t t = __umulhi(n, mul);
    return (t + n) >> shift;
  }
};

}  // namespace lmpb
