// Per-element semantics of Lamp3's ops, shared verbatim by the nvcc-compiled
// eager kernels and the NVRTC-compiled fused kernels (this file is embedded
// into every generated program), so a fused chain rounds exactly like the
// same chain run op by op.  Self-contained: no standard headers.
//
// Semantics follow the reference's CPU functors
// (csrc/include/lamp3/tensor/cpu/kernels.hpp:22-172): operands are in the
// output type T; transcendental ops compute in T for floating T and in double
// for integral T, then convert back (math_acc_t, kernels.hpp:20-21);
// comparisons yield 1/0 in T.  + - * round once each (__fadd_rn & co.), so
// nvcc/NVRTC can never contract them into an FMA.
#pragma once

namespace lmpb_dev {

// op codes (same values as lmpb_binary_op / lmpb_unary_op in lmpb.h)
enum { B_ADD = 0, B_SUB, B_MUL, B_DIV, B_POW, B_EQ, B_NE, B_GE, B_LE, B_GT, B_LT, B_ABS_BW, B_CLAMP_BW };
enum { U_NEG = 0, U_EXP, U_LOG, U_SQRT, U_ABS, U_SIN, U_COS, U_TAN, U_CLAMP };

template <typename T> struct is_fp { static constexpr bool value = false; };
template <> struct is_fp<float> { static constexpr bool value = true; };
template <> struct is_fp<double> { static constexpr bool value = true; };

template <bool C, typename A, typename B> struct cond { using type = A; };
template <typename A, typename B> struct cond<false, A, B> { using type = B; };
template <typename T> using math_t = typename cond<is_fp<T>::value, T, double>::type;

__device__ __forceinline__ float m_pow(float a, float b) { return powf(a, b); }
__device__ __forceinline__ double m_pow(double a, double b) { return pow(a, b); }
__device__ __forceinline__ float m_exp(float a) { return expf(a); }
__device__ __forceinline__ double m_exp(double a) { return exp(a); }
__device__ __forceinline__ float m_log(float a) { return logf(a); }
__device__ __forceinline__ double m_log(double a) { return log(a); }
__device__ __forceinline__ float m_sqrt(float a) { return sqrtf(a); }
__device__ __forceinline__ double m_sqrt(double a) { return sqrt(a); }
__device__ __forceinline__ float m_abs(float a) { return fabsf(a); }
__device__ __forceinline__ double m_abs(double a) { return fabs(a); }
__device__ __forceinline__ float m_sin(float a) { return sinf(a); }
__device__ __forceinline__ double m_sin(double a) { return sin(a); }
__device__ __forceinline__ float m_cos(float a) { return cosf(a); }
__device__ __forceinline__ double m_cos(double a) { return cos(a); }
__device__ __forceinline__ float m_tan(float a) { return tanf(a); }
__device__ __forceinline__ double m_tan(double a) { return tan(a); }

// Smallest finite value of T: the identity of a max reduction (the
// numeric_limits<T>::lowest() the eager reductions start from).
template <typename T> __device__ __forceinline__ T lowest();
template <> __device__ __forceinline__ bool lowest<bool>() { return false; }
template <> __device__ __forceinline__ short lowest<short>() { return (short)-32768; }
template <> __device__ __forceinline__ int lowest<int>() { return -2147483647 - 1; }
template <> __device__ __forceinline__ long long lowest<long long>() { return -9223372036854775807ll - 1; }
template <> __device__ __forceinline__ float lowest<float>() { return -3.40282346638528859812e+38f; }
template <> __device__ __forceinline__ double lowest<double>() { return -1.79769313486231570815e+308; }

template <typename T> __device__ __forceinline__ T r_add(T a, T b) { return a + b; }
template <typename T> __device__ __forceinline__ T r_sub(T a, T b) { return a - b; }
template <typename T> __device__ __forceinline__ T r_mul(T a, T b) { return a * b; }
template <> __device__ __forceinline__ float r_add<float>(float a, float b) { return __fadd_rn(a, b); }
template <> __device__ __forceinline__ float r_sub<float>(float a, float b) { return __fsub_rn(a, b); }
template <> __device__ __forceinline__ float r_mul<float>(float a, float b) { return __fmul_rn(a, b); }
template <> __device__ __forceinline__ double r_add<double>(double a, double b) { return __dadd_rn(a, b); }
template <> __device__ __forceinline__ double r_sub<double>(double a, double b) { return __dsub_rn(a, b); }
template <> __device__ __forceinline__ double r_mul<double>(double a, double b) { return __dmul_rn(a, b); }

// Integral pow.  The reference computes std::pow in double and truncates
// (PowFunctor, kernels.hpp:36-41); glibc's pow is exact whenever the result is
// an exactly representable double, CUDA's device pow is not (3^1 can come out
// as 2.9999999999999996 and truncate to 2).  For an integral exponent >= 0 the
// power is built by binary exponentiation in double, exact up to 2^53; a
// negative exponent gives |result| < 1 (truncates to 0) except for bases 1/-1.
template <typename T>
__device__ __forceinline__ T int_pow(T a, T b) {
  long long e = static_cast<long long>(b);
  if (e < 0) {
    if (a == T(1)) return T(1);
    if (a == static_cast<T>(-1)) return (e & 1) ? static_cast<T>(-1) : T(1);
    if (a == T(0)) return static_cast<T>(1.0 / 0.0);
    return T(0);
  }
  double base = static_cast<double>(a), r = 1.0;
  while (e) {
    if (e & 1) r *= base;
    e >>= 1;
    if (e) base *= base;
  }
  return static_cast<T>(r);
}

template <int OP, typename T>
__device__ __forceinline__ T binary_apply(T a, T b, T lo, T hi) {
  if constexpr (OP == B_ADD) return static_cast<T>(r_add(a, b));
  else if constexpr (OP == B_SUB) return static_cast<T>(r_sub(a, b));
  else if constexpr (OP == B_MUL) return static_cast<T>(r_mul(a, b));
  else if constexpr (OP == B_DIV) {
    if constexpr (is_fp<T>::value) return a / b;
    else return b == T(0) ? T(0) : static_cast<T>(a / b);  // the CPU traps on x/0; a GPU must not
  }
  else if constexpr (OP == B_POW) {
    if constexpr (is_fp<T>::value) return m_pow(a, b);
    else return int_pow<T>(a, b);
  }
  else if constexpr (OP == B_EQ) return static_cast<T>(a == b);
  else if constexpr (OP == B_NE) return static_cast<T>(a != b);
  else if constexpr (OP == B_GE) return static_cast<T>(a >= b);
  else if constexpr (OP == B_LE) return static_cast<T>(a <= b);
  else if constexpr (OP == B_GT) return static_cast<T>(a > b);
  else if constexpr (OP == B_LT) return static_cast<T>(a < b);
  else if constexpr (OP == B_ABS_BW)  // (input, grad): sign(input)*grad, 0 at 0
    return a > T(0) ? b : (a < T(0) ? static_cast<T>(-b) : T(0));
  else  // B_CLAMP_BW: grad where lo < input < hi (strict), else 0
    return (a > lo && a < hi) ? b : T(0);
}

template <int OP, typename T>
__device__ __forceinline__ T unary_apply(T a, T lo, T hi) {
  if constexpr (OP == U_NEG) return static_cast<T>(-a);
  else if constexpr (OP == U_EXP) return static_cast<T>(m_exp(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_LOG) return static_cast<T>(m_log(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_SQRT) return static_cast<T>(m_sqrt(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_ABS) return static_cast<T>(m_abs(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_SIN) return static_cast<T>(m_sin(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_COS) return static_cast<T>(m_cos(static_cast<math_t<T>>(a)));
  else if constexpr (OP == U_TAN) return static_cast<T>(m_tan(static_cast<math_t<T>>(a)));
  else return a < lo ? lo : (a > hi ? hi : a);  // U_CLAMP
}

}  // namespace lmpb_dev
