/*
 * lamp3_oracle.c — TEST INFRASTRUCTURE ONLY (see lamp3_oracle.h).
 *
 * CPU restatement of the reference Lamp3 kernels, each function citing the
 * reference code it follows (paths relative to the rushlite project root).
 * Compiled with -ffp-contract=off so every float op rounds once, which is
 * the per-op rounding of the reference's functors.
 */
#include "lamp3_oracle.h"

#include <math.h>
#include <stdbool.h>
#include <stdlib.h>
#include <string.h>

enum { D_BOOL, D_I16, D_I32, D_I64, D_F32, D_F64 };
enum { B_ADD, B_SUB, B_MUL, B_DIV, B_POW, B_EQ, B_NE, B_GE, B_LE, B_GT, B_LT, B_ABS_BW, B_CLAMP_BW };
enum { U_NEG, U_EXP, U_LOG, U_SQRT, U_ABS, U_SIN, U_COS, U_TAN, U_CLAMP };
enum { R_SUM, R_MAX, R_MIN, R_PROD };

#define MAXD 16

/* Loads element i of a `dt` array as double/int64 then converts to the
 * target in each typed section below (ptr_pack.hpp:12-17: static_cast<OutT>). */
#define LOAD_AS(T, p, dt, i)                                     \
  ((dt) == D_BOOL  ? (T)(((const bool*)(p))[i])                  \
   : (dt) == D_I16 ? (T)(((const int16_t*)(p))[i])               \
   : (dt) == D_I32 ? (T)(((const int32_t*)(p))[i])               \
   : (dt) == D_I64 ? (T)(((const int64_t*)(p))[i])               \
   : (dt) == D_F32 ? (T)(((const float*)(p))[i])                 \
                   : (T)(((const double*)(p))[i]))

/* Saturating double -> integral conversion for clamp bounds (the reference's
 * static_cast is undefined outside the range; the backend saturates). */
#define SAT(T, LO, HI, v) ((v) != (v) ? (T)0 : (v) >= (double)(HI) ? (T)(HI) : (v) <= (double)(LO) ? (T)(LO) : (T)(v))

/* Broadcast offsets: init_padded_strides (csrc/src/tensor/cpu/offset_util.cpp:7-28)
 * and CPUOffsetUtil::get (offset_util.cpp:46-63). */
static void padded(const int64_t* shape, int nd, int ond, int64_t* out) {
  int64_t s = 1;
  for (int i = 0; i < ond; ++i) out[i] = 0;
  for (int k = 0; k < nd; ++k) {
    int src = nd - 1 - k, dst = ond - 1 - k;
    out[dst] = shape[src] == 1 ? 0 : s;
    s *= shape[src];
  }
}

static int bshape(const int64_t* a, int an, const int64_t* b, int bn, int64_t* o, int* on) {
  int nd = an > bn ? an : bn;
  if (nd > MAXD) return 1;
  for (int k = 0; k < nd; ++k) {
    int ai = an - 1 - k, bi = bn - 1 - k;
    int64_t av = ai >= 0 ? a[ai] : 1, bv = bi >= 0 ? b[bi] : 1;
    if (!(av == 1 || bv == 1 || av == bv)) return 1;
    o[nd - 1 - k] = av != 1 ? av : bv;
  }
  *on = nd;
  return 0;
}

/* Functors: csrc/include/lamp3/tensor/cpu/kernels.hpp:22-156. */
#define DEF_BINARY(T, NAME, ISF, POWF, ABSF, LO, HI)                                              \
  static void NAME(int op, const void* a, int adt, const int64_t* ash, int an, const void* b,    \
                   int bdt, const int64_t* bsh, int bn, T* out, const int64_t* osh, int on,      \
                   double p0, double p1) {                                                       \
    int64_t sa[MAXD], sb[MAXD], so[MAXD], n = 1;                                                 \
    padded(ash, an, on, sa);                                                                     \
    padded(bsh, bn, on, sb);                                                                     \
    for (int d = on - 1; d >= 0; --d) { so[d] = n; n *= osh[d]; }                               \
    T lo = ISF ? (T)p0 : SAT(T, LO, HI, p0), hi = ISF ? (T)p1 : SAT(T, LO, HI, p1);              \
    for (int64_t i = 0; i < n; ++i) {                                                            \
      int64_t idx = i, oa = 0, ob = 0;                                                           \
      for (int d = 0; d < on; ++d) {                                                             \
        int64_t c = idx / so[d];                                                                 \
        idx %= so[d];                                                                            \
        oa += c * sa[d];                                                                         \
        ob += c * sb[d];                                                                         \
      }                                                                                          \
      T x = LOAD_AS(T, a, adt, oa), y = LOAD_AS(T, b, bdt, ob), r;                               \
      switch (op) {                                                                              \
        case B_ADD: r = (T)(x + y); break;                                                       \
        case B_SUB: r = (T)(x - y); break;                                                       \
        case B_MUL: r = (T)(x * y); break;                                                       \
        case B_DIV: r = ISF ? (T)(x / y) : (y == 0 ? (T)0 : (T)(x / y)); break;                  \
        case B_POW: r = (T)POWF(x, y); break;                                                    \
        case B_EQ: r = (T)(x == y); break;                                                       \
        case B_NE: r = (T)(x != y); break;                                                       \
        case B_GE: r = (T)(x >= y); break;                                                       \
        case B_LE: r = (T)(x <= y); break;                                                       \
        case B_GT: r = (T)(x > y); break;                                                        \
        case B_LT: r = (T)(x < y); break;                                                        \
        case B_ABS_BW: r = x > (T)0 ? y : (x < (T)0 ? (T)(-y) : (T)0); break;                   \
        default: r = (x > lo && x < hi) ? y : (T)0; break;                                       \
      }                                                                                          \
      out[i] = r;                                                                                \
    }                                                                                            \
  }                                                                                              \
  static void NAME##_un(int op, const T* in, T* out, int64_t n, double p0, double p1) {          \
    T lo = ISF ? (T)p0 : SAT(T, LO, HI, p0), hi = ISF ? (T)p1 : SAT(T, LO, HI, p1);              \
    for (int64_t i = 0; i < n; ++i) {                                                            \
      T x = in[i], r;                                                                            \
      switch (op) {                                                                              \
        case U_NEG: r = (T)(-x); break;                                                          \
        case U_EXP: r = ISF ? (T)(sizeof(T) == 4 ? expf((float)x) : exp((double)x)) : (T)exp((double)x); break;  \
        case U_LOG: r = ISF ? (T)(sizeof(T) == 4 ? logf((float)x) : log((double)x)) : (T)log((double)x); break;  \
        case U_SQRT: r = ISF ? (T)(sizeof(T) == 4 ? sqrtf((float)x) : sqrt((double)x)) : (T)sqrt((double)x); break; \
        case U_ABS: r = (T)ABSF(x); break;                                                       \
        case U_SIN: r = ISF ? (T)(sizeof(T) == 4 ? sinf((float)x) : sin((double)x)) : (T)sin((double)x); break;  \
        case U_COS: r = ISF ? (T)(sizeof(T) == 4 ? cosf((float)x) : cos((double)x)) : (T)cos((double)x); break;  \
        case U_TAN: r = ISF ? (T)(sizeof(T) == 4 ? tanf((float)x) : tan((double)x)) : (T)tan((double)x); break;  \
        default: r = x < lo ? lo : (x > hi ? hi : x); break;                                     \
      }                                                                                          \
      out[i] = r;                                                                                \
    }                                                                                            \
  }

static double powd(double a, double b) { return pow(a, b); }
static float powf2(float a, float b) { return powf(a, b); }
static double fabsd(double a) { return fabs(a); }
static float fabsf2(float a) { return fabsf(a); }

DEF_BINARY(bool, bin_b, 0, powd, fabsd, 0, 1)
DEF_BINARY(int16_t, bin_i16, 0, powd, fabsd, INT16_MIN, INT16_MAX)
DEF_BINARY(int32_t, bin_i32, 0, powd, fabsd, INT32_MIN, INT32_MAX)
DEF_BINARY(int64_t, bin_i64, 0, powd, fabsd, INT64_MIN, INT64_MAX)
DEF_BINARY(float, bin_f32, 1, powf2, fabsf2, 0, 0)
DEF_BINARY(double, bin_f64, 1, powd, fabsd, 0, 0)

int lo_binary(int op, int out_dt, const void* a, int a_dt, const int64_t* a_shape, int a_nd,
              const void* b, int b_dt, const int64_t* b_shape, int b_nd, void* out, double p0,
              double p1) {
  int64_t osh[MAXD];
  int on = 0;
  if (bshape(a_shape, a_nd, b_shape, b_nd, osh, &on)) return 1;
  switch (out_dt) {
    case D_BOOL: bin_b(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    case D_I16: bin_i16(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    case D_I32: bin_i32(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    case D_I64: bin_i64(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    case D_F32: bin_f32(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    case D_F64: bin_f64(op, a, a_dt, a_shape, a_nd, b, b_dt, b_shape, b_nd, out, osh, on, p0, p1); break;
    default: return 1;
  }
  return 0;
}

int lo_unary(int op, int dt, const void* in, void* out, int64_t n, double p0, double p1) {
  switch (dt) {
    case D_BOOL: bin_b_un(op, in, out, n, p0, p1); break;
    case D_I16: bin_i16_un(op, in, out, n, p0, p1); break;
    case D_I32: bin_i32_un(op, in, out, n, p0, p1); break;
    case D_I64: bin_i64_un(op, in, out, n, p0, p1); break;
    case D_F32: bin_f32_un(op, in, out, n, p0, p1); break;
    case D_F64: bin_f64_un(op, in, out, n, p0, p1); break;
    default: return 1;
  }
  return 0;
}

/* vectorized_reduct_kernel (csrc/src/tensor/cpu/reduct.cpp:7-20): output i
 * walks its reduced elements in order; identities from kernels.hpp:153-172. */
#define DEF_REDUCE(T, NAME, LOWEST, HIGHEST)                                                     \
  static void NAME(int op, const T* in, const int64_t* shape, int nd, int axis, T* out) {      \
    int64_t outer = 1, inner = 1, R = shape[axis];                                               \
    for (int i = 0; i < axis; ++i) outer *= shape[i];                                            \
    for (int i = axis + 1; i < nd; ++i) inner *= shape[i];                                       \
    for (int64_t o = 0; o < outer; ++o)                                                          \
      for (int64_t c = 0; c < inner; ++c) {                                                      \
        T acc = op == R_SUM ? (T)0 : op == R_PROD ? (T)1 : op == R_MAX ? (T)(LOWEST) : (T)(HIGHEST); \
        for (int64_t r = 0; r < R; ++r) {                                                        \
          T x = in[(o * R + r) * inner + c];                                                     \
          switch (op) {                                                                          \
            case R_SUM: acc = (T)(acc + x); break;                                               \
            case R_PROD: acc = (T)(acc * x); break;                                              \
            case R_MAX: acc = (acc < x) ? x : acc; break;                                        \
            default: acc = (x < acc) ? x : acc; break;                                           \
          }                                                                                      \
        }                                                                                        \
        out[o * inner + c] = acc;                                                                \
      }                                                                                          \
  }

#include <float.h>
DEF_REDUCE(bool, red_b, 0, 1)
DEF_REDUCE(int16_t, red_i16, INT16_MIN, INT16_MAX)
DEF_REDUCE(int32_t, red_i32, INT32_MIN, INT32_MAX)
DEF_REDUCE(int64_t, red_i64, INT64_MIN, INT64_MAX)
DEF_REDUCE(float, red_f32, -FLT_MAX, FLT_MAX)
DEF_REDUCE(double, red_f64, -DBL_MAX, DBL_MAX)

int lo_reduce(int op, int dt, const void* in, const int64_t* shape, int nd, int axis, void* out) {
  if (axis < 0 || axis >= nd) return 1;
  switch (dt) {
    case D_BOOL: red_b(op, in, shape, nd, axis, out); break;
    case D_I16: red_i16(op, in, shape, nd, axis, out); break;
    case D_I32: red_i32(op, in, shape, nd, axis, out); break;
    case D_I64: red_i64(op, in, shape, nd, axis, out); break;
    case D_F32: red_f32(op, in, shape, nd, axis, out); break;
    case D_F64: red_f64(op, in, shape, nd, axis, out); break;
    default: return 1;
  }
  return 0;
}

/* cpuMatmulKernel (csrc/src/tensor/cpu/matrix.cpp:8-19): sum in the output
 * type over k in order. */
#define DEF_MATMUL(T, NAME)                                                                      \
  static void NAME(const void* A, int adt, const void* B, int bdt, T* C, int64_t m, int64_t k,  \
                   int64_t n) {                                                                  \
    for (int64_t i = 0; i < m; ++i)                                                              \
      for (int64_t j = 0; j < n; ++j) {                                                          \
        T sum = 0;                                                                               \
        for (int64_t t = 0; t < k; ++t)                                                          \
          sum = (T)(sum + (T)(LOAD_AS(T, A, adt, i * k + t) * LOAD_AS(T, B, bdt, t * n + j)));   \
        C[i * n + j] = sum;                                                                      \
      }                                                                                          \
  }
DEF_MATMUL(bool, mm_b)
DEF_MATMUL(int16_t, mm_i16)
DEF_MATMUL(int32_t, mm_i32)
DEF_MATMUL(int64_t, mm_i64)
DEF_MATMUL(float, mm_f32)
DEF_MATMUL(double, mm_f64)

int lo_matmul(int out_dt, const void* A, int a_dt, const void* B, int b_dt, void* C, int64_t m,
              int64_t k, int64_t n) {
  switch (out_dt) {
    case D_BOOL: mm_b(A, a_dt, B, b_dt, C, m, k, n); break;
    case D_I16: mm_i16(A, a_dt, B, b_dt, C, m, k, n); break;
    case D_I32: mm_i32(A, a_dt, B, b_dt, C, m, k, n); break;
    case D_I64: mm_i64(A, a_dt, B, b_dt, C, m, k, n); break;
    case D_F32: mm_f32(A, a_dt, B, b_dt, C, m, k, n); break;
    case D_F64: mm_f64(A, a_dt, B, b_dt, C, m, k, n); break;
    default: return 1;
  }
  return 0;
}

/* cpuTransposeKernel (csrc/src/tensor/cpu/matrix.cpp:21-25). */
int lo_transpose(int dt, const void* in, void* out, int64_t m, int64_t n) {
  static const size_t sz[] = {1, 2, 4, 8, 4, 8};
  if (dt < 0 || dt > 5) return 1;
  size_t es = sz[dt];
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j)
      memcpy((char*)out + (j * m + i) * es, (const char*)in + (i * n + j) * es, es);
  return 0;
}
