/*
 * lamp3_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference Lamp3 CPU kernels, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline as the checker.  It is
 * never linked into, or called by, the product (rushlite_b200).
 *
 * Pinned against: the reference's own CPU build (oracle/_ref, compiled from
 * the reference sources by oracle/Makefile) on seeded inputs, and the golden
 * vectors in tests/golden/ transcribed from the reference's C++ known-answer
 * tests (csrc/tests/tensor_tests.cpp, csrc/tests/autograd_tests.cpp).
 *
 * dtype / op codes are those of include/lmpb.h.  All arrays are row-major
 * contiguous host memory.
 */
#ifndef LAMP3_ORACLE_H_
#define LAMP3_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out = op(a, b) with broadcasting; both operands converted to out_dt first. */
int lo_binary(int op, int out_dt, const void* a, int a_dt, const int64_t* a_shape, int a_nd,
              const void* b, int b_dt, const int64_t* b_shape, int b_nd, void* out, double p0,
              double p1);
/* out[i] = op(in[i]), same dtype. */
int lo_unary(int op, int dt, const void* in, void* out, int64_t n, double p0, double p1);
/* keep-dim reduction along axis, sequential per output like the reference. */
int lo_reduce(int op, int dt, const void* in, const int64_t* shape, int nd, int axis, void* out);
/* C[m,n] = A[m,k] B[k,n], accumulated in out_dt over k in order. */
int lo_matmul(int out_dt, const void* A, int a_dt, const void* B, int b_dt, void* C, int64_t m,
              int64_t k, int64_t n);
int lo_transpose(int dt, const void* in, void* out, int64_t m, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
