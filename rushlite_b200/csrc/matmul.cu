// Matmul entry points.  fp32 x fp32 -> fp32 goes to the tcgen05 split-fp16 GEMM
// (gemm_sm100.cu); every other dtype combination runs the SIMT kernel here,
// which accumulates in the output dtype over k in order, like the
// reference's cpuMatmulKernel (csrc/src/tensor/cpu/matrix.cpp:8-19).
#include "common.cuh"

namespace lmpb {

// Declared in gemm_sm100.cu.
lmpb_status gemm_f32_sm100(int trans_a, int trans_b, const float* A, const float* B, float* C,
                           int64_t m, int64_t n, int64_t k, float beta, cudaStream_t st,
                           const float* bias = nullptr, int clamp = 0, double lo = 0.0, double hi = 0.0);
unsigned int gemm_take_error();

namespace {

constexpr int TS = 16;

template <typename O>
__global__ void __launch_bounds__(TS* TS)
    matmul_simt_kernel(const void* __restrict__ A, int adt, const void* __restrict__ B, int bdt,
                       O* __restrict__ C, int64_t m, int64_t k, int64_t n) {
  __shared__ O As[TS][TS + 1];
  __shared__ O Bs[TS][TS + 1];
  const int tx = threadIdx.x % TS, ty = threadIdx.x / TS;
  const int64_t row = (int64_t)blockIdx.y * TS + ty;
  const int64_t col = (int64_t)blockIdx.x * TS + tx;
  O acc = O(0);
  for (int64_t k0 = 0; k0 < k; k0 += TS) {
    const int64_t ka = k0 + tx, kb = k0 + ty;
    As[ty][tx] = (row < m && ka < k) ? load_as<O>(A, adt, row * k + ka) : O(0);
    Bs[ty][tx] = (kb < k && col < n) ? load_as<O>(B, bdt, kb * n + col) : O(0);
    __syncthreads();
    const int kk = (int)((k - k0) < TS ? (k - k0) : TS);
    for (int t = 0; t < kk; ++t) acc = static_cast<O>(r_add(acc, static_cast<O>(r_mul(As[ty][t], Bs[t][tx]))));
    __syncthreads();
  }
  if (row < m && col < n) C[row * n + col] = acc;
}

}  // namespace
}  // namespace lmpb

using namespace lmpb;

extern "C" lmpb_status lmpb_matmul(int out_dtype, const void* A, int a_dtype, const void* B,
                                   int b_dtype, void* C, int64_t m, int64_t k, int64_t n,
                                   void* stream) {
  LMPB_CHECK_ARG(valid_dtype(out_dtype) && valid_dtype(a_dtype) && valid_dtype(b_dtype),
                 "lmpb_matmul: invalid dtype");
  LMPB_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "lmpb_matmul: negative size");
  if (m == 0 || n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(C != nullptr && (k == 0 || (A && B)), "lmpb_matmul: null pointer");
  cudaStream_t st = as_stream(stream);
  if (k == 0) return lmpb_fill(out_dtype, C, m * n, 0.0, stream);
  if (out_dtype == LMPB_FLOAT32 && a_dtype == LMPB_FLOAT32 && b_dtype == LMPB_FLOAT32)
    return gemm_f32_sm100(0, 0, (const float*)A, (const float*)B, (float*)C, m, n, k, 0.f, st);
  LMPB_CHECK_ARG((m + TS - 1) / TS <= 65535, "lmpb_matmul: m too large for the SIMT path");
  dim3 grid((unsigned)((n + TS - 1) / TS), (unsigned)((m + TS - 1) / TS));
  LMPB_DISPATCH_DTYPE(out_dtype, O, {
    matmul_simt_kernel<O><<<grid, TS * TS, 0, st>>>(A, a_dtype, B, b_dtype, (O*)C, m, k, n);
    return launch_status("matmul_simt_kernel");
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_matmul: invalid dtype");
}

extern "C" lmpb_status lmpb_gemm_f32(int trans_a, int trans_b, const float* A, const float* B,
                                     float* C, int64_t m, int64_t n, int64_t k, float beta,
                                     void* stream) {
  LMPB_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "lmpb_gemm_f32: negative size");
  LMPB_CHECK_ARG(beta == 0.f || beta == 1.f, "lmpb_gemm_f32: beta must be 0 or 1");
  if (m == 0 || n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(C != nullptr && (k == 0 || (A && B)), "lmpb_gemm_f32: null pointer");
  if (k == 0) return beta == 0.f ? lmpb_fill(LMPB_FLOAT32, C, m * n, 0.0, stream) : LMPB_OK;
  return gemm_f32_sm100(trans_a, trans_b, A, B, C, m, n, k, beta, as_stream(stream));
}

extern "C" lmpb_status lmpb_gemm_f32_bias_act(int trans_a, int trans_b, const float* A, const float* B,
                                              float* C, int64_t m, int64_t n, int64_t k, const float* bias,
                                              int clamp, double lo, double hi, void* stream) {
  LMPB_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "lmpb_gemm_f32_bias_act: negative size");
  if (m == 0 || n == 0) return LMPB_OK;
  LMPB_CHECK_ARG(C != nullptr && (k == 0 || (A && B)), "lmpb_gemm_f32_bias_act: null pointer");
  if (k == 0) {  // the product is zero: C = clamp(0 + bias)
    cudaStream_t st = as_stream(stream);
    lmpb_status s = lmpb_fill(LMPB_FLOAT32, C, m * n, 0.0, st);
    if (s == LMPB_OK && bias) {
      const int64_t cs[2] = {m, n}, bs[1] = {n};
      s = lmpb_binary(LMPB_ADD, LMPB_FLOAT32, C, LMPB_FLOAT32, cs, 2, bias, LMPB_FLOAT32, bs, 1, C, 0.0, 0.0, st);
    }
    if (s == LMPB_OK && clamp) s = lmpb_unary(LMPB_CLAMP, LMPB_FLOAT32, C, C, m * n, lo, hi, st);
    return s;
  }
  return gemm_f32_sm100(trans_a, trans_b, A, B, C, m, n, k, 0.f, as_stream(stream), bias, clamp, lo, hi);
}

namespace lmpb {
unsigned peer_take_error();
}
using lmpb::peer_take_error;

extern "C" lmpb_status lmpb_device_error(void) {
  LMPB_CUDA_TRY(cudaDeviceSynchronize());
  const unsigned int e = gemm_take_error();
  const unsigned int pe = peer_take_error();
  if (pe != 0)
    return set_error(LMPB_ERR_TIMEOUT, "fused reduce + all-reduce: a bounded wait for another GPU expired (code " +
                                           std::to_string(pe) + ")");
  if (e == 0) return LMPB_OK;
  return set_error(LMPB_ERR_TIMEOUT, "tensor-core GEMM: a bounded wait expired (code " + std::to_string(e) + ")");
}
