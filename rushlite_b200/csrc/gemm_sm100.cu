// fp32 GEMM entry used by lmpb_matmul / lmpb_gemm_f32.
#include "common.cuh"

namespace lmpb {

lmpb_status gemm_f32_simt(int ta, int tb, const float* A, const float* B, float* C, int64_t m,
                          int64_t n, int64_t k, float beta, cudaStream_t st);

lmpb_status gemm_f32_sm100(int trans_a, int trans_b, const float* A, const float* B, float* C,
                           int64_t m, int64_t n, int64_t k, float beta, cudaStream_t st) {
  return gemm_f32_simt(trans_a, trans_b, A, B, C, m, n, k, beta, st);
}

}  // namespace lmpb
