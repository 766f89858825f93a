// fp32 SIMT GEMM with transposes and beta, used for shapes the tensor-core
// path cannot describe with TMA (a row pitch that is not a multiple of 16
// bytes, e.g. the README MLP's N = 10) and for tiny problems where a 128x128
// tensor-core tile would be mostly padding.
//
// 64x64 CTA tile, k-step 16, 256 threads each owning a 4x4 register block.
// The fp32 product is accumulated with explicit round-to-nearest multiply and
// add (no FMA), k in order, like the reference's sequential dot product.
#include "common.cuh"

namespace lmpb {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

__global__ void __launch_bounds__(256)
    gemm_simt_kernel(int ta, int tb, const float* __restrict__ A, const float* __restrict__ B,
                     float* __restrict__ C, int64_t m, int64_t n, int64_t k, float beta) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 4 x 4 each
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int64_t k0 = 0; k0 < k; k0 += BK) {
    // A tile: BM x BK, 1024 elements, 4 per thread
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int idx = tid + e * 256;
      int r, c;
      if (ta) { r = idx % BM; c = idx / BM; } else { r = idx / BK; c = idx % BK; }
      int64_t gr = m0 + r, gc = k0 + c;
      float v = 0.f;
      if (gr < m && gc < k) v = ta ? A[gc * m + gr] : A[gr * k + gc];
      As[c][r] = v;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int idx = tid + e * 256;
      int r, c;  // r over k, c over n
      if (tb) { r = idx % BK; c = idx / BK; } else { r = idx / BN; c = idx % BN; }
      int64_t gr = k0 + r, gc = n0 + c;
      float v = 0.f;
      if (gr < k && gc < n) v = tb ? B[gc * k + gr] : B[gr * n + gc];
      Bs[r][c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < BK; ++t) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[t][tr * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[t][tc * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t r = m0 + tr * 4 + i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t c = n0 + tc * 4 + j;
      if (c >= n) continue;
      float v = acc[i][j];
      if (beta != 0.f) v = __fadd_rn(C[r * n + c], v);
      C[r * n + c] = v;
    }
  }
}

}  // namespace

lmpb_status gemm_f32_simt(int ta, int tb, const float* A, const float* B, float* C, int64_t m,
                          int64_t n, int64_t k, float beta, cudaStream_t st) {
  if ((m + BM - 1) / BM > 65535)
    return set_error(LMPB_ERR_UNSUPPORTED, "gemm_f32_simt: m too large");
  dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
  gemm_simt_kernel<<<grid, 256, 0, st>>>(ta, tb, A, B, C, m, n, k, beta);
  return launch_status("gemm_simt_kernel");
}

}  // namespace lmpb
