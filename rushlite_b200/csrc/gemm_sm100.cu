// fp32 GEMM on the B200 tensor cores: three fp16 products per operand pair
// (tcgen05.mma kind::f16, fp32 accumulation in TMEM), TMA-fed.
//
//   C[m,n] = op(A)[m,k] · op(B)[k,n] (+ C when beta = 1), fp32 in and out.
//
// fp32 accuracy from fp16 tensor cores (the split of Ootomo & Yokota, 2022,
// "Recovering single precision accuracy from Tensor Cores while surpassing
// the FP32 theoretical peak performance", with a power-of-two scale per row):
// every row r of op(A) (and every column of op(B)) is scaled by 2^e_r so its
// largest finite magnitude lies in [2^14, 2^15); each scaled element x becomes
//     hi = fp16(x),  lo = fp16((x - hi) * 2^11)        (round to nearest)
// and the tile accumulates big = hi·hi and small = hi·lo + lo·hi in two fp32
// TMEM accumulators; the epilogue forms (big + small * 2^-11) * 2^-(e_r+e_c).
// hi and lo each carry 11 significant bits, as tf32 would, but kind::f16
// runs at twice the kind::tf32 rate.  The dropped lo·lo term is 2^-22
// relative.  Scales are exact powers of two; a scaled element below
// 2^-13 (2^-27 of its row's maximum) loses bits of lo to fp16 subnormals,
// an absolute error under 2^-40 of the row's largest product.  Inf and NaN
// pass through: the scale ignores non-finite values and lo is 0 where hi is inf.
//
// 1. A split pass per operand: the row maxima (a column-max kernel when the
//    operand must be transposed), then hi/lo fp16 planes, K-major (rows of K
//    contiguous, K padded to the k-block), transposing when the caller's
//    layout is not K-major.  It reads each input element twice (the second
//    read mostly from L2) and writes 4 bytes.
// 2. The GEMM kernels.  For m >= 256 the CTA-pair kernel: 2-CTA clusters,
//    persistent, each pair walking 256 x BN output tiles in grouped order
//    with tcgen05.mma.cta_group::2 (M = 256); each CTA loads its own 128
//    rows of A and 128 rows (half) of B per k-block, so B is loaded once per
//    pair.  10 warps per CTA:
//      warp 0     TMA producer (one elected thread): 4 tiles per k-block
//                 (A hi/lo, B hi/lo) into a 6-deep shared-memory ring,
//                 64-byte swizzled; the bytes of both CTAs complete on the
//                 leader CTA's mbarrier;
//      warp 1     owns two TMEM accumulators (128 lanes x BN fp32 columns
//                 each: hi*hi and the cross terms); in the leader CTA one
//                 thread issues 3 products x BK/16 MMAs per k-block, then a
//                 tcgen05.commit that frees the stage in both CTAs;
//      warps 2-9  epilogue: two warps per TMEM lane quarter, one per
//                 128-column half, pull their combined values into registers
//                 and release the accumulators, then unscale, add C, apply
//                 the optional bias/clamp and store (overlapping the next
//                 tile's MMAs).  Long K may be split in two; see the split-K
//                 note in the pair kernel.
//    For 64 <= m < 256 a single-CTA kernel with 128 x BN tiles (6 warps:
//    producer, MMA issuer, 4 epilogue warps) does the same per tile.
//    Every mbarrier wait is bounded (clock64); on expiry the kernel records
//    an error code in a device word, stops issuing, frees TMEM and returns.
//    No TMA load is multicast: each CTA loads its own tiles; only the
//    commit's mbarrier arrival is multicast to the pair.
// Shapes that TMA cannot describe or that are too small for a 128-row tile
// use the SIMT kernel (gemm_simt.cu).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <vector>
#include <string>

#include "common.cuh"

namespace lmpb {

lmpb_status gemm_f32_simt(int ta, int tb, const float* A, const float* B, float* C, int64_t m,
                          int64_t n, int64_t k, float beta, cudaStream_t st);

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 32;      // 32 fp16 = 64 bytes per row = one 64B swizzle atom
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr int A_TILE = BM * BK * 2;  // 8 KB
constexpr int B_TILE = BN * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // 48 KB
// Two accumulators per tile: hi*hi in columns [0, BN), the cross terms
// hi*lo + lo*hi (scaled by 2^11) in [BN, 2BN).  Keeping them apart also keeps
// the tensor core's truncating fp32 accumulation to one product per add in
// the big accumulator.
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// CTA-pair kernel (cta_group::2): 256 x BN tiles, each CTA loading 128 rows
// of A and 128 rows (half) of B per k-block.
constexpr int P_STAGES = 6;
constexpr int P_A_TILE = 128 * BK * 2;                       // 8 KB
constexpr int P_B_TILE = 128 * BK * 2;                       // 8 KB: half of N
constexpr int P_STAGE_BYTES = 2 * P_A_TILE + 2 * P_B_TILE;  // 32 KB per CTA
constexpr int P_EPI_BYTES = 8 * 32 * 32 * 4;  // per epilogue warp a 32 x 32 fp32 staging block
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256 + P_EPI_BYTES;
constexpr int P_TM = 256;  // output tile rows per pair
constexpr int kThreadsP = 320;  // producer, MMA, 8 epilogue warps

constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

// Device error word: 0 = ok, else the code of the first bounded wait that expired.
__device__ unsigned int g_gemm_error = 0;

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the error word set to `code`) after kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned code) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicCAS(&g_gemm_error, 0u, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major, 64B-swizzled tile: rows of 64 bytes, 8-row atoms 512 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);  // start address
  d |= (uint64_t)1 << 16;                  // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;         // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;                  // SWIZZLE_64B
  return d;
}

// kind::f16 instruction descriptor: D f32, A and B both f16 (format 0), both
// K-major, M=128, N=BN.
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])::"memory");  // uses of r stay after the wait
}

// tcgen05.ld without the wait, so several loads can be in flight.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Orders every use of r after the preceding tcgen05.wait::ld: the registers
// of an asynchronous tcgen05.ld are only valid once the wait has returned.
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])::"memory");
}

// ------------------------------------------------------------ split pass

// |x| for finite x, else 0: row scales ignore Inf and NaN.
__device__ __forceinline__ float finite_abs(float x) {
  const float a = fabsf(x);
  return a < INFINITY ? a : 0.f;
}

// e such that mx * 2^e lies in [2^14, 2^15); 0 for a row without finite
// non-zero values.
__host__ __device__ __forceinline__ int row_exp(float mx) {
  if (!(mx > 0.f) || !(mx < INFINITY)) return 0;
  int p;
  frexpf(mx, &p);  // mx = f * 2^p, f in [0.5, 1)
  return 15 - p;
}

// x * 2^e, exact unless the result is subnormal.  Row exponents lie in
// [-114, 163], so the epilogue's e = -(e_row + e_col) stays within +-330:
// outside one power of two's range, three steps of at most 2^+-126 each.
// The steps share e's sign, so every intermediate lies between x and the
// result, and only a subnormal result can be rounded (possibly twice).  The
// steps are plain multiplies: the epilogue inlines this 128 times per
// thread, and a library call there bloats the kernel past the instruction
// cache (measured on B200, the 1024 x 4096 x 4096 product with its split
// pass: 182 us with ldexpf in the rare branch, 146 us without).
__device__ __forceinline__ float pow2_scale(float x, int e) {
  if (e >= -126 && e <= 127) return x * __int_as_float((e + 127) << 23);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int s = max(-126, min(126, e));
    x *= __int_as_float((s + 127) << 23);
    e -= s;
  }
  return x;
}

// Scaled element -> (hi, lo): hi = fp16(xs), lo = fp16((xs - hi) * 2^11).
__device__ __forceinline__ void split16(float xs, __half& hi, __half& lo) {
  hi = __float2half_rn(xs);
  const float h = __half2float(hi);
  lo = __hisinf(hi) ? __float2half_rn(0.f) : __float2half_rn(__fsub_rn(xs, h) * 2048.f);
}

__device__ __forceinline__ float block_max256(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  __syncthreads();  // red is reused by the next row
  return m;
}

// src is [rows, K] row-major (K-major already).  One CTA per row at a time:
// the row's finite max-abs, then hi/lo [rows, Kp] with zero padding; rowmax
// receives the max and expo the row's scale exponent (for the epilogue).  vec: K % 4 == 0 and src 16-byte aligned.
template <bool vec>
__global__ void __launch_bounds__(256)
    split_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp, __half* __restrict__ hi,
                      __half* __restrict__ lo, float* __restrict__ rowmax, int* __restrict__ expo) {
  __shared__ float red[8];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = src + r * K;
    float mx = 0.f;
    if (vec) {
      const float4* row4 = reinterpret_cast<const float4*>(row);
      for (int64_t c = threadIdx.x; c < K / 4; c += 256) {
        const float4 v = __ldg(row4 + c);
        mx = fmaxf(fmaxf(mx, fmaxf(finite_abs(v.x), finite_abs(v.y))), fmaxf(finite_abs(v.z), finite_abs(v.w)));
      }
    } else {
      for (int64_t c = threadIdx.x; c < K; c += 256) mx = fmaxf(mx, finite_abs(__ldg(row + c)));
    }
    mx = block_max256(mx, red);
    const int e = row_exp(mx);
    if (threadIdx.x == 0) {
      rowmax[r] = mx;
      expo[r] = e;
    }
    __half* hrow = hi + r * Kp;
    __half* lrow = lo + r * Kp;
    if (vec) {  // Kp % 4 == 0; 4 halves = 8 bytes per store
      const float4* row4 = reinterpret_cast<const float4*>(row);
      for (int64_t c = threadIdx.x; c < Kp / 4; c += 256) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c * 4 < K) v = __ldg(row4 + c);
        __half h[4], l[4];
        split16(pow2_scale(v.x, e), h[0], l[0]);
        split16(pow2_scale(v.y, e), h[1], l[1]);
        split16(pow2_scale(v.z, e), h[2], l[2]);
        split16(pow2_scale(v.w, e), h[3], l[3]);
        *reinterpret_cast<uint2*>(hrow + c * 4) = *reinterpret_cast<const uint2*>(h);
        *reinterpret_cast<uint2*>(lrow + c * 4) = *reinterpret_cast<const uint2*>(l);
      }
    } else {
      for (int64_t c = threadIdx.x; c < Kp; c += 256) {
        __half h = __float2half_rn(0.f), l = h;
        if (c < K) split16(pow2_scale(row[c], e), h, l);
        hrow[c] = h;
        lrow[c] = l;
      }
    }
  }
}

// split_rows_kernel<true> for rows of at most NV * 1024 floats: the row is
// read once into registers (NV 16-byte loads per thread, all in flight), its
// max taken there, then split from the registers; same results.
template <int NV>
__global__ void __launch_bounds__(256)
    split_rows_reg_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp, __half* __restrict__ hi,
                          __half* __restrict__ lo, float* __restrict__ rowmax, int* __restrict__ expo) {
  __shared__ float red[8];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4* row4 = reinterpret_cast<const float4*>(src + r * K);
    float4 v[NV];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t c = threadIdx.x + i * 256;
      v[i] = c * 4 < K ? __ldg(row4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < NV; ++i)
      mx = fmaxf(fmaxf(mx, fmaxf(finite_abs(v[i].x), finite_abs(v[i].y))), fmaxf(finite_abs(v[i].z), finite_abs(v[i].w)));
    mx = block_max256(mx, red);
    const int e = row_exp(mx);
    if (threadIdx.x == 0) {
      rowmax[r] = mx;
      expo[r] = e;
    }
    __half* hrow = hi + r * Kp;
    __half* lrow = lo + r * Kp;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t c = threadIdx.x + i * 256;
      if (c * 4 < Kp) {
        __half h[4], l[4];
        split16(pow2_scale(v[i].x, e), h[0], l[0]);
        split16(pow2_scale(v[i].y, e), h[1], l[1]);
        split16(pow2_scale(v[i].z, e), h[2], l[2]);
        split16(pow2_scale(v[i].w, e), h[3], l[3]);
        *reinterpret_cast<uint2*>(hrow + c * 4) = *reinterpret_cast<const uint2*>(h);
        *reinterpret_cast<uint2*>(lrow + c * 4) = *reinterpret_cast<const uint2*>(l);
      }
    }
  }
}

// src is [K, rows] row-major (the operand transposed): the finite max-abs of
// every column r over K, as float bits into colmax[r] (zeroed beforehand;
// non-negative floats order like their bits).  CTA = 64 columns x 256 k.
__global__ void __launch_bounds__(256)
    colmax_kernel(const float* __restrict__ src, int64_t rows, int64_t K, unsigned* __restrict__ colmax) {
  __shared__ float part[4][64];
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  const int64_t r = (int64_t)blockIdx.x * 64 + tx;
  const int64_t k0 = (int64_t)blockIdx.y * 256, k1 = k0 + 256 < K ? k0 + 256 : K;
  float mx = 0.f;
  if (r < rows)
    for (int64_t k = k0 + ty; k < k1; k += 4) mx = fmaxf(mx, finite_abs(__ldg(src + k * rows + r)));
  part[ty][tx] = mx;
  __syncthreads();
  if (ty == 0 && r < rows) {
    mx = fmaxf(fmaxf(part[0][tx], part[1][tx]), fmaxf(part[2][tx], part[3][tx]));
    if (mx > 0.f) atomicMax(colmax + r, __float_as_uint(mx));
  }
}

// colmax_kernel with 16-byte loads (rows % 4 == 0, src 16-byte aligned): a
// CTA is 16 column quads (64 columns) x 16 k-lanes over one k chunk (a multiple of 64), each thread
// with 4 loads in flight.  Max is order-free, so the maxima are the same.
__global__ void __launch_bounds__(256)
    colmax4_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int kchunk, unsigned* __restrict__ colmax) {
  __shared__ float4 part[16][16];
  const int tq = threadIdx.x & 15, tk = threadIdx.x >> 4;
  const int64_t r = (int64_t)blockIdx.x * 64 + 4 * tq;
  const int64_t k0 = (int64_t)blockIdx.y * kchunk, k1 = k0 + kchunk < K ? k0 + kchunk : K;
  float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r < rows) {
    const float* base = src + r;
    int64_t k = k0 + tk;
    for (; k + 48 < k1; k += 64) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(reinterpret_cast<const float4*>(base + (k + 16 * u) * rows));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        m.x = fmaxf(m.x, finite_abs(v[u].x));
        m.y = fmaxf(m.y, finite_abs(v[u].y));
        m.z = fmaxf(m.z, finite_abs(v[u].z));
        m.w = fmaxf(m.w, finite_abs(v[u].w));
      }
    }
    for (; k < k1; k += 16) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(base + k * rows));
      m.x = fmaxf(m.x, finite_abs(v.x));
      m.y = fmaxf(m.y, finite_abs(v.y));
      m.z = fmaxf(m.z, finite_abs(v.z));
      m.w = fmaxf(m.w, finite_abs(v.w));
    }
  }
  part[tk][tq] = m;
  __syncthreads();
  if (threadIdx.x < 64) {
    const int q = threadIdx.x >> 2, c = threadIdx.x & 3;
    const int64_t col = (int64_t)blockIdx.x * 64 + threadIdx.x;
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v = part[i][q];
      mx = fmaxf(mx, c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w);
    }
    if (col < rows && mx > 0.f) atomicMax(colmax + col, __float_as_uint(mx));
  }
}

// src is [K, rows] row-major: hi/lo [rows, Kp] through 64 x 64 shared-memory
// tiles, scaled by the column maxima; reads along rows and half2 writes along
// K both coalesced.
__global__ void __launch_bounds__(256)
    split_transpose_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp,
                           const float* __restrict__ colmax, __half* __restrict__ hi, __half* __restrict__ lo,
                           int* __restrict__ expo) {
  __shared__ float tile[64][65];
  const int64_t k0 = (int64_t)blockIdx.y * 64, r0 = (int64_t)blockIdx.x * 64;
  {
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
#pragma unroll
    for (int j = ty; j < 64; j += 4) {
      const int64_t k = k0 + j, r = r0 + tx;
      tile[j][tx] = (k < K && r < rows) ? __ldg(src + k * rows + r) : 0.f;
    }
  }
  __syncthreads();
  const int kx = threadIdx.x & 31, ry = threadIdx.x >> 5;  // 32 k-pairs x 8 rows
  const int64_t k = k0 + 2 * kx;
#pragma unroll
  for (int j = ry; j < 64; j += 8) {
    const int64_t r = r0 + j;
    if (r < rows && k < Kp) {  // Kp is even, so k + 1 < Kp too
      const int e = row_exp(__ldg(colmax + r));
      if (blockIdx.y == 0 && kx == 0) expo[r] = e;  // once per row
      __half h0, h1, l0, l1;
      split16(pow2_scale(tile[2 * kx][j], e), h0, l0);
      split16(pow2_scale(tile[2 * kx + 1][j], e), h1, l1);
      *reinterpret_cast<__half2*>(hi + r * Kp + k) = __halves2half2(h0, h1);
      *reinterpret_cast<__half2*>(lo + r * Kp + k) = __halves2half2(l0, l1);
    }
  }
}

// split_transpose_kernel with 16-byte traffic both ways (rows % 4 == 0, src
// 16-byte aligned): the 64 x 64 tile is filled by float4 loads along the
// rows, and each thread writes 8 adjacent k (16 bytes) of one output row.
__global__ void __launch_bounds__(256)
    split_transpose4_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp,
                            const float* __restrict__ colmax, __half* __restrict__ hi, __half* __restrict__ lo,
                            int* __restrict__ expo) {
  __shared__ float tile[64][65];
  const int64_t k0 = (int64_t)blockIdx.y * 64, r0 = (int64_t)blockIdx.x * 64;
  {
    const int tq = threadIdx.x & 15, tk = threadIdx.x >> 4;  // 16 column-quads x 16 k
#pragma unroll
    for (int j = tk; j < 64; j += 16) {
      const int64_t k = k0 + j, r = r0 + 4 * tq;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < K && r < rows) v = __ldg(reinterpret_cast<const float4*>(src + k * rows + r));
      tile[j][4 * tq] = v.x;
      tile[j][4 * tq + 1] = v.y;
      tile[j][4 * tq + 2] = v.z;
      tile[j][4 * tq + 3] = v.w;
    }
  }
  __syncthreads();
  const int kg = threadIdx.x & 7, ry = threadIdx.x >> 3;  // 8 groups of 8 k x 32 rows
  const int64_t k = k0 + 8 * kg;
#pragma unroll
  for (int j = ry; j < 64; j += 32) {
    const int64_t r = r0 + j;
    if (r < rows && k < Kp) {  // Kp is a multiple of 32, so all 8 are inside
      const int e = row_exp(__ldg(colmax + r));
      if (blockIdx.y == 0 && kg == 0) expo[r] = e;  // once per row
      __half h[8], l[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) split16(pow2_scale(tile[8 * kg + i][j], e), h[i], l[i]);
      *reinterpret_cast<uint4*>(hi + r * Kp + k) = *reinterpret_cast<const uint4*>(h);
      *reinterpret_cast<uint4*>(lo + r * Kp + k) = *reinterpret_cast<const uint4*>(l);
    }
  }
}

// ------------------------------------------------------------ GEMM kernel

// Tile t of a tiles_m x tiles_n grid in grouped order: 8 row-tiles at a time
// walk the column tiles, so concurrently running CTAs share B panels in L2.
// Work schedule, shared by the kernels and the host (and exported below so
// that tests check the very code the kernels run).
//
// Output tiles are visited in groups of 8 tile rows: tile t of a group walks
// down the group's rows first, so consecutive tiles share B columns in L2.
__host__ __device__ __forceinline__ void sched_tile(int t, int tiles_m, int tiles_n, int tm, int tn, int& m0,
                                                    int& n0) {
  const int group = 8;
  const int g = t / (group * tiles_n);
  const int first_m = g * group;
  const int gsize = min(tiles_m - first_m, group);
  const int local = t % (group * tiles_n);
  m0 = (first_m + local % gsize) * tm;
  n0 = (local / gsize) * tn;
}

// Split-K units: unit u is tile u / splits over k-blocks [kb0, kb1) of
// split u % splits, each split ceil(num_kb / splits) k-blocks long.
__host__ __device__ __forceinline__ void sched_unit(int u, int splits, int num_kb, int& t, int& kb0, int& kb1) {
  const int kb_per = (num_kb + splits - 1) / splits;
  t = u / splits;
  kb0 = (u % splits) * kb_per;
  kb1 = min(num_kb, kb0 + kb_per);
}

// A requested split count, reduced until every unit has a k-block: the last
// unit starts at (splits - 1) * kb_per, which must be below num_kb.
__host__ __device__ __forceinline__ int sched_clamp_splits(int splits, int num_kb) {
  splits = max(1, min(splits, max(1, num_kb)));
  while (splits > 1 && (splits - 1) * ((num_kb + splits - 1) / splits) >= num_kb) --splits;
  return splits;
}

// The split count the pair kernel runs with: forced > 0 is a tuning override
// (clamped as above); otherwise K is split in two when the run gets >= 5 %
// shorter, time ~ rounds(units) / splits with rounds = ceil(units / clusters),
// and only for long K (>= 256 k-blocks, K >= 8192): measured on B200, a split
// unit costs more than its share of the MMAs (4096^3: 2 splits 0.50 ms vs
// 0.46 ms unsplit, 4 splits 1.1 ms; 4096 x 8192 x 4096: 0.80 vs 0.84 ms;
// K = 32768: 2.8 vs 3.35 ms).
inline int sched_choose_splits(int64_t ntiles, int num_kb, int clusters, int forced) {
  if (clusters <= 0) return 1;
  if (forced > 0) return sched_clamp_splits(forced, num_kb);
  auto cost = [&](int sp) { return (double)((ntiles * sp + clusters - 1) / clusters) / sp; };
  return (num_kb >= 256 && cost(2) < cost(1) * 0.95) ? 2 : 1;
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& m0, int& n0) {
  sched_tile(t, tiles_m, tiles_n, BM, BN, m0, n0);
}

// As tile_coords, for the pair kernel's 256-row tiles.
__device__ __forceinline__ void tile_coords_pair(int t, int tiles_m, int tiles_n, int& m0, int& n0) {
  sched_tile(t, tiles_m, tiles_n, P_TM, BN, m0, n0);
}

// Optional epilogue after the product: + bias[col] (a row of n, fp32) then
// clamp(lo, hi), each rounding and comparing as the eager elementwise kernels
// do (fp32 add; a < lo ? lo : (a > hi ? hi : a)), so a fused Linear+ReLU is
// bit-identical to matmul, + bias, clamp run one after another.
struct Epilogue {
  const float* bias;  // null: none
  int clamp;
  float lo, hi;
};

__device__ __forceinline__ float epilogue_apply(const Epilogue& ep, float v, int col) {
  if (ep.bias) v = __fadd_rn(v, __ldg(ep.bias + col));
  if (ep.clamp) v = v < ep.lo ? ep.lo : (v > ep.hi ? ep.hi : v);
  return v;
}

// Epilogue of one tile for one thread: TMEM lane `taddr` (this warp's lane
// quarter) holds output row `row`, columns [n0, n0 + BN): big accumulator at
// column offset 0, cross terms at BN.  Combines, unscales, adds C when beta,
// stores.  Every thread of the warp must call it (tcgen05.ld is warp-wide).
__device__ __forceinline__ void drain_tile(uint32_t taddr, int row, int n0, int M, int N,
                                           const int* __restrict__ eA, const int* __restrict__ eB,
                                           float* __restrict__ C, int beta, bool ok, const Epilogue& ep) {
  const bool vec = (N & 3) == 0;
  const int erow = row < M ? __ldg(eA + row) : 0;
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    uint32_t r[16], rs[16];
    tmem_ld16(taddr + c, r);
    tmem_ld16(taddr + BN + c, rs);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      // an infinite hi*hi sum stands: its cross terms may hold inf*0 = NaN
      const float big = __uint_as_float(r[j]);
      r[j] = __float_as_uint(isinf(big) ? big : __fmaf_rn(__uint_as_float(rs[j]), 0x1p-11f, big));
    }
    if (!ok || row >= M) continue;
    float* crow = C + (int64_t)row * N + n0 + c;
    const int ncols = min(16, N - (n0 + c));
    if (ncols <= 0) continue;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int col = min(n0 + c + j, N - 1);
      r[j] = __float_as_uint(pow2_scale(__uint_as_float(r[j]), -(erow + __ldg(eB + col))));
    }
    if (vec && ncols == 16) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                               __uint_as_float(r[j + 3]));
        if (beta) {
          const float4 o = *reinterpret_cast<const float4*>(crow + j);
          v.x = __fadd_rn(o.x, v.x);
          v.y = __fadd_rn(o.y, v.y);
          v.z = __fadd_rn(o.z, v.z);
          v.w = __fadd_rn(o.w, v.w);
        }
        if (ep.bias || ep.clamp) {
          const int col = n0 + c + j;
          v.x = epilogue_apply(ep, v.x, col);
          v.y = epilogue_apply(ep, v.y, col + 1);
          v.z = epilogue_apply(ep, v.z, col + 2);
          v.w = epilogue_apply(ep, v.w, col + 3);
        }
        *reinterpret_cast<float4*>(crow + j) = v;
      }
    } else {
      for (int j = 0; j < ncols; ++j) {
        float v = __uint_as_float(r[j]);
        if (beta) v = __fadd_rn(crow[j], v);
        crow[j] = epilogue_apply(ep, v, n0 + c + j);
      }
    }
  }
}

// Persistent: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
__global__ void __launch_bounds__(kThreads, 1)
    gemm_f16x3_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                      const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                      const int* __restrict__ eA, const int* __restrict__ eB, float* __restrict__ C, int M,
                      int N, int num_kb, int beta, int tiles_m, int tiles_n, Epilogue ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // accumulators ready for the epilogue
  uint64_t* tempty = tfull + 2;      // accumulators drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(&tfull[0]), 1);
    mbar_init(smem_u32(&tempty[0]), 128);  // every epilogue thread arrives
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: one ring position per k-block, continuing across tiles
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tAh)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tAl)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tBh)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tBl)) : "memory");
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int m0, n0;
      tile_coords(t, tiles_m, tiles_n, m0, n0);
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t phase = (it / STAGES) & 1;
        if (!mbar_wait(smem_u32(&empty[s]), phase ^ 1, 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        const uint32_t bar = smem_u32(&full[s]);
        mbar_expect_tx(bar, STAGE_BYTES);
        tma_load_2d(smem_u32(st), &tAh, kb * BK, m0, bar);
        tma_load_2d(smem_u32(st + A_TILE), &tAl, kb * BK, m0, bar);
        tma_load_2d(smem_u32(st + 2 * A_TILE), &tBh, kb * BK, n0, bar);
        tma_load_2d(smem_u32(st + 2 * A_TILE + B_TILE), &tBl, kb * BK, n0, bar);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = instr_desc();
    uint32_t it = 0;
    bool ok = true;
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++lt) {
      const uint32_t aphase = lt & 1;
      if (!mbar_wait(smem_u32(&tempty[0]), aphase ^ 1, 4)) break;  // epilogue drained the accumulators
      tc_fence_after();
      const uint32_t dbig = tmem, dsmall = tmem + (uint32_t)BN;
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t phase = (it / STAGES) & 1;
        if (!mbar_wait(smem_u32(&full[s]), phase, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        const uint64_t dAh = smem_desc(base), dAl = smem_desc(base + A_TILE);
        const uint64_t dBh = smem_desc(base + 2 * A_TILE), dBl = smem_desc(base + 2 * A_TILE + B_TILE);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);  // 16 fp16 = 32 bytes along the swizzled row
          const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
          mma_f16(dsmall, dAl + off, dBh + off, idesc, first);
          mma_f16(dsmall, dAh + off, dBl + off, idesc, 1u);
          mma_f16(dbig, dAh + off, dBh + off, idesc, first);
        }
        mma_commit(smem_u32(&empty[s]));
      }
      mma_commit(smem_u32(&tfull[0]));
    }
  } else if (warp >= 2) {
    // ---- epilogue: TMEM -> registers -> global, one tile behind the MMAs
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const uint32_t aphase = lt & 1;
      const bool ok = mbar_wait(smem_u32(&tfull[0]), aphase, 3);
      tc_fence_after();
      int m0, n0;
      tile_coords(t, tiles_m, tiles_n, m0, n0);
      const int row = m0 + q * 32 + lane;
      drain_tile(tmem + ((uint32_t)(q * 32) << 16), row, n0, M, N, eA, eB, C, beta, ok, ep);
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[0]));
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------ CTA-pair kernel
//
// Two CTAs of a cluster compute one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA loads its own 128 rows of A
// and its half (128 rows) of B, so a k-block costs each SM 32 KB of loads
// instead of 48 KB, and six stages fit where four did.  The even CTA (the
// leader) issues the MMAs; its `full` barriers collect the load bytes of
// both CTAs (the .cta_group::2 form of the TMA load signals the leader's
// barrier; no load is multicast), and its commits arrive on the `empty` and
// `tfull` barriers of both CTAs.  Each CTA's TMEM holds its 128 rows; both
// epilogues drain their own half and arrive on the leader's `tempty`.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `cta` of the cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t addr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(cta));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA tile load into this CTA's shared memory; completion bytes go to the
// mbarrier at `bar` (a cluster address, here the leader's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on the barrier at this shared offset in both CTAs of the pair once
// the leader's issued MMAs complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// kind::f16, D f32, A and B f16, K-major, M = 256 (across the pair), N = BN.
__host__ __device__ constexpr uint32_t instr_desc_pair() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(P_TM >> 4) << 24);
}

// The pair kernel's epilogue writes each warp's 32 rows 32 columns at a
// time through a 32 x 32 fp32 staging block in shared memory: every lane
// parks four scaled sums of its own row (float4 j of row r at slot
// j ^ (r & 7), so neither side conflicts on banks), then the warp unscales
// and writes the block out row-wise, 8 lanes per 128-byte row segment, so
// every store is coalesced.  The unscale sits in the write-out loop, which
// is not unrolled: the code exists once, not once per value held.
__device__ __forceinline__ void stage_quad(float4* sw, int lane, int j, float4 v) {
  sw[lane * 8 + (j ^ (lane & 7))] = v;
}

// Rows wrow0 .. wrow0 + 31, columns col0 .. col0 + 31 of C from the staging
// block: unscaled by 2^-(e_row + e_col), + C when beta, then the bias and
// clamp epilogue.
__device__ __forceinline__ void flush_block(const float4* sw, int lane, int wrow0, int col0, int M, int N, bool vec,
                                            int beta, const Epilogue& ep, const int* __restrict__ eA,
                                            const int* __restrict__ eB, float* __restrict__ C) {
  const int j = lane & 7, col = col0 + 4 * j;
  // eB holds n exponents in a buffer padded to 64: the lanes past n read
  // padding, and their columns are never stored
  const int4 ec = col < N ? __ldg(reinterpret_cast<const int4*>(eB + col)) : make_int4(0, 0, 0, 0);
#pragma unroll 1
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3), grow = wrow0 + r;
    if (grow >= M || col >= N) continue;
    const float4 raw = sw[r * 8 + (j ^ (r & 7))];
    const int erow = __ldg(eA + grow);
    float4 o = make_float4(pow2_scale(raw.x, -(erow + ec.x)), pow2_scale(raw.y, -(erow + ec.y)),
                           pow2_scale(raw.z, -(erow + ec.z)), pow2_scale(raw.w, -(erow + ec.w)));
    if (!vec) {  // a row pitch that is not a multiple of 16 bytes
      float* dst = C + (int64_t)grow * N + col;
      const float ov[4] = {o.x, o.y, o.z, o.w};
      for (int e = 0; e < 4 && col + e < N; ++e)
        dst[e] = epilogue_apply(ep, beta ? __fadd_rn(dst[e], ov[e]) : ov[e], col + e);
      continue;
    }
    float4* dst = reinterpret_cast<float4*>(C + (int64_t)grow * N + col);
    if (beta) {
      const float4 p = *dst;
      o.x = __fadd_rn(p.x, o.x);
      o.y = __fadd_rn(p.y, o.y);
      o.z = __fadd_rn(p.z, o.z);
      o.w = __fadd_rn(p.w, o.w);
    }
    if (ep.bias || ep.clamp) {
      o.x = epilogue_apply(ep, o.x, col);
      o.y = epilogue_apply(ep, o.y, col + 1);
      o.z = epilogue_apply(ep, o.z, col + 2);
      o.w = epilogue_apply(ep, o.w, col + 3);
    }
    *dst = o;
  }
}

__global__ void __launch_bounds__(kThreadsP, 1)
    gemm_f16x3_pair_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                           const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                           const int* __restrict__ eA, const int* __restrict__ eB, float* __restrict__ C, int M,
                           int N, int num_kb, int beta, int tiles_m, int tiles_n, Epilogue ep, int splits,
                           float* __restrict__ part, unsigned* __restrict__ arrivals) {
  extern __shared__ uint8_t smem_raw[];
  // The same offsets in both CTAs: the pair MMA addresses the peer's tiles
  // and the commits address the peer's barriers by the local offset.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
  float4* epi_stage = reinterpret_cast<float4*>(smem + P_STAGES * P_STAGE_BYTES + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // Work units: tile t = u / splits covers k-blocks [ks * kb_per, ...) with
  // ks = u % splits; with splits > 1 the unit that finishes a tile last sums
  // the partials (see the epilogue).
  const int num_units = tiles_m * tiles_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);   // the leader's expect_tx
      mbar_init(smem_u32(&empty[s]), 1);  // the leader's commit
    }
    mbar_init(smem_u32(&tfull[0]), 1);
    mbar_init(smem_u32(&tempty[0]), 16);  // one arrive per epilogue warp, both CTAs
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer, both CTAs
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tAh)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tAl)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tBh)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tBl)) : "memory");
    uint32_t it = 0;
    bool ok = true;
    for (int u = pair; u < num_units && ok; u += npairs) {
      int t, kb0, kb1, m0, n0;
      sched_unit(u, splits, num_kb, t, kb0, kb1);
      tile_coords_pair(t, tiles_m, tiles_n, m0, n0);
      const int ya = m0 + (int)rank * 128, yb = n0 + (int)rank * 128;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % P_STAGES;
        const uint32_t phase = (it / P_STAGES) & 1;
        if (!mbar_wait(smem_u32(&empty[s]), phase ^ 1, 5)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * P_STAGE_BYTES;
        const uint32_t bar_local = smem_u32(&full[s]);
        if (leader) mbar_expect_tx(bar_local, 2 * P_STAGE_BYTES);
        const uint32_t bar = map_to_cta(bar_local, 0);
        tma_load_2d_pair(smem_u32(st), &tAh, kb * BK, ya, bar);
        tma_load_2d_pair(smem_u32(st + P_A_TILE), &tAl, kb * BK, ya, bar);
        tma_load_2d_pair(smem_u32(st + 2 * P_A_TILE), &tBh, kb * BK, yb, bar);
        tma_load_2d_pair(smem_u32(st + 2 * P_A_TILE + P_B_TILE), &tBl, kb * BK, yb, bar);
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer, leader only
    constexpr uint32_t idesc = instr_desc_pair();
    uint32_t it = 0;
    bool ok = true;
    int lt = 0;
    for (int u = pair; u < num_units && ok; u += npairs, ++lt) {
      int t_unused, kb0, kb1;
      sched_unit(u, splits, num_kb, t_unused, kb0, kb1);
      if (!mbar_wait(smem_u32(&tempty[0]), (lt & 1) ^ 1, 6)) break;  // both epilogues drained
      tc_fence_after();
      const uint32_t dbig = tmem, dsmall = tmem + (uint32_t)BN;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % P_STAGES;
        const uint32_t phase = (it / P_STAGES) & 1;
        if (!mbar_wait(smem_u32(&full[s]), phase, 7)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * P_STAGE_BYTES);
        const uint64_t dAh = smem_desc(base), dAl = smem_desc(base + P_A_TILE);
        const uint64_t dBh = smem_desc(base + 2 * P_A_TILE), dBl = smem_desc(base + 2 * P_A_TILE + P_B_TILE);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);
          const uint32_t first = (kb == kb0 && kk == 0) ? 0u : 1u;
          mma_f16_pair(dsmall, dAl + off, dBh + off, idesc, first);
          mma_f16_pair(dsmall, dAh + off, dBl + off, idesc, 1u);
          mma_f16_pair(dbig, dAh + off, dBh + off, idesc, first);
        }
        mma_commit_pair(smem_u32(&empty[s]));
      }
      mma_commit_pair(smem_u32(&tfull[0]));
    }
  } else if (warp >= 2) {
    // ---- epilogue, both CTAs: this CTA's 128 rows of the pair's tile.  Two
    // warps per TMEM lane quarter, one per 128-column half.  Each thread
    // pulls its 128 combined values into registers and releases the
    // accumulators before unscaling and storing, so the stores overlap the
    // next tile's MMAs.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const uint32_t tempty_leader = map_to_cta(smem_u32(&tempty[0]), 0);
    const bool vec = (N & 3) == 0;
    int lt = 0;
    for (int u = pair; u < num_units; u += npairs, ++lt) {
      const int t = u / splits, ks = u % splits;
      const bool ok = mbar_wait(smem_u32(&tfull[0]), lt & 1, 8);
      tc_fence_after();
      int m0, n0;
      tile_coords_pair(t, tiles_m, tiles_n, m0, n0);
      const int row = m0 + (int)rank * 128 + q * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 128);
      float v[128];
#pragma unroll
      for (int c = 0; c < 128; c += 16) {
        uint32_t rb[16], rs[16];
        tmem_ld16_issue(taddr + c, rb);
        tmem_ld16_issue(taddr + BN + c, rs);
        tmem_ld_wait();
        tmem_regs_ready(rb);
        tmem_regs_ready(rs);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          // an infinite hi*hi sum stands: its cross terms may hold inf*0 = NaN
          const float big = __uint_as_float(rb[j]);
          v[c + j] = isinf(big) ? big : __fmaf_rn(__uint_as_float(rs[j]), 0x1p-11f, big);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader);
      if (splits > 1) {
        // Split-K: every unit leaves its 32 x 128 block of (pre-scale)
        // partial sums in `part`; the unit whose arrival completes the
        // count adds the splits' partials in split order and finishes, so
        // the result does not depend on which unit came last.  No unit
        // waits for another.
        const int blk = (int)rank * 8 + (warp - 2);
        const size_t bsz = 32 * 128;
        float4* mine = reinterpret_cast<float4*>(part + ((size_t)u * 16 + blk) * bsz);
#pragma unroll
        for (int c = 0; c < 128; c += 4) mine[(c >> 2) * 32 + lane] = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(arrivals + (size_t)t * 16 + blk, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)(splits - 1) && ok) {
          __threadfence();
          const int c0 = n0 + h * 128;
          const int wrow0 = m0 + (int)rank * 128 + q * 32;
          float4* sw = epi_stage + (warp - 2) * 256;
          const float4* tp = reinterpret_cast<const float4*>(part + ((size_t)t * splits * 16 + blk) * bsz);
#pragma unroll 1
          for (int cc = 0; cc < 128; cc += 32) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int at = ((cc >> 2) + j) * 32 + lane;
              float4 a = __ldcg(tp + at);
              for (int k = 1; k < splits; ++k) {
                const float4 b = __ldcg(tp + (size_t)k * 16 * (bsz / 4) + at);
                a.x = __fadd_rn(a.x, b.x);
                a.y = __fadd_rn(a.y, b.y);
                a.z = __fadd_rn(a.z, b.z);
                a.w = __fadd_rn(a.w, b.w);
              }
              stage_quad(sw, lane, j, a);
            }
            __syncwarp();
            flush_block(sw, lane, wrow0, c0 + cc, M, N, vec, beta, ep, eA, eB, C);
            __syncwarp();
          }
        }
      } else if (ok) {
        const int c0 = n0 + h * 128;
        const int wrow0 = m0 + (int)rank * 128 + q * 32;
        float4* sw = epi_stage + (warp - 2) * 256;
#pragma unroll
        for (int cc = 0; cc < 128; cc += 32) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            stage_quad(sw, lane, j, make_float4(v[cc + 4 * j], v[cc + 4 * j + 1], v[cc + 4 * j + 2], v[cc + 4 * j + 3]));
          __syncwarp();
          flush_block(sw, lane, wrow0, c0 + cc, M, N, vec, beta, ep, eA, eB, C);
          __syncwarp();
        }
      }
      (void)ks;
      if (!ok) break;
    }
  }
  // Neither CTA may leave while the other can still reach its shared memory
  // or TMEM.
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------ host side

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiled) nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// Tensor map over a [rows, Kp] fp16 plane, box = box_rows x BK, 64B swizzle.
lmpb_status make_map(CUtensorMap* map, const __half* base, int64_t rows, int64_t Kp, int box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(LMPB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Kp * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LMPB_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return LMPB_OK;
}

// How many CTA pairs of the pair kernel can be resident at once on the
// current device (the persistent grid's size in pairs); 0 if none.
int pair_clusters() {
  static int cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cached[dev] > 0) return cached[dev];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)sm_count());
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_f16x3_pair_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cached[dev] = n;
  return n;
}

// One operand -> scaled fp16 hi/lo planes [rows, Kp] and its row maxima.
// kmajor: src is [rows, K]; else src is [K, rows].  rowmax must be zeroed
// beforehand when !kmajor.
lmpb_status split_operand(const float* src, bool kmajor, int64_t rows, int64_t K, int64_t Kp, __half* hi,
                          __half* lo, float* rowmax, int* expo, cudaStream_t st) {
  if (kmajor) {
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(rows, (int64_t)sm_count() * 8));
    static const bool two_pass = getenv("LMPB_GEMM_SPLIT2PASS") != nullptr;  // A/B switch
    const bool vec = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    if (vec && !two_pass && Kp <= 4096)
      split_rows_reg_kernel<4><<<grid, 256, 0, st>>>(src, rows, K, Kp, hi, lo, rowmax, expo);
    else if (vec)
      split_rows_kernel<true><<<grid, 256, 0, st>>>(src, rows, K, Kp, hi, lo, rowmax, expo);
    else
      split_rows_kernel<false><<<grid, 256, 0, st>>>(src, rows, K, Kp, hi, lo, rowmax, expo);
    return launch_status("gemm split pass (rows)");
  }
  if ((Kp + 63) / 64 > 65535 || (K + 255) / 256 > 65535)
    return set_error(LMPB_ERR_UNSUPPORTED, "gemm: K too large for the split pass");
  const bool quad = (rows & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  static const bool scalar_colmax = getenv("LMPB_GEMM_COLMAX1") != nullptr;  // A/B switch
  if (quad && !scalar_colmax) {
    // k chunks (multiples of 64) sized so that the grid holds about 8 CTAs
    // per SM: a [1024, 4096] operand is 64 column blocks, 16 chunks of 64
    const int64_t gx = (rows + 63) / 64;
    const int64_t ky = std::max<int64_t>(1, ((int64_t)sm_count() * 8 + gx - 1) / gx);
    const int64_t kchunk = std::max<int64_t>(64, ((K + ky - 1) / ky + 63) / 64 * 64);
    colmax4_kernel<<<dim3((unsigned)gx, (unsigned)((K + kchunk - 1) / kchunk)), 256, 0, st>>>(
        src, rows, K, (int)kchunk, reinterpret_cast<unsigned*>(rowmax));
  }
  else
    colmax_kernel<<<dim3((unsigned)((rows + 63) / 64), (unsigned)((K + 255) / 256)), 256, 0, st>>>(
        src, rows, K, reinterpret_cast<unsigned*>(rowmax));
  lmpb_status s = launch_status("gemm split pass (column maxima)");
  if (s != LMPB_OK) return s;
  const dim3 grid((unsigned)((rows + 63) / 64), (unsigned)((Kp + 63) / 64));
  if (quad)
    split_transpose4_kernel<<<grid, 256, 0, st>>>(src, rows, K, Kp, rowmax, hi, lo, expo);
  else
    split_transpose_kernel<<<grid, 256, 0, st>>>(src, rows, K, Kp, rowmax, hi, lo, expo);
  return launch_status("gemm split pass (transpose)");
}

}  // namespace

// Tensor-core path for problems that fill 128-row tiles; SIMT otherwise.
lmpb_status gemm_f32_sm100(int trans_a, int trans_b, const float* A, const float* B, float* C, int64_t m,
                           int64_t n, int64_t k, float beta, cudaStream_t st, const float* bias, int clamp,
                           double lo, double hi) {
  const Epilogue ep{bias, clamp, (float)lo, (float)hi};
  const bool small = m < 64 || n < 64 || k < 32 || (double)m * n * k < 2.0e6;
  if (small || m > (1ll << 30) || n > (1ll << 30) || getenv("LMPB_GEMM_SIMT"))
  {
    lmpb_status s = gemm_f32_simt(trans_a, trans_b, A, B, C, m, n, k, beta, st);
    // the eager elementwise kernels, in place: the same values as the fused epilogue
    if (s == LMPB_OK && bias) {
      const int64_t cs[2] = {m, n}, bs[1] = {n};
      s = lmpb_binary(LMPB_ADD, LMPB_FLOAT32, C, LMPB_FLOAT32, cs, 2, bias, LMPB_FLOAT32, bs, 1, C, 0.0, 0.0, st);
    }
    if (s == LMPB_OK && clamp) s = lmpb_unary(LMPB_CLAMP, LMPB_FLOAT32, C, C, m * n, lo, hi, st);
    return s;
  }
  // The shared-memory opt-in is per device: set it the first time each
  // device (the current one) runs the tensor-core path.
  {
    static std::mutex mu;
    static std::vector<char> ready;
    int dev = 0;
    LMPB_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if ((int)ready.size() <= dev) ready.resize(dev + 1, 0);
    if (!ready[dev]) {
      cudaError_t ae = cudaFuncSetAttribute(gemm_f16x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      if (ae == cudaSuccess)
        ae = cudaFuncSetAttribute(gemm_f16x3_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
      if (ae != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("gemm smem attribute: ") + cudaGetErrorString(ae));
      ready[dev] = 1;
    }
  }
  const int64_t Kp = (k + BK - 1) / BK * BK;
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t plane_a = up((size_t)m * Kp * 2), plane_b = up((size_t)n * Kp * 2);
  const size_t max_a = up((size_t)m * 4), max_b = up((size_t)n * 4);  // row maxima, then row exponents
  char* ws = nullptr;
  LMPB_CUDA_TRY(stream_alloc((void**)&ws, 2 * plane_a + 2 * plane_b + 2 * (max_a + max_b), st));
  __half* Ah = reinterpret_cast<__half*>(ws);
  __half* Al = reinterpret_cast<__half*>(ws + plane_a);
  __half* Bh = reinterpret_cast<__half*>(ws + 2 * plane_a);
  __half* Bl = reinterpret_cast<__half*>(ws + 2 * plane_a + plane_b);
  float* mxA = reinterpret_cast<float*>(ws + 2 * plane_a + 2 * plane_b);
  float* mxB = reinterpret_cast<float*>(ws + 2 * plane_a + 2 * plane_b + max_a);
  int* exA = reinterpret_cast<int*>(ws + 2 * plane_a + 2 * plane_b + max_a + max_b);
  int* exB = reinterpret_cast<int*>(ws + 2 * plane_a + 2 * plane_b + 2 * max_a + max_b);
  // op(A) is [m,k]: K-major as stored unless transposed; the MMA's B operand
  // is op(B)^T = [n,k]: K-major as stored only when trans_b.
  const bool ka = !trans_a, kb = trans_b != 0;
  lmpb_status s = LMPB_OK;
  if (!ka || !kb) {  // column maxima accumulate by atomicMax from zero
    const cudaError_t e = cudaMemsetAsync(ws + 2 * plane_a + 2 * plane_b, 0, max_a + max_b, st);
    if (e != cudaSuccess) s = set_error(LMPB_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (s == LMPB_OK) s = split_operand(A, ka, m, k, Kp, Ah, Al, mxA, exA, st);
  if (s == LMPB_OK) s = split_operand(B, kb, n, k, Kp, Bh, Bl, mxB, exB, st);
  // Pair kernel when there are 256 rows to pair up; the single-CTA kernel
  // otherwise (LMPB_GEMM_PAIR=0 forces it, for comparison).
  static const bool pair_off = [] {
    const char* v = getenv("LMPB_GEMM_PAIR");
    return v && v[0] == '0';
  }();
  const bool pair = m >= P_TM && !pair_off;
  int splits = 1;  // split-K for the pair kernel, chosen below
  CUtensorMap mAh, mAl, mBh, mBl;
  const int b_box = pair ? BN / 2 : BN;
  if (s == LMPB_OK) s = make_map(&mAh, Ah, m, Kp, BM);
  if (s == LMPB_OK) s = make_map(&mAl, Al, m, Kp, BM);
  if (s == LMPB_OK) s = make_map(&mBh, Bh, n, Kp, b_box);
  if (s == LMPB_OK) s = make_map(&mBl, Bl, n, Kp, b_box);
  const int64_t tiles_n = (n + BN - 1) / BN, tiles_m = (m + (pair ? P_TM : BM) - 1) / (pair ? P_TM : BM);
  if (s == LMPB_OK && tiles_m * tiles_n > 0x7FFFFFFF) s = set_error(LMPB_ERR_UNSUPPORTED, "gemm: too many tiles");
  const int64_t ntiles = tiles_m * tiles_n;
  const int nkb = (int)(Kp / BK), bflag = beta != 0.f ? 1 : 0;
  if (s == LMPB_OK && pair) {
    int clusters = pair_clusters();
    const char* force = getenv("LMPB_GEMM_SPLITK");  // tuning override: the split count (1 = none)
    splits = sched_choose_splits(ntiles, nkb, clusters, force ? std::max(1, atoi(force)) : 0);
    void* sk = nullptr;
    float* part = nullptr;
    unsigned* arrivals = nullptr;
    if (clusters > 0 && splits > 1) {
      const size_t pbytes = (size_t)ntiles * splits * 16 * 32 * 128 * 4, abytes = (size_t)ntiles * 16 * 4;
      cudaError_t ae = stream_alloc(&sk, pbytes + abytes, st);
      if (ae == cudaSuccess) ae = cudaMemsetAsync(static_cast<char*>(sk) + pbytes, 0, abytes, st);
      if (ae != cudaSuccess) {
        s = set_error(LMPB_ERR_CUDA, std::string("gemm split-K workspace: ") + cudaGetErrorString(ae));
      } else {
        part = static_cast<float*>(sk);
        arrivals = reinterpret_cast<unsigned*>(static_cast<char*>(sk) + pbytes);
      }
    }
    if (s != LMPB_OK) {
    } else if (clusters <= 0) {
      s = set_error(LMPB_ERR_CUDA, "gemm: no CTA-pair cluster fits on this device");
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(ntiles * splits, clusters)));
      cfg.blockDim = dim3(kThreadsP);
      cfg.dynamicSmemBytes = P_SMEM_BYTES;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const cudaError_t le = cudaLaunchKernelEx(&cfg, gemm_f16x3_pair_kernel, mAh, mAl, mBh, mBl, (const int*)exA,
                                                (const int*)exB, C, (int)m, (int)n, nkb, bflag, (int)tiles_m,
                                                (int)tiles_n, ep, splits, part, arrivals);
      s = le != cudaSuccess ? set_error(LMPB_ERR_CUDA, std::string("gemm pair launch: ") + cudaGetErrorString(le))
                            : launch_status("gemm_f16x3_pair_kernel");
    }
    if (sk) cudaFreeAsync(sk, st);
  } else if (s == LMPB_OK) {
    const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sm_count());
    gemm_f16x3_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(mAh, mAl, mBh, mBl, exA, exB, C, (int)m, (int)n, nkb, bflag,
                                                          (int)tiles_m, (int)tiles_n, ep);
    s = launch_status("gemm_f16x3_kernel");
  }
  cudaError_t e = cudaFreeAsync(ws, st);
  if (s == LMPB_OK && e != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("cudaFreeAsync: ") + cudaGetErrorString(e));
  return s;
}

// Reads and clears the device error word of the tensor-core GEMM (0 = none).
unsigned int gemm_take_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof v) != cudaSuccess) return 0xFFFFFFFFu;
  if (v) cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof zero);
  return v;
}

}  // namespace lmpb

// The schedule helpers above, for tests (no counterpart in the reference).
extern "C" void lmpb_gemm_sched_tile(int t, int tiles_m, int tiles_n, int tm, int tn, int* m0, int* n0) {
  lmpb::sched_tile(t, tiles_m, tiles_n, tm, tn, *m0, *n0);
}
extern "C" void lmpb_gemm_sched_unit(int u, int splits, int num_kb, int* t, int* kb0, int* kb1) {
  lmpb::sched_unit(u, splits, num_kb, *t, *kb0, *kb1);
}
extern "C" int lmpb_gemm_sched_splits(int64_t ntiles, int num_kb, int clusters, int forced) {
  return lmpb::sched_choose_splits(ntiles, num_kb, clusters, forced);
}
