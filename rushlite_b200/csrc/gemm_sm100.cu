// fp32 GEMM on the B200 tensor cores: 3xTF32 with tcgen05, TMEM and TMA.
//
//   C[m,n] = op(A)[m,k] · op(B)[k,n] (+ C when beta = 1), fp32 in and out.
//
// fp32 accuracy is kept by splitting every operand element x into
// hi = tf32(x) and lo = tf32(x - hi) (round to nearest) and accumulating
// hi·hi + hi·lo + lo·hi in fp32 in TMEM; the dropped lo·lo term and the tf32
// rounding of lo are O(2^-22) relative, below fp32 accumulation error.
//
// 1. A split pass writes hi and lo planes of both operands, K-major (rows of
//    K contiguous fp32, K padded to the k-block), transposing op(A) / op(B)
//    on the way when the caller's layout is not K-major.  It reads each input
//    element once and writes 8 bytes; for 4096^3 that is ~1.5% of the GEMM.
// 2. The GEMM kernel: persistent, one CTA per SM walking 128 x BN output
//    tiles in grouped order, 6 warps:
//      warp 0     TMA producer (one elected thread): 4 tiles per k-block
//                 (A hi/lo, B hi/lo) into a STAGES-deep shared-memory ring,
//                 64-byte swizzled, completion on an mbarrier;
//      warp 1     owns two TMEM accumulators (128 lanes x BN fp32 columns
//                 each: hi*hi and the cross terms) and
//                 issues the tcgen05.mma.kind::tf32 instructions (one thread),
//                 3 products x BK/8 MMAs per k-block, then tcgen05.commit
//                 frees the stage;
//      warps 2-5  epilogue: tcgen05.ld 32x32b from TMEM (each warp reads the
//                 32 lanes its rank in the warpgroup may access), optional
//                 + C, 16-byte stores.
//    Every mbarrier wait is bounded (clock64); on expiry the kernel records
//    an error code in a device word, stops issuing, frees TMEM and returns.
//    No cluster launch and no multicast: each CTA loads its own tiles.
// Shapes that TMA cannot describe or that are too small for a 128-row tile
// use the SIMT kernel (gemm_simt.cu).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"

namespace lmpb {

lmpb_status gemm_f32_simt(int ta, int tb, const float* A, const float* B, float* C, int64_t m,
                          int64_t n, int64_t k, float beta, cudaStream_t st);

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 16;      // 16 fp32 = 64 bytes per row = one 64B swizzle atom
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr int A_TILE = BM * BK * 4;  // 8 KB
constexpr int B_TILE = BN * BK * 4;  // 16 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // 48 KB
// Two accumulators per tile: hi*hi in columns [0, BN), the small cross terms
// hi*lo + lo*hi in [BN, 2BN).  The tensor core's fp32 accumulation truncates,
// so its error grows with the number of additions into one accumulator;
// keeping the cross terms apart cuts the big accumulator's additions by 3x.
// The epilogue adds the two with round-to-nearest.
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
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

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major, M=128, N=BN.
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
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
}

// ------------------------------------------------------------ split pass

// Round to the nearest tf32 value (10 explicit mantissa bits), ties to even.
__device__ __forceinline__ float tf32_rne(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) != 0x7F800000u) {  // finite
    u += 0x0FFFu + ((u >> 13) & 1u);
    u &= 0xFFFFE000u;
  }
  return __uint_as_float(u);
}

__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  hi = tf32_rne(x);
  lo = tf32_rne(__fsub_rn(x, hi));
}

// src is [rows, K] row-major, K == Kp: a flat float4 stream. Each CTA owns
// 1024 consecutive float4s and each thread keeps four loads in flight.
__global__ void __launch_bounds__(256)
    split_flat_kernel(const float4* __restrict__ src, int64_t n4, float4* __restrict__ hi, float4* __restrict__ lo) {
  const int64_t base = (int64_t)blockIdx.x * 1024 + threadIdx.x;
  float4 x[4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (base + u * 256 < n4) x[u] = __ldg(src + base + u * 256);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t i = base + u * 256;
    if (i < n4) {
      float4 h, l;
      split(x[u].x, h.x, l.x);
      split(x[u].y, h.y, l.y);
      split(x[u].z, h.z, l.z);
      split(x[u].w, h.w, l.w);
      hi[i] = h;
      lo[i] = l;
    }
  }
}

// src is [rows, K] row-major, K < Kp: one CTA row-walk per row, zero padding.
__global__ void __launch_bounds__(256)
    split_kmajor_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp,
                        float* __restrict__ hi, float* __restrict__ lo) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
    for (int64_t c = threadIdx.x; c < Kp; c += 256) {
      float h = 0.f, l = 0.f;
      if (c < K) split(src[r * K + c], h, l);
      hi[r * Kp + c] = h;
      lo[r * Kp + c] = l;
    }
}

// src is [K, rows] row-major (the operand transposed): hi/lo [rows, Kp].
// 64 x 64 tiles through shared memory, 16 elements per thread, both the
// read (along rows) and the writes (along K) coalesced.
__global__ void __launch_bounds__(256)
    split_transpose_kernel(const float* __restrict__ src, int64_t rows, int64_t K, int64_t Kp,
                           float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[64][65];
  const int64_t k0 = (int64_t)blockIdx.y * 64, r0 = (int64_t)blockIdx.x * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
#pragma unroll
  for (int j = ty; j < 64; j += 4) {
    const int64_t k = k0 + j, r = r0 + tx;
    tile[j][tx] = (k < K && r < rows) ? __ldg(src + k * rows + r) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int j = ty; j < 64; j += 4) {
    const int64_t r = r0 + j, k = k0 + tx;
    if (r < rows && k < Kp) {
      float h, l;
      split(tile[tx][j], h, l);
      hi[r * Kp + k] = h;
      lo[r * Kp + k] = l;
    }
  }
}

// ------------------------------------------------------------ GEMM kernel

// Tile t of a tiles_m x tiles_n grid in grouped order: 8 row-tiles at a time
// walk the column tiles, so concurrently running CTAs share B panels in L2.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& m0, int& n0) {
  const int group = 8;
  const int g = t / (group * tiles_n);
  const int first_m = g * group;
  const int gsize = min(tiles_m - first_m, group);
  const int local = t % (group * tiles_n);
  m0 = (first_m + local % gsize) * BM;
  n0 = (local / gsize) * BN;
}

// Persistent: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
__global__ void __launch_bounds__(kThreads, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                       const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                       float* __restrict__ C, int M, int N, int num_kb, int beta, int tiles_m, int tiles_n) {
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
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes along the swizzled row
          const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
          mma_tf32(dsmall, dAl + off, dBh + off, idesc, first);
          mma_tf32(dsmall, dAh + off, dBl + off, idesc, 1u);
          mma_tf32(dbig, dAh + off, dBh + off, idesc, first);
        }
        mma_commit(smem_u32(&empty[s]));
      }
      mma_commit(smem_u32(&tfull[0]));
    }
  } else if (warp >= 2) {
    // ---- epilogue: TMEM -> registers -> global, one tile behind the MMAs
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool vec = (N & 3) == 0;
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const uint32_t aphase = lt & 1;
      const bool ok = mbar_wait(smem_u32(&tfull[0]), aphase, 3);
      tc_fence_after();
      int m0, n0;
      tile_coords(t, tiles_m, tiles_n, m0, n0);
      const int row = m0 + q * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16], rs[16];
        tmem_ld16(taddr + c, r);
        tmem_ld16(taddr + BN + c, rs);
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(rs[j])));
        if (!ok || row >= M) continue;
        float* crow = C + (int64_t)row * N + n0 + c;
        const int ncols = min(16, N - (n0 + c));
        if (ncols <= 0) continue;
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
            *reinterpret_cast<float4*>(crow + j) = v;
          }
        } else {
          for (int j = 0; j < ncols; ++j) {
            float v = __uint_as_float(r[j]);
            if (beta) v = __fadd_rn(crow[j], v);
            crow[j] = v;
          }
        }
      }
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

// Tensor map over a [rows, Kp] fp32 plane, box = box_rows x BK, 128B swizzle.
lmpb_status make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t Kp, int box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(LMPB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Kp * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LMPB_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return LMPB_OK;
}

lmpb_status split_operand(const float* src, bool kmajor, int64_t rows, int64_t K, int64_t Kp, float* hi,
                          float* lo, cudaStream_t st) {
  const int64_t cap = (int64_t)sm_count() * 8;
  if (kmajor && K == Kp && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
    const int64_t n4 = rows * K / 4;  // K is a multiple of BK, so of 4
    const int64_t blocks = (n4 + 1023) / 1024;
    if (blocks > INT32_MAX) return set_error(LMPB_ERR_UNSUPPORTED, "gemm: operand too large for the split pass");
    split_flat_kernel<<<(unsigned)std::max<int64_t>(1, blocks), 256, 0, st>>>(
        reinterpret_cast<const float4*>(src), n4, reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo));
  } else if (kmajor) {
    split_kmajor_kernel<<<(int)std::max<int64_t>(1, std::min<int64_t>(rows, cap)), 256, 0, st>>>(src, rows, K, Kp,
                                                                                               hi, lo);
  } else {
    if ((Kp + 63) / 64 > 65535) return set_error(LMPB_ERR_UNSUPPORTED, "gemm: K too large for the split pass");
    dim3 grid((unsigned)((rows + 63) / 64), (unsigned)((Kp + 63) / 64));
    split_transpose_kernel<<<grid, 256, 0, st>>>(src, rows, K, Kp, hi, lo);
  }
  return launch_status("gemm split pass");
}

}  // namespace

// Tensor-core path for problems that fill 128-row tiles; SIMT otherwise.
lmpb_status gemm_f32_sm100(int trans_a, int trans_b, const float* A, const float* B, float* C, int64_t m,
                           int64_t n, int64_t k, float beta, cudaStream_t st) {
  const bool small = m < 64 || n < 64 || k < 32 || (double)m * n * k < 2.0e6;
  if (small || m > (1ll << 30) || n > (1ll << 30) || getenv("LMPB_GEMM_SIMT"))
    return gemm_f32_simt(trans_a, trans_b, A, B, C, m, n, k, beta, st);
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("gemm smem attribute: ") + cudaGetErrorString(attr_err));
  const int64_t Kp = (k + BK - 1) / BK * BK;
  const size_t plane_a = (size_t)m * Kp * 4, plane_b = (size_t)n * Kp * 4;
  void* ws = nullptr;
  LMPB_CUDA_TRY(stream_alloc((void**)&ws, 2 * plane_a + 2 * plane_b, st));
  float* Ah = static_cast<float*>(ws);
  float* Al = reinterpret_cast<float*>(static_cast<char*>(ws) + plane_a);
  float* Bh = reinterpret_cast<float*>(static_cast<char*>(ws) + 2 * plane_a);
  float* Bl = reinterpret_cast<float*>(static_cast<char*>(ws) + 2 * plane_a + plane_b);
  // op(A) is [m,k]: K-major as stored unless transposed; the MMA's B operand
  // is op(B)^T = [n,k]: K-major as stored only when trans_b.
  lmpb_status s = split_operand(A, !trans_a, m, k, Kp, Ah, Al, st);
  if (s == LMPB_OK) s = split_operand(B, trans_b != 0, n, k, Kp, Bh, Bl, st);
  CUtensorMap mAh, mAl, mBh, mBl;
  if (s == LMPB_OK) s = make_map(&mAh, Ah, m, Kp, BM);
  if (s == LMPB_OK) s = make_map(&mAl, Al, m, Kp, BM);
  if (s == LMPB_OK) s = make_map(&mBh, Bh, n, Kp, BN);
  if (s == LMPB_OK) s = make_map(&mBl, Bl, n, Kp, BN);
  if (s == LMPB_OK) {
    const int64_t tiles_n = (n + BN - 1) / BN, tiles_m = (m + BM - 1) / BM;
    if (tiles_m * tiles_n > 0x7FFFFFFF) {
      s = set_error(LMPB_ERR_UNSUPPORTED, "gemm: too many tiles");
    } else {
      const int64_t ntiles = tiles_m * tiles_n;
      const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sm_count());
      gemm_3xtf32_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(mAh, mAl, mBh, mBl, C, (int)m, (int)n,
                                                             (int)(Kp / BK), beta != 0.f ? 1 : 0, (int)tiles_m,
                                                             (int)tiles_n);
      s = launch_status("gemm_3xtf32_kernel");
    }
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
