// Keep-dim reductions (sum / max / min / prod) along one axis.
//
// The input is viewed as [outer, R, inner] with R the reduced extent.
//  * inner == 1 (last axis): each row is reduced by one CTA (long rows) or
//    one warp (short rows) with 16-byte vector loads and a warp-shuffle tree.
//  * inner  > 1 (leading / middle axis): a thread owns a 16-byte vector of
//    adjacent columns and walks down the R rows, so every warp load is a
//    fully coalesced 512-byte segment.  When outer x column-blocks cannot fill
//    the 148 SMs, R is split into chunks.  With enough column blocks, the 8
//    chunks of a column block are one thread-block cluster: each CTA leaves
//    its partial in shared memory and the cluster's first CTA folds the 8
//    partials in chunk order through distributed shared memory, in the same
//    kernel.  Otherwise the S chunks' partials go to a workspace and a second
//    kernel combines them in chunk order.  No float atomics, so results are
//    identical run to run.
// Accumulation stays in the input dtype (the reference's functors are
// instantiated on the output type, csrc/src/tensor/cpu/reduct.cpp:33-49),
// which keeps int32 sums, max and min bit-exact with the reference; a float
// sum differs from the reference's sequential order only by rounding.
#include <cooperative_groups.h>

#include <cstdio>
#include <map>
#include <mutex>
#include <cstdlib>
#include <limits>

#include "common.cuh"

namespace lmpb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxPeerRanks = 8;
constexpr int64_t kPeerMaxBlocks = 16384;                // column blocks per flag table row
constexpr long long kPeerWaitCycles = 4000000000ll;      // ~2 s at 1.9 GHz

template <int OP, typename T>
struct RedOp {
  static __host__ __device__ __forceinline__ T identity() {
    if constexpr (OP == LMPB_SUM) return T(0);
    else if constexpr (OP == LMPB_PROD) return T(1);
    else if constexpr (OP == LMPB_MAX) return std::numeric_limits<T>::lowest();
    else return std::numeric_limits<T>::max();
  }
  // `acc` covers lower indices than `x`; max/min keep `acc` on ties like
  // std::max / std::min in the reference's sequential loop.
  static __device__ __forceinline__ T apply(T acc, T x) {
    if constexpr (OP == LMPB_SUM) return static_cast<T>(r_add(acc, x));
    else if constexpr (OP == LMPB_PROD) return static_cast<T>(r_mul(acc, x));
    else if constexpr (OP == LMPB_MAX) return (acc < x) ? x : acc;
    else return (x < acc) ? x : acc;
  }
};

template <typename T>
__device__ __forceinline__ T shfl_down(T v, int delta) {
  if constexpr (sizeof(T) < 4) {
    int t = static_cast<int>(v);
    return static_cast<T>(__shfl_down_sync(0xffffffffu, t, delta));
  } else {
    return __shfl_down_sync(0xffffffffu, v, delta);
  }
}

template <int OP, typename T>
__device__ __forceinline__ T warp_reduce(T v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = RedOp<OP, T>::apply(v, shfl_down(v, d));
  return v;
}

template <typename T>
struct V16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T v[N];
  };
};

// Reduces `len` contiguous elements starting at `row` with the threads
// [lane0, lane0 + nthreads); returns the per-thread partial.  The row is cut
// into packets of PW contiguous elements; thread `tid` takes packets tid,
// tid + nthreads, ... and folds each packet's elements in order.  This is the
// walk of the fused compiler's row reductions (csrc/fused.cpp, packet width
// `vec`), so an eager last-axis sum and a fused one add in the same order.
template <typename T, int PW>
struct alignas(PW * sizeof(T) >= 16 ? 16 : PW * sizeof(T)) RowPack {
  T v[PW];
};

template <int OP, typename T, int PW>
__device__ __forceinline__ T row_partial(const T* __restrict__ row, int64_t len, int tid, int nthreads) {
  using R = RedOp<OP, T>;
  using Pk = RowPack<T, PW>;
  T acc = R::identity();
  const Pk* pk = reinterpret_cast<const Pk*>(row);
  const int64_t np = len / PW;  // len % PW == 0 (the host picks PW so)
  int64_t i = tid;
  for (; i + 3 * nthreads < np; i += 4 * nthreads) {
    Pk x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = pk[i + u * nthreads];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < PW; ++j) acc = R::apply(acc, x[u].v[j]);
  }
  for (; i < np; i += nthreads) {
    const Pk x = pk[i];
#pragma unroll
    for (int j = 0; j < PW; ++j) acc = R::apply(acc, x.v[j]);
  }
  return acc;
}

// One CTA per row (grid-stride over rows).
template <int OP, typename T, int PW>
__global__ void __launch_bounds__(kThreads)
    reduce_rows_cta_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t rows,
                           int64_t len) {
  __shared__ T warp_part[kThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    T acc = row_partial<OP, T, PW>(in + r * len, len, threadIdx.x, kThreads);
    acc = warp_reduce<OP, T>(acc);
    if (lane == 0) warp_part[wid] = acc;
    __syncthreads();
    if (wid == 0) {
      T v = lane < kThreads / 32 ? warp_part[lane] : RedOp<OP, T>::identity();
      v = warp_reduce<OP, T>(v);
      if (lane == 0) out[r] = v;
    }
    __syncthreads();
  }
}

// One warp per row.
template <int OP, typename T, int PW>
__global__ void __launch_bounds__(kThreads)
    reduce_rows_warp_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t rows,
                            int64_t len) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t r = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    T acc = row_partial<OP, T, PW>(in + r * len, len, lane, 32);
    acc = warp_reduce<OP, T>(acc);
    if (lane == 0) out[r] = acc;
  }
}

// Column reduction of [outer, R, inner].  A CTA is CTX column threads x CTY
// row lanes: thread (tx, ty) owns VW adjacent columns and rows r0+ty,
// r0+ty+CTY, ... of chunk blockIdx.z (4 rows in flight); the CTY lane
// partials are folded in lane order through shared memory and the CTA's
// partial goes to dst[(chunk * outer + o) * inner + c].  Narrow CTAs (CTX*VW
// columns) fill the GPU with few row chunks, so the combine pass is small.
template <int OP, typename T, int VW, int CTX>
__global__ void __launch_bounds__(kThreads)
    reduce_cols_kernel(const T* __restrict__ in, T* __restrict__ dst, int64_t outer, int64_t R, int64_t inner,
                       int64_t rows_per_chunk) {
  constexpr int CTY = kThreads / CTX;
  using Rd = RedOp<OP, T>;
  __shared__ T part[CTY][CTX * VW];
  const int tx = threadIdx.x % CTX, ty = threadIdx.x / CTX;
  const int64_t c = ((int64_t)blockIdx.x * CTX + tx) * VW;
  const int64_t o = blockIdx.y;
  const int64_t chunk = blockIdx.z;
  const int64_t r0 = chunk * rows_per_chunk;
  const int64_t r1 = min(R, r0 + rows_per_chunk);
  T acc[VW];
#pragma unroll
  for (int j = 0; j < VW; ++j) acc[j] = Rd::identity();
  if (c < inner) {
    const T* base = in + (o * R) * inner + c;
    int64_t r = r0 + ty;
    if constexpr (VW > 1) {
      for (; r + 3 * CTY < r1; r += 4 * CTY) {
        V16<T> x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u].raw = __ldg(reinterpret_cast<const uint4*>(base + (r + u * CTY) * inner));
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x[u].v[j]);
      }
      for (; r < r1; r += CTY) {
        V16<T> x;
        x.raw = __ldg(reinterpret_cast<const uint4*>(base + r * inner));
#pragma unroll
        for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x.v[j]);
      }
    } else {
      for (; r < r1; r += CTY) acc[0] = Rd::apply(acc[0], base[r * inner]);
    }
  }
#pragma unroll
  for (int j = 0; j < VW; ++j) part[ty][tx * VW + j] = acc[j];
  __syncthreads();
  if (ty == 0 && c < inner) {
#pragma unroll
    for (int j = 0; j < VW; ++j) {
      T v = part[0][tx * VW + j];
      for (int k = 1; k < CTY; ++k) v = Rd::apply(v, part[k][tx * VW + j]);
      dst[(chunk * outer + o) * inner + c + j] = v;
    }
  }
}

// The column kernel for a cluster of kClusterChunks CTAs along the chunk
// axis: the CTAs walk their row chunks as reduce_cols_kernel does, fold their
// row lanes into `fin` in shared memory, and the cluster's rank-0 CTA folds
// the ranks' `fin` in rank (= chunk) order through distributed shared memory
// and writes the output: no workspace and no second launch.
constexpr int kClusterChunks = 8;

// Chunks per cluster: 8 (portable) or 16 (LMPB_REDUCE_CLUSTER=16, a
// non-portable cluster size B200 supports).
int cluster_chunks() {
  const char* e = getenv("LMPB_REDUCE_CLUSTER");
  return (e && atoi(e) == 16) ? 16 : kClusterChunks;
}

template <int OP, typename T, int VW, int CC, int CTX = 16, int DEPTH = 4>
__global__ void __launch_bounds__(kThreads)
    reduce_cols_cluster_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t R, int64_t inner,
                               int64_t rows_per_chunk) {
  namespace cg = cooperative_groups;
  constexpr int CTY = kThreads / CTX;
  using Rd = RedOp<OP, T>;
  __shared__ T part[CTY][CTX * VW];
  __shared__ T fin[CTX * VW];
  const int tx = threadIdx.x % CTX, ty = threadIdx.x / CTX;
  const int64_t c = ((int64_t)blockIdx.x * CTX + tx) * VW;
  const int64_t o = blockIdx.y;
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_chunk;
  const int64_t r1 = min(R, r0 + rows_per_chunk);
  T acc[VW];
#pragma unroll
  for (int j = 0; j < VW; ++j) acc[j] = Rd::identity();
  if (c < inner) {
    const T* base = in + (o * R) * inner + c;
    int64_t r = r0 + ty;
    for (; r + (DEPTH - 1) * CTY < r1; r += DEPTH * CTY) {
      V16<T> x[DEPTH];
#pragma unroll
      for (int u = 0; u < DEPTH; ++u) x[u].raw = __ldg(reinterpret_cast<const uint4*>(base + (r + u * CTY) * inner));
#pragma unroll
      for (int u = 0; u < DEPTH; ++u)
#pragma unroll
        for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x[u].v[j]);
    }
    for (; r < r1; r += CTY) {
      V16<T> x;
      x.raw = __ldg(reinterpret_cast<const uint4*>(base + r * inner));
#pragma unroll
      for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x.v[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < VW; ++j) part[ty][tx * VW + j] = acc[j];
  __syncthreads();
  if (ty == 0) {
#pragma unroll
    for (int j = 0; j < VW; ++j) {
      T v = part[0][tx * VW + j];
      for (int k = 1; k < CTY; ++k) v = Rd::apply(v, part[k][tx * VW + j]);
      fin[tx * VW + j] = v;
    }
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();  // every rank's fin is written
  if (cl.block_rank() == 0 && ty == 0 && c < inner) {
#pragma unroll
    for (int j = 0; j < VW; ++j) {
      T v = fin[tx * VW + j];
      for (int k = 1; k < CC; ++k) v = Rd::apply(v, cl.map_shared_rank(fin, k)[tx * VW + j]);
      out[o * inner + c + j] = v;
    }
  }
  cl.sync();  // the other ranks keep their shared memory until rank 0 has read it
}

// Combines S chunk partials: out[i] = op over s of part[s][i], in chunk order.
// A CTA owns 32 adjacent columns (lane = column, coalesced); its 8 warps take
// 8 contiguous runs of chunks, each with 8 independent loads in flight, and
// warp 0 folds the 8 run results in run order through shared memory.
template <int OP, typename T>
__global__ void __launch_bounds__(kThreads)
    reduce_combine_kernel(const T* __restrict__ part, T* __restrict__ out, int64_t n, int S) {
  using Rd = RedOp<OP, T>;
  __shared__ T run[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t i = (int64_t)blockIdx.x * 32 + lane;
  const int per = (S + 7) / 8;
  const int s0 = w * per, s1 = min(S, s0 + per);
  T acc = Rd::identity();
  if (i < n) {
    int s = s0;
    for (; s + 7 < s1; s += 8) {
      T v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[(int64_t)(s + u) * n + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = Rd::apply(acc, v[u]);
    }
    for (; s < s1; ++s) acc = Rd::apply(acc, part[(int64_t)s * n + i]);
  }
  run[w][lane] = acc;
  __syncthreads();
  if (w == 0 && i < n) {
    T r = run[0][lane];
#pragma unroll
    for (int k = 1; k < 8; ++k) r = Rd::apply(r, run[k][lane]);
    out[i] = r;
  }
}

// ---------------------------------------------------------------------------
// Leading-axis reduction fused with the all-reduce of its result across the
// GPUs of a row-partitioned job, over NVLink peer memory.  Each rank runs the
// cluster column walk on its own rows; a cluster's rank-0 CTA then pushes its
// 64-column partial into slot [rank] of every rank's exchange buffer (remote
// stores), fences, and raises its flag (the call's epoch) in every rank's flag
// table.  It waits, with a bound, until all ranks' flags for its column block
// carry the epoch, and folds the partials from its own buffer in rank order,
// so every rank writes identical results.  Buffers alternate between two
// halves by epoch parity: a rank reaches epoch e + 2 only after every rank
// signalled e + 1, i.e. finished reading epoch e.
struct PeerArgs {
  unsigned char* data[kMaxPeerRanks];  // each rank's exchange buffer (this process's mapping)
  unsigned* flags[kMaxPeerRanks];      // each rank's flag table [kMaxPeerRanks][kPeerMaxBlocks]
  int nranks, rank;
  unsigned epoch;
  int64_t slot_bytes;
};

__device__ unsigned int g_peer_error = 0;


template <int OP, typename T, int VW, int CC>
__global__ void __launch_bounds__(kThreads)
    reduce_cols_peer_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t R, int64_t inner,
                            int64_t rows_per_chunk, PeerArgs pa) {
  namespace cg = cooperative_groups;
  constexpr int CTX = 16, CTY = kThreads / CTX, DEPTH = 4;
  using Rd = RedOp<OP, T>;
  __shared__ T part[CTY][CTX * VW];
  __shared__ T fin[CTX * VW];
  const int tx = threadIdx.x % CTX, ty = threadIdx.x / CTX;
  const int64_t c = ((int64_t)blockIdx.x * CTX + tx) * VW;
  const int64_t r0 = (int64_t)blockIdx.z * rows_per_chunk;
  const int64_t r1 = min(R, r0 + rows_per_chunk);
  T acc[VW];
#pragma unroll
  for (int j = 0; j < VW; ++j) acc[j] = Rd::identity();
  if (c < inner) {
    const T* base = in + c;
    int64_t r = r0 + ty;
    for (; r + (DEPTH - 1) * CTY < r1; r += DEPTH * CTY) {
      V16<T> x[DEPTH];
#pragma unroll
      for (int u = 0; u < DEPTH; ++u) x[u].raw = __ldg(reinterpret_cast<const uint4*>(base + (r + u * CTY) * inner));
#pragma unroll
      for (int u = 0; u < DEPTH; ++u)
#pragma unroll
        for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x[u].v[j]);
    }
    for (; r < r1; r += CTY) {
      V16<T> x;
      x.raw = __ldg(reinterpret_cast<const uint4*>(base + r * inner));
#pragma unroll
      for (int j = 0; j < VW; ++j) acc[j] = Rd::apply(acc[j], x.v[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < VW; ++j) part[ty][tx * VW + j] = acc[j];
  __syncthreads();
  if (ty == 0) {
#pragma unroll
    for (int j = 0; j < VW; ++j) {
      T v = part[0][tx * VW + j];
      for (int k = 1; k < CTY; ++k) v = Rd::apply(v, part[k][tx * VW + j]);
      fin[tx * VW + j] = v;
    }
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  if (cl.block_rank() == 0 && ty == 0) {  // lanes 0..15 of warp 0
    T v[VW];
#pragma unroll
    for (int j = 0; j < VW; ++j) {
      v[j] = fin[tx * VW + j];
      for (int k = 1; k < CC; ++k) v[j] = Rd::apply(v[j], cl.map_shared_rank(fin, k)[tx * VW + j]);
    }
    const int half = (int)(pa.epoch & 1u);
    // push this rank's partial into slot [rank] of every rank's buffer
    if (c < inner) {  // one 16-byte store per rank (VW * sizeof(T) == 16 on this path)
      V16<T> pk;
#pragma unroll
      for (int j = 0; j < VW; ++j) pk.v[j] = v[j];
      for (int p = 0; p < pa.nranks; ++p) {
        T* dst = reinterpret_cast<T*>(pa.data[p] + ((int64_t)half * kMaxPeerRanks + pa.rank) * pa.slot_bytes) + c;
        *reinterpret_cast<uint4*>(dst) = pk.raw;
      }
    }
    __threadfence_system();  // the partials are visible everywhere before any flag
    __syncwarp(0xffffu);
    bool ok = true;
    if (tx == 0) {
      for (int p = 0; p < pa.nranks; ++p)
        *reinterpret_cast<volatile unsigned*>(pa.flags[p] + (int64_t)pa.rank * kPeerMaxBlocks + blockIdx.x) = pa.epoch;
      // wait (bounded) for every rank's partial of this column block: relaxed
      // polling, one system-scope fence once all flags are seen
      const volatile unsigned* mine = pa.flags[pa.rank];
      const long long t0 = clock64();
      for (int q = 0; q < pa.nranks && ok; ++q)
        while (mine[(int64_t)q * kPeerMaxBlocks + blockIdx.x] - pa.epoch > 0x7fffffffu) {
          if (clock64() - t0 > kPeerWaitCycles) {
            atomicExch(&g_peer_error, 1u);
            ok = false;
            break;
          }
        }
      __threadfence_system();
    }
    ok = __shfl_sync(0xffffu, ok, 0);
    if (ok && c < inner) {
      const unsigned char* mybuf = pa.data[pa.rank];
#pragma unroll
      for (int j = 0; j < VW; ++j) {
        T r = Rd::identity();
        for (int q = 0; q < pa.nranks; ++q) {
          const T* src = reinterpret_cast<const T*>(mybuf + ((int64_t)half * kMaxPeerRanks + q) * pa.slot_bytes) + c + j;
          const T x = *reinterpret_cast<const volatile T*>(src);
          r = q == 0 ? x : Rd::apply(r, x);
        }
        out[c + j] = r;
      }
    }
  }
  cl.sync();
}

template <int OP, typename T>
__global__ void fill_identity_kernel(T* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = RedOp<OP, T>::identity();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Column threads per CTA of the column kernel: wider CTAs read longer
// contiguous runs of each row (CTX * 16 bytes), narrower ones leave more
// CTAs to spread over the SMs when the tensor has few columns.
int pick_ctx(int64_t inner, int vw) {
  int ctx = 16;
  if (const char* e = getenv("LMPB_REDUCE_CTX")) {  // tuning override: 16, 32, 64 or 128
    const int v = atoi(e);
    if (v == 16 || v == 32 || v == 64 || v == 128) return v;
  }
  (void)inner;
  (void)vw;
  return ctx;
}

template <typename T>
int64_t pick_chunks(int64_t outer, int64_t R, int64_t inner, int vw, int ctx) {
  const int64_t colblocks = (inner / vw + ctx - 1) / ctx;
  const int64_t ctas = colblocks * outer;
  // one wave: at most 8 resident CTAs per SM (256 threads, 4 KB shared
  // memory each), so a chunk count that overshoots the slots leaves a second,
  // nearly empty wave (measured: 1216 CTAs for 1184 slots cost ~15 %)
  const int64_t target = (int64_t)sm_count() * 8;
  if (ctas >= target || R < 64) return 1;
  int64_t S = target / ctas;
  if (const char* e = getenv("LMPB_REDUCE_CEIL"))  // A/B switch: the previous rounding up
    if (atoi(e)) S = (target + ctas - 1) / ctas;
  if (S > R / 16) S = R / 16;  // keep >= 16 rows per chunk
  if (S < 1) S = 1;
  return S;
}

}  // namespace

// Reduction plan shared by the allocating and workspace-taking entry points.
struct ReducePlan {
  int64_t outer, R, inner;
  int64_t S;  // chunks (1 = no workspace)
  int vw;     // column vector width
  int ctx;    // column threads per CTA
  bool cluster;  // the chunks are one thread-block cluster (S = kClusterChunks, no workspace)
  int cfg = 0;   // cluster kernel variant: bit 0 = 8 column threads, bit 1 = 8 rows in flight
  size_t ws_bytes;
};

template <typename T>
static ReducePlan plan_reduce(const void* in, const void* out, int64_t outer, int64_t R, int64_t inner) {
  ReducePlan p{outer, R, inner, 1, 1, 16, false, 0};
  if (inner > 1) {
    constexpr int N = V16<T>::N;
    p.vw = (inner % N == 0 && aligned16(in) && aligned16(out)) ? N : 1;
    p.ctx = pick_ctx(inner, p.vw);
    p.S = pick_chunks<T>(outer, R, inner, p.vw, p.ctx);
    // enough column blocks for two cluster CTAs per SM: fold the chunks in
    // the cluster instead of through a workspace and a second kernel
    const int64_t colblocks = (inner / p.vw + 15) / 16;
    const char* e = getenv("LMPB_REDUCE_CLUSTER");  // A/B switch: 0 keeps the workspace path
    if (const char* c2 = getenv("LMPB_REDUCE_CLUSTER_CFG")) {  // tuning override "ctx,depth": 8|16, 4|8
      int cx = 16, dp = 4;
      if (sscanf(c2, "%d,%d", &cx, &dp) == 2) p.cfg = (cx == 8 ? 1 : 0) + (dp == 8 ? 2 : 0);
    }
    const int cc = cluster_chunks();
    if (p.S > 1 && p.vw == N && p.ctx == 16 && outer <= 65535 && R >= 16 * cc &&
        colblocks * outer * cc >= (int64_t)sm_count() * 2 && !(e && atoi(e) == 0)) {
      p.cluster = true;
      p.S = cc;
    }
    if (p.S > 1 && !p.cluster) p.ws_bytes = (size_t)p.S * outer * inner * sizeof(T);
  }
  return p;
}

template <int OP, typename T>
static lmpb_status run_reduce(const ReducePlan& p, const T* in, T* out, T* ws, cudaStream_t st) {
  const int64_t nout = p.outer * p.inner;
  if (p.R == 0) {
    fill_identity_kernel<OP, T><<<(int)std::min<int64_t>((nout + 255) / 256, 4096), 256, 0, st>>>(out, nout);
    return launch_status("fill_identity_kernel");
  }
  if (p.inner == 1) {
    // packet width as the fused compiler picks it for a row reduction: the
    // largest of 8, 4, 2 dividing the row, when input and output are 16-byte
    // aligned; otherwise one element
    int pw = 1;
    if (aligned16(in) && aligned16(out))
      for (int w = 8; w > 1; w >>= 1)
        if (p.R % w == 0) { pw = w; break; }
    const int64_t cap = (int64_t)sm_count() * 8;
    const bool cta = p.R >= 2048;
    const int grid = (int)(cta ? std::min<int64_t>(p.outer, cap) : std::min<int64_t>((p.outer + 7) / 8, cap));
    auto launch = [&](auto pw_c) {
      constexpr int PW = decltype(pw_c)::value;
      if (cta) reduce_rows_cta_kernel<OP, T, PW><<<grid, kThreads, 0, st>>>(in, out, p.outer, p.R);
      else reduce_rows_warp_kernel<OP, T, PW><<<grid, kThreads, 0, st>>>(in, out, p.outer, p.R);
    };
    switch (pw) {
      case 8: launch(std::integral_constant<int, 8>{}); break;
      case 4: launch(std::integral_constant<int, 4>{}); break;
      case 2: launch(std::integral_constant<int, 2>{}); break;
      default: launch(std::integral_constant<int, 1>{}); break;
    }
    return launch_status("reduce_rows_kernel");
  }
  constexpr int N = V16<T>::N;
  const int64_t colblocks = (p.inner / p.vw + p.ctx - 1) / p.ctx;
  const int64_t rows_per_chunk = (p.R + p.S - 1) / p.S;
  if (p.outer > 65535 || p.S > 65535)
    return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce: outer extent too large for the column kernel");
  dim3 grid((unsigned)colblocks, (unsigned)p.outer, (unsigned)p.S);
  if (p.cluster) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = (unsigned)p.S;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (p.cfg) {
      const int64_t cb = (p.inner / p.vw + ((p.cfg & 1) ? 7 : 15)) / ((p.cfg & 1) ? 8 : 16);
      cfg.gridDim = dim3((unsigned)cb, (unsigned)p.outer, (unsigned)p.S);
      switch (p.cfg) {
        case 1: e = cudaLaunchKernelEx(&cfg, reduce_cols_cluster_kernel<OP, T, N, kClusterChunks, 8, 4>, in, out, p.R, p.inner, rows_per_chunk); break;
        case 2: e = cudaLaunchKernelEx(&cfg, reduce_cols_cluster_kernel<OP, T, N, kClusterChunks, 16, 8>, in, out, p.R, p.inner, rows_per_chunk); break;
        default: e = cudaLaunchKernelEx(&cfg, reduce_cols_cluster_kernel<OP, T, N, kClusterChunks, 8, 8>, in, out, p.R, p.inner, rows_per_chunk); break;
      }
    } else if (p.S == 16) {
      auto k = reduce_cols_cluster_kernel<OP, T, N, 16>;
      e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, k, in, out, p.R, p.inner, rows_per_chunk);
    } else {
      e = cudaLaunchKernelEx(&cfg, reduce_cols_cluster_kernel<OP, T, N, kClusterChunks>, in, out, p.R, p.inner,
                             rows_per_chunk);
    }
    if (e != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("reduce_cols_cluster_kernel: ") + cudaGetErrorString(e));
    return launch_status("reduce_cols_cluster_kernel");
  }
  T* dst = p.S > 1 ? ws : out;
  auto launch = [&](auto vw_c, auto ctx_c) {
    reduce_cols_kernel<OP, T, decltype(vw_c)::value, decltype(ctx_c)::value>
        <<<grid, kThreads, 0, st>>>(in, dst, p.outer, p.R, p.inner, rows_per_chunk);
  };
  using I16 = std::integral_constant<int, 16>;
  using I32 = std::integral_constant<int, 32>;
  using I64 = std::integral_constant<int, 64>;
  using I128 = std::integral_constant<int, 128>;
  using VN = std::integral_constant<int, N>;
  using V1 = std::integral_constant<int, 1>;
  if (p.vw == N) {
    switch (p.ctx) {
      case 32: launch(VN{}, I32{}); break;
      case 64: launch(VN{}, I64{}); break;
      case 128: launch(VN{}, I128{}); break;
      default: launch(VN{}, I16{}); break;
    }
  } else {
    launch(V1{}, I16{});
  }
  lmpb_status s = launch_status("reduce_cols_kernel");
  if (s != LMPB_OK || p.S == 1) return s;
  const int64_t g2 = (nout + 31) / 32;
  if (g2 > 0x7FFFFFFFll) return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce: output too large to combine");
  reduce_combine_kernel<OP, T><<<(unsigned)g2, kThreads, 0, st>>>(ws, out, nout, (int)p.S);
  return launch_status("reduce_combine_kernel");
}

lmpb_status reduce_geometry(const int64_t* shape, int ndim, int axis, int64_t& outer, int64_t& R,
                            int64_t& inner) {
  LMPB_CHECK_ARG(ndim >= 1 && ndim <= LMPB_MAX_DIMS, "lmpb_reduce: bad ndim");
  LMPB_CHECK_ARG(axis >= 0 && axis < ndim, "lmpb_reduce: axis out of range");
  outer = 1;
  inner = 1;
  for (int i = 0; i < axis; ++i) outer *= shape[i];
  for (int i = axis + 1; i < ndim; ++i) inner *= shape[i];
  R = shape[axis];
  return LMPB_OK;
}

// Workspace bytes lmpb_reduce would need for this call (0 when none).
size_t reduce_workspace_bytes(int dtype, const void* in, const void* out, const int64_t* shape, int ndim,
                              int axis) {
  int64_t outer, R, inner;
  if (!valid_dtype(dtype) || reduce_geometry(shape, ndim, axis, outer, R, inner) != LMPB_OK) return 0;
  if (outer * inner == 0 || R == 0) return 0;
  LMPB_DISPATCH_DTYPE(dtype, T, return plan_reduce<T>(in, out, outer, R, inner).ws_bytes);
  return 0;
}

// Runs a planned reduction with a caller-provided workspace of at least
// plan.ws_bytes (may be null when ws_bytes == 0).
lmpb_status reduce_with_workspace(int op, int dtype, const void* in, const int64_t* shape,
                                  int ndim, int axis, void* out, void* ws, size_t ws_bytes,
                                  void* stream, bool allocate) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_reduce: invalid dtype");
  LMPB_CHECK_ARG(op >= LMPB_SUM && op <= LMPB_PROD, "lmpb_reduce: unknown op");
  int64_t outer, R, inner;
  lmpb_status s = reduce_geometry(shape, ndim, axis, outer, R, inner);
  if (s != LMPB_OK) return s;
  if (outer * inner == 0) return LMPB_OK;
  LMPB_CHECK_ARG(out && (in || R == 0), "lmpb_reduce: null pointer");  // an empty input may have no buffer
  cudaStream_t st = as_stream(stream);
  LMPB_DISPATCH_DTYPE(dtype, T, {
    ReducePlan p = plan_reduce<T>(in, out, outer, R, inner);
    void* w = ws;
    if (p.ws_bytes > 0) {
      if (allocate) {
        LMPB_CUDA_TRY(stream_alloc((void**)&w, p.ws_bytes, st));
      } else {
        LMPB_CHECK_ARG(w != nullptr && ws_bytes >= p.ws_bytes, "lmpb_reduce: workspace too small");
      }
    }
    switch (op) {
      case LMPB_SUM: s = run_reduce<LMPB_SUM, T>(p, (const T*)in, (T*)out, (T*)w, st); break;
      case LMPB_MAX: s = run_reduce<LMPB_MAX, T>(p, (const T*)in, (T*)out, (T*)w, st); break;
      case LMPB_MIN: s = run_reduce<LMPB_MIN, T>(p, (const T*)in, (T*)out, (T*)w, st); break;
      default: s = run_reduce<LMPB_PROD, T>(p, (const T*)in, (T*)out, (T*)w, st); break;
    }
    if (allocate && p.ws_bytes > 0) {
      cudaError_t e = cudaFreeAsync(w, st);
      if (s == LMPB_OK && e != cudaSuccess)
        return set_error(LMPB_ERR_CUDA, std::string("cudaFreeAsync: ") + cudaGetErrorString(e));
    }
    return s;
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_reduce: invalid dtype");
}

// ---------------------------------------------------------------- peer path

size_t peer_region_bytes(int64_t slot_bytes) {
  return (size_t)2 * kMaxPeerRanks * slot_bytes + (size_t)kMaxPeerRanks * kPeerMaxBlocks * sizeof(unsigned);
}
size_t peer_flags_offset(int64_t slot_bytes) { return (size_t)2 * kMaxPeerRanks * slot_bytes; }

unsigned peer_take_error() {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_peer_error, sizeof v) != cudaSuccess) return 0xFFFFFFFFu;
  if (v) cudaMemcpyToSymbol(g_peer_error, &zero, sizeof zero);
  return v;
}

// The fused reduce + all-reduce over the ranks' peer-mapped regions `bufs`
// (each peer_region_bytes(slot_bytes) long: two halves of kMaxPeerRanks data
// slots, then the flag table).  LMPB_ERR_UNSUPPORTED when this shape does not
// take the cluster column path, its result does not fit a slot, or its CTAs
// could not all be resident at once (a rank's waiting CTA must never keep a
// CTA another rank waits for from running).
lmpb_status reduce_allreduce_peer(int op, int dtype, const void* in, const int64_t* shape, int ndim, int axis,
                                  void* out, unsigned char* const* bufs, int nranks, int rank, unsigned epoch,
                                  int64_t slot_bytes, cudaStream_t st) {
  LMPB_CHECK_ARG(valid_dtype(dtype), "lmpb_reduce_allreduce: invalid dtype");
  LMPB_CHECK_ARG(op >= LMPB_SUM && op <= LMPB_PROD, "lmpb_reduce_allreduce: unknown op");
  LMPB_CHECK_ARG(nranks >= 1 && nranks <= kMaxPeerRanks && rank >= 0 && rank < nranks,
                 "lmpb_reduce_allreduce: bad rank count");
  int64_t outer, R, inner;
  lmpb_status s = reduce_geometry(shape, ndim, axis, outer, R, inner);
  if (s != LMPB_OK) return s;
  if (outer != 1 || inner <= 1 || R == 0)
    return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce_allreduce: only a leading-axis reduction of a matrix");
  LMPB_CHECK_ARG(in && out, "lmpb_reduce_allreduce: null pointer");
  LMPB_DISPATCH_DTYPE(dtype, T, {
    ReducePlan p = plan_reduce<T>(in, out, outer, R, inner);
    constexpr int N = V16<T>::N;
    if (!p.cluster || p.S != kClusterChunks || p.vw != N || inner * (int64_t)sizeof(T) > slot_bytes)
      return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce_allreduce: shape outside the fused path");
    const int64_t colblocks = (inner / N + 15) / 16;
    if (colblocks > kPeerMaxBlocks) return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce_allreduce: too many columns");
    PeerArgs pa{};
    for (int r = 0; r < nranks; ++r) {
      pa.data[r] = bufs[r];
      pa.flags[r] = reinterpret_cast<unsigned*>(bufs[r] + peer_flags_offset(slot_bytes));
    }
    pa.nranks = nranks;
    pa.rank = rank;
    pa.epoch = epoch;
    pa.slot_bytes = slot_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)colblocks, 1, (unsigned)kClusterChunks);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = kClusterChunks;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const int64_t rpc = (R + kClusterChunks - 1) / kClusterChunks;
    cudaError_t e = cudaSuccess;
    auto go = [&](auto kern) -> lmpb_status {
      // clusters that fit the GPU at once, per device and kernel (the query is slow)
      static std::mutex mu;
      static std::map<std::pair<int, const void*>, int> fits;
      int dev = 0;
      cudaGetDevice(&dev);
      int active = 0;
      {
        std::lock_guard<std::mutex> lk(mu);
        auto it = fits.find({dev, (const void*)kern});
        if (it != fits.end()) {
          active = it->second;
        } else {
          e = cudaOccupancyMaxActiveClusters(&active, kern, &cfg);
          if (e != cudaSuccess)
            return set_error(LMPB_ERR_CUDA, std::string("cudaOccupancyMaxActiveClusters: ") + cudaGetErrorString(e));
          fits[{dev, (const void*)kern}] = active;
        }
      }
      if (active < colblocks)
        return set_error(LMPB_ERR_UNSUPPORTED, "lmpb_reduce_allreduce: the grid does not fit the GPU at once");
      e = cudaLaunchKernelEx(&cfg, kern, (const T*)in, (T*)out, R, inner, rpc, pa);
      if (e != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("reduce_cols_peer_kernel: ") + cudaGetErrorString(e));
      return launch_status("reduce_cols_peer_kernel");
    };
    switch (op) {
      case LMPB_SUM: return go(reduce_cols_peer_kernel<LMPB_SUM, T, N, kClusterChunks>);
      case LMPB_MAX: return go(reduce_cols_peer_kernel<LMPB_MAX, T, N, kClusterChunks>);
      case LMPB_MIN: return go(reduce_cols_peer_kernel<LMPB_MIN, T, N, kClusterChunks>);
      default: return go(reduce_cols_peer_kernel<LMPB_PROD, T, N, kClusterChunks>);
    }
  });
  return set_error(LMPB_ERR_INVALID, "lmpb_reduce_allreduce: invalid dtype");
}

}  // namespace lmpb

extern "C" lmpb_status lmpb_reduce(int op, int dtype, const void* in, const int64_t* shape,
                                   int ndim, int axis, void* out, void* stream) {
  return lmpb::reduce_with_workspace(op, dtype, in, shape, ndim, axis, out, nullptr, 0, stream,
                                     true);
}
