// Host-side pieces of the C ABI: error strings, shape broadcasting, device
// queries.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "lmpb.h"

namespace lmpb {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

lmpb_status set_error(lmpb_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

lmpb_status launch_status(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(LMPB_ERR_CUDA, std::string(what) + " launch failed: " + cudaGetErrorString(e));
  return LMPB_OK;
}

bool valid_dtype(int dt) { return dt >= LMPB_BOOL && dt <= LMPB_FLOAT64; }

size_t dtype_size(int dt) {
  static const size_t sz[] = {1, 2, 4, 8, 4, 8};
  return valid_dtype(dt) ? sz[dt] : 0;
}

// Stream-ordered allocation from the device's default pool.  The first call on
// a device raises the pool's release threshold so freed blocks stay in the
// process for reuse instead of being returned to the driver at every
// synchronisation (which makes the next large allocation map memory again).
cudaError_t stream_alloc(void** p, size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static std::vector<char> ready;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    if ((int)ready.size() <= dev) ready.resize(dev + 1, 0);
    if (!ready[dev]) {
      cudaMemPool_t pool;
      if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      }
      ready[dev] = 1;
    }
  }
  return cudaMallocAsync(p, bytes, st);
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace lmpb

extern "C" const char* lmpb_last_error(void) { return lmpb::g_last_error.c_str(); }

extern "C" const char* lmpb_version(void) { return "lmpb 0.1 sm_100a"; }

extern "C" uint64_t lmpb_kernel_launches(void) { return lmpb::g_launches.load(); }

extern "C" lmpb_status lmpb_broadcast_shape(const int64_t* a_shape, int a_ndim,
                                            const int64_t* b_shape, int b_ndim,
                                            int64_t* out_shape, int* out_ndim) {
  if (a_ndim < 0 || b_ndim < 0 || a_ndim > LMPB_MAX_DIMS || b_ndim > LMPB_MAX_DIMS)
    return lmpb::set_error(LMPB_ERR_INVALID, "Too many dims");
  if ((a_ndim && !a_shape) || (b_ndim && !b_shape) || !out_shape || !out_ndim)
    return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_broadcast_shape: null pointer");
  const int nd = a_ndim > b_ndim ? a_ndim : b_ndim;
  for (int k = 0; k < nd; ++k) {
    const int ai = a_ndim - 1 - k, bi = b_ndim - 1 - k;
    const int64_t av = ai >= 0 ? a_shape[ai] : 1;
    const int64_t bv = bi >= 0 ? b_shape[bi] : 1;
    if (!(av == 1 || bv == 1 || av == bv))
      return lmpb::set_error(LMPB_ERR_INVALID, "calc_aligned_shape: Broadcast rule violation.");
    out_shape[nd - 1 - k] = av != 1 ? av : bv;
  }
  *out_ndim = nd;
  return LMPB_OK;
}
