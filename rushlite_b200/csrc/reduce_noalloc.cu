// lmpb_reduce_noalloc: lmpb_reduce for callers that cannot allocate device
// memory while they run.
//
// lmpb_reduce takes the split-row workspace of a large leading-axis reduction
// from CUDA's stream-ordered pool.  Some callers cannot allow that: code that
// runs under an allocator it does not own (a host framework that forbids
// allocation inside its own memory planner, an embedded runtime with a fixed
// device budget, or a real-time loop that must not hit a pool miss that ends
// in cudaMalloc).  This variant uses instead one fixed scratch array that
// lives in the library's device data for as long as the library is loaded,
// on every GPU that loads it (1 MiB each).
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace lmpb {

size_t reduce_workspace_bytes(int dtype, const void* in, const void* out, const int64_t* shape, int ndim,
                              int axis);
lmpb_status reduce_with_workspace(int op, int dtype, const void* in, const int64_t* shape, int ndim, int axis,
                                  void* out, void* ws, size_t ws_bytes, void* stream, bool allocate);

namespace {

// The split plan targets 8 CTAs per SM, each CTA 16 column threads of 16
// bytes, so its workspace is at most 8 x SMs x 256 B (0.3 MB on a 148-SM
// B200); 1 MiB covers it with margin.  The size check in
// lmpb_reduce_noalloc therefore cannot fail on a B200: it would take a GPU
// with more than 512 SMs.
constexpr size_t kNoAllocScratchBytes = 1u << 20;  // 1 MiB per device

// The scratch itself.  Host code must not pass `g_noalloc_scratch` to a
// kernel: on the host the name is only a stand-in for the symbol, not a
// device address.  scratch_ptr() looks the device address up.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::vector<void*> g_ptr;  // per device ordinal; filled on first use

lmpb_status scratch_ptr(void** out) {
  int dev = 0;
  LMPB_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_ptr.size() <= dev) g_ptr.resize(dev + 1, nullptr);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(LMPB_ERR_CUDA, std::string("lmpb_reduce_noalloc: cudaGetSymbolAddress failed: ") +
                                          cudaGetErrorString(e));
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return LMPB_OK;
}

}  // namespace
}  // namespace lmpb

extern "C" lmpb_status lmpb_reduce_noalloc(int op, int dtype, const void* in, const int64_t* shape, int ndim,
                                           int axis, void* out, void* stream) {
  using namespace lmpb;
  LMPB_CHECK_ARG(shape != nullptr || ndim == 0, "lmpb_reduce_noalloc: null shape");
  const size_t need = reduce_workspace_bytes(dtype, in, out, shape, ndim, axis);
  if (need > kNoAllocScratchBytes)
    return set_error(LMPB_ERR_INVALID, "lmpb_reduce_noalloc: this reduction needs " + std::to_string(need) +
                                           " bytes of scratch, more than the fixed " +
                                           std::to_string(kNoAllocScratchBytes) + "; use lmpb_reduce");
  void* ws = nullptr;
  if (need > 0) {
    lmpb_status s = scratch_ptr(&ws);
    if (s != LMPB_OK) return s;
  }
  // Every split partial is written before it is read, so the scratch needs
  // no clearing between calls.
  return reduce_with_workspace(op, dtype, in, shape, ndim, axis, out, ws, kNoAllocScratchBytes, stream, false);
}
