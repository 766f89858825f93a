// Peer-memory context of a row-partitioned multi-GPU job (one process per
// GPU): each rank's exchange region, mapped into every other rank's process
// through CUDA IPC, for the fused leading-axis reduce + all-reduce.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "lmpb.h"

namespace lmpb {
lmpb_status set_error(lmpb_status st, const std::string& msg);
size_t peer_region_bytes(int64_t slot_bytes);
lmpb_status reduce_allreduce_peer(int op, int dtype, const void* in, const int64_t* shape, int ndim, int axis,
                                  void* out, unsigned char* const* bufs, int nranks, int rank, unsigned epoch,
                                  int64_t slot_bytes, cudaStream_t st);
}  // namespace lmpb

namespace {

constexpr int kMaxRanks = 8;
constexpr int64_t kSlotBytes = 1 << 20;  // one rank's partial: up to 1 MiB (262,144 fp32 columns)

struct PeerCtx {
  unsigned char* own = nullptr;
  unsigned char* buf[kMaxRanks] = {};
  int nranks = 0, rank = -1, device = -1;
  unsigned epoch = 0;
  bool open = false;
};
std::mutex g_mu;
PeerCtx g_ctx;

lmpb_status cuda_fail(cudaError_t e, const char* what) {
  return lmpb::set_error(LMPB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" lmpb_status lmpb_peer_export(void* handle, size_t bytes) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!handle || bytes < sizeof(cudaIpcMemHandle_t))
    return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_peer_export: handle buffer smaller than LMPB_PEER_HANDLE_BYTES");
  if (!g_ctx.own) {
    const size_t n = lmpb::peer_region_bytes(kSlotBytes);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, n);
    if (e != cudaSuccess) return cuda_fail(e, "lmpb_peer_export: cudaMalloc");
    e = cudaMemset(p, 0, n);  // flags start below every epoch
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      cudaFree(p);
      return cuda_fail(e, "lmpb_peer_export: clearing the region");
    }
    g_ctx.own = static_cast<unsigned char*>(p);
    cudaGetDevice(&g_ctx.device);
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, g_ctx.own);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof h);
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_peer_import(const void* handles, int nranks, int rank) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!handles || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_peer_import: bad handles, rank or rank count");
  if (!g_ctx.own) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_peer_import: call lmpb_peer_export first");
  if (g_ctx.open) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_peer_import: already open");
  const unsigned char* hs = static_cast<const unsigned char*>(handles);
  for (int r = 0; r < nranks; ++r) {
    if (r == rank) {
      g_ctx.buf[r] = g_ctx.own;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)r * LMPB_PEER_HANDLE_BYTES, sizeof h);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != rank && g_ctx.buf[q]) cudaIpcCloseMemHandle(g_ctx.buf[q]);
      return cuda_fail(e, "cudaIpcOpenMemHandle");
    }
    g_ctx.buf[r] = static_cast<unsigned char*>(p);
  }
  g_ctx.nranks = nranks;
  g_ctx.rank = rank;
  g_ctx.epoch = 0;
  g_ctx.open = true;
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_peer_close(void) {
  std::lock_guard<std::mutex> g(g_mu);
  cudaDeviceSynchronize();
  if (g_ctx.open)
    for (int r = 0; r < g_ctx.nranks; ++r)
      if (r != g_ctx.rank && g_ctx.buf[r]) cudaIpcCloseMemHandle(g_ctx.buf[r]);
  if (g_ctx.own) cudaFree(g_ctx.own);
  g_ctx = PeerCtx{};
  return LMPB_OK;
}

extern "C" int lmpb_peer_size(void) { return g_ctx.open ? g_ctx.nranks : 0; }

extern "C" lmpb_status lmpb_reduce_allreduce(int op, int dtype, const void* in, const int64_t* shape, int ndim,
                                             int axis, void* out, void* stream) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_ctx.open) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_reduce_allreduce: no peer context (lmpb_peer_import)");
  const unsigned next = g_ctx.epoch + 1 == 0 ? 1 : g_ctx.epoch + 1;
  lmpb_status s = lmpb::reduce_allreduce_peer(op, dtype, in, shape, ndim, axis, out, g_ctx.buf, g_ctx.nranks,
                                              g_ctx.rank, next, kSlotBytes, reinterpret_cast<cudaStream_t>(stream));
  if (s == LMPB_OK) g_ctx.epoch = next;
  return s;
}
