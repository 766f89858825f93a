// Device collectives for the multi-GPU paths: an NCCL communicator per
// process (one process per GPU), all-reduce of device buffers on the
// caller's stream or overlapped on a per-device communication stream.
//
// Lamp3 itself is single-device; the sharded paths it gains here are the two
// exchange steps of a row-partitioned job: the leading-axis reduction's
// partials (one small all-reduce after the reduce kernel) and data-parallel
// training's gradient sum.  Both are issued on the stream the host layer
// computes on, so they are ordered after the kernels that produce their
// input and can be recorded into a CUDA graph together with the step.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2): the library loads, and
// everything single-GPU works, on a machine without it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>
#include <vector>

#include "lmpb.h"

namespace lmpb {
lmpb_status set_error(lmpb_status st, const std::string& msg);
}

namespace {

struct Nccl {
  void* so = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  const char* (*errorString)(ncclResult_t) = nullptr;
};

std::mutex g_mu;
Nccl g_nccl;
bool g_loaded = false;

// The communicator of this process and the device it was created on, plus a
// communication stream and the events of overlapped all-reduces not yet joined.
struct Comm {
  ncclComm_t comm = nullptr;
  int device = -1, nranks = 0, rank = 0;
  cudaStream_t stream = nullptr;
  std::vector<cudaEvent_t> pending, free_events;
};
Comm g_comm;

lmpb_status load() {
  if (g_loaded) return LMPB_OK;
  void* so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!so) return lmpb::set_error(LMPB_ERR_UNSUPPORTED, std::string("NCCL not available: ") + dlerror());
  Nccl n;
  n.so = so;
  bool ok = true;
  auto sym = [&](auto& fp, const char* name) {
    fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(so, name));
    ok = ok && fp;
  };
  sym(n.getUniqueId, "ncclGetUniqueId");
  sym(n.commInitRank, "ncclCommInitRank");
  sym(n.commDestroy, "ncclCommDestroy");
  sym(n.allReduce, "ncclAllReduce");
  sym(n.groupStart, "ncclGroupStart");
  sym(n.groupEnd, "ncclGroupEnd");
  sym(n.errorString, "ncclGetErrorString");
  if (!ok) return lmpb::set_error(LMPB_ERR_UNSUPPORTED, "libnccl.so.2 lacks an expected symbol");
  g_nccl = n;
  g_loaded = true;
  return LMPB_OK;
}

lmpb_status nccl_err(ncclResult_t r, const char* what) {
  return lmpb::set_error(LMPB_ERR_CUDA, std::string(what) + ": " + g_nccl.errorString(r));
}

bool nccl_type(int dt, ncclDataType_t* t) {
  switch (dt) {
    case LMPB_INT32: *t = ncclInt32; return true;
    case LMPB_INT64: *t = ncclInt64; return true;
    case LMPB_FLOAT32: *t = ncclFloat32; return true;
    case LMPB_FLOAT64: *t = ncclFloat64; return true;
    default: return false;
  }
}

bool nccl_op(int op, ncclRedOp_t* r) {
  switch (op) {
    case LMPB_SUM: *r = ncclSum; return true;
    case LMPB_MAX: *r = ncclMax; return true;
    case LMPB_MIN: *r = ncclMin; return true;
    case LMPB_PROD: *r = ncclProd; return true;
    default: return false;
  }
}

cudaEvent_t take_event() {
  if (!g_comm.free_events.empty()) {
    cudaEvent_t e = g_comm.free_events.back();
    g_comm.free_events.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  return e;
}

}  // namespace

extern "C" lmpb_status lmpb_comm_unique_id(void* out, size_t bytes) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!out || bytes < sizeof(ncclUniqueId))
    return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_comm_unique_id: buffer smaller than LMPB_COMM_ID_BYTES");
  lmpb_status st = load();
  if (st != LMPB_OK) return st;
  ncclUniqueId id;
  ncclResult_t r = g_nccl.getUniqueId(&id);
  if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
  memcpy(out, &id, sizeof(id));
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_comm_init(const void* id, int nranks, int rank) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!id || nranks < 1 || rank < 0 || rank >= nranks)
    return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_comm_init: bad id, rank or rank count");
  if (g_comm.comm) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_comm_init: a communicator already exists");
  lmpb_status st = load();
  if (st != LMPB_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return lmpb::set_error(LMPB_ERR_CUDA, "lmpb_comm_init: no device");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  ncclResult_t r = g_nccl.commInitRank(&c, nranks, uid, rank);
  if (r != ncclSuccess) return nccl_err(r, "ncclCommInitRank");
  cudaStream_t s = nullptr;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
    g_nccl.commDestroy(c);
    return lmpb::set_error(LMPB_ERR_CUDA, "lmpb_comm_init: stream");
  }
  g_comm.comm = c;
  g_comm.device = dev;
  g_comm.nranks = nranks;
  g_comm.rank = rank;
  g_comm.stream = s;
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_comm_destroy(void) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_comm.comm) return LMPB_OK;
  cudaStreamSynchronize(g_comm.stream);
  g_nccl.commDestroy(g_comm.comm);
  for (cudaEvent_t e : g_comm.pending) cudaEventDestroy(e);
  for (cudaEvent_t e : g_comm.free_events) cudaEventDestroy(e);
  cudaStreamDestroy(g_comm.stream);
  g_comm = Comm{};
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_allreduce(int dtype, void* const* bufs, const int64_t* counts, int nbufs, int op,
                                      int overlap, void* stream) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_comm.comm) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_allreduce: no communicator (lmpb_comm_init)");
  ncclDataType_t t;
  ncclRedOp_t r;
  if (!nccl_type(dtype, &t)) return lmpb::set_error(LMPB_ERR_UNSUPPORTED, "lmpb_allreduce: dtype");
  if (!nccl_op(op, &r)) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_allreduce: op");
  if (nbufs < 0 || (nbufs && (!bufs || !counts))) return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_allreduce: buffers");
  if (nbufs == 0) return LMPB_OK;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  cudaStream_t run = cs;
  if (overlap) {
    // the communication stream starts after the work queued on `stream`
    cudaEvent_t ready = take_event();
    if (cudaEventRecord(ready, cs) != cudaSuccess || cudaStreamWaitEvent(g_comm.stream, ready, 0) != cudaSuccess)
      return lmpb::set_error(LMPB_ERR_CUDA, "lmpb_allreduce: stream fork");
    g_comm.free_events.push_back(ready);
    run = g_comm.stream;
  }
  ncclResult_t e = g_nccl.groupStart();
  for (int i = 0; i < nbufs && e == ncclSuccess; ++i) {
    if (counts[i] < 0 || (counts[i] && !bufs[i])) {
      g_nccl.groupEnd();
      return lmpb::set_error(LMPB_ERR_INVALID, "lmpb_allreduce: bad buffer");
    }
    if (counts[i]) e = g_nccl.allReduce(bufs[i], bufs[i], (size_t)counts[i], t, r, g_comm.comm, run);
  }
  ncclResult_t e2 = g_nccl.groupEnd();
  if (e != ncclSuccess) return nccl_err(e, "ncclAllReduce");
  if (e2 != ncclSuccess) return nccl_err(e2, "ncclGroupEnd");
  if (overlap) {
    cudaEvent_t done = take_event();
    if (cudaEventRecord(done, g_comm.stream) != cudaSuccess)
      return lmpb::set_error(LMPB_ERR_CUDA, "lmpb_allreduce: event");
    g_comm.pending.push_back(done);
  }
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_comm_join(void* stream) {
  std::lock_guard<std::mutex> g(g_mu);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  for (cudaEvent_t e : g_comm.pending) {
    if (cudaStreamWaitEvent(cs, e, 0) != cudaSuccess) return lmpb::set_error(LMPB_ERR_CUDA, "lmpb_comm_join");
    g_comm.free_events.push_back(e);
  }
  g_comm.pending.clear();
  return LMPB_OK;
}

extern "C" int lmpb_comm_size(void) { return g_comm.comm ? g_comm.nranks : 0; }
