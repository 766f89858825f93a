/*
 * lmpb.h — C ABI of the Lamp3 B200 backend (sm_100a).
 *
 * This is the flat kernel layer that sits under Lamp3's CUDA dispatch.  Every
 * entry point takes plain device pointers, element counts and shapes, and a
 * cudaStream_t passed as `void*` (NULL = the legacy default stream).  No entry
 * point allocates an OUTPUT: the caller owns every input and output buffer,
 * exactly as the reference's `TensorMetaHandler` allocates the output before
 * the kernel runs (csrc/src/tensor/cpu/meta_handler.cpp:9-73).  Kernels are
 * launched asynchronously on the given stream; a host read must synchronise
 * that stream first.
 *
 * Each function names the reference interface it replaces (paths are relative
 * to the rushlite project root).  The reference registers one function pointer
 * per op and device in a `DispatchStub` table
 * (csrc/include/lamp3/tensor/dispatch_stub.hpp:21-64); a CUDA registration
 * unit built on this header wraps each stub signature around one call here
 * (allocate the output, call the lmpb_* function, throw on a non-OK status).
 *
 * Errors: every call returns an lmpb_status.  LMPB_ERR_INVALID mirrors the
 * reference's user-error LMP_CHECK (a throw of std::runtime_error,
 * csrc/include/lamp3/common/assert.hpp:89-90); the other codes replace
 * LMP_CUDA_CHECK's std::terminate (assert.hpp:95-102) by a status the caller
 * can turn into an exception.  lmpb_last_error() returns the calling thread's
 * message for its last failed call.
 */
#ifndef LMPB_H_
#define LMPB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LMPB_MAX_DIMS 16 /* csrc/include/lamp3/tensor/utils/align_utils.hpp:7 */

/* Element types, same numbering as lmp::tensor::DataType
 * (csrc/include/lamp3/tensor/data_type.hpp:25-32).  The output type of a
 * binary op is the larger enum value (type_upcast, data_type.hpp:77-80). */
typedef enum {
  LMPB_BOOL = 0,
  LMPB_INT16 = 1,
  LMPB_INT32 = 2,
  LMPB_INT64 = 3,
  LMPB_FLOAT32 = 4,
  LMPB_FLOAT64 = 5
} lmpb_dtype;

typedef enum {
  LMPB_OK = 0,
  LMPB_ERR_INVALID = 1,     /* bad argument: shape, dtype, op, null pointer */
  LMPB_ERR_CUDA = 2,        /* a CUDA runtime / driver call failed */
  LMPB_ERR_UNSUPPORTED = 3, /* valid request this build does not serve */
  LMPB_ERR_COMPILE = 4,     /* NVRTC rejected a generated fused kernel */
  LMPB_ERR_TIMEOUT = 5      /* a bounded device wait gave up */
} lmpb_status;

/* Binary ops: ops::add..lt (csrc/src/tensor/native/expand_ops.cpp:28-160),
 * functors csrc/include/lamp3/tensor/cpu/kernels.hpp:22-64.  Comparisons
 * produce 1/0 in the output dtype (not bool). */
typedef enum {
  LMPB_ADD = 0,
  LMPB_SUB = 1,
  LMPB_MUL = 2,
  LMPB_DIV = 3,
  LMPB_POW = 4,
  LMPB_EQ = 5,
  LMPB_NE = 6,
  LMPB_GE = 7,
  LMPB_LE = 8,
  LMPB_GT = 9,
  LMPB_LT = 10,
  /* the two same-shape backward kernels, unary_ops.hpp:103-105 */
  LMPB_ABS_BACKWARD = 11,
  LMPB_CLAMP_BACKWARD = 12
} lmpb_binary_op;

/* Unary ops: ops::neg..tan, clamp (csrc/src/tensor/native/unary_ops.cpp:23-55) */
typedef enum {
  LMPB_NEG = 0,
  LMPB_EXP = 1,
  LMPB_LOG = 2,
  LMPB_SQRT = 3,
  LMPB_ABS = 4,
  LMPB_SIN = 5,
  LMPB_COS = 6,
  LMPB_TAN = 7,
  LMPB_CLAMP = 8
} lmpb_unary_op;

/* Reductions: ops::sum/max/min/prod (csrc/src/tensor/native/reduct_ops.cpp:12-28) */
typedef enum { LMPB_SUM = 0, LMPB_MAX = 1, LMPB_MIN = 2, LMPB_PROD = 3 } lmpb_reduce_op;

/* Copy directions for lmpb_copy. */
typedef enum { LMPB_H2D = 0, LMPB_D2H = 1, LMPB_D2D = 2, LMPB_H2H = 3 } lmpb_copy_kind;

/* ---------------------------------------------------------------- errors */

/* Message of the calling thread's last failed call ("" if none). */
const char* lmpb_last_error(void);
/* Library version string; also proves the library loaded. */
const char* lmpb_version(void);
/* Number of kernels this library has launched in the process (all devices).
 * No counterpart in the reference; used to count launches in benchmarks. */
uint64_t lmpb_kernel_launches(void);

/* ------------------------------------------------------------ shapes */

/* NumPy broadcast of two shapes (AlignUtil::calc_aligned_shape,
 * csrc/src/tensor/utils/align_utils.cpp:18-40).  Writes out_shape (room for
 * LMPB_MAX_DIMS) and *out_ndim; LMPB_ERR_INVALID on a broadcast violation. */
lmpb_status lmpb_broadcast_shape(const int64_t* a_shape, int a_ndim, const int64_t* b_shape,
                                 int b_ndim, int64_t* out_shape, int* out_ndim);

/* ------------------------------------------------------- elementwise */

/* out = op(a, b) with NumPy broadcasting of row-major contiguous a and b.
 * Replaces add_cuda..lt_cuda (csrc/src/tensor/cuda/kernels.cu:13-64) and the
 * binary/expand dispatch handlers behind them (cuda/binary.cu:63-96,
 * cuda/expand.cu:38-59).  Both operands are converted to out_dtype before
 * the op (cuda/ptr_pack.cuh:12-17); out_dtype is normally
 * max(a_dtype, b_dtype).  `out` holds prod(broadcast shape) elements.
 * LMPB_ABS_BACKWARD / LMPB_CLAMP_BACKWARD take (input, grad) as (a, b) and
 * need equal shapes and dtypes (abs_backward_cuda / clamp_backward_cuda,
 * csrc/src/tensor/native/unary_ops.cpp:57-83); p0/p1 are clamp's min/max. */
lmpb_status lmpb_binary(int op, int out_dtype, const void* a, int a_dtype, const int64_t* a_shape,
                        int a_ndim, const void* b, int b_dtype, const int64_t* b_shape, int b_ndim,
                        void* out, double p0, double p1, void* stream);

/* out[i] = op(in[i]) for n elements, out and in of the same dtype
 * (infer_unary, csrc/src/tensor/infer_meta.cpp:11-17).  Replaces
 * neg_cuda..clamp_cuda (csrc/src/tensor/cuda/kernels.cu:31-64; cuda/unary.cu:13-82).
 * Integer inputs of exp/log/sqrt/sin/cos/tan compute in double and truncate
 * (cuda/kernels.cuh:24-25).  p0/p1 are clamp's min/max (ignored otherwise). */
lmpb_status lmpb_unary(int op, int dtype, const void* in, void* out, int64_t n, double p0,
                       double p1, void* stream);

/* ------------------------------------------------------- reductions */

/* Keep-dim reduction of row-major `in` (shape[ndim]) along `axis` into `out`
 * (shape with shape[axis] = 1), accumulating in the input dtype
 * (infer_reduct, csrc/src/tensor/infer_meta.cpp:35-44).  Replaces
 * sum_cuda..prod_cuda (csrc/src/tensor/cuda/kernels.cu:112-122) and
 * reduct_dispatch_handler (cuda/reduct.cu:213-260).  Integer sums, max and min
 * are bit-exact with the reference; float sums and products differ only by
 * summation order.  Results are deterministic run to run.  A large reduction
 * over a leading axis uses a split workspace that the library takes from
 * CUDA's stream-ordered pool (cudaMallocAsync) on `stream`. */
lmpb_status lmpb_reduce(int op, int dtype, const void* in, const int64_t* shape, int ndim,
                        int axis, void* out, void* stream);

/* lmpb_reduce for callers that must not allocate device memory during the
 * call (a framework whose memory planner owns every allocation, a runtime
 * with a fixed device budget, a loop that cannot risk a pool miss turning
 * into cudaMalloc).  Same arguments and results as lmpb_reduce, but the
 * split-row workspace is a fixed 1 MiB scratch array inside the library,
 * held on every GPU that loads it until the process exits; nothing is
 * allocated or freed.  A reduction needing more than 1 MiB of scratch
 * (outer x inner x chunks x element size) returns LMPB_ERR_INVALID.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  All calls share the one array:
 * calls whose kernels may overlap on the GPU (other streams, other host
 * threads) race on it, so serialise them.  No counterpart in the reference. */
lmpb_status lmpb_reduce_noalloc(int op, int dtype, const void* in, const int64_t* shape, int ndim,
                                int axis, void* out, void* stream);

/* ----------------------------------------------------------- matmul */

/* C[m,n] = A[m,k] · B[k,n], row-major, converted to out_dtype
 * (matmul_cuda, csrc/src/tensor/cuda/kernels.cu:83-110; cuda/matrix.cu:178-199).
 * fp32 × fp32 → fp32 runs on the tcgen05 tensor cores: every row of A and
 * column of B is scaled by a power of two into fp16 range and split into
 * fp16 hi and lo parts, and hi·hi + hi·lo + lo·hi accumulate in fp32 in TMEM
 * (fp32-level accuracy, Inf/NaN propagate); other dtype combinations use a
 * SIMT kernel that accumulates in out_dtype like the reference. */
lmpb_status lmpb_matmul(int out_dtype, const void* A, int a_dtype, const void* B, int b_dtype,
                        void* C, int64_t m, int64_t k, int64_t n, void* stream);

/* fp32 GEMM with operand transposes and accumulate, on the same
 * tensor-core path:  C[m,n] = op(A)·op(B) + beta·C, op(X) = X or Xᵀ of a
 * row-major array (A is [m,k] or, with trans_a, [k,m]; B is [k,n] or, with
 * trans_b, [n,k]).  beta is 0 or 1.  This lets autograd compute
 * dA = G·Bᵀ and dB = Aᵀ·G and accumulate them into the grad buffers without
 * materialising the transposes that MatrixMultiplicationBackward builds
 * (csrc/src/autograd/functions/matrix_ops.cpp:8-24). */
lmpb_status lmpb_gemm_f32(int trans_a, int trans_b, const float* A, const float* B, float* C,
                          int64_t m, int64_t n, int64_t k, float beta, void* stream);

/* C[m,n] = clamp(op(A)·op(B) + bias, lo, hi) in one tensor-core GEMM: the
 * bias row (n fp32 values, broadcast over the rows; null for none) and the
 * clamp (when `clamp` is non-zero) run in the GEMM's epilogue, rounding and
 * comparing exactly as the eager ADD and CLAMP kernels do, so the result is
 * bit-identical to lmpb_gemm_f32 followed by lmpb_binary(ADD, C, bias) and
 * lmpb_unary(CLAMP).  This is the Linear(+ReLU) of the reference's layers
 * (matmul, broadcast add, clamp(0, DBL_MAX): python layers/linear.py,
 * layers/activation.py) without writing and re-reading the product.  No
 * single counterpart in the reference, which runs the three ops apart. */
lmpb_status lmpb_gemm_f32_bias_act(int trans_a, int trans_b, const float* A, const float* B, float* C,
                                   int64_t m, int64_t n, int64_t k, const float* bias, int clamp,
                                   double lo, double hi, void* stream);

/* The tensor-core GEMM's work schedule, the same functions its kernels run,
 * exported so that tests can check it without a GPU.  Output tile t (tiles
 * of tm x tn, tile rows grouped by 8) starts at (*m0, *n0); split-K unit u
 * covers tile *t over k-blocks [*kb0, *kb1); lmpb_gemm_sched_splits returns
 * the split count for ntiles tiles of num_kb k-blocks on `clusters` CTA pairs
 * (forced > 0: a requested count, reduced until no unit is empty).  No
 * counterpart in the reference. */
void lmpb_gemm_sched_tile(int t, int tiles_m, int tiles_n, int tm, int tn, int* m0, int* n0);
void lmpb_gemm_sched_unit(int u, int splits, int num_kb, int* t, int* kb0, int* kb1);
int lmpb_gemm_sched_splits(int64_t ntiles, int num_kb, int clusters, int forced);

/* LMPB_ERR_TIMEOUT if a bounded device wait inside a kernel expired since
 * the last call (the kernel then stopped early and its output is invalid),
 * else LMPB_OK.  Synchronises the current device.  No counterpart in the
 * reference, whose kernels have no device-side waits. */
lmpb_status lmpb_device_error(void);

/* out[n,m] = in[m,n]ᵀ (transpose_cuda, csrc/src/tensor/cuda/kernels.cu:66-81). */
lmpb_status lmpb_transpose(int dtype, const void* in, void* out, int64_t m, int64_t n,
                           void* stream);

/* ----------------------------------------------------------- memory */

/* Device allocation from CUDA's stream-ordered pool; replaces empty_cuda and
 * the caching allocator (csrc/src/tensor/cuda/memory.cu:56-65,
 * cuda/allocator.cu:39-138).  Blocks are 256-byte aligned.  These are the
 * only calls that allocate, and a caller with its own allocator can skip them. */
lmpb_status lmpb_malloc(void** ptr, size_t bytes, void* stream);
lmpb_status lmpb_free(void* ptr, void* stream);

/* fill_cuda (csrc/src/tensor/cuda/memory.cu:67-73): ptr[0..n) = (T)value. */
lmpb_status lmpb_fill(int dtype, void* ptr, int64_t n, double value, void* stream);

/* copy_cuda (csrc/src/tensor/cuda/memory.cu:126-174): casting copy of n
 * elements between host and device.  A host side must stay valid until the
 * stream reaches the copy (pinned memory makes it asynchronous). */
lmpb_status lmpb_copy(int kind, const void* src, int src_dtype, void* dst, int dst_dtype,
                      int64_t n, void* stream);

/* add_inplace_cuda (csrc/src/tensor/cuda/memory.cu:22-83): dst[i] += src[i],
 * the gradient accumulation of Variable::incr_grad
 * (csrc/src/autograd/variable.cpp:30-35). */
lmpb_status lmpb_add_inplace(int dtype, void* dst, const void* src, int64_t n, void* stream);

/* ------------------------------------------------- multi-GPU collectives */

/* The reference is single-device; these serve the exchange steps of the
 * row-partitioned multi-GPU paths built on it (one process per GPU): the
 * all-reduce of a leading-axis reduction's partials and of data-parallel
 * gradients.  NCCL underneath, loaded at run time; LMPB_ERR_UNSUPPORTED when
 * it is absent.  No counterpart in the reference. */
#define LMPB_COMM_ID_BYTES 128

/* Writes a new communicator id (LMPB_COMM_ID_BYTES bytes) for rank 0 to
 * share with the other ranks (through the launcher's store, for example). */
lmpb_status lmpb_comm_unique_id(void* id, size_t bytes);
/* Joins this process, on the current CUDA device, to the communicator of
 * `nranks` ranks named by `id`.  One communicator per process. */
lmpb_status lmpb_comm_init(const void* id, int nranks, int rank);
lmpb_status lmpb_comm_destroy(void);
/* Number of ranks of the communicator (0 before lmpb_comm_init). */
int lmpb_comm_size(void);
/* In-place all-reduce (`op` an lmpb_reduce_op) of `nbufs` device buffers of
 * `dtype` (int32, int64, float32, float64) in one grouped launch.  With
 * overlap = 0 it runs on `stream`, after the work already queued there.  With
 * overlap = 1 it runs on the library's communication stream, still after the
 * work queued on `stream`, so later kernels on `stream` proceed meanwhile;
 * lmpb_comm_join(stream) then makes `stream` wait for every overlapped
 * all-reduce issued so far.  Both forms can be recorded by stream capture. */
lmpb_status lmpb_allreduce(int dtype, void* const* bufs, const int64_t* counts, int nbufs, int op, int overlap,
                           void* stream);
lmpb_status lmpb_comm_join(void* stream);

/* Leading-axis reduction fused with the all-reduce of its result across the
 * GPUs of a row-partitioned job, in ONE kernel over NVLink peer memory: each
 * rank reduces its own rows (`in`, shape[ndim], along `axis` with all dims
 * before it of extent 1), pushes its partial into every rank's exchange
 * region, and every rank folds the partials in rank order, so all ranks write
 * identical `out` (the reduction over all ranks' rows).  Replaces, for the
 * sharded C3 dim-0 case, sum_cuda..prod_cuda (csrc/src/tensor/cuda/kernels.cu:112-122)
 * followed by a separate all-reduce; the reference itself is single-device.
 * Setup, once, collectively: every rank calls lmpb_peer_export (allocates its
 * region, LMPB_PEER_HANDLE_BYTES of CUDA IPC handle out), the handles are
 * exchanged out of band (rank order), then every rank calls lmpb_peer_import.
 * Every rank must make the same sequence of lmpb_reduce_allreduce calls; the
 * kernel waits for the other ranks with a bound (~2 s), after which it stops
 * and lmpb_device_error reports LMPB_ERR_TIMEOUT.  One rank per GPU.
 * LMPB_ERR_UNSUPPORTED when the shape is outside the fused path (the caller
 * then reduces with lmpb_reduce and all-reduces with lmpb_allreduce). */
#define LMPB_PEER_HANDLE_BYTES 64
lmpb_status lmpb_peer_export(void* handle, size_t bytes);
lmpb_status lmpb_peer_import(const void* handles, int nranks, int rank);
lmpb_status lmpb_peer_close(void);
/* Number of ranks of the peer context (0 when none is open). */
int lmpb_peer_size(void);
lmpb_status lmpb_reduce_allreduce(int op, int dtype, const void* in, const int64_t* shape, int ndim, int axis,
                                  void* out, void* stream);

/* ------------------------------------------------------ fused kernels */

/* The lazy-fusion compiler behind capture_on / capture.  Replaces the NVRTC
 * inductor (build_fused_graph csrc/src/inductor/nvrtc/fused_graph.cpp:6-35,
 * codegen_kernel codegen.cpp:21-61, NVRTCInductorBackend::realize
 * nvrtc_backend.cpp:145-190).  Unlike the reference, a fused region may
 * contain broadcast leaves, constant fills, and reductions of its result over
 * broadcast axes, and may write several outputs from one pass.
 *
 * A program is a DAG of lmpb_fnode in topological order over one iteration
 * space `iter_shape`.  Leaves are device arrays whose shapes broadcast to the
 * iteration space.  Every node computes in its own dtype after converting its
 * inputs to that dtype (codegen.cpp:45-55).  Each output names a node and a
 * mode: STORE writes the full iteration space, ACCUM adds into an existing
 * full-size buffer (add_inplace fused in), REDUCE_SUM / REDUCE_SUM_ACCUM sum
 * the node over the axes where out_shape is 1 (the sum_broadcast_axis of
 * csrc/src/autograd/utils/grad_utils.cpp:10-36), add the optional addend
 * node, and store or accumulate. */
typedef enum {
  LMPB_FN_LEAF = 0,   /* reads leaf slot `a` */
  LMPB_FN_CONST = 1,  /* the constant p0 */
  LMPB_FN_BINARY = 2, /* binary op `sub` on nodes a, b (params p0/p1 for clamp_backward) */
  LMPB_FN_UNARY = 3,  /* unary op `sub` on node a (p0/p1 for clamp) */
  LMPB_FN_ROWRED = 4  /* LMPB_SUM or LMPB_MAX (`sub`) of node a over the last
                         iteration dim; the same value along that dim.  The
                         max and sum of a row softmax (layers/activation.py:26-40
                         of the reference's Python layer) fuse with what reads
                         them; equal bit for bit to the separate reduction */
} lmpb_fnode_kind;

typedef struct {
  int32_t kind;  /* lmpb_fnode_kind */
  int32_t sub;   /* lmpb_binary_op / lmpb_unary_op */
  int32_t dtype; /* lmpb_dtype the node computes in */
  int32_t a, b;  /* input node indices (or leaf slot for LEAF) */
  double p0, p1;
} lmpb_fnode;

typedef struct {
  int32_t dtype;
  int32_t ndim;
  int64_t shape[LMPB_MAX_DIMS]; /* right-aligned broadcast to the iteration space */
} lmpb_fleaf;

typedef enum {
  LMPB_OUT_STORE = 0,
  LMPB_OUT_ACCUM = 1,
  LMPB_OUT_REDUCE_SUM = 2,
  LMPB_OUT_REDUCE_SUM_ACCUM = 3
} lmpb_fout_mode;

typedef struct {
  int32_t node;
  int32_t mode;    /* lmpb_fout_mode */
  int32_t dtype;   /* dtype of the output buffer */
  int32_t addend;  /* REDUCE_* only: node added to the sum (-1: none); it must
                      not vary along the reduced axes, e.g. the elementwise
                      terms of a gradient that also receives a broadcast sum */
  int32_t ndim;
  int32_t reserved;
  int64_t shape[LMPB_MAX_DIMS]; /* == iter shape, or with 1s on reduced axes */
} lmpb_fout;

typedef struct lmpb_fused_s* lmpb_fused;

/* Compile (or fetch from the in-process and on-disk caches) a fused kernel.
 * The handle is valid until lmpb_fused_release. */
lmpb_status lmpb_fused_build(const lmpb_fnode* nodes, int n_nodes, const lmpb_fleaf* leaves,
                             int n_leaves, const lmpb_fout* outs, int n_outs,
                             const int64_t* iter_shape, int iter_ndim, lmpb_fused* handle);
/* Launch it: leaf_ptrs[n_leaves] inputs, out_ptrs[n_outs] outputs. */
lmpb_status lmpb_fused_launch(lmpb_fused handle, const void* const* leaf_ptrs,
                              void* const* out_ptrs, void* stream);
lmpb_status lmpb_fused_release(lmpb_fused handle);
/* Generated CUDA source of a handle (for tests and debugging). */
const char* lmpb_fused_source(lmpb_fused handle);

#ifdef __cplusplus
}
#endif

#endif /* LMPB_H_ */
