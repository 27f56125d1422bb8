/*
 * rmsnorm_b200.h -- C ABI of the B200 (sm_100a) RMSNorm forward/backward library.
 *
 * This is the whole native boundary of the package: plain pointers, sizes and
 * status codes. No C++ exception crosses it, no torch type appears in it, and
 * the library never allocates device memory on a call: the caller owns every
 * buffer (inputs, outputs, backward workspace) and the stream.
 *
 * Interfaces of the reference (Int21-AI/RMSNorm-H100) that it replaces:
 *   rmsnorm_b200_fwd        <- rmsnorm_cuda_fwd (rmsnorm/csrc/ptx_rmsnorm_kernels.cu:7296-7321)
 *                              reached through the pybind entry points fwd_, fwd_fast and
 *                              fwd_residual_fast (rmsnorm/csrc/torch_bindings.cpp:120-194, 268-310)
 *   rmsnorm_b200_bwd        <- rmsnorm_cuda_bwd (ptx_rmsnorm_kernels.cu:7323-7351) reached
 *                              through bwd_ and bwd_fast (torch_bindings.cpp:196-266, 312-352)
 *   rmsnorm_b200_bwd_workspace_size
 *                           <- rmsnorm_cuda_bwd_partial_blocks / rmsnorm_cuda_bwd_reduce_chunks
 *                              (ptx_rmsnorm_kernels.cu:7275-7281), which the bindings used to
 *                              size dw_partial (torch_bindings.cpp:241-254, 317-340)
 *   rmsnorm_b200_strerror   <- the TORCH_CHECK / CUDA_CHECK messages that the reference threw
 *                              across its extern "C" boundary (ptx_rmsnorm_kernels.cu:42-50,
 *                              7232-7234; torch_bindings.cpp:50-70)
 *   rmsnorm_b200_device_status, rmsnorm_b200_set_wait_timeout_ns,
 *   rmsnorm_b200_selftest_wait_timeout
 *                           <- no counterpart: the reference's mbarrier waits are unbounded
 *                              (ptx_rmsnorm_kernels.cu:957-986). Every wait here is bounded
 *                              and reports through a device status word.
 *   rmsnorm_b200_abi_version, rmsnorm_b200_launch_count, rmsnorm_b200_last_plan,
 *   rmsnorm_b200_max_active_clusters
 *                           <- no counterpart (introspection for tests and benchmarks).
 *   rmsnorm_b200_debug_bounds_build, rmsnorm_b200_debug_report
 *                           <- no counterpart: the bounds-checked build's report (the
 *                              reference's only memory check was its standalone verifier's
 *                              element-wise compare, ptx_rmsnorm_kernels.cu:6723-6787).
 *
 * Semantics (identical to the reference's fp32 math, rmsnorm/rmsnorm.py:230-271, 390-399):
 *   rows are the flattened leading dimensions; row r uses affine head (r % heads).
 *   fwd:  h = x (+ residual) in fp32; rstd = rsqrt(mean(h^2) + eps);
 *         out = h * rstd * weight (+ bias); residual_out = h; rstd[r] = rstd.
 *   bwd:  xhat = x * rstd; wdy = dout * weight;  c = mean(xhat * wdy);
 *         dx = (wdy - xhat * c) * rstd (+ dresidual_out); dresidual = dx;
 *         dweight = sum_rows(dout * xhat); dbias = sum_rows(dout), reduced in a fixed
 *         order (bitwise reproducible run to run on the same device model).
 */
#ifndef RMSNORM_B200_H_
#define RMSNORM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RMSNORM_B200_ABI_VERSION 1

/* dtype codes: same numbering as the reference's dtype_code() (torch_bindings.cpp:37-48). */
enum {
  RMSNORM_B200_F16 = 0,
  RMSNORM_B200_BF16 = 1,
  RMSNORM_B200_F32 = 2
};

/* status codes */
enum {
  RMSNORM_B200_OK = 0,
  RMSNORM_B200_ERR_INVALID_ARGUMENT = 1,
  RMSNORM_B200_ERR_UNSUPPORTED = 2,
  RMSNORM_B200_ERR_WORKSPACE = 3,
  RMSNORM_B200_ERR_CUDA = 4,
  RMSNORM_B200_ERR_DEVICE_TIMEOUT = 5,
  RMSNORM_B200_ERR_NO_DEVICE = 6,
  RMSNORM_B200_ERR_SCRATCH_LIMIT = 7
};

/* Forward arguments. Pointers marked nullable may be NULL. All row-major, contiguous. */
typedef struct rmsnorm_b200_fwd_args {
  int64_t rows;               /* M >= 0 (rows after flattening; tokens*heads when per-head) */
  int64_t hidden;             /* N >= 1 */
  int32_t heads;              /* H >= 1; rows % H == 0; row r uses affine head r % H */
  int32_t x_dtype;
  const void* x;              /* [rows, hidden] */
  const void* residual;       /* nullable, [rows, hidden] */
  int32_t residual_dtype;
  int32_t weight_dtype;
  const void* weight;         /* nullable, [weight_heads, hidden] */
  int32_t weight_heads;       /* 1 (shared) or heads (per-head) */
  int32_t bias_dtype;
  const void* bias;           /* nullable, [bias_heads, hidden] */
  int32_t bias_heads;         /* 1 or heads */
  int32_t out_dtype;
  void* out;                  /* [rows, hidden] */
  void* residual_out;         /* nullable, [rows, hidden]; receives x (+ residual) */
  int32_t residual_out_dtype;
  int32_t reserved0;
  float* rstd;                /* nullable, [rows] fp32 */
  float eps;
  int32_t reserved1;
} rmsnorm_b200_fwd_args;

/* Backward arguments. */
typedef struct rmsnorm_b200_bwd_args {
  int64_t rows;
  int64_t hidden;
  int32_t heads;
  int32_t x_dtype;
  const void* x;              /* [rows, hidden]: the normalised input (x or residual_out) */
  const void* dout;           /* [rows, hidden] */
  int32_t dout_dtype;
  int32_t weight_dtype;
  const float* rstd;          /* [rows] fp32 */
  const void* weight;         /* nullable, [weight_heads, hidden] */
  int32_t weight_heads;
  int32_t dresidual_out_dtype;
  const void* dresidual_out;  /* nullable, [rows, hidden]; added to dx */
  void* dx;                   /* [rows, hidden] */
  int32_t dx_dtype;
  int32_t dresidual_dtype;
  void* dresidual;            /* nullable, [rows, hidden]; a second copy of dx */
  void* dweight;              /* nullable (requires weight), [weight_heads, hidden] */
  int32_t dweight_dtype;
  int32_t dbias_dtype;
  void* dbias;                /* nullable, [dbias_heads, hidden]: sum of dout over rows */
  int32_t dbias_heads;        /* 1 or heads */
  int32_t reserved0;
} rmsnorm_b200_bwd_args;

/* Enqueue the forward on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Uses the current CUDA device. Returns a status code; never blocks the host. */
int rmsnorm_b200_fwd(const rmsnorm_b200_fwd_args* args, void* stream);

/* Bytes of device workspace rmsnorm_b200_bwd needs for these arguments on the current
 * device (0 when no dweight/dbias is requested). The size depends on the device's SM count. */
int rmsnorm_b200_bwd_workspace_size(const rmsnorm_b200_bwd_args* args, size_t* bytes);

/* Enqueue the backward on `stream`. `workspace` must be device memory of at least
 * rmsnorm_b200_bwd_workspace_size() bytes, 16-byte aligned; its contents on entry are
 * ignored and it may be reused as soon as the stream has passed this call. */
int rmsnorm_b200_bwd(const rmsnorm_b200_bwd_args* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Backward that allocates nothing: the same kernels as rmsnorm_b200_bwd, with the
 * dweight/dbias partial sums kept in a scratch buffer built into the library instead of a
 * caller-provided workspace. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory at call time: a plugin inside a host
 * framework that has reserved all device memory for its own pool, or code that must not
 * allocate once it is running (allocation can block, fail, or synchronise the device).
 *
 * The buffer is RMSNORM_B200_NOALLOC_SCRATCH_BYTES of device memory, one per device,
 * reserved by every GPU that loads the library until the process exits. Problems whose
 * partial sums need more return RMSNORM_B200_ERR_SCRATCH_LIMIT without running (every
 * streaming-kernel problem fits on a B200; only very wide rows on the generic path can
 * exceed it). Where rmsnorm_b200_bwd's plan would keep more partial rows than fit (its
 * dbias kernels with the sums in tensor memory keep one per row group of every CTA), this
 * entry point runs the kernels that keep the sums in registers instead. The first call on a device looks up the buffer's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture. All calls on a
 * device share the one buffer, so calls whose kernels overlap on the GPU (different
 * streams, no ordering between them) race and give wrong dweight/dbias; calls ordered on
 * one stream are fine. Nothing in the buffer needs to be zero between calls: every
 * partial sum is written before it is read. */
#define RMSNORM_B200_NOALLOC_SCRATCH_BYTES (16u << 20)
int rmsnorm_b200_bwd_noalloc(const rmsnorm_b200_bwd_args* args, void* stream);

/* ---- Row-sharded backward over the GPUs of one node (one process per GPU) ----
 * No counterpart in the reference (single-GPU). A row-sharded training step sums every
 * rank's dweight / dbias; rmsnorm_b200_bwd_allreduce does that sum in the same kernel as
 * the backward's final fixed-order reduction of the partial rows: each rank pushes its
 * column sums, tagged, into every rank's exchange buffer over NVLink (peer stores, no
 * multicast) and sums the ranks' values in rank order, so every rank gets identical bits.
 *
 * Set-up, once per group: every rank calls rmsnorm_b200_peer_group_create (allocates and
 * zeroes its exchange buffer, returns its CUDA IPC handle), the ranks exchange the handles
 * (e.g. an all-gather over the process group), then every rank calls
 * rmsnorm_b200_peer_group_connect with all handles in rank order. Every rank must then
 * make the same sequence of rmsnorm_b200_bwd_allreduce calls with the same gradient shapes.
 * A rank waits for its peers at most the peer timeout (rmsnorm_b200_set_peer_timeout_ns,
 * default 10 s); a wait that runs out records RMSNORM_B200_ERR_DEVICE_TIMEOUT in the device
 * status word and the group must be re-created. */
#define RMSNORM_B200_IPC_HANDLE_BYTES 64
#define RMSNORM_B200_MAX_PEERS 8
typedef struct rmsnorm_b200_peer_group rmsnorm_b200_peer_group;

/* Bytes of the exchange buffer of a rank in a group of `world` ranks whose calls sum at
 * most `max_grad_floats` gradient values (dweight + dbias elements). */
int rmsnorm_b200_peer_buffer_size(int32_t world, int64_t max_grad_floats, size_t* bytes);

/* Creates this rank's member of a group on the current device: allocates (cudaMalloc,
 * set-up only) and zeroes its exchange buffer and writes the buffer's CUDA IPC handle
 * (RMSNORM_B200_IPC_HANDLE_BYTES bytes) to `ipc_handle`. */
int rmsnorm_b200_peer_group_create(int32_t rank, int32_t world, int64_t max_grad_floats, void* ipc_handle,
                                   rmsnorm_b200_peer_group** group);

/* Maps the other ranks' buffers: `ipc_handles` holds world handles in rank order (this
 * rank's own entry is ignored). */
int rmsnorm_b200_peer_group_connect(rmsnorm_b200_peer_group* group, const void* ipc_handles);

/* The same with device pointers this device can address for each rank's buffer (world
 * entries in rank order; this rank's own entry is ignored), for callers that map the
 * buffers themselves. */
int rmsnorm_b200_peer_group_connect_buffers(rmsnorm_b200_peer_group* group, void* const* buffers);

/* Device address of this rank's exchange buffer (for rmsnorm_b200_peer_group_connect_buffers
 * of the other ranks when they share this process's address space). */
int rmsnorm_b200_peer_group_buffer(rmsnorm_b200_peer_group* group, void** buffer);

/* Unmaps the peers' buffers and frees this rank's buffer. No call may be in flight. */
int rmsnorm_b200_peer_group_destroy(rmsnorm_b200_peer_group* group);

/* Longest wait for the peers inside rmsnorm_b200_bwd_allreduce (at least 1 ms). */
int rmsnorm_b200_set_peer_timeout_ns(uint64_t timeout_ns);

/* rmsnorm_b200_bwd on this rank's rows, with dweight / dbias summed over the group's
 * ranks (identical on every rank). Same arguments and workspace as rmsnorm_b200_bwd; the
 * group's device must be current. */
int rmsnorm_b200_bwd_allreduce(const rmsnorm_b200_bwd_args* args, void* workspace, size_t workspace_bytes,
                               rmsnorm_b200_peer_group* group, void* stream);

/* LayerNorm forward over rows of `hidden` elements: mean, variance as the mean of squared
 * deviations (fp32), out = (x - mean) * rsqrt(var + eps) * weight + bias. Replaces the
 * PyTorch implementation of layernorm_fwd (rmsnorm/rmsnorm.py:655-676); the reference has
 * no native kernel for it. */
typedef struct rmsnorm_b200_ln_fwd_args {
  int64_t rows;               /* >= 0 */
  int64_t hidden;             /* >= 1 (the normalised size) */
  int32_t x_dtype;
  int32_t weight_dtype;
  const void* x;              /* [rows, hidden] */
  const void* weight;         /* nullable (ones), [hidden] */
  const void* bias;           /* nullable (zeros), [hidden] */
  int32_t bias_dtype;
  int32_t out_dtype;
  void* out;                  /* nullable (statistics only), [rows, hidden] */
  float* mean;                /* nullable, [rows] fp32 */
  float* rstd;                /* nullable, [rows] fp32 */
  float eps;
  int32_t reserved0;
} rmsnorm_b200_ln_fwd_args;

int rmsnorm_b200_layernorm_fwd(const rmsnorm_b200_ln_fwd_args* args, void* stream);

/* Static, human-readable message for a status code. */
const char* rmsnorm_b200_strerror(int status);

/* Reads (and optionally clears) the current device's status word, in stream order:
 * 0 when no kernel has reported a problem, RMSNORM_B200_ERR_DEVICE_TIMEOUT when a bounded
 * device-side wait ran out. Synchronises `stream`. */
int rmsnorm_b200_device_status(void* stream, int32_t* status, int32_t* where, int32_t clear);

/* Upper bound of every device-side wait on the current device (default 2 s; at least 1 ms,
 * smaller values return RMSNORM_B200_ERR_INVALID_ARGUMENT). After a failure a kernel still
 * waits up to max(limit, 2 s) for its in-flight copies before it exits. */
int rmsnorm_b200_set_wait_timeout_ns(uint64_t timeout_ns);

/* Failure-detection self test: launches one CTA that waits, with the given bound, on an
 * mbarrier nothing ever arrives at. The wait runs out, the kernel records
 * RMSNORM_B200_ERR_DEVICE_TIMEOUT in the status word and returns; nothing faults. */
int rmsnorm_b200_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

int rmsnorm_b200_abi_version(void);

/* Bounds-checked build (librmsnorm_b200_debug.so, compiled with -DRMSB_DEBUG_BOUNDS; a
 * stand-in for a memory checker, not for production). Every API call registers the byte
 * ranges of its tensors, workspace and internal arrays; every load, store and copy of its
 * kernels checks its bytes against them (global memory) or against the end of the CTA's
 * shared memory, and a failed check is counted, the first one recorded, and the access
 * skipped (loads read zeros; nothing traps). rmsnorm_b200_debug_bounds_build returns 1 in
 * that build and 0 otherwise. rmsnorm_b200_debug_report synchronises `stream` and returns
 * the number of failed checks since the last clear and the first one's site (1 vector
 * load, 2 vector store, 3 bulk-copy source, 4 bulk-copy destination, 5 async copy, 6
 * scalar load, 7 scalar store, 8 exchange record, 9 peer word, 10 partial-row load, 11 L2
 * prefetch), address and size; clear != 0 resets them. The release build returns
 * RMSNORM_B200_ERR_UNSUPPORTED. */
int rmsnorm_b200_debug_bounds_build(void);
int rmsnorm_b200_debug_report(void* stream, uint64_t* violations, int32_t* site, uint64_t* address,
                              uint32_t* bytes, int32_t clear);

/* How many clusters of `cluster_size` CTAs of the streaming kernels (512 threads, the full
 * shared-memory carve-out) the current device can hold at once; 1 CTA per SM. Used by the
 * planner to size grids; exported for tests and benchmarks. */
int rmsnorm_b200_max_active_clusters(int32_t cluster_size, int32_t* clusters);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t rmsnorm_b200_launch_count(void);

/* Describes the plan of the last fwd/bwd call on this host thread (kernel family,
 * cluster size, grid, stage layout). Returns the full length; writes at most len-1 chars. */
int rmsnorm_b200_last_plan(char* buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* RMSNORM_B200_H_ */
