// device_common.cuh -- sm_100a building blocks shared by every kernel of the library:
// inline-PTX wrappers for mbarriers, TMA bulk copies (cp.async.bulk, no tensor map, no
// multicast), cluster / distributed-shared-memory access, bounded waits that report
// through a device status word, and dtype-generic 8-element vector load/store.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "rmsnorm_b200.h"

namespace rmsb200 {

// ---------------------------------------------------------------------------------------
// Device status word (one per device: file-scope __device__ variables live in each
// device's copy of the module). 0 = OK; otherwise the first error recorded. The library
// is a single translation unit, so the variables are defined here.
// ---------------------------------------------------------------------------------------
__device__ int g_status = 0;
__device__ int g_status_where = 0;
__device__ unsigned long long g_wait_timeout_ns = 2000000000ull;

// Where a bounded wait gave up (reported through rmsnorm_b200_device_status).
enum WaitSite : int {
  kSiteFwdFull = 1,
  kSiteFwdEmpty = 2,
  kSiteFwdCluster = 3,
  kSiteBwdFull = 4,
  kSiteBwdEmpty = 5,
  kSiteBwdCluster = 6,
  kSiteDrain = 7,
  kSiteSelftest = 8,
  kSitePeer = 9,  // a rank's dweight / dbias sums in the peer all-reduce
};

__device__ __forceinline__ void record_error(int code, int where) {
  if (atomicCAS(&g_status, 0, code) == 0) {
    atomicExch(&g_status_where, where);
  }
}

// Programmatic dependent launch. pdl_wait: blocks until the grids this launch depends on
// have completed and their memory operations are visible (a no-op for a launch without
// the programmatic-serialization attribute); every global access of a streaming kernel
// follows it. pdl_launch_dependents: lets the next launch in the stream be scheduled
// (its CTAs then run their shared-memory prologue as this grid's CTAs retire).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Dynamic shared memory of the streaming kernels (every extern __shared__ array aliases its
// start).
extern __shared__ __align__(128) unsigned char rmsb_dyn_smem[];

// ---------------------------------------------------------------------------------------
// Bounds-checked build (compiled with -DRMSB_DEBUG_BOUNDS into librmsnorm_b200_debug.so;
// the stand-in for a memory checker). Every API call registers the byte ranges of its
// tensors, workspace and internal arrays (g_dbg_ranges, written by a one-thread kernel
// ahead of the call's kernels on the same stream). Each vector / scalar load and store,
// bulk copy (source and shared-memory destination), async copy and exchange access then
// checks its bytes: global addresses must lie inside one registered range, shared
// addresses below the end of the CTA's dynamic shared memory. A failed check records the
// first bad access (site, address, size) and the count in g_dbg_report and SKIPS the
// access (loads read zeros; a skipped bulk copy still completes its bytes on the
// mbarrier, so no wait hangs). Nothing traps. Runs of non-bulk async copies are checked as
// a whole before the first copy (and are plain copies in this build: see cp_async_4). In the release build every check is the
// constant true and compiles away.
// ---------------------------------------------------------------------------------------
enum DbgSite : int {
  kDbgVecLoad = 1,
  kDbgVecStore = 2,
  kDbgBulkSrc = 3,
  kDbgBulkDst = 4,
  kDbgAsyncCopy = 5,
  kDbgScalarLoad = 6,
  kDbgScalarStore = 7,
  kDbgRecord = 8,
  kDbgPeerWord = 9,
  kDbgPartialLoad = 10,
  kDbgPrefetch = 11,
};
constexpr int kDbgMaxRanges = 24;
struct DbgRanges {
  int32_t n;
  int32_t clip_site;  // unused by the device; keeps the layout 8-byte aligned
  unsigned long long lo[kDbgMaxRanges];
  unsigned long long hi[kDbgMaxRanges];
};

#ifdef RMSB_DEBUG_BOUNDS
__device__ DbgRanges g_dbg_ranges;
__device__ unsigned long long g_dbg_report[4];  // violations, first site, first address, first size

__device__ __noinline__ bool dbg_check(const void* p, uint32_t bytes, int site) {
  const unsigned long long a = reinterpret_cast<unsigned long long>(p);
  bool ok = true;
  if (__isShared(p)) {
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    const uint32_t off = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    const uint32_t end = static_cast<uint32_t>(__cvta_generic_to_shared(rmsb_dyn_smem)) + dyn;
    ok = off + bytes <= end;
  } else if (__isGlobal(p)) {
    ok = false;
    const int n = g_dbg_ranges.n;
    for (int i = 0; i < n && i < kDbgMaxRanges; ++i)
      if (a >= g_dbg_ranges.lo[i] && a + bytes <= g_dbg_ranges.hi[i]) ok = true;
  }
  if (!ok && atomicAdd(&g_dbg_report[0], 1ull) == 0) {
    g_dbg_report[1] = static_cast<unsigned long long>(site);
    g_dbg_report[2] = a;
    g_dbg_report[3] = bytes;
  }
  return ok;
}

__global__ void dbg_ranges_kernel(const DbgRanges r) {
  if (threadIdx.x == 0) g_dbg_ranges = r;
}
#define RMSB_DBG_OK(p, bytes, site) ::rmsb200::dbg_check((p), (bytes), (site))
#else
#define RMSB_DBG_OK(p, bytes, site) true
#endif

// Scalar stores / loads of the streaming and generic kernels, checked in the debug build.
template <typename T>
__device__ __forceinline__ void st1(T* p, T v) {
  if (RMSB_DBG_OK(p, sizeof(T), kDbgScalarStore)) *p = v;
}
template <typename T>
__device__ __forceinline__ T ld1(const T* p) {
  return RMSB_DBG_OK(p, sizeof(T), kDbgScalarLoad) ? *p : T{};
}

// One float4 of a partial row (the dweight / dbias reductions).
__device__ __forceinline__ float4 ld_partial4(const float* p) {
  if (!RMSB_DBG_OK(p, 16, kDbgPartialLoad)) return make_float4(0.f, 0.f, 0.f, 0.f);
  return *reinterpret_cast<const float4*>(p);
}

__device__ __forceinline__ bool abort_requested() {
  return *reinterpret_cast<volatile int*>(&g_status) != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------
// Shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async proxy and to the other CTAs of
// the cluster.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One probe of phase `parity`; the hardware may suspend the thread for a short while.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Same, with cluster-scope acquire: used where peers of the cluster complete the phase
// with st.async ... complete_tx into this CTA's shared memory.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Smallest wait limit the host may set, and the floor of the drain after a failure: a CTA
// never leaves while a bulk copy may still be landing in its shared memory, whatever limit
// the caller chose for ordinary waits.
constexpr unsigned long long kMinWaitTimeoutNs = 1000000ull;        // 1 ms
constexpr unsigned long long kDrainTimeoutFloorNs = 2000000000ull;  // 2 s

// Bounded wait, slow path: returns false (after recording the error) when the phase has
// not completed within g_wait_timeout_ns, or -- when `honor_abort` -- as soon as another
// thread of any CTA has recorded an error. The drain (honor_abort false) waits at least
// kDrainTimeoutFloorNs.
template <bool kClusterScope>
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int where, bool honor_abort) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = honor_abort ? g_wait_timeout_ns
                                     : (g_wait_timeout_ns > kDrainTimeoutFloorNs ? g_wait_timeout_ns
                                                                                  : kDrainTimeoutFloorNs);
  while (true) {
    if (kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) {
      return true;
    }
    if (honor_abort && abort_requested()) return false;
    if (globaltimer_ns() - t0 > limit) {
      record_error(RMSNORM_B200_ERR_DEVICE_TIMEOUT, where);
      return false;
    }
  }
}

// Bounded wait: one inline probe, then the out-of-line bounded loop.
template <bool kClusterScope = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int where, bool honor_abort = true) {
  if (kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow<kClusterScope>(bar, parity, where, honor_abort);
}

// ---------------------------------------------------------------------------------------
// TMA bulk copy (global -> this CTA's shared memory), completion counted in bytes on an
// mbarrier. Source and destination 16-byte aligned, size a multiple of 16. No multicast.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Orders this CTA's earlier generic-proxy accesses to shared memory before later
// async-proxy (TMA) writes to it: issued before a stage is refilled.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar, uint64_t policy) {
#ifdef RMSB_DEBUG_BOUNDS
  if (!RMSB_DBG_OK(gsrc, bytes, kDbgBulkSrc) || !RMSB_DBG_OK(smem_dst, bytes, kDbgBulkDst)) {
    // the bytes the consumers wait for are completed without a copy
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
    return;
  }
#endif
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of global memory into L2 (no shared-memory destination, no completion):
// warms the lines a later bulk_load of the same range will read. Source 16-byte aligned,
// size a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
  if (!RMSB_DBG_OK(gsrc, bytes, kDbgPrefetch)) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// Non-bulk async copy of 4 or 16 bytes; completion is attached to an mbarrier with
// cp_async_arrive (which raises the barrier's expected arrivals by one first, so the
// phase cannot complete before these copies land).
// The bounds-checked build checks a run of these copies as a whole before issuing it, and
// makes them plain synchronous copies with no arrive of their own: its out-of-line checker
// calls, falling between async copies and their tracking arrive, left that arrive
// undelivered on B200 (a wait that timed out). The issuing thread's copies then precede
// its expect-tx arrive on the slot, which the consumers acquire.
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gsrc) {
#ifdef RMSB_DEBUG_BOUNDS
  *static_cast<uint32_t*>(smem_dst) = *static_cast<const uint32_t*>(gsrc);
#else
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
#endif
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
#ifdef RMSB_DEBUG_BOUNDS
  *static_cast<uint4*>(smem_dst) = *static_cast<const uint4*>(gsrc);
#else
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
#endif
}

__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
#ifdef RMSB_DEBUG_BOUNDS
  (void)bar;  // the copies above were synchronous: the phase needs no extra arrival
#else
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
#endif
}

// ---------------------------------------------------------------------------------------
// Clusters / distributed shared memory
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// All threads of all CTAs of the cluster. Used once, at kernel start, so that every
// CTA's mbarriers are initialised before any peer signals them.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

__device__ __forceinline__ uint32_t map_peer(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}

// 4-byte store into a peer CTA's shared memory that completes 4 tx-bytes on the peer's
// mbarrier (the peer waits for the bytes, not for an arrival).
__device__ __forceinline__ void st_async_peer(uint32_t remote_addr, float v, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
          remote_addr),
      "r"(__float_as_uint(v)), "r"(remote_bar)
      : "memory");
}

// Global-memory accesses of the cross-CTA exchange (gpu scope; not cached in L1).
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  if (!RMSB_DBG_OK(p, 8, kDbgRecord)) return;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  if (!RMSB_DBG_OK(p, 8, kDbgRecord)) return 0ull;
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------------------------------
// Tensor memory (TMEM) as per-thread accumulator storage. TMEM is 128 lanes x 512 columns
// of 32-bit cells per SM, normally the tensor cores' accumulator; a streaming kernel has
// no MMA, so it can keep per-column running sums there instead of in registers. A warp may
// access only the 32 lanes of its quarter (warp index % 4); with the 32x32b shape, lane i
// of the warp reads / writes TMEM lane (quarter * 32 + i), `n` consecutive columns.
// Allocation and deallocation are issued by one whole warp; every tcgen05.ld / st is
// issued by all 32 lanes of a warp together (the .sync.aligned forms).
// ---------------------------------------------------------------------------------------
// Allocates `ncols` columns (a power of two, 32..512) for this CTA and writes the TMEM
// address to `dst` in shared memory; then gives up the right to allocate again, so other
// CTAs on the SM are never kept waiting by this one.
__device__ __forceinline__ void tmem_alloc_warp(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_warp(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Orders this thread's earlier tcgen05 operations before a following thread barrier, and
// the barrier before this thread's later tcgen05 operations.
__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive columns of this lane, as 8 float pairs (element 2i in .x, 2i+1 in .y).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float2 (&v)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float2 (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0].x)), "r"(__float_as_uint(v[0].y)), "r"(__float_as_uint(v[1].x)),
      "r"(__float_as_uint(v[1].y)), "r"(__float_as_uint(v[2].x)), "r"(__float_as_uint(v[2].y)),
      "r"(__float_as_uint(v[3].x)), "r"(__float_as_uint(v[3].y)), "r"(__float_as_uint(v[4].x)),
      "r"(__float_as_uint(v[4].y)), "r"(__float_as_uint(v[5].x)), "r"(__float_as_uint(v[5].y)),
      "r"(__float_as_uint(v[6].x)), "r"(__float_as_uint(v[6].y)), "r"(__float_as_uint(v[7].x)),
      "r"(__float_as_uint(v[7].y))
      : "memory");
}

// Blocks until this thread's earlier tcgen05.ld (wait_ld) / tcgen05.st (wait_st) are done.
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------------------
// 8-element vectors. Every tensor of a row is handled in groups of 8 consecutive
// elements: 16 bytes for fp16/bf16, 32 bytes for fp32.
// ---------------------------------------------------------------------------------------
template <typename T>
struct Vec8;

template <>
struct Vec8<float> {
  static constexpr int kBytes = 32;
  __device__ __forceinline__ static void load(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ static void load_global(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ static void store(void* p, const float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecStore)) return;
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
    __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[4], v[5], v[6], v[7]));
  }
};

__device__ __forceinline__ void unpack_bf16x2(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xffff0000u);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void unpack_f16x2(uint32_t u, float& lo, float& hi) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct Vec8<__nv_bfloat16> {
  static constexpr int kBytes = 16;
  __device__ __forceinline__ static void unpack(const uint4 u, float (&v)[8]) {
    unpack_bf16x2(u.x, v[0], v[1]);
    unpack_bf16x2(u.y, v[2], v[3]);
    unpack_bf16x2(u.z, v[4], v[5]);
    unpack_bf16x2(u.w, v[6], v[7]);
  }
  __device__ __forceinline__ static void load(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ __forceinline__ static void load_global(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), v);
  }
  __device__ __forceinline__ static void store(void* p, const float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecStore)) return;
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    __stcs(reinterpret_cast<uint4*>(p), u);
  }
};

template <>
struct Vec8<__half> {
  static constexpr int kBytes = 16;
  __device__ __forceinline__ static void unpack(const uint4 u, float (&v)[8]) {
    unpack_f16x2(u.x, v[0], v[1]);
    unpack_f16x2(u.y, v[2], v[3]);
    unpack_f16x2(u.z, v[4], v[5]);
    unpack_f16x2(u.w, v[6], v[7]);
  }
  __device__ __forceinline__ static void load(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ __forceinline__ static void load_global(const void* p, float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float& e : v) e = 0.f; return; }
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), v);
  }
  __device__ __forceinline__ static void store(void* p, const float (&v)[8]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecStore)) return;
    uint4 u;
    u.x = pack_f16x2(v[0], v[1]);
    u.y = pack_f16x2(v[2], v[3]);
    u.z = pack_f16x2(v[4], v[5]);
    u.w = pack_f16x2(v[6], v[7]);
    __stcs(reinterpret_cast<uint4*>(p), u);
  }
};

// The same 8-element vectors held as 4 float pairs, for the paired fp32 instructions of
// sm_100 (__ffma2_rn / __fmul2_rn / __fadd2_rn: two lanes per instruction, each rounded
// exactly as the scalar instruction). Pair i holds elements 2i and 2i+1.
template <typename T>
struct Pair8;

template <>
struct Pair8<float> {
  __device__ __forceinline__ static void load(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = make_float2(a.x, a.y); v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(b.x, b.y); v[3] = make_float2(b.z, b.w);
  }
  __device__ __forceinline__ static void load_global(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = make_float2(a.x, a.y); v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(b.x, b.y); v[3] = make_float2(b.z, b.w);
  }
  __device__ __forceinline__ static void store(void* p, const float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 32, kDbgVecStore)) return;
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
    __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[2].x, v[2].y, v[3].x, v[3].y));
  }
};

__device__ __forceinline__ float2 unpack_bf16x2_pair(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

__device__ __forceinline__ uint32_t pack_bf16x2_pair(float2 v) {
  __nv_bfloat162 h = __float22bfloat162_rn(v);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_f16x2_pair(uint32_t u) {
  return __half22float2(*reinterpret_cast<__half2*>(&u));
}

__device__ __forceinline__ uint32_t pack_f16x2_pair(float2 v) {
  __half2 h = __float22half2_rn(v);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct Pair8<__nv_bfloat16> {
  __device__ __forceinline__ static void unpack(const uint4 u, float2 (&v)[4]) {
    v[0] = unpack_bf16x2_pair(u.x); v[1] = unpack_bf16x2_pair(u.y);
    v[2] = unpack_bf16x2_pair(u.z); v[3] = unpack_bf16x2_pair(u.w);
  }
  __device__ __forceinline__ static void load(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ __forceinline__ static void load_global(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), v);
  }
  __device__ __forceinline__ static void store(void* p, const float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecStore)) return;
    uint4 u;
    u.x = pack_bf16x2_pair(v[0]); u.y = pack_bf16x2_pair(v[1]);
    u.z = pack_bf16x2_pair(v[2]); u.w = pack_bf16x2_pair(v[3]);
    __stcs(reinterpret_cast<uint4*>(p), u);
  }
};

template <>
struct Pair8<__half> {
  __device__ __forceinline__ static void unpack(const uint4 u, float2 (&v)[4]) {
    v[0] = unpack_f16x2_pair(u.x); v[1] = unpack_f16x2_pair(u.y);
    v[2] = unpack_f16x2_pair(u.z); v[3] = unpack_f16x2_pair(u.w);
  }
  __device__ __forceinline__ static void load(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ __forceinline__ static void load_global(const void* p, float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecLoad)) { for (float2& e : v) e = make_float2(0.f, 0.f); return; }
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), v);
  }
  __device__ __forceinline__ static void store(void* p, const float2 (&v)[4]) {
    if (!RMSB_DBG_OK(p, 16, kDbgVecStore)) return;
    uint4 u;
    u.x = pack_f16x2_pair(v[0]); u.y = pack_f16x2_pair(v[1]);
    u.z = pack_f16x2_pair(v[2]); u.w = pack_f16x2_pair(v[3]);
    __stcs(reinterpret_cast<uint4*>(p), u);
  }
};

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }

// Tag type for a tensor that is absent from a kernel instantiation.
struct NoT {};
template <typename T>
struct Present {
  static constexpr bool value = true;
};
template <>
struct Present<NoT> {
  static constexpr bool value = false;
};

// Runtime-dtype variants for tensors whose dtype is not a template parameter (outputs
// of secondary dtype, affine parameters loaded once). `e` is the element index.
__device__ __forceinline__ int dtype_bytes(int dt) { return dt == RMSNORM_B200_F32 ? 4 : 2; }

__device__ __forceinline__ void load8_rt(const void* base, int dt, int64_t e, float (&v)[8],
                                         bool global) {
  if (dt == RMSNORM_B200_F32) {
    const float* p = reinterpret_cast<const float*>(base) + e;
    if (global) Vec8<float>::load_global(p, v); else Vec8<float>::load(p, v);
  } else if (dt == RMSNORM_B200_BF16) {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(base) + e;
    if (global) Vec8<__nv_bfloat16>::load_global(p, v); else Vec8<__nv_bfloat16>::load(p, v);
  } else {
    const __half* p = reinterpret_cast<const __half*>(base) + e;
    if (global) Vec8<__half>::load_global(p, v); else Vec8<__half>::load(p, v);
  }
}

// Paired form of load8_rt (affine parameters of the streaming kernels, read from global
// memory once per kernel).
__device__ __forceinline__ void load8p_rt(const void* base, int dt, int64_t e, float2 (&v)[4]) {
  if (dt == RMSNORM_B200_F32) {
    Pair8<float>::load_global(reinterpret_cast<const float*>(base) + e, v);
  } else if (dt == RMSNORM_B200_BF16) {
    Pair8<__nv_bfloat16>::load_global(reinterpret_cast<const __nv_bfloat16*>(base) + e, v);
  } else {
    Pair8<__half>::load_global(reinterpret_cast<const __half*>(base) + e, v);
  }
}

__device__ __forceinline__ void store8_rt(void* base, int dt, int64_t e, const float (&v)[8]) {
  if (dt == RMSNORM_B200_F32) {
    Vec8<float>::store(reinterpret_cast<float*>(base) + e, v);
  } else if (dt == RMSNORM_B200_BF16) {
    Vec8<__nv_bfloat16>::store(reinterpret_cast<__nv_bfloat16*>(base) + e, v);
  } else {
    Vec8<__half>::store(reinterpret_cast<__half*>(base) + e, v);
  }
}

// Scalar runtime-dtype access (generic kernels).
__device__ __forceinline__ float load1_rt(const void* base, int dt, int64_t e) {
  if (!RMSB_DBG_OK(static_cast<const char*>(base) + e * dtype_bytes(dt), dtype_bytes(dt), kDbgScalarLoad)) return 0.f;
  if (dt == RMSNORM_B200_F32) return reinterpret_cast<const float*>(base)[e];
  if (dt == RMSNORM_B200_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[e]);
  return __half2float(reinterpret_cast<const __half*>(base)[e]);
}

__device__ __forceinline__ void store1_rt(void* base, int dt, int64_t e, float v) {
  if (!RMSB_DBG_OK(static_cast<char*>(base) + e * dtype_bytes(dt), dtype_bytes(dt), kDbgScalarStore)) return;
  if (dt == RMSNORM_B200_F32) {
    reinterpret_cast<float*>(base)[e] = v;
  } else if (dt == RMSNORM_B200_BF16) {
    reinterpret_cast<__nv_bfloat16*>(base)[e] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(base)[e] = __float2half_rn(v);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

}  // namespace rmsb200
