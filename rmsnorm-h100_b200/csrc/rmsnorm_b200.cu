// rmsnorm_b200.cu -- C ABI, per-device state, launch planner and dispatch.
//
// Dispatch (replaces launch_fwd / launch_bwd of the reference,
// rmsnorm/csrc/ptx_rmsnorm_kernels.cu:4941-6600, and its per-(dtype, N) thread tables):
//   * streaming kernels (stream_kernels.cuh) for every shape whose rows are 8-element
//     vectorisable and 16-byte aligned, in the specialised dtype combinations;
//   * generic kernels (generic_kernels.cuh) for everything else;
//   * backward dweight/dbias: per-(CTA, row group) fp32 partial rows written by the main
//     kernel, summed in a fixed order by reduce_partials_kernel (deterministic; the
//     reference used fp32 atomics on several paths, ptx_rmsnorm_kernels.cu:3288-3291).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <type_traits>
#include <string>
#include <tuple>
#include <vector>

#include "generic_kernels.cuh"
#include "peer_allreduce.cuh"
#include "stream_kernels.cuh"

// One rank's member of a peer group (opaque in the C ABI): the exchange buffers of the
// fused dweight / dbias all-reduce (peer_allreduce.cuh).
struct rmsnorm_b200_peer_group {
  int rank = 0;
  int world = 0;
  int device = -1;
  int64_t max_floats = 0;                                 // words per (parity, source) slot
  void* buffer = nullptr;                                 // this rank's exchange buffer (owned)
  void* opened[RMSNORM_B200_MAX_PEERS] = {};              // IPC mappings of the peers' buffers
  unsigned long long* recv[RMSNORM_B200_MAX_PEERS] = {};  // each rank's receive area, as this device sees it
  bool connected = false;
};
static_assert(sizeof(cudaIpcMemHandle_t) == RMSNORM_B200_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(RMSNORM_B200_MAX_PEERS == rmsb200::kMaxPeers, "peer count");

namespace rmsb200 {
namespace {

std::atomic<uint64_t> g_launches{0};
thread_local std::string t_last_plan;

// Shared memory an SM offers (228 KB), the opt-in maximum per CTA (227 KB), and the
// 1 KB the runtime reserves per resident CTA.
constexpr int kSmemPerSm = 233472;
constexpr int kSmemOptIn = 232448;
constexpr int kSmemSysReserve = 1024;

struct BlockCfg {
  int threads;
  int ctas_per_sm;
  int smem_budget;  // bytes of stages one CTA may use (barrier area excluded)
};
constexpr BlockCfg kLarge = {kBlockLarge, 1, kSmemOptIn - kSmemReserve};
constexpr BlockCfg kSmall = {kBlockSmall, 2, kSmemPerSm / 2 - kSmemSysReserve - kSmemReserve};

int elem_bytes(int dt) { return dt == RMSNORM_B200_F32 ? 4 : 2; }
bool valid_dt(int dt) { return dt == RMSNORM_B200_F16 || dt == RMSNORM_B200_BF16 || dt == RMSNORM_B200_F32; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------------------------
// Per-device state: SM count, kernel attributes set once per (device, kernel), cached
// occupancy queries. Kernel attributes are per device, so they are set lazily for each
// device a call runs on (the reference set them once per process, which is wrong with
// more than one GPU: ptx_rmsnorm_kernels.cu:5471-5475).
// ------------------------------------------------------------------------------------
struct DeviceState {
  int sm_count = 0;
  void* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch on this device
  XRecord* xrec = nullptr;          // device address of g_xrec on this device
  uint32_t* xgen = nullptr;         // device address of g_xgen on this device
  uint32_t xepoch = 0;              // launches that used the global-memory exchange
  std::mutex mu;
  std::map<const void*, bool> attrs_done;
  std::map<std::tuple<const void*, int, int, int>, int> occupancy;  // (kernel, P, smem, threads)
};

std::mutex g_devices_mu;
std::vector<std::unique_ptr<DeviceState>> g_devices;

int get_device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RMSNORM_B200_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_devices_mu);
  if (static_cast<int>(g_devices.size()) <= dev) g_devices.resize(dev + 1);
  if (!g_devices[dev]) {
    auto st = std::make_unique<DeviceState>();
    if (cudaDeviceGetAttribute(&st->sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return RMSNORM_B200_ERR_NO_DEVICE;
    g_devices[dev] = std::move(st);
  }
  *out = g_devices[dev].get();
  return RMSNORM_B200_OK;
}

// Scratch for rmsnorm_b200_bwd_noalloc: a file-scope device array, one per device that
// loads the library. In host code `g_noalloc_scratch` only names a host-side stand-in, so
// its device address is looked up (per device, with that device current) and passed on.
static __device__ __align__(256) unsigned char g_noalloc_scratch[RMSNORM_B200_NOALLOC_SCRATCH_BYTES];

int noalloc_scratch(DeviceState* ds, void** out) {
  std::lock_guard<std::mutex> lock(ds->mu);
  if (!ds->noalloc_scratch) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
      cudaGetLastError();
      return RMSNORM_B200_ERR_CUDA;
    }
    ds->noalloc_scratch = ptr;
  }
  *out = ds->noalloc_scratch;
  return RMSNORM_B200_OK;
}

// Records of the global-memory row-total exchange (split rows on a cooperative grid): a
// file-scope device array, kXRecSets sets used round-robin by launch, so launches that
// overlap at their ends (at most a few on one device) use different sets. Within a set,
// records and generation counters are kept per group size P: the records of a CTA then
// belong to one CTA group, whose counter gives each of its executions a fresh generation
// (drawn on the device), so neither another launch nor an earlier replay of the same
// captured launch can supply a record with the awaited tag.
static __device__ XRecord g_xrec[kXRecSets * kXGroupSizes * kXRecMaxCtas * kXSlots];
static __device__ uint32_t g_xgen[kXRecSets * kXGroupSizes * kXRecMaxCtas];

// Next record set (round robin): the records and generation counters of group size P.
int next_xset(DeviceState* ds, int P, XRecord** rec, uint32_t** gen) {
  int pidx = 0;
  while ((2 << pidx) < P) ++pidx;
  if ((2 << pidx) != P || pidx >= kXGroupSizes) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(ds->mu);
  if (!ds->xrec) {
    void* ptr = nullptr;
    void* gptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_xrec) != cudaSuccess || !ptr ||
        cudaGetSymbolAddress(&gptr, g_xgen) != cudaSuccess || !gptr) {
      cudaGetLastError();
      return RMSNORM_B200_ERR_CUDA;
    }
    ds->xrec = static_cast<XRecord*>(ptr);
    ds->xgen = static_cast<uint32_t*>(gptr);
  }
  const size_t slot = static_cast<size_t>(ds->xepoch++ % kXRecSets) * kXGroupSizes + pidx;
  *rec = ds->xrec + slot * kXRecMaxCtas * kXSlots;
  *gen = ds->xgen + slot * kXRecMaxCtas;
  return RMSNORM_B200_OK;
}

int ensure_attrs(DeviceState* ds, const void* kernel) {
  std::lock_guard<std::mutex> lock(ds->mu);
  if (ds->attrs_done.count(kernel)) return RMSNORM_B200_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemOptIn) != cudaSuccess)
    return RMSNORM_B200_ERR_CUDA;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return RMSNORM_B200_ERR_CUDA;
  ds->attrs_done[kernel] = true;
  return RMSNORM_B200_OK;
}

// Clusters of P CTAs (P > 1) or CTAs (P == 1) that can be resident at once.
int resident_units(DeviceState* ds, const void* kernel, int P, int smem, int threads) {
  const auto key = std::make_tuple(kernel, P, smem, threads);
  {
    std::lock_guard<std::mutex> lock(ds->mu);
    auto it = ds->occupancy.find(key);
    if (it != ds->occupancy.end()) return it->second;
  }
  int n = 0;
  if (P == 1) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess) n = 0;
    n *= ds->sm_count;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P * ds->sm_count);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = P;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a refused query must not poison the caller's next check
  std::lock_guard<std::mutex> lock(ds->mu);
  ds->occupancy[key] = n;
  return n;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : dflt;
}

int pow2_ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

int log2i(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// L2 prefetch distance: each refill of a ring slot can also prefetch the unit S further
// on, so a unit's bytes are requested about 2S units before they are consumed while only S
// units of shared memory hold them. Measured on B200 it pays only where a row slice fills
// shared memory and streams as chunks (K > 1); elsewhere the extra L2 traffic costs more
// than the deeper pipeline gains.
void set_prefetch(StreamPlan& pl) {
  const int force = env_int("RMSNORM_B200_L2_PREFETCH", -1);  // units; 0 = off
  pl.pf = force >= 0 ? force : (pl.K > 1 ? pl.S : 0);
}

// Builds the thread/tile/stage/cluster plan for a streaming kernel launched with block
// shape `bc`. `in_bytes[k]` is the element size of staged input k (0 = absent);
// `rstd_staged` adds the per-row rstd block (backward); `max_vecs` is the kernel's vectors
// per thread. `force_p` (0 = free) pins the cluster size. Returns false (with a reason)
// when the shape is outside what the streaming kernels take.
bool make_stream_plan(int64_t rows, int64_t N64, int H, const int in_bytes[3], bool rstd_staged,
                      int max_vecs, const BlockCfg& bc, int force_p, StreamPlan* out, std::string* why,
                      bool one_sweep = false, bool col_mode = false) {
  StreamPlan pl = {};
  if (N64 % 8 != 0 || N64 > (int64_t(1) << 30)) { *why = "hidden % 8 != 0"; return false; }
  const int N = static_cast<int>(N64);
  const int64_t W = static_cast<int64_t>(H) * N;
  if (W / 8 > (int64_t(1) << 24)) { *why = "row too long"; return false; }
  const int vrow = static_cast<int>(W / 8);
  const int T = bc.threads;
  const int budget = bc.smem_budget;
  pl.T = T;
  pl.heads = H;
  pl.N = N;
  pl.W = W;
  pl.nrows = rows / H;
  int P = 1;
  pl.cols = max_vecs;
  if (H > 1) {
    const int vs = N / 8;
    if (!is_pow2(vs) || vs > 32) { *why = "per-head segment not a power of two <= 32 vectors"; return false; }
    // column mode (col_mode): the fewest columns per thread whose group fits the CTA, each
    // thread then covering max_vecs / cols super-rows of a sweep
    int cols = max_vecs;
    if (col_mode)
      for (int c = 1; c < max_vecs; c <<= 1) {
        const int per = (vrow + c - 1) / c;
        if (vs * ((per + vs - 1) / vs) <= T) { cols = c; break; }
      }
    const int per_thread_min = (vrow + cols - 1) / cols;
    const int G = vs * ((per_thread_min + vs - 1) / vs);
    if (G > T) { *why = "per-head super-row too wide"; return false; }
    pl.seg_mode = 1;
    pl.vs = vs;
    pl.G = G;
    pl.vslice = vrow;
    pl.cols = cols;
  } else if (vrow <= 32) {
    pl.seg_mode = 1;
    pl.vs = pow2_ceil(vrow);
    pl.G = pl.vs;
    pl.vslice = vrow;
  } else {
    pl.seg_mode = 0;
    pl.vs = 1;
    int bytes_per_vec = 0;
    for (int k = 0; k < 3; ++k) bytes_per_vec += 8 * in_bytes[k];
    const int max_p = std::min(kMaxCluster, env_int("RMSNORM_B200_MAX_CLUSTER", kMaxCluster));
    P = 0;
    for (int cand = 1; cand <= max_p; cand <<= 1) {
      if (force_p && cand != force_p) continue;
      if (vrow % cand) continue;
      const int vs_ = vrow / cand;
      if (vs_ > T * max_vecs) continue;
      const int64_t slice_bytes = static_cast<int64_t>(vs_) * bytes_per_vec + (rstd_staged ? 16 : 0);
      if (slice_bytes > budget) continue;
      // prefer a split that leaves room for at least two stages
      if (slice_bytes * 2 > budget && cand < max_p && !force_p && vrow % (cand * 2) == 0 &&
          (vrow / (cand * 2)) >= 32)
        continue;
      P = cand;
      break;
    }
    if (P == 0) { *why = "no cluster split fits"; return false; }
    pl.vslice = vrow / P;
    const int per_thread_min = (pl.vslice + max_vecs - 1) / max_vecs;
    pl.G = std::min(T, static_cast<int>(align_up(static_cast<uint32_t>(per_thread_min), 32u)));
  }
  pl.vs_shift = log2i(pl.vs);
  pl.P = P;
  pl.rps = P > 1 ? 1 : T / pl.G;
  if (pl.rps < 1) { *why = "group wider than the CTA"; return false; }
  pl.lag = 0;
  pl.xpair = 0;
  pl.xbcast = 0;
  pl.K = 1;
  pl.kpc_shift = log2i(max_vecs);

  if (P > 1) {
    // Split-row ring: a row slice streams as K chunks (ring units). K = 1 (lag 1) when two
    // slices fit; otherwise the slice is cut into the fewest chunks of >= 32 KB that leave
    // at least one chunk of the next row loading behind the current row (K > 1 needs every
    // thread to own max_vecs vectors of the slice, so a chunk holds whole thread vectors).
    const bool full = pl.vslice == pl.G * max_vecs;
    auto chunk_bytes = [&](int k) {
      uint32_t off = 0;
      for (int t = 0; t < 3; ++t) off = align_up(off + static_cast<uint32_t>(pl.vslice / k) * 8u * in_bytes[t], 128);
      return off + (rstd_staged ? 128u : 0u);
    };
    const int force_k = env_int("RMSNORM_B200_FORCE_K", 0);
    int K = 1;
    if (force_k > 0) {
      if (!is_pow2(force_k) || force_k > max_vecs || (force_k > 1 && !full)) {
        *why = "forced chunk count does not divide the thread vectors";
        return false;
      }
      K = force_k;
    } else if (budget / static_cast<int>(chunk_bytes(1)) < 2 && full) {
      for (int k = 2; k <= max_vecs; k <<= 1) {
        if (chunk_bytes(k) < 32u * 1024u) break;
        K = k;
        if (budget / static_cast<int>(chunk_bytes(k)) >= k + 1) break;
      }
    }
    pl.K = K;
    pl.kpc_shift = log2i(max_vecs / K);
    pl.R = 1;
    uint32_t off = 0;
    for (int t = 0; t < 3; ++t) {
      pl.row_bytes[t] = static_cast<uint32_t>(pl.vslice / K) * 8u * in_bytes[t];
      pl.off[t] = off;
      off = align_up(off + pl.row_bytes[t], 128);
    }
    pl.off[3] = off;
    if (rstd_staged) off += 128;
    pl.stage_bytes = off;
    const int max_s = std::max(1, std::min(kMaxStages, env_int("RMSNORM_B200_MAX_STAGES", kMaxStages)));
    pl.S = std::min<int>(max_s, budget / static_cast<int>(off));
    if (pl.S < K) { *why = "no split-row ring fits"; return false; }
    // Exchange lag: rows i-lag..i stay resident while row i's total is exchanged, which
    // needs S >= (lag + 1) * K ring units; a deeper lag lets a CTA run ahead of its
    // slowest peer.
    const int force_lag = env_int("RMSNORM_B200_FORCE_LAG", -1);
    int lag = pl.S >= 2 * K ? 1 : 0;
    if (force_lag >= 0) lag = std::min(force_lag, rmsb200::kMaxLag);
    while (lag > 0 && pl.S < (lag + 1) * K) --lag;
    pl.lag = lag;
    pl.ntiles = pl.nrows;
    set_prefetch(pl);
    *out = pl;
    return true;
  }

  uint32_t per_row = 0;
  for (int k = 0; k < 3; ++k) {
    pl.row_bytes[k] = static_cast<uint32_t>(pl.vslice) * 8u * in_bytes[k];
    per_row += pl.row_bytes[k];
  }
  const int rstd_per_row = pl.seg_mode ? H : 1;
  if (rstd_staged) per_row += 4u * rstd_per_row;
  // Tile (stage) size and ring depth, measured on B200: a ring of about 100 KB in at least
  // two stages streams best (deeper rings delay the first tiles of small problems and gain
  // nothing on large ones); per-head rows (seg mode) amortise their per-tile work over
  // bigger tiles.
  const int dflt_stage = (pl.seg_mode ? (rstd_staged ? 128 : 64) : 48) * 1024;
  const int target = env_int("RMSNORM_B200_STAGE_BYTES", dflt_stage) * T / kBlockLarge;
  const int rstep = pl.rps * (max_vecs / pl.cols);  // super-rows per sweep
  int R = rstep;
  if (P == 1 && !one_sweep) {  // one_sweep: one row per row group per tile
    const int64_t m = std::max<int64_t>(1, target / (static_cast<int64_t>(rstep) * per_row));
    R = static_cast<int>(rstep * m);
    const int64_t rows_needed = (pl.nrows + rstep - 1) / rstep * rstep;
    if (R > rows_needed) R = static_cast<int>(std::max<int64_t>(rstep, rows_needed));
  }
  auto layout = [&](int r) {
    uint32_t off = 0;
    for (int k = 0; k < 3; ++k) {
      pl.off[k] = off;
      off = align_up(off + static_cast<uint32_t>(r) * pl.row_bytes[k], 128);
    }
    pl.off[3] = off;
    if (rstd_staged) off = align_up(off + 4u * r * rstd_per_row, 128);
    return off;
  };
  uint32_t stage = layout(R);
  while (2 * stage > static_cast<uint32_t>(budget) && R > rstep) {  // keep two stages
    R -= rstep;
    stage = layout(R);
  }
  if (stage > static_cast<uint32_t>(budget)) { *why = "stage does not fit shared memory"; return false; }
  pl.R = R;
  pl.stage_bytes = stage;
  const int max_s = std::max(1, std::min(kMaxStages, env_int("RMSNORM_B200_MAX_STAGES", kMaxStages)));
  // per-head backwards in column mode with 16-bit inputs stream best from three tiles
  // (measured on B200: +1.0 % to +1.6 %; fp32 -2 %)
  const int dflt_ring = (pl.cols < max_vecs && rstd_staged && in_bytes[0] <= 2) ? 200 * 1024 : 100 * 1024;
  const int ring = env_int("RMSNORM_B200_RING_BYTES", dflt_ring) * T / kBlockLarge;
  const int s_fit = std::max(1, std::min<int>(max_s, budget / static_cast<int>(stage)));
  pl.S = std::min(s_fit, std::max(2, ring / static_cast<int>(stage)));
  // Row-mode rows pipelined one tile deep keep two tiles resident, so the ring gets one more
  // slot. Measured on B200: a gain for forwards whose CTA holds several row groups (cfg 1:
  // +2 %), a loss where one row fills the CTA (-1 % to -5 %) and for backwards (-6 % at
  // N = 4096), so by default only the former pipeline (LayerNorm always does).
  pl.pipe_rows = 0;
  const int pipe = env_int("RMSNORM_B200_PIPE_ROWS", -1);  // -1 auto, 0 off, 1 on
  if (!pl.seg_mode && R == pl.rps && (pipe == 1 || (pipe < 0 && pl.rps >= 2 && !rstd_staged))) {
    pl.pipe_rows = 1;
    pl.S = std::min(s_fit, pl.S + 1);
  }
  pl.ntiles = (pl.nrows + R - 1) / R;
  set_prefetch(pl);
  *out = pl;
  return true;
}

int smem_bytes(const StreamPlan& pl) { return pl.S * static_cast<int>(pl.stage_bytes) + kSmemReserve; }


std::string describe(const char* kind, const StreamPlan& pl, int grid) {
  char buf[512];
  std::snprintf(buf, sizeof(buf),
                "%s mode=%s P=%d x=%s grid=%d clusters=%d T=%d G=%d rps=%d R=%d S=%d stage=%u "
                "vslice=%d vs=%d cols=%d K=%d lag=%d%s pf=%d tiles=%lld",
                kind, pl.seg_mode ? "seg" : "row", pl.P,
                pl.P == 1 ? "none" : (pl.xmode == kXGlobal ? "global" : "cluster"), grid, pl.nclusters, pl.T, pl.G,
                pl.rps,
                pl.R, pl.S, pl.stage_bytes, pl.vslice, pl.vs, pl.cols, pl.K, pl.lag, pl.xpair ? " pairs" : "", pl.pf,
                static_cast<long long>(pl.ntiles));
  return buf;
}

#ifdef RMSB_DEBUG_BOUNDS
// Bounds-checked build: the byte ranges the kernels of one API call may access, written to
// the device (dbg_ranges_kernel) on the call's stream before its first launch. The
// internal record arrays of the split-row exchange are always included.
struct DbgList {
  DbgRanges r{};
  void add(const void* p, size_t bytes) {
    if (!p || bytes == 0 || r.n >= kDbgMaxRanges) return;
    r.lo[r.n] = reinterpret_cast<uintptr_t>(p);
    r.hi[r.n] = r.lo[r.n] + bytes;
    ++r.n;
  }
};

int dbg_register(DbgList& l, cudaStream_t stream) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_xrec) == cudaSuccess) l.add(p, sizeof(g_xrec));
  if (cudaGetSymbolAddress(&p, g_xgen) == cudaSuccess) l.add(p, sizeof(g_xgen));
  cudaGetLastError();
  dbg_ranges_kernel<<<1, 32, 0, stream>>>(l.r);
  return cudaGetLastError() == cudaSuccess ? RMSNORM_B200_OK : RMSNORM_B200_ERR_CUDA;
}

// Self test of the checker: RMSNORM_B200_DEBUG_CLIP_OUT=k registers the output tensor of a
// forward k bytes short, so the kernel's (in-bounds) stores to its last k bytes are
// reported and skipped.
size_t dbg_clip(size_t bytes) {
  const int c = env_int("RMSNORM_B200_DEBUG_CLIP_OUT", 0);
  return c > 0 && static_cast<size_t>(c) < bytes ? bytes - static_cast<size_t>(c) : bytes;
}
#endif

// Sizes the grid (persistent: as many clusters or groups as can be resident, at most one
// per tile), picks the row-total exchange for split rows and, unless dry_run, launches.
// Clusters of 4, 8 or 16 CTAs fit fewer times on the GPU than the SM count allows (on
// B200: 33 x 4, 15 x 8, 7 x 16 of 148 SMs); where groups of P CTAs of a cooperative grid
// keep more SMs busy, those exchange through global memory instead. Returns UNSUPPORTED
// when no cluster of this shape fits.
template <typename Params>
int launch_stream(DeviceState* ds, void (*kernel)(const Params), Params params, StreamPlan& pl,
                  cudaStream_t stream, const char* kind, bool dry_run, int* grid_out) {
  const int smem = smem_bytes(pl);
  if (ensure_attrs(ds, reinterpret_cast<const void*>(kernel)) != RMSNORM_B200_OK) return RMSNORM_B200_ERR_CUDA;
  const void* kfn = reinterpret_cast<const void*>(kernel);
  const int64_t ntiles = std::max<int64_t>(pl.ntiles, 1);
  int units = resident_units(ds, kfn, pl.P, smem, pl.T);
  pl.xmode = kXCluster;
  if (pl.P > 1) {
    const int ctas = std::min(resident_units(ds, kfn, 1, smem, pl.T), kXRecMaxCtas);
    const int groups = ctas / pl.P;
    const int force = env_int("RMSNORM_B200_XMODE", -1);  // 0 cluster, 1 global
    const bool global = force == kXGlobal ||
                        (force < 0 && std::min<int64_t>(ntiles, groups) > std::min<int64_t>(ntiles, units));
    if (global && groups > 0) {
      pl.xmode = kXGlobal;
      units = groups;
    }
  }
  // Global records: warp 0 polls for the CTA and the other warps wait on shared memory (the
  // CTA-wide row sum keeps the warps in step: row groups of more than one warp). Measured on
  // B200, 32 KB row slices: bf16 cfg 5 forward +5.3 %, backward +8.7 %, cfg 3 +3.0 %; 64 KB
  // fp32 slices: backward level, forward -1.6 %, so those keep every warp polling.
  pl.xbcast = pl.P > 1 && pl.xmode == kXGlobal && pl.G > 32 &&
              static_cast<int64_t>(pl.row_bytes[0]) * pl.K <= 32768 && env_int("RMSNORM_B200_XBCAST", 1);
  if constexpr (std::is_same_v<Params, FwdParams>) {
    if (params.res || params.ro) pl.xbcast = 0;  // compiled into the residual-free forwards only
  }
  if (units <= 0) return RMSNORM_B200_ERR_UNSUPPORTED;
  const int64_t nclusters = std::min<int64_t>(ntiles, units);
  pl.nclusters = static_cast<int>(nclusters);
  const int grid = static_cast<int>(nclusters * pl.P);
  if (grid_out) *grid_out = grid;
  if (dry_run) return RMSNORM_B200_OK;
  params.xrec = nullptr;
  params.xgen = nullptr;
  if (pl.xmode == kXGlobal) {
    const int st = next_xset(ds, pl.P, &params.xrec, &params.xgen);
    if (st != RMSNORM_B200_OK) return st;
  }
  params.pl = pl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(pl.T);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pl.P == 1 && env_int("RMSNORM_B200_PDL", 1)) {
    // programmatic dependent launch: the grid may be scheduled while the previous kernel
    // in the stream retires; the kernel waits for it before its first global access
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  } else if (pl.P > 1 && pl.xmode == kXCluster) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = pl.P;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.numAttrs = 1;
  } else if (pl.P > 1) {
    // the P CTAs of a group wait for one another: all CTAs must be resident at once
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = attr;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, params);
  if (err != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  t_last_plan = describe(kind, pl, grid);
  if (pl.xbcast) t_last_plan += " bcast";
  return RMSNORM_B200_OK;
}

// ---------------------------------------------------------------------------------------
// Kernel tables: the specialised dtype combinations (absent tensor = -1 / NoT)
// ---------------------------------------------------------------------------------------
using FwdKernel = void (*)(const FwdParams);
using BwdKernel = void (*)(const BwdParams);
using h16 = __half;
using b16 = __nv_bfloat16;
constexpr int H = RMSNORM_B200_F16, B = RMSNORM_B200_BF16, F = RMSNORM_B200_F32, NA = -1;

// (x, residual, out, residual_out)
FwdKernel pick_fwd(int x, int r, int o, int ro, bool bias) {
#define RMSB_FWD(XT, XC, RT, RC, OT, OC, ROT, ROC)                              \
  if (x == XC && r == RC && o == OC && ro == ROC)                               \
    return bias ? fwd_stream_kernel<XT, RT, OT, ROT, true, false, kMaxVecs, kBlockLarge, 1>  \
                : fwd_stream_kernel<XT, RT, OT, ROT, false, false, kMaxVecs, kBlockLarge, 1>;
  RMSB_FWD(b16, B, NoT, NA, b16, B, NoT, NA)
  RMSB_FWD(h16, H, NoT, NA, h16, H, NoT, NA)
  RMSB_FWD(float, F, NoT, NA, float, F, NoT, NA)
  RMSB_FWD(b16, B, b16, B, b16, B, b16, B)
  RMSB_FWD(h16, H, h16, H, h16, H, h16, H)
  RMSB_FWD(float, F, float, F, float, F, float, F)
  RMSB_FWD(b16, B, b16, B, b16, B, float, F)
  RMSB_FWD(h16, H, h16, H, h16, H, float, F)
  RMSB_FWD(b16, B, float, F, b16, B, float, F)
  RMSB_FWD(h16, H, float, F, h16, H, float, F)
  // out_dtype = float32 from half/bf16 inputs
  RMSB_FWD(b16, B, NoT, NA, float, F, NoT, NA)
  RMSB_FWD(h16, H, NoT, NA, float, F, NoT, NA)
#undef RMSB_FWD
  return nullptr;
}

// Per-head column mode (x and out of one dtype, no residual): `cols` columns and
// kMaxVecs / cols super-rows per thread per sweep.
FwdKernel pick_fwd_cols(int x, int o, bool bias, int cols) {
  if (x != o) return nullptr;
#define RMSB_FWD_COLS(XT, XC, C)                                                                  \
  if (x == XC && cols == C)                                                                       \
    return bias ? fwd_stream_kernel<XT, NoT, XT, NoT, true, false, kMaxVecs, kBlockLarge, 1, C>    \
                : fwd_stream_kernel<XT, NoT, XT, NoT, false, false, kMaxVecs, kBlockLarge, 1, C>;
  RMSB_FWD_COLS(b16, B, 1)
  RMSB_FWD_COLS(h16, H, 1)
  RMSB_FWD_COLS(float, F, 1)
  RMSB_FWD_COLS(b16, B, 2)
  RMSB_FWD_COLS(h16, H, 2)
  RMSB_FWD_COLS(float, F, 2)
#undef RMSB_FWD_COLS
  return nullptr;
}

// LayerNorm: x and out of one dtype, no residual.
FwdKernel pick_ln(int x, int o, bool bias) {
  if (x != o) return nullptr;
#define RMSB_LN(XT, XC)                                                                              \
  if (x == XC)                                                                                       \
    return bias ? fwd_stream_kernel<XT, NoT, XT, NoT, true, true, kMaxVecs, kBlockLarge, 1>          \
                : fwd_stream_kernel<XT, NoT, XT, NoT, false, true, kMaxVecs, kBlockLarge, 1>;
  RMSB_LN(b16, B)
  RMSB_LN(h16, H)
  RMSB_LN(float, F)
#undef RMSB_LN
  return nullptr;
}

// Vectors per thread: the dbias variants keep a third register array, so they own two
// vectors per super-row slice instead of four to stay within 128 registers.
constexpr int kBwdVecsDb = 2;
int bwd_max_vecs(bool has_db) { return has_db ? kBwdVecsDb : kMaxVecs; }

// (x, dout, dx, dresidual_out, dresidual), dbias, launch shape
// Per-head backward (x, dy and dx of one dtype, no residual gradients): kernels that stage
// each tile's rstd block with one bulk copy.
BwdKernel pick_bwd_per_head(int x, int dy, int dx, bool db, bool small) {
  if (x != dy || x != dx) return nullptr;
#define RMSB_BWD_PH(XT, XC, BLK, MINB)                                                                  \
  if (x == XC)                                                                                        \
    return db ? bwd_stream_kernel<XT, XT, XT, NoT, NoT, true, kBwdVecsDb, BLK, MINB, true>            \
              : bwd_stream_kernel<XT, XT, XT, NoT, NoT, false, kMaxVecs, BLK, MINB, true>;
  if (small) {
    RMSB_BWD_PH(b16, B, kBlockSmall, 2)
    RMSB_BWD_PH(h16, H, kBlockSmall, 2)
    RMSB_BWD_PH(float, F, kBlockSmall, 2)
    return nullptr;
  }
  RMSB_BWD_PH(b16, B, kBlockLarge, 1)
  RMSB_BWD_PH(h16, H, kBlockLarge, 1)
  RMSB_BWD_PH(float, F, kBlockLarge, 1)
#undef RMSB_BWD_PH
  return nullptr;
}

// Per-head column mode (x, dy and dx of one dtype, no residual gradients; bulk rstd
// staging): `cols` columns and kMaxVecs / cols super-rows per thread per sweep. With one
// or two columns the dbias variants keep four vectors per thread.
BwdKernel pick_bwd_cols(int x, int dy, int dx, bool db, int cols) {
  if (x != dy || x != dx) return nullptr;
#define RMSB_BWD_COLS(XT, XC, C)                                                                       \
  if (x == XC && cols == C)                                                                            \
    return db ? bwd_stream_kernel<XT, XT, XT, NoT, NoT, true, kMaxVecs, kBlockLarge, 1, true, C>        \
              : bwd_stream_kernel<XT, XT, XT, NoT, NoT, false, kMaxVecs, kBlockLarge, 1, true, C>;
  RMSB_BWD_COLS(b16, B, 1)
  RMSB_BWD_COLS(h16, H, 1)
  RMSB_BWD_COLS(float, F, 1)
  RMSB_BWD_COLS(b16, B, 2)
  RMSB_BWD_COLS(h16, H, 2)
  RMSB_BWD_COLS(float, F, 2)
#undef RMSB_BWD_COLS
  return nullptr;
}

BwdKernel pick_bwd(int x, int dy, int dx, int dro, int dres, bool db, bool small) {
#define RMSB_BWD_SHAPE(XT, XC, DT, DC, DXT, DXC, AT, AC, ST, SC, BLK, MINB)                       \
  if (x == XC && dy == DC && dx == DXC && dro == AC && dres == SC)                                 \
    return db ? bwd_stream_kernel<XT, DT, DXT, AT, ST, true, kBwdVecsDb, BLK, MINB>                \
              : bwd_stream_kernel<XT, DT, DXT, AT, ST, false, kMaxVecs, BLK, MINB>;
  if (small) {
#define RMSB_BWD(...) RMSB_BWD_SHAPE(__VA_ARGS__, kBlockSmall, 2)
    RMSB_BWD(b16, B, b16, B, b16, B, NoT, NA, NoT, NA)
    RMSB_BWD(h16, H, h16, H, h16, H, NoT, NA, NoT, NA)
    RMSB_BWD(float, F, float, F, float, F, NoT, NA, NoT, NA)
    RMSB_BWD(float, F, b16, B, b16, B, NoT, NA, NoT, NA)
    RMSB_BWD(float, F, h16, H, h16, H, NoT, NA, NoT, NA)
#undef RMSB_BWD
    return nullptr;
  }
#define RMSB_BWD(...) RMSB_BWD_SHAPE(__VA_ARGS__, kBlockLarge, 1)
  RMSB_BWD(b16, B, b16, B, b16, B, NoT, NA, NoT, NA)
  RMSB_BWD(h16, H, h16, H, h16, H, NoT, NA, NoT, NA)
  RMSB_BWD(float, F, float, F, float, F, NoT, NA, NoT, NA)
  RMSB_BWD(b16, B, b16, B, b16, B, b16, B, b16, B)
  RMSB_BWD(h16, H, h16, H, h16, H, h16, H, h16, H)
  RMSB_BWD(float, F, float, F, float, F, float, F, float, F)
  RMSB_BWD(float, F, b16, B, b16, B, NoT, NA, NoT, NA)
  RMSB_BWD(float, F, h16, H, h16, H, NoT, NA, NoT, NA)
  RMSB_BWD(float, F, b16, B, b16, B, float, F, b16, B)
  RMSB_BWD(float, F, h16, H, h16, H, float, F, h16, H)
  RMSB_BWD(float, F, b16, B, b16, B, NoT, NA, float, F)
  RMSB_BWD(float, F, h16, H, h16, H, NoT, NA, float, F)
  RMSB_BWD(float, F, b16, B, b16, B, float, F, float, F)
  RMSB_BWD(float, F, h16, H, h16, H, float, F, float, F)
  // the public rmsnorm_bwd on a saved fp32 residual_out returns dx in the saved dtype
  RMSB_BWD(float, F, b16, B, float, F, NoT, NA, NoT, NA)
  RMSB_BWD(float, F, h16, H, float, F, NoT, NA, NoT, NA)
#undef RMSB_BWD
#undef RMSB_BWD_SHAPE
  return nullptr;
}

// dbias backwards with the dweight / dbias sums in tensor memory (4 vectors per thread,
// rows not split, 512-thread CTAs): the same dtype combinations as pick_bwd's large shape.
BwdKernel pick_bwd_tmem(int x, int dy, int dx, int dro, int dres) {
#define RMSB_BWD_TM(XT, XC, DT, DC, DXT, DXC, AT, AC, ST, SC)                                         \
  if (x == XC && dy == DC && dx == DXC && dro == AC && dres == SC)                                   \
    return bwd_stream_kernel<XT, DT, DXT, AT, ST, true, kMaxVecs, kBlockLarge, 1, false, kMaxVecs, true>;
  RMSB_BWD_TM(b16, B, b16, B, b16, B, NoT, NA, NoT, NA)
  RMSB_BWD_TM(h16, H, h16, H, h16, H, NoT, NA, NoT, NA)
  RMSB_BWD_TM(float, F, float, F, float, F, NoT, NA, NoT, NA)
  RMSB_BWD_TM(b16, B, b16, B, b16, B, b16, B, b16, B)
  RMSB_BWD_TM(h16, H, h16, H, h16, H, h16, H, h16, H)
  RMSB_BWD_TM(float, F, float, F, float, F, float, F, float, F)
  RMSB_BWD_TM(float, F, b16, B, b16, B, NoT, NA, NoT, NA)
  RMSB_BWD_TM(float, F, h16, H, h16, H, NoT, NA, NoT, NA)
  RMSB_BWD_TM(float, F, b16, B, b16, B, float, F, b16, B)
  RMSB_BWD_TM(float, F, h16, H, h16, H, float, F, h16, H)
  RMSB_BWD_TM(float, F, b16, B, b16, B, NoT, NA, float, F)
  RMSB_BWD_TM(float, F, h16, H, h16, H, NoT, NA, float, F)
  RMSB_BWD_TM(float, F, b16, B, b16, B, float, F, float, F)
  RMSB_BWD_TM(float, F, h16, H, h16, H, float, F, float, F)
  RMSB_BWD_TM(float, F, b16, B, float, F, NoT, NA, NoT, NA)
  RMSB_BWD_TM(float, F, h16, H, float, F, NoT, NA, NoT, NA)
#undef RMSB_BWD_TM
  return nullptr;
}

// ---------------------------------------------------------------------------------------
// Argument validation
// ---------------------------------------------------------------------------------------
int check_common(int64_t rows, int64_t hidden, int heads) {
  if (rows < 0 || hidden < 1 || heads < 1) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (rows % heads != 0) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  return RMSNORM_B200_OK;
}

int check_fwd(const rmsnorm_b200_fwd_args* a) {
  if (!a) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  int st = check_common(a->rows, a->hidden, a->heads);
  if (st) return st;
  if (!valid_dt(a->x_dtype) || !valid_dt(a->out_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->rows > 0 && (!a->x || !a->out)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->residual && !valid_dt(a->residual_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->residual_out && !valid_dt(a->residual_out_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->weight && (!valid_dt(a->weight_dtype) || (a->weight_heads != 1 && a->weight_heads != a->heads)))
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->bias && (!valid_dt(a->bias_dtype) || (a->bias_heads != 1 && a->bias_heads != a->heads)))
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->heads > 1) {
    const bool wh = a->weight && a->weight_heads == a->heads;
    const bool bh = a->bias && a->bias_heads == a->heads;
    if (!wh && !bh) return RMSNORM_B200_ERR_INVALID_ARGUMENT;  // heads only come from an affine tensor
  }
  return RMSNORM_B200_OK;
}

int check_bwd(const rmsnorm_b200_bwd_args* a) {
  if (!a) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  int st = check_common(a->rows, a->hidden, a->heads);
  if (st) return st;
  if (a->rows > 0 && (!a->x || !a->dout || !a->rstd || !a->dx)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (!valid_dt(a->x_dtype) || !valid_dt(a->dout_dtype) || !valid_dt(a->dx_dtype))
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->weight && (!valid_dt(a->weight_dtype) || (a->weight_heads != 1 && a->weight_heads != a->heads)))
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->dweight && (!a->weight || !valid_dt(a->dweight_dtype))) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->dbias && (!valid_dt(a->dbias_dtype) || (a->dbias_heads != 1 && a->dbias_heads != a->heads)))
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->dresidual_out && !valid_dt(a->dresidual_out_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->dresidual && !valid_dt(a->dresidual_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  return RMSNORM_B200_OK;
}

// ---------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------
int launch_fwd_generic(DeviceState* ds, const rmsnorm_b200_fwd_args* a, cudaStream_t stream,
                       const std::string& why) {
  GenFwdParams g = {};
  g.rows = a->rows; g.N = a->hidden; g.H = a->heads;
  g.x = a->x; g.x_dt = a->x_dtype;
  g.res = a->residual; g.res_dt = a->residual_dtype;
  g.w = a->weight; g.w_dt = a->weight_dtype; g.w_ph = a->weight && a->weight_heads > 1;
  g.b = a->bias; g.b_dt = a->bias_dtype; g.b_ph = a->bias && a->bias_heads > 1;
  g.out = a->out; g.out_dt = a->out_dtype;
  g.ro = a->residual_out; g.ro_dt = a->residual_out_dtype;
  g.rstd = a->rstd; g.eps = a->eps;
  const int64_t grid = std::min<int64_t>(a->rows, static_cast<int64_t>(ds->sm_count) * 8);
  fwd_generic_kernel<<<static_cast<unsigned>(grid), kGenericThreads, 0, stream>>>(g);
  if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  t_last_plan = "fwd_generic (" + why + ") grid=" + std::to_string(grid);
  return RMSNORM_B200_OK;
}

int do_fwd(const rmsnorm_b200_fwd_args* a, cudaStream_t stream) {
  int st = check_fwd(a);
  if (st) return st;
  if (a->rows == 0) { t_last_plan = "fwd empty"; return RMSNORM_B200_OK; }
  DeviceState* ds = nullptr;
  st = get_device_state(&ds);
  if (st) return st;
#ifdef RMSB_DEBUG_BOUNDS
  {
    DbgList l;
    const size_t n = static_cast<size_t>(a->rows) * static_cast<size_t>(a->hidden);
    const size_t hd = static_cast<size_t>(a->hidden);
    l.add(a->x, n * elem_bytes(a->x_dtype));
    if (a->residual) l.add(a->residual, n * elem_bytes(a->residual_dtype));
    if (a->weight) l.add(a->weight, std::max(a->weight_heads, 1) * hd * elem_bytes(a->weight_dtype));
    if (a->bias) l.add(a->bias, std::max(a->bias_heads, 1) * hd * elem_bytes(a->bias_dtype));
    l.add(a->out, dbg_clip(n * elem_bytes(a->out_dtype)));
    if (a->residual_out) l.add(a->residual_out, n * elem_bytes(a->residual_out_dtype));
    if (a->rstd) l.add(a->rstd, static_cast<size_t>(a->rows) * 4);
    st = dbg_register(l, stream);
    if (st) return st;
  }
#endif
  std::string why;
  FwdKernel kernel = nullptr;
  if (env_int("RMSNORM_B200_FORCE_GENERIC", 0)) {
    why = "forced";
  } else if (a->hidden % 8) {
    why = "hidden % 8";
  } else {
    const void* ptrs[] = {a->x, a->residual, a->weight, a->bias, a->out, a->residual_out};
    for (const void* p : ptrs)
      if (p && !aligned16(p)) why = "unaligned pointer";
    if (why.empty()) {
      kernel = pick_fwd(a->x_dtype, a->residual ? a->residual_dtype : NA, a->out_dtype,
                        a->residual_out ? a->residual_out_dtype : NA, a->bias != nullptr);
      if (!kernel) why = "dtype combination";
    }
  }
  if (kernel) {
    StreamPlan pl;
    const int in_bytes[3] = {elem_bytes(a->x_dtype), a->residual ? elem_bytes(a->residual_dtype) : 0, 0};
    bool planned = false;
    // Per-head rows without a residual: column mode, where its kernel exists. Measured on
    // B200 at (16384, 32, 128) fp16 with per-head weight and bias: the four-column kernel
    // holds 64 registers of weight / bias and issues about a third more instructions.
    if (a->heads > 1 && !a->residual && !a->residual_out && env_int("RMSNORM_B200_COL_MODE", 1) &&
        make_stream_plan(a->rows, a->hidden, a->heads, in_bytes, false, kMaxVecs, kLarge, 0, &pl, &why, false,
                         true) &&
        pl.cols < kMaxVecs && pl.S >= 2) {
      if (FwdKernel kc = pick_fwd_cols(a->x_dtype, a->out_dtype, a->bias != nullptr, pl.cols)) {
        kernel = kc;
        planned = true;
      }
    }
    if (!planned)
      planned = make_stream_plan(a->rows, a->hidden, a->heads, in_bytes, false, kMaxVecs, kLarge,
                                 env_int("RMSNORM_B200_FORCE_CLUSTER", 0), &pl, &why);
    if (planned) {
      // Split rows whose ring holds two pairs of row slices and two more loading go in pairs
      // (residual-free forwards). Measured on B200 (bf16, CUDA-graph replays, two repeats,
      // bitwise equal to the row loop): P = 16 +21 % (cfg 5: 4550 -> 5510 GB/s), P = 8 +21 %,
      // P = 4 +21 %, P = 2 +14 %. Before warp 0 alone polled the global records, pairs lost at
      // P = 8 and 16 (every warp polled twice as many records per exchange).
      if (pl.P > 1 && pl.K == 1 && pl.P <= 16 && pl.S >= 6 && !a->residual && !a->residual_out &&
          env_int("RMSNORM_B200_XPAIR", 1) && env_int("RMSNORM_B200_FORCE_LAG", -1) < 0) {
        pl.xpair = 1;
        pl.lag = 1;
      }
      FwdParams p = {};
      p.x = a->x; p.res = a->residual; p.w = a->weight; p.b = a->bias;
      p.out = a->out; p.ro = a->residual_out; p.rstd = a->rstd;
      p.w_dt = a->weight_dtype; p.b_dt = a->bias_dtype;
      p.w_per_head = a->weight && a->weight_heads > 1;
      p.b_per_head = a->bias && a->bias_heads > 1;
      p.eps = a->eps;
      st = launch_stream(ds, kernel, p, pl, stream, "fwd_stream", false, nullptr);
      if (st != RMSNORM_B200_ERR_UNSUPPORTED) return st;
      why = "cluster not schedulable";
    }
  }
  return launch_fwd_generic(ds, a, stream, why);
}

// ---------------------------------------------------------------------------------------
// LayerNorm forward
// ---------------------------------------------------------------------------------------
int check_ln(const rmsnorm_b200_ln_fwd_args* a) {
  if (!a) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  int st = check_common(a->rows, a->hidden, 1);
  if (st) return st;
  if (!valid_dt(a->x_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->rows > 0 && !a->x) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->out && !valid_dt(a->out_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->weight && !valid_dt(a->weight_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  if (a->bias && !valid_dt(a->bias_dtype)) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  return RMSNORM_B200_OK;
}

int do_ln(const rmsnorm_b200_ln_fwd_args* a, cudaStream_t stream) {
  int st = check_ln(a);
  if (st) return st;
  if (a->rows == 0) { t_last_plan = "ln empty"; return RMSNORM_B200_OK; }
  DeviceState* ds = nullptr;
  st = get_device_state(&ds);
  if (st) return st;
#ifdef RMSB_DEBUG_BOUNDS
  {
    DbgList l;
    const size_t n = static_cast<size_t>(a->rows) * static_cast<size_t>(a->hidden);
    l.add(a->x, n * elem_bytes(a->x_dtype));
    if (a->weight) l.add(a->weight, static_cast<size_t>(a->hidden) * elem_bytes(a->weight_dtype));
    if (a->bias) l.add(a->bias, static_cast<size_t>(a->hidden) * elem_bytes(a->bias_dtype));
    if (a->out) l.add(a->out, dbg_clip(n * elem_bytes(a->out_dtype)));
    if (a->mean) l.add(a->mean, static_cast<size_t>(a->rows) * 4);
    if (a->rstd) l.add(a->rstd, static_cast<size_t>(a->rows) * 4);
    st = dbg_register(l, stream);
    if (st) return st;
  }
#endif
  std::string why;
  FwdKernel kernel = nullptr;
  if (env_int("RMSNORM_B200_FORCE_GENERIC", 0)) {
    why = "forced";
  } else if (a->hidden % 8) {
    why = "hidden % 8";
  } else if (!a->out) {
    why = "statistics only";
  } else {
    const void* ptrs[] = {a->x, a->weight, a->bias, a->out};
    for (const void* p : ptrs)
      if (p && !aligned16(p)) why = "unaligned pointer";
    if (why.empty()) {
      kernel = pick_ln(a->x_dtype, a->out_dtype, a->bias != nullptr);
      if (!kernel) why = "dtype combination";
    }
  }
  if (kernel) {
    StreamPlan pl;
    const int in_bytes[3] = {elem_bytes(a->x_dtype), 0, 0};
    // rows are never split across CTAs: a row that does not fit one CTA takes the generic path
    // one row per row group per tile: the LayerNorm row loop pipelines rows tile by tile
    if (make_stream_plan(a->rows, a->hidden, 1, in_bytes, false, kMaxVecs, kLarge, 1, &pl, &why, true)) {
      FwdParams p = {};
      p.x = a->x; p.w = a->weight; p.b = a->bias; p.out = a->out;
      p.rstd = a->rstd; p.mean = a->mean;
      p.w_dt = a->weight_dtype; p.b_dt = a->bias_dtype;
      p.eps = a->eps;
      st = launch_stream(ds, kernel, p, pl, stream, "ln_stream", false, nullptr);
      if (st != RMSNORM_B200_ERR_UNSUPPORTED) return st;
      why = "not schedulable";
    }
  }
  GenLnParams g = {};
  g.rows = a->rows; g.N = a->hidden;
  g.x = a->x; g.x_dt = a->x_dtype;
  g.w = a->weight; g.w_dt = a->weight_dtype;
  g.b = a->bias; g.b_dt = a->bias_dtype;
  g.out = a->out; g.out_dt = a->out_dtype;
  g.mean = a->mean; g.rstd = a->rstd; g.eps = a->eps;
  const int64_t grid = std::min<int64_t>(a->rows, static_cast<int64_t>(ds->sm_count) * 8);
  ln_generic_kernel<<<static_cast<unsigned>(grid), kGenericThreads, 0, stream>>>(g);
  if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  t_last_plan = "ln_generic (" + why + ") grid=" + std::to_string(grid);
  return RMSNORM_B200_OK;
}

// ---------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------
struct BwdPlan {
  bool stream = false;
  StreamPlan pl = {};
  BwdKernel kernel = nullptr;
  int grid = 0;
  int64_t nparts = 0;        // partial rows per requested gradient
  int64_t chunk_rows = 0;    // generic: super-rows per chunk
  int64_t W = 0;
  bool need_dw = false, need_db = false;
  bool tmem = false;         // the dweight / dbias sums of the streaming kernel live in TMEM
  std::string why;
};

// Tries one (block shape, kernel) candidate; on success fills bp and returns true.
// col_mode: per-head column mode, the kernel picked by the plan's column count.
// max_vecs: vectors per thread of the kernel (0 = the default of its dbias variant).
bool try_bwd_stream(DeviceState* ds, const rmsnorm_b200_bwd_args* a, BwdKernel kernel, const BlockCfg& bc,
                    int force_p, BwdPlan* bp, std::string* why, bool col_mode = false, int max_vecs = 0) {
  if (!kernel && !col_mode) return false;
  const int in_bytes[3] = {elem_bytes(a->x_dtype), elem_bytes(a->dout_dtype),
                           a->dresidual_out ? elem_bytes(a->dresidual_out_dtype) : 0};
  StreamPlan pl;
  if (max_vecs == 0) max_vecs = col_mode ? kMaxVecs : bwd_max_vecs(bp->need_db);
  if (!make_stream_plan(a->rows, a->hidden, a->heads, in_bytes, true, max_vecs, bc, force_p, &pl, why, false,
                        col_mode))
    return false;
  if (col_mode) {
    // column mode needs whole sweeps of kMaxVecs / cols rows per tile; where only one such
    // tile fits (fp32 at 4096-wide rows) the plan without it streams better (-7.5 %)
    if (pl.cols >= kMaxVecs || pl.S < 2) return false;
    kernel = pick_bwd_cols(a->x_dtype, a->dout_dtype, a->dx_dtype, bp->need_db, pl.cols);
    if (!kernel) return false;
  }
  int grid = 0;
  BwdParams dummy = {};
  if (launch_stream(ds, kernel, dummy, pl, nullptr, "bwd_stream", true, &grid) != RMSNORM_B200_OK) {
    *why = "cluster not schedulable";
    return false;
  }
  bp->stream = true;
  bp->kernel = kernel;
  bp->pl = pl;
  bp->grid = grid;
  bp->nparts = static_cast<int64_t>(pl.nclusters) * pl.rps;
  return true;
}

// allow_tmem false: plan without the TMEM-accumulator kernels (their plans can keep more
// partial rows: one per row group of each of the SM-count CTAs).
int plan_bwd(DeviceState* ds, const rmsnorm_b200_bwd_args* a, BwdPlan* bp, bool allow_tmem = true) {
  bp->W = a->hidden * a->heads;
  bp->need_dw = a->dweight != nullptr;
  bp->need_db = a->dbias != nullptr;
  std::string why;
  bool ok = env_int("RMSNORM_B200_FORCE_GENERIC", 0) == 0;
  if (!ok) why = "forced";
  if (ok && a->hidden % 8) { ok = false; why = "hidden % 8"; }
  if (ok) {
    const void* ptrs[] = {a->x, a->dout, a->weight, a->dresidual_out, a->dx, a->dresidual};
    for (const void* p : ptrs)
      if (p && !aligned16(p)) { ok = false; why = "unaligned pointer"; }
  }
  if (ok) {
    const int dro = a->dresidual_out ? a->dresidual_out_dtype : NA;
    const int dres = a->dresidual ? a->dresidual_dtype : NA;
    BwdKernel large = pick_bwd(a->x_dtype, a->dout_dtype, a->dx_dtype, dro, dres, bp->need_db, false);
    BwdKernel small = pick_bwd(a->x_dtype, a->dout_dtype, a->dx_dtype, dro, dres, bp->need_db, true);
    if (a->heads > 1 && dro == NA && dres == NA) {  // per-head rows: bulk rstd staging
      BwdKernel ph_large = pick_bwd_per_head(a->x_dtype, a->dout_dtype, a->dx_dtype, bp->need_db, false);
      BwdKernel ph_small = pick_bwd_per_head(a->x_dtype, a->dout_dtype, a->dx_dtype, bp->need_db, true);
      if (ph_large) large = ph_large;
      if (ph_small) small = ph_small;
    }
    const int force_p = env_int("RMSNORM_B200_FORCE_CLUSTER", 0);
    const int shape = env_int("RMSNORM_B200_BWD_SHAPE", 0);  // 0 auto, 1 large only, 2 small only
    if (a->heads > 1 && dro == NA && dres == NA && shape == 0 && env_int("RMSNORM_B200_COL_MODE", 1)) {
      BwdPlan cand = *bp;
      std::string why_c;
      if (try_bwd_stream(ds, a, nullptr, kLarge, 0, &cand, &why_c, true)) { *bp = cand; return RMSNORM_B200_OK; }
    }
    // dbias backwards: the 4-vector kernel with its sums in TMEM when a row fits one CTA in
    // row mode (up to 16384 columns with 512 threads); the 2-vector register kernel otherwise
    if (bp->need_db && shape != 2 && allow_tmem && env_int("RMSNORM_B200_TMEM_ACC", 1)) {
      if (BwdKernel tk = pick_bwd_tmem(a->x_dtype, a->dout_dtype, a->dx_dtype, dro, dres)) {
        BwdPlan cand = *bp;
        std::string why_t;
        if (try_bwd_stream(ds, a, tk, kLarge, force_p, &cand, &why_t, false, kMaxVecs) && cand.pl.P == 1 &&
            !cand.pl.seg_mode) {
          cand.tmem = true;
          *bp = cand;
          return RMSNORM_B200_OK;
        }
      }
    }
    if (!large && !small) why = "dtype combination";
    // A row split across a cluster waits once per row for its peers. With two CTAs of
    // 256 threads per SM, two such row pipelines overlap on every SM; prefer that shape
    // when the cluster split it needs keeps at least as many SMs busy.
    BwdPlan cand_large = *bp, cand_small = *bp;
    std::string why_l, why_s;
    const bool have_large = shape != 2 && try_bwd_stream(ds, a, large, kLarge, force_p, &cand_large, &why_l);
    bool have_small = false;
    if (shape != 1 && small && (!have_large || cand_large.pl.P > 1 || shape == 2))
      have_small = try_bwd_stream(ds, a, small, kSmall, force_p, &cand_small, &why_s);
    if (have_small && have_large) {
      const int64_t sms_large = static_cast<int64_t>(cand_large.grid);
      const int64_t sms_small = static_cast<int64_t>(cand_small.grid) / kSmall.ctas_per_sm;
      if (sms_small <= sms_large) have_small = false;
    }
    if (have_small) { *bp = cand_small; return RMSNORM_B200_OK; }
    if (have_large) { *bp = cand_large; return RMSNORM_B200_OK; }
    if (why.empty()) why = why_l.empty() ? why_s : why_l;
  }
  bp->stream = false;
  bp->why = why;
  const int64_t nsup = a->rows / a->heads;
  const int64_t col_blocks = (bp->W + kGenericThreads - 1) / kGenericThreads;
  int64_t target = std::max<int64_t>(1, (4 * ds->sm_count + col_blocks - 1) / col_blocks);
  target = std::min<int64_t>(target, 1024);
  bp->chunk_rows = std::max<int64_t>(1, (nsup + target - 1) / target);
  bp->nparts = nsup > 0 ? (nsup + bp->chunk_rows - 1) / bp->chunk_rows : 0;
  return RMSNORM_B200_OK;
}

size_t workspace_for(const BwdPlan& bp) {
  const size_t per = static_cast<size_t>(bp.nparts) * static_cast<size_t>(bp.W) * sizeof(float);
  return (bp.need_dw ? per : 0) + (bp.need_db ? per : 0);
}

// Gradient values (dweight + dbias elements) a backward with these arguments produces.
int64_t grad_floats(const rmsnorm_b200_bwd_args* a) {
  const int64_t W = a->hidden * a->heads;
  int64_t n = 0;
  if (a->dweight) n += (a->weight_heads == 1 && a->heads > 1) ? a->hidden : W;
  if (a->dbias) n += (a->dbias_heads == 1 && a->heads > 1) ? a->hidden : W;
  return n;
}

// group: when not null, the dweight / dbias sums are all-reduced over the group's ranks by
// the fused reduction kernel instead of reduce_partials_kernel.
int do_bwd(const rmsnorm_b200_bwd_args* a, void* ws, size_t ws_bytes, cudaStream_t stream,
           rmsnorm_b200_peer_group* group = nullptr, bool allow_tmem = true) {
  int st = check_bwd(a);
  if (st) return st;
  if (group != nullptr) {  // checked before anything is launched: the ranks stay in step
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != group->device || !group->connected)
      return RMSNORM_B200_ERR_INVALID_ARGUMENT;
    if (grad_floats(a) > group->max_floats) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  }
  DeviceState* ds = nullptr;
  st = get_device_state(&ds);
  if (st) return st;
  BwdPlan bp;
  st = plan_bwd(ds, a, &bp, allow_tmem);
  if (st) return st;
  const size_t need = workspace_for(bp);
  if (need > ws_bytes || (need > 0 && (!ws || !aligned16(ws)))) return RMSNORM_B200_ERR_WORKSPACE;
#ifdef RMSB_DEBUG_BOUNDS
  {
    DbgList l;
    const size_t n = static_cast<size_t>(a->rows) * static_cast<size_t>(a->hidden);
    const size_t hd = static_cast<size_t>(a->hidden);
    l.add(a->x, n * elem_bytes(a->x_dtype));
    l.add(a->dout, n * elem_bytes(a->dout_dtype));
    l.add(a->rstd, static_cast<size_t>(a->rows) * 4);
    if (a->weight) l.add(a->weight, std::max(a->weight_heads, 1) * hd * elem_bytes(a->weight_dtype));
    if (a->dresidual_out) l.add(a->dresidual_out, n * elem_bytes(a->dresidual_out_dtype));
    l.add(a->dx, n * elem_bytes(a->dx_dtype));
    if (a->dresidual) l.add(a->dresidual, n * elem_bytes(a->dresidual_dtype));
    if (a->dweight) l.add(a->dweight, std::max(a->weight_heads, 1) * hd * elem_bytes(a->dweight_dtype));
    if (a->dbias) l.add(a->dbias, std::max(a->dbias_heads, 1) * hd * elem_bytes(a->dbias_dtype));
    l.add(ws, ws_bytes);
    if (group)
      for (int q = 0; q < group->world; ++q)
        l.add(group->recv[q], 2ull * static_cast<size_t>(group->world) * static_cast<size_t>(group->max_floats) * 8ull);
    st = dbg_register(l, stream);
    if (st) return st;
  }
#endif
  float* dw_part = bp.need_dw ? static_cast<float*>(ws) : nullptr;
  float* db_part = bp.need_db ? static_cast<float*>(ws) + (bp.need_dw ? bp.nparts * bp.W : 0) : nullptr;

  if (a->rows > 0) {
    if (bp.stream) {
      BwdParams p = {};
      p.x = a->x; p.dy = a->dout; p.dro = a->dresidual_out; p.rstd = a->rstd; p.w = a->weight;
      p.dx = a->dx; p.dres = a->dresidual; p.dw_part = dw_part; p.db_part = db_part;
      p.w_dt = a->weight_dtype;
      p.w_per_head = a->weight && a->weight_heads > 1;
      StreamPlan pl = bp.pl;
      st = launch_stream(ds, bp.kernel, p, pl, stream, "bwd_stream", false, nullptr);
      if (st) return st;
      if (bp.tmem) t_last_plan += " acc=tmem";
    } else {
      GenBwdParams g = {};
      g.rows = a->rows; g.N = a->hidden; g.H = a->heads;
      g.x = a->x; g.x_dt = a->x_dtype; g.dy = a->dout; g.dy_dt = a->dout_dtype;
      g.rstd = a->rstd; g.w = a->weight; g.w_dt = a->weight_dtype;
      g.w_ph = a->weight && a->weight_heads > 1;
      g.dro = a->dresidual_out; g.dro_dt = a->dresidual_out_dtype;
      g.dx = a->dx; g.dx_dt = a->dx_dtype; g.dres = a->dresidual; g.dres_dt = a->dresidual_dtype;
      const int64_t grid = std::min<int64_t>(a->rows, static_cast<int64_t>(ds->sm_count) * 8);
      bwd_generic_dx_kernel<<<static_cast<unsigned>(grid), kGenericThreads, 0, stream>>>(g);
      if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
      g_launches.fetch_add(1, std::memory_order_relaxed);
      if ((dw_part || db_part) && bp.nparts > 0) {
        dim3 pg(static_cast<unsigned>((bp.W + kGenericThreads - 1) / kGenericThreads),
                static_cast<unsigned>(bp.nparts));
        bwd_generic_partials_kernel<<<pg, kGenericThreads, 0, stream>>>(g, bp.chunk_rows, dw_part, db_part);
        if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
        g_launches.fetch_add(1, std::memory_order_relaxed);
      }
      t_last_plan = "bwd_generic (" + bp.why + ") grid=" + std::to_string(grid) +
                    " chunks=" + std::to_string(bp.nparts);
    }
  } else {
    t_last_plan = "bwd empty";
  }

  // dweight and dbias: fixed-order column sums of the partial rows, one launch for both
  ReduceParams rp = {};
  rp.C = a->rows > 0 ? bp.nparts : 0;
  rp.W = bp.W;
  rp.N = a->hidden;
  int njobs = 0;
  auto add_job = [&](const float* part, void* outp, int out_dt, int out_heads) {
    ReduceJob& jb = rp.job[njobs++];
    jb.fold = (out_heads == 1 && a->heads > 1) ? a->heads : 1;
    jb.wout = jb.fold > 1 ? a->hidden : bp.W;
    jb.part = part;
    jb.out = outp;
    jb.out_dt = out_dt;
  };
  if (a->dweight) add_job(dw_part, a->dweight, a->dweight_dtype, a->weight_heads);
  if (a->dbias) add_job(db_part, a->dbias, a->dbias_dtype, a->dbias_heads);
  if (njobs > 0 && group != nullptr) {
    PeerParams pp = {};
    for (int q = 0; q < group->world; ++q) pp.recv[q] = group->recv[q];
    pp.seq = static_cast<uint32_t*>(group->buffer);
    pp.rank = group->rank;
    pp.world = group->world;
    pp.stride = group->max_floats;
    reduce_allreduce_kernel<<<kARBlocks, kARThreads, 0, stream>>>(rp, pp);
    if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    t_last_plan += " allreduce=peer world=" + std::to_string(group->world);
  } else if (njobs > 0) {
    int64_t blocks = 0;  // column blocks of the widest job (per-job block width: see reduce_vectorised)
    for (int i = 0; i < njobs; ++i) {
      const int64_t cols = reduce_vectorised(rp.job[i], rp.W) ? kReduceVCols : kReduceCols;
      blocks = std::max(blocks, (rp.job[i].wout + cols - 1) / cols);
    }
    const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(njobs));
    reduce_partials_kernel<<<grid, kReduceThreads, 0, stream>>>(rp);
    if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  return RMSNORM_B200_OK;
}

}  // namespace
}  // namespace rmsb200

// =========================================================================================
// C ABI
// =========================================================================================
using namespace rmsb200;

extern "C" int rmsnorm_b200_fwd(const rmsnorm_b200_fwd_args* args, void* stream) {
  return do_fwd(args, static_cast<cudaStream_t>(stream));
}

extern "C" int rmsnorm_b200_layernorm_fwd(const rmsnorm_b200_ln_fwd_args* args, void* stream) {
  return do_ln(args, static_cast<cudaStream_t>(stream));
}

extern "C" int rmsnorm_b200_bwd_workspace_size(const rmsnorm_b200_bwd_args* args, size_t* bytes) {
  if (!bytes) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  int st = check_bwd(args);
  if (st) return st;
  DeviceState* ds = nullptr;
  st = get_device_state(&ds);
  if (st) return st;
  BwdPlan bp;
  st = plan_bwd(ds, args, &bp);
  if (st) return st;
  *bytes = workspace_for(bp);
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_bwd(const rmsnorm_b200_bwd_args* args, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return do_bwd(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int rmsnorm_b200_peer_buffer_size(int32_t world, int64_t max_grad_floats, size_t* bytes) {
  if (!bytes || world < 1 || world > RMSNORM_B200_MAX_PEERS || max_grad_floats < 1)
    return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  *bytes = static_cast<size_t>(kPeerBufferHeader) + 2ull * static_cast<size_t>(world) *
                                                        static_cast<size_t>(max_grad_floats) * 8ull;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_peer_group_create(int32_t rank, int32_t world, int64_t max_grad_floats,
                                              void* ipc_handle, rmsnorm_b200_peer_group** group) {
  if (!group || !ipc_handle || rank < 0 || rank >= world) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  *group = nullptr;
  size_t bytes = 0;
  int st = rmsnorm_b200_peer_buffer_size(world, max_grad_floats, &bytes);
  if (st) return st;
  auto g = std::make_unique<rmsnorm_b200_peer_group>();
  if (cudaGetDevice(&g->device) != cudaSuccess) return RMSNORM_B200_ERR_NO_DEVICE;
  g->rank = rank;
  g->world = world;
  g->max_floats = max_grad_floats;
  if (cudaMalloc(&g->buffer, bytes) != cudaSuccess) {
    cudaGetLastError();
    return RMSNORM_B200_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  // zeroed before any peer can reach it: the handle leaves this call only afterwards
  if (cudaMemset(g->buffer, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, g->buffer) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(g->buffer);
    return RMSNORM_B200_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  g->recv[rank] = reinterpret_cast<unsigned long long*>(static_cast<char*>(g->buffer) + kPeerBufferHeader);
  *group = g.release();
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_peer_group_connect(rmsnorm_b200_peer_group* g, const void* ipc_handles) {
  if (!g || !ipc_handles || g->connected) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != g->device) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < g->world; ++q) {
    if (q == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(ipc_handles) + static_cast<size_t>(q) * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess || !p) {
      cudaGetLastError();
      for (int r = 0; r < q; ++r)
        if (g->opened[r]) { cudaIpcCloseMemHandle(g->opened[r]); g->opened[r] = nullptr; }
      return RMSNORM_B200_ERR_CUDA;
    }
    g->opened[q] = p;
    g->recv[q] = reinterpret_cast<unsigned long long*>(static_cast<char*>(p) + kPeerBufferHeader);
  }
  g->connected = true;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_peer_group_connect_buffers(rmsnorm_b200_peer_group* g, void* const* buffers) {
  if (!g || !buffers || g->connected) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < g->world; ++q)
    if (q != g->rank && !buffers[q]) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < g->world; ++q)
    if (q != g->rank)
      g->recv[q] = reinterpret_cast<unsigned long long*>(static_cast<char*>(buffers[q]) + kPeerBufferHeader);
  g->connected = true;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_peer_group_buffer(rmsnorm_b200_peer_group* g, void** buffer) {
  if (!g || !buffer) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  *buffer = g->buffer;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_peer_group_destroy(rmsnorm_b200_peer_group* g) {
  if (!g) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  int st = RMSNORM_B200_OK;
  for (int q = 0; q < g->world; ++q)
    if (g->opened[q] && cudaIpcCloseMemHandle(g->opened[q]) != cudaSuccess) st = RMSNORM_B200_ERR_CUDA;
  if (g->buffer && cudaFree(g->buffer) != cudaSuccess) st = RMSNORM_B200_ERR_CUDA;
  cudaGetLastError();
  delete g;
  return st;
}

extern "C" int rmsnorm_b200_set_peer_timeout_ns(uint64_t timeout_ns) {
  if (timeout_ns < kMinWaitTimeoutNs) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  unsigned long long v = timeout_ns;
  if (cudaMemcpyToSymbol(g_peer_timeout_ns, &v, sizeof(v)) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_bwd_allreduce(const rmsnorm_b200_bwd_args* args, void* workspace, size_t workspace_bytes,
                                          rmsnorm_b200_peer_group* group, void* stream) {
  if (!group) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  return do_bwd(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), group);
}

extern "C" int rmsnorm_b200_bwd_noalloc(const rmsnorm_b200_bwd_args* args, void* stream) {
  int st = check_bwd(args);
  if (st) return st;
  DeviceState* ds = nullptr;
  st = get_device_state(&ds);
  if (st) return st;
  void* scratch = nullptr;
  st = noalloc_scratch(ds, &scratch);
  if (st) return st;
  BwdPlan bp;
  st = plan_bwd(ds, args, &bp);
  if (st) return st;
  // a plan whose partial rows do not fit the buffer falls back to the register-accumulator
  // kernels, which keep fewer partial rows (one per CTA group instead of one per row group
  // of every CTA)
  bool allow_tmem = true;
  if (workspace_for(bp) > RMSNORM_B200_NOALLOC_SCRATCH_BYTES && bp.tmem) {
    allow_tmem = false;
    st = plan_bwd(ds, args, &bp, false);
    if (st) return st;
  }
  if (workspace_for(bp) > RMSNORM_B200_NOALLOC_SCRATCH_BYTES) return RMSNORM_B200_ERR_SCRATCH_LIMIT;
  return do_bwd(args, scratch, RMSNORM_B200_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream), nullptr,
                allow_tmem);
}

extern "C" const char* rmsnorm_b200_strerror(int status) {
  switch (status) {
    case RMSNORM_B200_OK: return "ok";
    case RMSNORM_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RMSNORM_B200_ERR_UNSUPPORTED: return "unsupported configuration";
    case RMSNORM_B200_ERR_WORKSPACE: return "workspace missing, too small or misaligned";
    case RMSNORM_B200_ERR_CUDA: return "CUDA launch or runtime error";
    case RMSNORM_B200_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case RMSNORM_B200_ERR_NO_DEVICE: return "no CUDA device";
    case RMSNORM_B200_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the library's built-in no-allocation buffer holds";
    default: return "unknown status";
  }
}

extern "C" int rmsnorm_b200_device_status(void* stream, int32_t* status, int32_t* where, int32_t clear) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = 0, wh = 0;
  if (cudaMemcpyFromSymbolAsync(&st, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyFromSymbolAsync(&wh, g_status_where, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return RMSNORM_B200_ERR_CUDA;
  if (clear) {
    static const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_status_where, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
      return RMSNORM_B200_ERR_CUDA;
  }
  if (cudaStreamSynchronize(s) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  if (status) *status = st;
  if (where) *where = wh;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_set_wait_timeout_ns(uint64_t timeout_ns) {
  if (timeout_ns < kMinWaitTimeoutNs) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  unsigned long long v = timeout_ns;
  if (cudaMemcpyToSymbol(g_wait_timeout_ns, &v, sizeof(v)) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
  if (cudaGetLastError() != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_max_active_clusters(int32_t cluster_size, int32_t* clusters) {
  if (!clusters || cluster_size < 1 || cluster_size > kMaxCluster) return RMSNORM_B200_ERR_INVALID_ARGUMENT;
  DeviceState* ds = nullptr;
  int st = get_device_state(&ds);
  if (st) return st;
  const void* k = reinterpret_cast<const void*>(pick_fwd(B, NA, B, NA, false));
  if (ensure_attrs(ds, k)) return RMSNORM_B200_ERR_CUDA;
  *clusters = resident_units(ds, k, cluster_size, kSmemOptIn, kBlockLarge);
  return RMSNORM_B200_OK;
}

extern "C" int rmsnorm_b200_abi_version(void) { return RMSNORM_B200_ABI_VERSION; }

extern "C" int rmsnorm_b200_debug_bounds_build(void) {
#ifdef RMSB_DEBUG_BOUNDS
  return 1;
#else
  return 0;
#endif
}

extern "C" int rmsnorm_b200_debug_report(void* stream, uint64_t* violations, int32_t* site, uint64_t* address,
                                         uint32_t* bytes, int32_t clear) {
#ifdef RMSB_DEBUG_BOUNDS
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  unsigned long long rep[4] = {0, 0, 0, 0};
  if (cudaMemcpyFromSymbol(rep, g_dbg_report, sizeof(rep)) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  if (violations) *violations = rep[0];
  if (site) *site = static_cast<int32_t>(rep[1]);
  if (address) *address = rep[2];
  if (bytes) *bytes = static_cast<uint32_t>(rep[3]);
  if (clear) {
    const unsigned long long z[4] = {0, 0, 0, 0};
    if (cudaMemcpyToSymbol(g_dbg_report, z, sizeof(z)) != cudaSuccess) return RMSNORM_B200_ERR_CUDA;
  }
  return RMSNORM_B200_OK;
#else
  (void)stream; (void)violations; (void)site; (void)address; (void)bytes; (void)clear;
  return RMSNORM_B200_ERR_UNSUPPORTED;
#endif
}

extern "C" uint64_t rmsnorm_b200_launch_count(void) { return g_launches.load(); }

extern "C" int rmsnorm_b200_last_plan(char* buf, size_t len) {
  const std::string& s = t_last_plan;
  if (buf && len > 0) {
    const size_t n = std::min(len - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(s.size());
}
