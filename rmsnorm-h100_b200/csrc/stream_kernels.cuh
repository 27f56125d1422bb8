// stream_kernels.cuh -- the persistent, TMA-staged forward and backward kernels.
//
// Structure (both directions):
//   * one CTA of T = 512 threads per SM (or one cluster of P CTAs on P SMs), persistent
//     over tiles assigned round-robin (tile = cluster id + k * clusters);
//   * thread 0 streams each tile HBM -> shared memory with cp.async.bulk (one bulk copy
//     per tensor per tile when P == 1, one per row slice when P > 1) into an S-deep ring of
//     stages; each stage's "full" mbarrier counts the bytes landing. Right after the
//     CTA-wide barrier that opens tile i, thread 0 refills the stage tile i-1 used with
//     tile i-1+S, so S-1 tiles are always in flight behind the one being computed;
//   * threads read 8-element vectors from shared memory, reduce the row (xor shuffles in a
//     warp, named barriers across the warps of a row group, st.async + mbarrier exchange
//     through distributed shared memory across the CTAs of a cluster), then re-read the
//     stage and write outputs with 16-byte coalesced streaming stores;
//   * affine parameters live in registers for the whole kernel (each thread always owns
//     the same columns), so dweight/dbias accumulate in registers and are written once
//     per (CTA, row group) as a partial row; a second kernel sums the partials in a fixed
//     order.
// Every wait is bounded; a wait that gives up records an error in the device status word
// and the CTA leaves its loop at the next CTA-wide vote (after its in-flight copies land).
#pragma once

#include "device_common.cuh"
#include "stream_plan.h"

namespace rmsb200 {

struct SmemLayout {
  uint64_t* full;   // [kMaxStages]
  uint64_t* xbar;   // [2] cluster exchange barriers
  float* xpart;     // [2][kMaxCluster] partial sums received from the cluster
  float* red;       // [2][32] per-warp partials (double buffered)
  float* bc;        // [2] cluster total broadcast to the row group
  int* bcf;         // [2] ... and whether the exchange completed
};

__device__ __forceinline__ SmemLayout carve_smem(unsigned char* smem, const StreamPlan& pl) {
  SmemLayout L;
  unsigned char* tail = smem + static_cast<size_t>(pl.S) * pl.stage_bytes;
  L.full = reinterpret_cast<uint64_t*>(tail);
  L.xbar = L.full + kMaxStages;
  L.xpart = reinterpret_cast<float*>(L.xbar + 2);
  L.red = L.xpart + 2 * kMaxCluster;
  L.bc = L.red + 64;
  L.bcf = reinterpret_cast<int*>(L.bc + 2);
  return L;
}

__device__ __forceinline__ void init_barriers(const SmemLayout& L, const StreamPlan& pl) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < pl.S; ++s) mbar_init(&L.full[s], 1);
    mbar_init(&L.xbar[0], 1);
    mbar_init(&L.xbar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (pl.P > 1) cluster_sync_all();
}

// Sum of `v` over the G threads of a whole-slice row group (G a multiple of 32), then over
// the P CTAs of the cluster. Every thread of the group returns the same total (summed in
// warp order, then in cluster-rank order, so every CTA of the cluster gets the same bits).
// Returns false, uniformly over the group, when the cluster exchange gave up.
__device__ __forceinline__ bool row_group_sum(float& v, const StreamPlan& pl, const SmemLayout& L,
                                              int gid, int gl, uint32_t seq, uint32_t rank,
                                              int site) {
  v = warp_sum(v);
  const uint32_t par = seq & 1u;
  if (pl.G > 32) {
    const int nw = pl.G >> 5;
    float* red = L.red + par * 32 + gid * nw;
    if ((gl & 31) == 0) red[gl >> 5] = v;
    named_barrier(1 + gid, pl.G);
    float t = 0.f;
    for (int j = 0; j < nw; ++j) t += red[j];
    v = t;
  }
  if (pl.P > 1) {
    const uint32_t parity = (seq >> 1) & 1u;
    float* xp = L.xpart + par * kMaxCluster;
    if (gl == 0) {
      xp[rank] = v;
      mbar_arrive_expect_tx(&L.xbar[par], static_cast<uint32_t>(pl.P - 1) * 4u);
      const uint32_t my_slot = smem_u32(&xp[rank]);
      const uint32_t my_bar = smem_u32(&L.xbar[par]);
      for (int q = 0; q < pl.P; ++q) {
        if (q == static_cast<int>(rank)) continue;
        st_async_peer(map_peer(my_slot, q), v, map_peer(my_bar, q));
      }
      const bool ok = mbar_wait<true>(&L.xbar[par], parity, site);
      float t = 0.f;
      for (int q = 0; q < pl.P; ++q) t += xp[q];
      L.bc[par] = t;
      L.bcf[par] = ok ? 1 : 0;
    }
    if (pl.G > 32) named_barrier(1 + gid, pl.G); else __syncwarp();
    v = L.bc[par];
    return L.bcf[par] != 0;
  }
  return true;
}

// xor-shuffle sum over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float seg_sum(float v, int width, unsigned mask) {
  for (int off = width >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(mask, v, off);
  return v;
}

// Ring bookkeeping for thread 0: issues tiles in order and remembers how many it issued.
struct Ring {
  int64_t issued = 0;  // tiles issued so far (index in this cluster's tile sequence)
};

// Waits (bounded) for the copies of tiles [consumed, issued) after a failure.
__device__ __forceinline__ void drain_ring(const StreamPlan& pl, const SmemLayout& L, int64_t consumed,
                                           int64_t issued) {
  for (int64_t j = consumed; j < issued; ++j)
    mbar_wait(&L.full[j % pl.S], static_cast<uint32_t>(j / pl.S) & 1u, kSiteDrain);
}

// =======================================================================================
// Forward
// =======================================================================================
template <typename X, typename RT>
__device__ __forceinline__ void fwd_issue(const FwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                          unsigned char* smem, int64_t tile, int s,
                                          int64_t slice_elt0, uint64_t pol) {
  unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
  const int64_t row0 = tile * pl.R;
  const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
  fence_proxy_async_smem();
  const uint32_t bx = static_cast<uint32_t>(rows) * pl.row_bytes[0];
  const uint32_t br = p.res != nullptr ? static_cast<uint32_t>(rows) * pl.row_bytes[1] : 0u;
  mbar_arrive_expect_tx(&L.full[s], bx + br);
  const int64_t e0 = row0 * pl.W + slice_elt0;  // P > 1 implies R == 1
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, bx, &L.full[s], pol);
  if (p.res != nullptr)
    bulk_load(st + pl.off[1], static_cast<const RT*>(p.res) + e0, br, &L.full[s], pol);
}

template <typename X, typename RT>
__global__ void __launch_bounds__(kBlockThreads, 1) fwd_stream_kernel(const FwdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const StreamPlan& pl = p.pl;
  const SmemLayout L = carve_smem(smem, pl);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  uint32_t rank = 0;
  int64_t cid = blockIdx.x;
  int64_t ncl = gridDim.x;
  if (pl.P > 1) {
    rank = cluster_ctarank();
    cid = cluster_id_x();
    ncl = cluster_count_x();
  }
  init_barriers(L, pl);

  const bool has_res = p.res != nullptr;
  constexpr int sx = sizeof(X);
  constexpr int sr = sizeof(RT);
  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const uint64_t pol = l2_policy_evict_first();

  int64_t issued = 0;
  if (tid == 0) {
    for (int j = 0; j < pl.S; ++j) {
      const int64_t t = cid + j * ncl;
      if (t >= pl.ntiles) break;
      fwd_issue<X, RT>(p, pl, L, smem, t, j, slice_elt0, pol);
      ++issued;
    }
  }

  const int gid = tid / pl.G;
  const int gl = tid - gid * pl.G;
  const bool in_group = gid < pl.rps;
  const int N = pl.N;
  const float n_f = static_cast<float>(N);

  float wr[kMaxVecs][8];
  float br_[kMaxVecs][8];
#pragma unroll
  for (int k = 0; k < kMaxVecs; ++k) {
    const int v = gl + k * pl.G;
    const int64_t c = slice_elt0 + static_cast<int64_t>(v) * 8;
    const bool valid = in_group && v < pl.vslice;
#pragma unroll
    for (int e = 0; e < 8; ++e) { wr[k][e] = 1.f; br_[k][e] = 0.f; }
    if (valid && p.w != nullptr) load8_rt(p.w, p.w_dt, p.w_per_head ? c : c % N, wr[k], true);
    if (valid && p.b != nullptr) load8_rt(p.b, p.b_dt, p.b_per_head ? c : c % N, br_[k], true);
  }

  uint32_t seq = 0;  // rows processed by this group (parity of scratch slots, cluster phases)
  int64_t i = 0;
  bool failed = false;
  for (int64_t tile = cid; tile < pl.ntiles; tile += ncl, ++i) {
    const int s = static_cast<int>(i % pl.S);
    const bool ok = mbar_wait(&L.full[s], static_cast<uint32_t>(i / pl.S) & 1u, kSiteFwdFull);
    if (__syncthreads_or(!ok || failed)) { failed = true; break; }
    if (tid == 0 && i > 0 && pl.S > 1) {  // everyone is past tile i-1: its stage is free
      const int64_t t = cid + (i - 1 + pl.S) * ncl;
      if (t < pl.ntiles) { fwd_issue<X, RT>(p, pl, L, smem, t, static_cast<int>((i - 1) % pl.S), slice_elt0, pol); ++issued; }
    }
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const int64_t row0 = tile * pl.R;
    const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
    for (int sw = 0; sw < pl.R; sw += pl.rps) {
      const int lr = sw + gid;
      const bool active = in_group && lr < rows;
      const unsigned amask = __ballot_sync(0xffffffffu, active);
      if (!active) continue;
      const unsigned char* xs = st + pl.off[0] + static_cast<size_t>(lr) * pl.row_bytes[0];
      const unsigned char* rs = st + pl.off[1] + static_cast<size_t>(lr) * pl.row_bytes[1];
      const int64_t row = row0 + lr;
      const int64_t g0 = row * pl.W + slice_elt0;  // global element index of the slice

      float part[kMaxVecs];
#pragma unroll
      for (int k = 0; k < kMaxVecs; ++k) {
        const int v = gl + k * pl.G;
        float acc = 0.f;
        if (v < pl.vslice) {
          float h[8];
          Vec8<X>::load(xs + v * 8 * sx, h);
          if (has_res) {
            float r[8];
            Vec8<RT>::load(rs + v * 8 * sr, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] += r[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc = fmaf(h[e], h[e], acc);
        }
        part[k] = acc;
      }

      float rstd_k[kMaxVecs];
      if (pl.seg_mode) {
#pragma unroll
        for (int k = 0; k < kMaxVecs; ++k) {
          const float ss = seg_sum(part[k], pl.vs, amask);
          rstd_k[k] = rsqrtf(ss / n_f + p.eps);
        }
      } else {
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxVecs; ++k) ss += part[k];
        const bool red_ok = row_group_sum(ss, pl, L, gid, gl, seq, rank, kSiteFwdCluster);
        ++seq;
        if (!red_ok) { failed = true; break; }
        const float r = rsqrtf(ss / n_f + p.eps);
#pragma unroll
        for (int k = 0; k < kMaxVecs; ++k) rstd_k[k] = r;
      }

#pragma unroll
      for (int k = 0; k < kMaxVecs; ++k) {
        const int v = gl + k * pl.G;
        if (v < pl.vslice) {
          float h[8];
          Vec8<X>::load(xs + v * 8 * sx, h);
          if (has_res) {
            float r[8];
            Vec8<RT>::load(rs + v * 8 * sr, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] += r[e];
          }
          const int64_t ge = g0 + static_cast<int64_t>(v) * 8;
          if (p.ro != nullptr) store8_rt(p.ro, p.ro_dt, ge, h);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = fmaf(h[e] * rstd_k[k], wr[k][e], br_[k][e]);
          store8_rt(p.out, p.out_dt, ge, y);
          if (p.rstd != nullptr) {
            if (pl.seg_mode) {
              if ((v & (pl.vs - 1)) == 0) p.rstd[row * pl.heads + v / pl.vs] = rstd_k[k];
            } else if (v == 0 && rank == 0) {
              p.rstd[row] = rstd_k[k];
            }
          }
        }
      }
    }
    if (pl.S == 1) {  // a single stage is refilled once everyone is done with it
      __syncthreads();
      const int64_t t = cid + (i + 1) * ncl;
      if (tid == 0 && t < pl.ntiles) { fwd_issue<X, RT>(p, pl, L, smem, t, 0, slice_elt0, pol); ++issued; }
    }
  }
  failed = __syncthreads_or(failed);
  if (failed && tid == 0) drain_ring(pl, L, i, issued);
  (void)lane;
}

// =======================================================================================
// Backward: dx in one pass from the saved rstd; dweight / dbias per-CTA partial rows.
// =======================================================================================
template <typename X, typename DY>
__device__ __forceinline__ void bwd_issue(const BwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                          unsigned char* smem, int64_t tile, int s,
                                          int64_t slice_elt0, int rstd_per_row, int sdro,
                                          uint64_t pol) {
  unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
  const int64_t row0 = tile * pl.R;
  const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
  fence_proxy_async_smem();
  // rstd of the tile's rows: plain async copies, tracked by the same mbarrier
  float* rdst = reinterpret_cast<float*>(st + pl.off[3]);
  const float* rsrc = p.rstd + row0 * rstd_per_row;
  const int cnt = rows * rstd_per_row;
  int j = 0;
  if ((reinterpret_cast<uintptr_t>(rsrc) & 15u) == 0)
    for (; j + 4 <= cnt; j += 4) cp_async_16(rdst + j, rsrc + j);
  for (; j < cnt; ++j) cp_async_4(rdst + j, rsrc + j);
  cp_async_arrive(&L.full[s]);
  const uint32_t b0 = static_cast<uint32_t>(rows) * pl.row_bytes[0];
  const uint32_t b1 = static_cast<uint32_t>(rows) * pl.row_bytes[1];
  const uint32_t b2 = p.dro != nullptr ? static_cast<uint32_t>(rows) * pl.row_bytes[2] : 0u;
  mbar_arrive_expect_tx(&L.full[s], b0 + b1 + b2);
  const int64_t e0 = row0 * pl.W + slice_elt0;
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, b0, &L.full[s], pol);
  bulk_load(st + pl.off[1], static_cast<const DY*>(p.dy) + e0, b1, &L.full[s], pol);
  if (p.dro != nullptr)
    bulk_load(st + pl.off[2], static_cast<const unsigned char*>(p.dro) + e0 * sdro, b2, &L.full[s], pol);
}

template <typename X, typename DY, bool kHasDb, int kVecs>
__global__ void __launch_bounds__(kBlockThreads, 1) bwd_stream_kernel(const BwdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const StreamPlan& pl = p.pl;
  const SmemLayout L = carve_smem(smem, pl);
  const int tid = threadIdx.x;
  uint32_t rank = 0;
  int64_t cid = blockIdx.x;
  int64_t ncl = gridDim.x;
  if (pl.P > 1) {
    rank = cluster_ctarank();
    cid = cluster_id_x();
    ncl = cluster_count_x();
  }
  init_barriers(L, pl);

  const bool has_dro = p.dro != nullptr;
  constexpr int sx = sizeof(X);
  constexpr int sd = sizeof(DY);
  const int sdro = has_dro ? dtype_bytes(p.dro_dt) : 0;
  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const int rstd_per_row = pl.seg_mode ? pl.heads : 1;
  const uint64_t pol = l2_policy_evict_first();

  int64_t issued = 0;
  if (tid == 0) {
    for (int j = 0; j < pl.S; ++j) {
      const int64_t t = cid + j * ncl;
      if (t >= pl.ntiles) break;
      bwd_issue<X, DY>(p, pl, L, smem, t, j, slice_elt0, rstd_per_row, sdro, pol);
      ++issued;
    }
  }

  const int gid = tid / pl.G;
  const int gl = tid - gid * pl.G;
  const bool in_group = gid < pl.rps;
  const int N = pl.N;
  const float n_f = static_cast<float>(N);
  const bool has_w = p.w != nullptr;

  float wr[kVecs][8];
  float dw[kVecs][8];
  float db[kHasDb ? kVecs : 1][8];
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    const int v = gl + k * pl.G;
    const int64_t c = slice_elt0 + static_cast<int64_t>(v) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) { wr[k][e] = 1.f; dw[k][e] = 0.f; }
    if (kHasDb) {
#pragma unroll
      for (int e = 0; e < 8; ++e) db[kHasDb ? k : 0][e] = 0.f;
    }
    if (in_group && v < pl.vslice && has_w) load8_rt(p.w, p.w_dt, p.w_per_head ? c : c % N, wr[k], true);
  }

  uint32_t seq = 0;
  int64_t i = 0;
  bool failed = false;
  for (int64_t tile = cid; tile < pl.ntiles; tile += ncl, ++i) {
    const int s = static_cast<int>(i % pl.S);
    const bool ok = mbar_wait(&L.full[s], static_cast<uint32_t>(i / pl.S) & 1u, kSiteBwdFull);
    if (__syncthreads_or(!ok || failed)) { failed = true; break; }
    if (tid == 0 && i > 0 && pl.S > 1) {
      const int64_t t = cid + (i - 1 + pl.S) * ncl;
      if (t < pl.ntiles) {
        bwd_issue<X, DY>(p, pl, L, smem, t, static_cast<int>((i - 1) % pl.S), slice_elt0, rstd_per_row, sdro, pol);
        ++issued;
      }
    }
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const float* rs_stage = reinterpret_cast<const float*>(st + pl.off[3]);
    const int64_t row0 = tile * pl.R;
    const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
    for (int sw = 0; sw < pl.R; sw += pl.rps) {
      const int lr = sw + gid;
      const bool active = in_group && lr < rows;
      const unsigned amask = __ballot_sync(0xffffffffu, active);
      if (!active) continue;
      const unsigned char* xs = st + pl.off[0] + static_cast<size_t>(lr) * pl.row_bytes[0];
      const unsigned char* ds = st + pl.off[1] + static_cast<size_t>(lr) * pl.row_bytes[1];
      const unsigned char* as = st + pl.off[2] + static_cast<size_t>(lr) * pl.row_bytes[2];
      const int64_t row = row0 + lr;
      const int64_t g0 = row * pl.W + slice_elt0;

      float rstd_k[kVecs];
      float part[kVecs];
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        const int v = gl + k * pl.G;
        float acc = 0.f;
        rstd_k[k] = 0.f;
        if (v < pl.vslice) {
          const float r = rs_stage[lr * rstd_per_row + (pl.seg_mode ? v / pl.vs : 0)];
          rstd_k[k] = r;
          float xv[8], dv[8];
          Vec8<X>::load(xs + v * 8 * sx, xv);
          Vec8<DY>::load(ds + v * 8 * sd, dv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float xh = xv[e] * r;
            acc = fmaf(xh, dv[e] * wr[k][e], acc);
            dw[k][e] = fmaf(dv[e], xh, dw[k][e]);
            if (kHasDb) db[kHasDb ? k : 0][e] += dv[e];
          }
        }
        part[k] = acc;
      }

      float c_k[kVecs];
      if (pl.seg_mode) {
#pragma unroll
        for (int k = 0; k < kVecs; ++k) c_k[k] = seg_sum(part[k], pl.vs, amask) / n_f;
      } else {
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) dot += part[k];
        const bool red_ok = row_group_sum(dot, pl, L, gid, gl, seq, rank, kSiteBwdCluster);
        ++seq;
        if (!red_ok) { failed = true; break; }
        const float c = dot / n_f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) c_k[k] = c;
      }

#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        const int v = gl + k * pl.G;
        if (v < pl.vslice) {
          const float r = rstd_k[k];
          float xv[8], dv[8], g[8];
          Vec8<X>::load(xs + v * 8 * sx, xv);
          Vec8<DY>::load(ds + v * 8 * sd, dv);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] = (dv[e] * wr[k][e] - (xv[e] * r) * c_k[k]) * r;
          if (has_dro) {
            float a[8];
            load8_rt(as + v * 8 * sdro, p.dro_dt, 0, a, false);
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] += a[e];
          }
          const int64_t ge = g0 + static_cast<int64_t>(v) * 8;
          store8_rt(p.dx, p.dx_dt, ge, g);
          if (p.dres != nullptr) store8_rt(p.dres, p.dres_dt, ge, g);
        }
      }
    }
    if (pl.S == 1) {
      __syncthreads();
      const int64_t t = cid + (i + 1) * ncl;
      if (tid == 0 && t < pl.ntiles) {
        bwd_issue<X, DY>(p, pl, L, smem, t, 0, slice_elt0, rstd_per_row, sdro, pol);
        ++issued;
      }
    }
  }
  failed = __syncthreads_or(failed);
  if (failed) {
    if (tid == 0) drain_ring(pl, L, i, issued);
    return;
  }

  // one partial row per (cluster, row group): the groups of a CTA own the same columns.
  // Every owned column is written, zeros included, so the reduction reads no stale data.
  const int64_t prow = (cid * pl.rps + gid) * pl.W;
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    const int v = gl + k * pl.G;
    if (in_group && v < pl.vslice) {
      const int64_t c = slice_elt0 + static_cast<int64_t>(v) * 8;
      if (p.dw_part != nullptr) Vec8<float>::store(p.dw_part + prow + c, dw[k]);
      if (kHasDb && p.db_part != nullptr) Vec8<float>::store(p.db_part + prow + c, db[kHasDb ? k : 0]);
    }
  }
}

}  // namespace rmsb200
