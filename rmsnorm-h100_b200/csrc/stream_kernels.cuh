// stream_kernels.cuh -- the persistent, TMA-staged forward and backward kernels.
//
// Structure (both directions):
//   * one CTA of 512 threads per SM, or two CTAs of 256 threads per SM (launch variant for
//     rows split across clusters, so that two independent row pipelines share each SM);
//     persistent over tiles assigned round-robin (tile = cluster id + k * clusters);
//   * thread 0 streams each tile HBM -> shared memory with cp.async.bulk (one bulk copy
//     per tensor per tile when P == 1, one per row slice when P > 1) into an S-deep ring of
//     stages; each stage's "full" mbarrier counts the bytes landing. Right after the
//     CTA-wide vote that opens tile i, thread 0 refills the stage tile i-1 used with tile
//     i-1+S, so S-1 tiles are always in flight behind the one being computed;
//   * threads read 8-element vectors from shared memory, reduce the row (xor shuffles in a
//     warp, one named barrier + one shared load + a second shuffle tree across the warps of
//     a row group, st.async + mbarrier exchange through distributed shared memory across
//     the CTAs of a cluster), then re-read the stage and write outputs with 16-byte
//     coalesced streaming stores;
//   * every per-element dtype is a template parameter (absent tensors are `NoT`), so the
//     inner loops carry no runtime type dispatch;
//   * affine parameters live in registers for the whole kernel (each thread always owns
//     the same columns), so dweight/dbias accumulate in registers and are written once
//     per (cluster, row group) as a partial row; a second kernel sums the partials in a
//     fixed order.
// Every wait is bounded; a wait that gives up records an error in the device status word
// and the CTA leaves its loop at the next CTA-wide vote (after its in-flight copies land).
#pragma once

#include <type_traits>

#include "device_common.cuh"
#include "stream_plan.h"

namespace rmsb200 {

constexpr int kXSlots = 4;  // cluster exchange slots (sequence number mod 4)

struct SmemLayout {
  uint64_t* full;   // [kMaxStages]
  uint64_t* xbar;   // [kXSlots] cluster exchange barriers
  float* xpart;     // [kXSlots][kMaxCluster] partial sums received from the cluster
  float* red;       // [2][32] per-warp partials (double buffered)
  float* bc;        // [kXSlots] cluster total broadcast to the row group
  int* bcf;         // [kXSlots] ... and whether the exchange completed
};

__device__ __forceinline__ SmemLayout carve_smem(unsigned char* smem, const StreamPlan& pl) {
  SmemLayout L;
  unsigned char* tail = smem + static_cast<size_t>(pl.S) * pl.stage_bytes;
  L.full = reinterpret_cast<uint64_t*>(tail);
  L.xbar = L.full + kMaxStages;
  L.xpart = reinterpret_cast<float*>(L.xbar + kXSlots);
  L.red = L.xpart + kXSlots * kMaxCluster;
  L.bc = L.red + 64;
  L.bcf = reinterpret_cast<int*>(L.bc + kXSlots);
  return L;
}

__device__ __forceinline__ void init_barriers(const SmemLayout& L, const StreamPlan& pl) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < pl.S; ++s) mbar_init(&L.full[s], 1);
    for (int s = 0; s < kXSlots; ++s) mbar_init(&L.xbar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (pl.P > 1) cluster_sync_all();
}

// Sum of `v` over the G threads of row group `gid` (G a multiple of 32). Every thread of
// the group gets the same bits: lanes load the per-warp partials in warp order and run the
// same shuffle tree.
__device__ __forceinline__ float group_sum(float v, const StreamPlan& pl, const SmemLayout& L, int gid,
                                           int gl, uint32_t seq) {
  v = warp_sum(v);
  if (pl.G > 32) {
    const int nw = pl.G >> 5;
    const int lane = gl & 31;
    float* red = L.red + (seq & 1u) * 32 + gid * nw;
    if (lane == 0) red[gl >> 5] = v;
    named_barrier(1 + gid, pl.G);
    v = warp_sum(lane < nw ? red[lane] : 0.f);
  }
  return v;
}

// Sum of the group totals of the P CTAs of the cluster, in rank order (every CTA gets the
// same bits). One thread sends this CTA's total into every peer's shared memory with
// st.async (completing 4 tx-bytes on the peer's mbarrier), waits (bounded) for the peers'
// totals, and broadcasts the result to the group. Returns false, uniformly over the
// group, when the exchange gave up.
__device__ __forceinline__ bool cluster_sum(float& v, const StreamPlan& pl, const SmemLayout& L, int gid,
                                            int gl, uint32_t seq, uint32_t rank, int site) {
  const uint32_t slot = seq & (kXSlots - 1);
  const uint32_t parity = (seq / kXSlots) & 1u;
  float* xp = L.xpart + slot * kMaxCluster;
  if (gl == 0) {
    xp[rank] = v;
    mbar_arrive_expect_tx(&L.xbar[slot], static_cast<uint32_t>(pl.P - 1) * 4u);
    const uint32_t my_slot = smem_u32(&xp[rank]);
    const uint32_t my_bar = smem_u32(&L.xbar[slot]);
    for (int q = 0; q < pl.P; ++q) {
      if (q == static_cast<int>(rank)) continue;
      st_async_peer(map_peer(my_slot, q), v, map_peer(my_bar, q));
    }
    const bool ok = mbar_wait<true>(&L.xbar[slot], parity, site);
    float t = 0.f;
    for (int q = 0; q < pl.P; ++q) t += xp[q];
    L.bc[slot] = t;
    L.bcf[slot] = ok ? 1 : 0;
  }
  if (pl.G > 32) named_barrier(1 + gid, pl.G); else __syncwarp();
  v = L.bc[slot];
  return L.bcf[slot] != 0;
}

// Split form of cluster_sum for the pipelined split-row loop: cluster_send posts this
// CTA's total for row `seq` (thread gl == 0 only, no wait); cluster_recv waits (bounded)
// for the peers' totals of row `seq`, sums them in rank order and broadcasts the result to
// the group. Four slots (seq mod 4) make two rows in flight safe: a peer can only post row
// seq + 4 after it received this CTA's row seq + 2, which this CTA sends after it has read
// row seq.
__device__ __forceinline__ void cluster_send(float v, const StreamPlan& pl, const SmemLayout& L, int gl,
                                             uint32_t seq, uint32_t rank) {
  if (gl != 0) return;
  const uint32_t slot = seq & (kXSlots - 1);
  float* xp = L.xpart + slot * kMaxCluster;
  xp[rank] = v;
  mbar_arrive_expect_tx(&L.xbar[slot], static_cast<uint32_t>(pl.P - 1) * 4u);
  const uint32_t my_slot = smem_u32(&xp[rank]);
  const uint32_t my_bar = smem_u32(&L.xbar[slot]);
  for (int q = 0; q < pl.P; ++q) {
    if (q == static_cast<int>(rank)) continue;
    st_async_peer(map_peer(my_slot, q), v, map_peer(my_bar, q));
  }
}

__device__ __forceinline__ bool cluster_recv(float& v, const StreamPlan& pl, const SmemLayout& L, int gid,
                                             int gl, uint32_t seq, int site) {
  const uint32_t slot = seq & (kXSlots - 1);
  if (gl == 0) {
    const bool ok = mbar_wait<true>(&L.xbar[slot], (seq / kXSlots) & 1u, site);
    const float* xp = L.xpart + slot * kMaxCluster;
    float t = 0.f;
    for (int q = 0; q < pl.P; ++q) t += xp[q];
    L.bc[slot] = t;
    L.bcf[slot] = ok ? 1 : 0;
  }
  if (pl.G > 32) named_barrier(1 + gid, pl.G); else __syncwarp();
  v = L.bc[slot];
  return L.bcf[slot] != 0;
}

// xor-shuffle sum over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float seg_sum(float v, int width, unsigned mask) {
  for (int off = width >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(mask, v, off);
  return v;
}

// Waits (bounded) for the copies of tiles [consumed, issued) after a failure.
__device__ __forceinline__ void drain_ring(const StreamPlan& pl, const SmemLayout& L, int64_t consumed,
                                           int64_t issued) {
  for (int64_t j = consumed; j < issued; ++j)
    mbar_wait(&L.full[j % pl.S], static_cast<uint32_t>(j / pl.S) & 1u, kSiteDrain);
}

template <typename T>
using Elt = typename std::conditional<Present<T>::value, T, float>::type;

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
  const uint32_t br = Present<RT>::value ? static_cast<uint32_t>(rows) * pl.row_bytes[1] : 0u;
  mbar_arrive_expect_tx(&L.full[s], bx + br);
  const int64_t e0 = row0 * pl.W + slice_elt0;  // P > 1 implies R == 1
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, bx, &L.full[s], pol);
  if constexpr (Present<RT>::value)
    bulk_load(st + pl.off[1], static_cast<const RT*>(p.res) + e0, br, &L.full[s], pol);
}

// Split-row pipeline: sub-chunk j of the row slice of tile `tile` into ring slot `slot`.
template <typename X, typename RT>
__device__ __forceinline__ void fwd_issue_chunk(const FwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                                unsigned char* smem, int64_t tile, int j, int slot,
                                                int64_t slice_elt0, uint64_t pol) {
  unsigned char* st = smem + static_cast<size_t>(slot) * pl.stage_bytes;
  fence_proxy_async_smem();
  const uint32_t bx = pl.row_bytes[0];
  const uint32_t br = Present<RT>::value ? pl.row_bytes[1] : 0u;
  mbar_arrive_expect_tx(&L.full[slot], bx + br);
  const int64_t e0 = tile * pl.W + slice_elt0 + static_cast<int64_t>(j) * (pl.vslice / pl.K) * 8;
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, bx, &L.full[slot], pol);
  if constexpr (Present<RT>::value)
    bulk_load(st + pl.off[1], static_cast<const RT*>(p.res) + e0, br, &L.full[slot], pol);
}

// X: input dtype; RT: residual dtype (NoT = none); OT: output dtype; ROT: residual_out
// dtype (NoT = not written).
template <typename X, typename RT, typename OT, typename ROT, int kVecs, int kBlock, int kMinBlocks>
__global__ void __launch_bounds__(kBlock, kMinBlocks) fwd_stream_kernel(const FwdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr bool kRes = Present<RT>::value;
  constexpr bool kRO = Present<ROT>::value;
  using RTe = Elt<RT>;
  using ROe = Elt<ROT>;
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

  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const uint64_t pol = l2_policy_evict_first();
  int64_t issued = 0;
  if (tid == 0 && pl.P == 1) {
    for (int j = 0; j < pl.S; ++j) {
      const int64_t t = cid + j * ncl;
      if (t >= pl.ntiles) break;
      fwd_issue<X, RT>(p, pl, L, smem, t, j, slice_elt0, pol);
      ++issued;
    }
  }

  const int G = pl.G;
  const int G8 = G * 8;
  const int gid = tid / G;
  const int gl = tid - gid * G;
  const bool in_group = gid < pl.rps;
  const float n_f = static_cast<float>(pl.N);
  unsigned vmask = 0;
#pragma unroll
  for (int k = 0; k < kVecs; ++k)
    if (in_group && gl + k * G < pl.vslice) vmask |= 1u << k;

  float wr[kVecs][8];
  float br[kVecs][8];
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    const int64_t c = slice_elt0 + static_cast<int64_t>(gl + k * G) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) { wr[k][e] = 1.f; br[k][e] = 0.f; }
    if ((vmask >> k) & 1u) {
      if (p.w != nullptr) load8_rt(p.w, p.w_dt, p.w_per_head ? c : c % pl.N, wr[k], true);
      if (p.b != nullptr) load8_rt(p.b, p.b_dt, p.b_per_head ? c : c % pl.N, br[k], true);
    }
  }

  if (pl.P > 1) {
    // ------------- split-row pipeline (row slices across a cluster, R = 1) -------------
    // Row slices are streamed as K sub-chunks through an S-slot ring. Iteration i runs
    // pass 1 of row i and posts its partial sum to the cluster, then (lag 1) receives
    // row i-1's total and runs its pass 2, so the exchange overlaps a whole pass 1.
    const int K = pl.K;
    const int S = pl.S;
    const int kpc_mask = (1 << pl.kpc_shift) - 1;
    const int64_t n_local = cid < pl.ntiles ? (pl.ntiles - 1 - cid) / ncl + 1 : 0;
    const int64_t total_q = n_local * K;
    const bool grp = tid < G;
    // ring positions are tracked incrementally (no 64-bit division in the loop)
    int iss_slot = 0, iss_j = 0;
    int64_t iss_tile = cid;
    auto issue_upto = [&](int64_t lim) {
      while (issued < lim) {
        fwd_issue_chunk<X, RT>(p, pl, L, smem, iss_tile, iss_j, iss_slot, slice_elt0, pol);
        ++issued;
        if (++iss_slot == S) iss_slot = 0;
        if (++iss_j == K) { iss_j = 0; iss_tile += ncl; }
      }
    };
    if (tid == 0) issue_upto(min(total_q, static_cast<int64_t>(S)));
    auto slot_ptr = [&](int base, int k, uint32_t off) -> const unsigned char* {
      int sl = base + (k >> pl.kpc_shift);
      if (sl >= S) sl -= S;
      return smem + static_cast<size_t>(sl) * pl.stage_bytes + off;
    };
    int row_slot = 0;       // ring slot of sub-chunk 0 of row i
    uint32_t row_phase = 0;  // its mbarrier phase parity
    bool failed = false;
    int64_t i = 0;
    for (; i < n_local + pl.lag; ++i) {
      bool ok = true;
      if (i < n_local) {
        for (int j = 0; j < K; ++j) {
          int sl = row_slot + j;
          uint32_t ph = row_phase;
          if (sl >= S) { sl -= S; ph ^= 1u; }
          ok = mbar_wait(&L.full[sl], ph, kSiteFwdFull) && ok;
        }
      }
      if (__syncthreads_or(!ok || failed)) { failed = true; break; }
      if (grp) {
        const int xo = gl * 8;
        if (i < n_local) {
          float ss = 0.f;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            if ((vmask >> k) & 1u) {
              const int vo = xo + (k & kpc_mask) * G8;
              float h[8];
              Vec8<X>::load(reinterpret_cast<const X*>(slot_ptr(row_slot, k, pl.off[0])) + vo, h);
              if constexpr (kRes) {
                float r[8];
                Vec8<RTe>::load(reinterpret_cast<const RTe*>(slot_ptr(row_slot, k, pl.off[1])) + vo, r);
#pragma unroll
                for (int e = 0; e < 8; ++e) h[e] += r[e];
              }
#pragma unroll
              for (int e = 0; e < 8; ++e) ss = fmaf(h[e], h[e], ss);
            }
          }
          ss = group_sum(ss, pl, L, 0, gl, static_cast<uint32_t>(i));
          cluster_send(ss, pl, L, gl, static_cast<uint32_t>(i), rank);
        }
        const int64_t r2 = i - pl.lag;
        if (r2 >= 0 && r2 < n_local) {
          int base2 = row_slot - pl.lag * K;
          if (base2 < 0) base2 += S;
          float tot;
          if (!cluster_recv(tot, pl, L, 0, gl, static_cast<uint32_t>(r2), kSiteFwdCluster)) {
            failed = true;
          } else {
            const float rs = rsqrtf(tot / n_f + p.eps);
            const int64_t row = cid + r2 * ncl;
            const int64_t g0 = row * pl.W + slice_elt0 + xo;
            OT* op = static_cast<OT*>(p.out) + g0;
            ROe* rop = static_cast<ROe*>(p.ro) + g0;
#pragma unroll
            for (int k = 0; k < kVecs; ++k) {
              if ((vmask >> k) & 1u) {
                const int vo = xo + (k & kpc_mask) * G8;
                float h[8];
                Vec8<X>::load(reinterpret_cast<const X*>(slot_ptr(base2, k, pl.off[0])) + vo, h);
                if constexpr (kRes) {
                  float r[8];
                  Vec8<RTe>::load(reinterpret_cast<const RTe*>(slot_ptr(base2, k, pl.off[1])) + vo, r);
#pragma unroll
                  for (int e = 0; e < 8; ++e) h[e] += r[e];
                }
                if constexpr (kRO) Vec8<ROe>::store(rop + k * G8, h);
                float y[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = fmaf(h[e] * rs, wr[k][e], br[k][e]);
                Vec8<OT>::store(op + k * G8, y);
              }
            }
            if (p.rstd != nullptr && gl == 0 && rank == 0) p.rstd[row] = rs;
          }
        }
      }
      __syncthreads();  // pass 2 of row i - lag is done: its slots are free
      if (tid == 0) issue_upto(min(total_q, max(static_cast<int64_t>(0), i + 1 - pl.lag) * K + S));
      if (i < n_local) {
        row_slot += K;
        if (row_slot >= S) { row_slot -= S; row_phase ^= 1u; }
      }
    }
    failed = __syncthreads_or(failed);
    if (failed && tid == 0) drain_ring(pl, L, i * K, issued);
    return;
  }

  const int xs_stride = static_cast<int>(pl.row_bytes[0] / sizeof(X));  // elements per staged row
  uint32_t seq = 0;  // rows reduced by this group (parity of scratch slots, cluster phases)
  int64_t i = 0;
  bool failed = false;
  for (int64_t tile = cid; tile < pl.ntiles; tile += ncl, ++i) {
    const int s = static_cast<int>(i % pl.S);
    const bool ok = mbar_wait(&L.full[s], static_cast<uint32_t>(i / pl.S) & 1u, kSiteFwdFull);
    if (__syncthreads_or(!ok || failed)) { failed = true; break; }
    if (tid == 0 && i > 0 && pl.S > 1) {  // everyone is past tile i-1: its stage is free
      const int64_t t = cid + (i - 1 + pl.S) * ncl;
      if (t < pl.ntiles) {
        fwd_issue<X, RT>(p, pl, L, smem, t, static_cast<int>((i - 1) % pl.S), slice_elt0, pol);
        ++issued;
      }
    }
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const X* xs0 = reinterpret_cast<const X*>(st + pl.off[0]) + gl * 8;
    const RTe* rs0 = reinterpret_cast<const RTe*>(st + pl.off[1]) + gl * 8;
    const int64_t row0 = tile * pl.R;
    const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
    for (int sw = 0; sw < pl.R; sw += pl.rps) {
      const int lr = sw + gid;
      const bool active = in_group && lr < rows;
      const unsigned amask = __ballot_sync(0xffffffffu, active);
      if (!active) continue;
      const X* xs = xs0 + lr * xs_stride;
      const RTe* rs = rs0 + lr * xs_stride;
      const int64_t row = row0 + lr;
      const int64_t g0 = row * pl.W + slice_elt0 + gl * 8;

      float part[kVecs];
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        part[k] = 0.f;
        if ((vmask >> k) & 1u) {
          float h[8];
          Vec8<X>::load(xs + k * G8, h);
          if constexpr (kRes) {
            float r[8];
            Vec8<RTe>::load(rs + k * G8, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] += r[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) part[k] = fmaf(h[e], h[e], part[k]);
        }
      }

      float rstd_k[kVecs];
      if (pl.seg_mode) {
#pragma unroll
        for (int k = 0; k < kVecs; ++k) rstd_k[k] = rsqrtf(seg_sum(part[k], pl.vs, amask) / n_f + p.eps);
      } else {
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) ss += part[k];
        ss = group_sum(ss, pl, L, gid, gl, seq);
        if (pl.P > 1 && !cluster_sum(ss, pl, L, gid, gl, seq, rank, kSiteFwdCluster)) {
          failed = true;
          ++seq;
          break;
        }
        ++seq;
        const float r = rsqrtf(ss / n_f + p.eps);
#pragma unroll
        for (int k = 0; k < kVecs; ++k) rstd_k[k] = r;
      }

      OT* op = static_cast<OT*>(p.out) + g0;
      ROe* rop = static_cast<ROe*>(p.ro) + g0;
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        if ((vmask >> k) & 1u) {
          float h[8];
          Vec8<X>::load(xs + k * G8, h);
          if constexpr (kRes) {
            float r[8];
            Vec8<RTe>::load(rs + k * G8, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] += r[e];
          }
          if constexpr (kRO) Vec8<ROe>::store(rop + k * G8, h);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = fmaf(h[e] * rstd_k[k], wr[k][e], br[k][e]);
          Vec8<OT>::store(op + k * G8, y);
        }
      }
      if (p.rstd != nullptr) {
        if (pl.seg_mode) {
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            const int v = gl + k * G;
            if (((vmask >> k) & 1u) && (v & (pl.vs - 1)) == 0)
              p.rstd[row * pl.heads + (v >> pl.vs_shift)] = rstd_k[k];
          }
        } else if (gl == 0 && rank == 0) {
          p.rstd[row] = rstd_k[0];
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
}

// =======================================================================================
// Backward: dx in one pass from the saved rstd; dweight / dbias per-CTA partial rows.
// =======================================================================================
template <typename X, typename DY, typename DROT>
__device__ __forceinline__ void bwd_issue(const BwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                          unsigned char* smem, int64_t tile, int s,
                                          int64_t slice_elt0, int rstd_per_row, uint64_t pol) {
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
  const uint32_t b2 = Present<DROT>::value ? static_cast<uint32_t>(rows) * pl.row_bytes[2] : 0u;
  mbar_arrive_expect_tx(&L.full[s], b0 + b1 + b2);
  const int64_t e0 = row0 * pl.W + slice_elt0;
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, b0, &L.full[s], pol);
  bulk_load(st + pl.off[1], static_cast<const DY*>(p.dy) + e0, b1, &L.full[s], pol);
  if constexpr (Present<DROT>::value)
    bulk_load(st + pl.off[2], static_cast<const DROT*>(p.dro) + e0, b2, &L.full[s], pol);
}

// Split-row pipeline: sub-chunk j of the row slice of tile `tile` into ring slot `slot`;
// sub-chunk 0 also brings the row's rstd.
template <typename X, typename DY, typename DROT>
__device__ __forceinline__ void bwd_issue_chunk(const BwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                                unsigned char* smem, int64_t tile, int j, int slot,
                                                int64_t slice_elt0, uint64_t pol) {
  unsigned char* st = smem + static_cast<size_t>(slot) * pl.stage_bytes;
  fence_proxy_async_smem();
  if (j == 0) {
    cp_async_4(st + pl.off[3], p.rstd + tile);
    cp_async_arrive(&L.full[slot]);
  }
  const uint32_t b0 = pl.row_bytes[0];
  const uint32_t b1 = pl.row_bytes[1];
  const uint32_t b2 = Present<DROT>::value ? pl.row_bytes[2] : 0u;
  mbar_arrive_expect_tx(&L.full[slot], b0 + b1 + b2);
  const int64_t e0 = tile * pl.W + slice_elt0 + static_cast<int64_t>(j) * (pl.vslice / pl.K) * 8;
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, b0, &L.full[slot], pol);
  bulk_load(st + pl.off[1], static_cast<const DY*>(p.dy) + e0, b1, &L.full[slot], pol);
  if constexpr (Present<DROT>::value)
    bulk_load(st + pl.off[2], static_cast<const DROT*>(p.dro) + e0, b2, &L.full[slot], pol);
}

// X: saved input dtype; DY: dout dtype; DXT: dx dtype; DROT: dresidual_out dtype (NoT =
// none); DREST: dresidual dtype (NoT = not written).
template <typename X, typename DY, typename DXT, typename DROT, typename DREST, bool kHasDb, int kVecs,
          int kBlock, int kMinBlocks>
__global__ void __launch_bounds__(kBlock, kMinBlocks) bwd_stream_kernel(const BwdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr bool kDro = Present<DROT>::value;
  constexpr bool kDres = Present<DREST>::value;
  using DROe = Elt<DROT>;
  using DRESe = Elt<DREST>;
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

  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const int rstd_per_row = pl.seg_mode ? pl.heads : 1;
  const uint64_t pol = l2_policy_evict_first();
  int64_t issued = 0;
  if (tid == 0 && pl.P == 1) {
    for (int j = 0; j < pl.S; ++j) {
      const int64_t t = cid + j * ncl;
      if (t >= pl.ntiles) break;
      bwd_issue<X, DY, DROT>(p, pl, L, smem, t, j, slice_elt0, rstd_per_row, pol);
      ++issued;
    }
  }

  const int G = pl.G;
  const int G8 = G * 8;
  const int gid = tid / G;
  const int gl = tid - gid * G;
  const bool in_group = gid < pl.rps;
  const float n_f = static_cast<float>(pl.N);
  unsigned vmask = 0;
#pragma unroll
  for (int k = 0; k < kVecs; ++k)
    if (in_group && gl + k * G < pl.vslice) vmask |= 1u << k;

  float wr[kVecs][8];
  float dw[kVecs][8];
  float db[kHasDb ? kVecs : 1][8];
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    const int64_t c = slice_elt0 + static_cast<int64_t>(gl + k * G) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) { wr[k][e] = 1.f; dw[k][e] = 0.f; }
    if constexpr (kHasDb) {
#pragma unroll
      for (int e = 0; e < 8; ++e) db[kHasDb ? k : 0][e] = 0.f;
    }
    if (((vmask >> k) & 1u) && p.w != nullptr) load8_rt(p.w, p.w_dt, p.w_per_head ? c : c % pl.N, wr[k], true);
  }

  bool failed = false;
  int64_t i = 0;
  if (pl.P > 1) {
    // ------------- split-row pipeline (row slices across a cluster, R = 1) -------------
    // As in the forward: K sub-chunks per row slice through an S-slot ring; pass 1 of row
    // i (dot product, dweight/dbias accumulation) overlaps the cluster exchange of row
    // i-1, whose pass 2 (dx) follows.
    const int K = pl.K;
    const int S = pl.S;
    const int kpc_mask = (1 << pl.kpc_shift) - 1;
    const int64_t n_local = cid < pl.ntiles ? (pl.ntiles - 1 - cid) / ncl + 1 : 0;
    const int64_t total_q = n_local * K;
    const bool grp = tid < G;
    int iss_slot = 0, iss_j = 0;
    int64_t iss_tile = cid;
    auto issue_upto = [&](int64_t lim) {
      while (issued < lim) {
        bwd_issue_chunk<X, DY, DROT>(p, pl, L, smem, iss_tile, iss_j, iss_slot, slice_elt0, pol);
        ++issued;
        if (++iss_slot == S) iss_slot = 0;
        if (++iss_j == K) { iss_j = 0; iss_tile += ncl; }
      }
    };
    if (tid == 0) issue_upto(min(total_q, static_cast<int64_t>(S)));
    auto slot_base = [&](int base, int k) -> const unsigned char* {
      int sl = base + (k >> pl.kpc_shift);
      if (sl >= S) sl -= S;
      return smem + static_cast<size_t>(sl) * pl.stage_bytes;
    };
    int row_slot = 0;
    uint32_t row_phase = 0;
    for (; i < n_local + pl.lag; ++i) {
      bool ok = true;
      if (i < n_local) {
        for (int j = 0; j < K; ++j) {
          int sl = row_slot + j;
          uint32_t ph = row_phase;
          if (sl >= S) { sl -= S; ph ^= 1u; }
          ok = mbar_wait(&L.full[sl], ph, kSiteBwdFull) && ok;
        }
      }
      if (__syncthreads_or(!ok || failed)) { failed = true; break; }
      if (grp) {
        const int xo = gl * 8;
        if (i < n_local) {
          const float r = *reinterpret_cast<const float*>(slot_base(row_slot, 0) + pl.off[3]);
          float dot = 0.f;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            if ((vmask >> k) & 1u) {
              const int vo = xo + (k & kpc_mask) * G8;
              const unsigned char* sb = slot_base(row_slot, k);
              float xv[8], dv[8];
              Vec8<X>::load(reinterpret_cast<const X*>(sb + pl.off[0]) + vo, xv);
              Vec8<DY>::load(reinterpret_cast<const DY*>(sb + pl.off[1]) + vo, dv);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float xh = xv[e] * r;
                dot = fmaf(xh, dv[e] * wr[k][e], dot);
                dw[k][e] = fmaf(dv[e], xh, dw[k][e]);
                if constexpr (kHasDb) db[kHasDb ? k : 0][e] += dv[e];
              }
            }
          }
          dot = group_sum(dot, pl, L, 0, gl, static_cast<uint32_t>(i));
          cluster_send(dot, pl, L, gl, static_cast<uint32_t>(i), rank);
        }
        const int64_t r2 = i - pl.lag;
        if (r2 >= 0 && r2 < n_local) {
          int base2 = row_slot - pl.lag * K;
          if (base2 < 0) base2 += S;
          float tot;
          if (!cluster_recv(tot, pl, L, 0, gl, static_cast<uint32_t>(r2), kSiteBwdCluster)) {
            failed = true;
          } else {
            const float c = tot / n_f;
            const float r = *reinterpret_cast<const float*>(slot_base(base2, 0) + pl.off[3]);
            const int64_t g0 = (cid + r2 * ncl) * pl.W + slice_elt0 + xo;
            DXT* dxp = static_cast<DXT*>(p.dx) + g0;
            DRESe* drp = static_cast<DRESe*>(p.dres) + g0;
#pragma unroll
            for (int k = 0; k < kVecs; ++k) {
              if ((vmask >> k) & 1u) {
                const int vo = xo + (k & kpc_mask) * G8;
                const unsigned char* sb = slot_base(base2, k);
                float xv[8], dv[8], g[8];
                Vec8<X>::load(reinterpret_cast<const X*>(sb + pl.off[0]) + vo, xv);
                Vec8<DY>::load(reinterpret_cast<const DY*>(sb + pl.off[1]) + vo, dv);
#pragma unroll
                for (int e = 0; e < 8; ++e) g[e] = (dv[e] * wr[k][e] - (xv[e] * r) * c) * r;
                if constexpr (kDro) {
                  float a[8];
                  Vec8<DROe>::load(reinterpret_cast<const DROe*>(sb + pl.off[2]) + vo, a);
#pragma unroll
                  for (int e = 0; e < 8; ++e) g[e] += a[e];
                }
                Vec8<DXT>::store(dxp + k * G8, g);
                if constexpr (kDres) Vec8<DRESe>::store(drp + k * G8, g);
              }
            }
          }
        }
      }
      __syncthreads();  // pass 2 of row i - lag is done: its slots are free
      if (tid == 0) issue_upto(min(total_q, max(static_cast<int64_t>(0), i + 1 - pl.lag) * K + S));
      if (i < n_local) {
        row_slot += K;
        if (row_slot >= S) { row_slot -= S; row_phase ^= 1u; }
      }
    }
    failed = __syncthreads_or(failed);
    if (failed) {
      if (tid == 0) drain_ring(pl, L, i * K, issued);
      return;
    }
  } else {
  const int x_stride = static_cast<int>(pl.row_bytes[0] / sizeof(X));
  uint32_t seq = 0;
  for (int64_t tile = cid; tile < pl.ntiles; tile += ncl, ++i) {
    const int s = static_cast<int>(i % pl.S);
    const bool ok = mbar_wait(&L.full[s], static_cast<uint32_t>(i / pl.S) & 1u, kSiteBwdFull);
    if (__syncthreads_or(!ok || failed)) { failed = true; break; }
    if (tid == 0 && i > 0 && pl.S > 1) {
      const int64_t t = cid + (i - 1 + pl.S) * ncl;
      if (t < pl.ntiles) {
        bwd_issue<X, DY, DROT>(p, pl, L, smem, t, static_cast<int>((i - 1) % pl.S), slice_elt0, rstd_per_row, pol);
        ++issued;
      }
    }
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const X* xs0 = reinterpret_cast<const X*>(st + pl.off[0]) + gl * 8;
    const DY* ds0 = reinterpret_cast<const DY*>(st + pl.off[1]) + gl * 8;
    const DROe* as0 = reinterpret_cast<const DROe*>(st + pl.off[2]) + gl * 8;
    const float* rs_stage = reinterpret_cast<const float*>(st + pl.off[3]);
    const int64_t row0 = tile * pl.R;
    const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
    for (int sw = 0; sw < pl.R; sw += pl.rps) {
      const int lr = sw + gid;
      const bool active = in_group && lr < rows;
      const unsigned amask = __ballot_sync(0xffffffffu, active);
      if (!active) continue;
      const X* xs = xs0 + lr * x_stride;
      const DY* ds = ds0 + lr * x_stride;
      const DROe* as = as0 + lr * x_stride;
      const int64_t g0 = (row0 + lr) * pl.W + slice_elt0 + gl * 8;

      float rstd_k[kVecs];
      float part[kVecs];
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        part[k] = 0.f;
        rstd_k[k] = 0.f;
        if ((vmask >> k) & 1u) {
          const float r = rs_stage[lr * rstd_per_row + (pl.seg_mode ? ((gl + k * G) >> pl.vs_shift) : 0)];
          rstd_k[k] = r;
          float xv[8], dv[8];
          Vec8<X>::load(xs + k * G8, xv);
          Vec8<DY>::load(ds + k * G8, dv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float xh = xv[e] * r;
            part[k] = fmaf(xh, dv[e] * wr[k][e], part[k]);
            dw[k][e] = fmaf(dv[e], xh, dw[k][e]);
            if constexpr (kHasDb) db[kHasDb ? k : 0][e] += dv[e];
          }
        }
      }

      float c_k[kVecs];
      if (pl.seg_mode) {
#pragma unroll
        for (int k = 0; k < kVecs; ++k) c_k[k] = seg_sum(part[k], pl.vs, amask) / n_f;
      } else {
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) dot += part[k];
        dot = group_sum(dot, pl, L, gid, gl, seq);
        if (pl.P > 1 && !cluster_sum(dot, pl, L, gid, gl, seq, rank, kSiteBwdCluster)) {
          failed = true;
          ++seq;
          break;
        }
        ++seq;
        const float c = dot / n_f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) c_k[k] = c;
      }

      DXT* dxp = static_cast<DXT*>(p.dx) + g0;
      DRESe* drp = static_cast<DRESe*>(p.dres) + g0;
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        if ((vmask >> k) & 1u) {
          const float r = rstd_k[k];
          float xv[8], dv[8], g[8];
          Vec8<X>::load(xs + k * G8, xv);
          Vec8<DY>::load(ds + k * G8, dv);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] = (dv[e] * wr[k][e] - (xv[e] * r) * c_k[k]) * r;
          if constexpr (kDro) {
            float a[8];
            Vec8<DROe>::load(as + k * G8, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] += a[e];
          }
          Vec8<DXT>::store(dxp + k * G8, g);
          if constexpr (kDres) Vec8<DRESe>::store(drp + k * G8, g);
        }
      }
    }
    if (pl.S == 1) {
      __syncthreads();
      const int64_t t = cid + (i + 1) * ncl;
      if (tid == 0 && t < pl.ntiles) {
        bwd_issue<X, DY, DROT>(p, pl, L, smem, t, 0, slice_elt0, rstd_per_row, pol);
        ++issued;
      }
    }
  }
  failed = __syncthreads_or(failed);
  if (failed) {
    if (tid == 0) drain_ring(pl, L, i, issued);
    return;
  }
  }  // tile loop

  // one partial row per (cluster, row group): the groups of a CTA own the same columns.
  // Every owned column is written, zeros included, so the reduction reads no stale data.
  const int64_t pbase = (cid * pl.rps + gid) * pl.W + slice_elt0 + gl * 8;
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    if ((vmask >> k) & 1u) {
      if (p.dw_part != nullptr) Vec8<float>::store(p.dw_part + pbase + k * G8, dw[k]);
      if constexpr (kHasDb) {
        if (p.db_part != nullptr) Vec8<float>::store(p.db_part + pbase + k * G8, db[kHasDb ? k : 0]);
      }
    }
  }
}

}  // namespace rmsb200
