// stream_kernels.cuh -- the persistent, TMA-staged forward (RMSNorm and LayerNorm) and
// backward kernels.
//
// Structure:
//   * one CTA of 512 threads per SM (or 256 threads, two per SM, for some backwards),
//     persistent over tiles assigned round-robin (local tile q of CTA group c is tile
//     c + q * groups);
//   * tiles stream HBM -> shared memory with cp.async.bulk (TMA bulk copies, no tensor map,
//     no multicast; one copy per tensor per tile) into an S-slot ring; each slot's "full"
//     mbarrier counts the landing bytes. There is no CTA-wide barrier per tile: every warp
//     waits on the slot's mbarrier, and when it is done with the slot it bumps the slot's
//     shared-memory counter; the last warp to finish refills the slot with tile q + S;
//   * threads read 8-element vectors from shared memory and reduce each row:
//       - per-head rows of up to 32 vectors ("seg" mode): xor shuffles inside a lane
//         segment, transposed so a thread's values for several heads share the levels;
//         per-head super-rows of up to 2 x T vectors run in column mode (kCols < kVecs:
//         a thread owns 1-2 vector columns across several super-rows of the sweep, so
//         fewer weight / bias / dweight registers stay live);
//       - whole rows ("row" mode): warp shuffles and one named barrier per row group, or,
//         for pipelined rows, split-phase reductions through per-group mbarriers so the
//         output pass of the previous row hides the wait (LayerNorm always, RMSNorm
//         forwards with several row groups per CTA);
//       - rows split over P CTAs: warp 0 sends the CTA's total to the peers (st.async into
//         the cluster's shared memory, or tagged 64-bit records in global memory for
//         groups of a cooperative grid) and every warp sums the P totals; pass 1 of row i
//         and its exchange overlap pass 2 of row i - lag;
//     then they re-read the slot and write outputs with 16-byte streaming stores;
//   * every launch waits (griddepcontrol.wait) before its first global access, so it may
//     be launched as a programmatic dependent of the previous kernel in the stream;
//   * every per-element dtype, the bias and the LayerNorm mode are template parameters
//     (absent tensors are `NoT`), so the inner loops carry no runtime type dispatch; the
//     arithmetic uses sm_100's paired fp32 instructions where that measured faster;
//   * affine parameters live in registers for the whole kernel (each thread always owns
//     the same columns), so dweight/dbias accumulate in registers and are written once
//     per (CTA group, row group) as a partial row; a second kernel sums the partials in a
//     fixed order.
// Every wait is bounded. A wait that gives up records an error in the device status word;
// from then on every wait of every CTA returns at once, so the kernel runs to its end on
// the same control flow (results undefined, status reported), lets its in-flight copies
// land, and exits.
#pragma once

#include <type_traits>

#include "device_common.cuh"
#include "stream_plan.h"

namespace rmsb200 {

constexpr int kXSlots = 8;  // cluster exchange slots (row sequence number mod 8)
constexpr int kMaxLag = 3;  // deepest exchange lag the slots allow: kXSlots >= 2 * lag + 2

constexpr int kGroupRed = 4;  // split-phase reductions per row group: 2 statistics x 2 rows in flight

// Dynamic shared memory (rmsb_dyn_smem, declared with the device helpers): the S ring
// stages, then the barrier / reduction area laid out by carve_smem.

// Byte offset, within the area after the stages, of the global-memory exchange's tag base
// (after full, xbar, xpart, red, done, gbar and gpart).
constexpr uint32_t kXTagOff = kMaxStages * 8 + kXSlots * 8 + kXSlots * kMaxCluster * 4 + 64 * 4 + kMaxStages * 4 +
                              16 * kGroupRed * 8 + kGroupRed * 16 * 4;
static_assert(kXTagOff + 8 <= kSmemReserve, "barrier area exceeds its reserve");

struct SmemLayout {
  uint64_t* full;   // [kMaxStages] slot filled
  uint64_t* xbar;   // [kXSlots] cluster exchange barriers
  float* xpart;     // [kXSlots][kMaxCluster] row totals of the cluster's CTAs
  float* red;       // [2][32] per-warp partials (double buffered)
  int* done;        // [kMaxStages] warps finished with the slot's current tile
  uint64_t* gbar;   // [16 groups][kGroupRed] split-phase row-group reductions (LayerNorm)
  float* gpart;     // [kGroupRed][16 warps] their per-warp partials
  uint32_t* xgen;   // [1] the execution generation of the global-memory exchange
  uint32_t* tmem;   // [1] TMEM address of the backward's accumulators (kTmemAcc kernels)
};

__device__ __forceinline__ SmemLayout carve_smem(unsigned char* smem, const StreamPlan& pl) {
  SmemLayout L;
  unsigned char* tail = smem + static_cast<size_t>(pl.S) * pl.stage_bytes;
  L.full = reinterpret_cast<uint64_t*>(tail);
  L.xbar = L.full + kMaxStages;
  L.xpart = reinterpret_cast<float*>(L.xbar + kXSlots);
  L.red = L.xpart + kXSlots * kMaxCluster;
  L.done = reinterpret_cast<int*>(L.red + 64);
  L.gbar = reinterpret_cast<uint64_t*>(L.done + kMaxStages);
  L.gpart = reinterpret_cast<float*>(L.gbar + 16 * kGroupRed);
  L.xgen = reinterpret_cast<uint32_t*>(tail + kXTagOff);
  L.tmem = L.xgen + 1;
  return L;
}

__device__ __forceinline__ void init_barriers(const SmemLayout& L, const StreamPlan& pl, bool group_red = false) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < pl.S; ++s) {
      mbar_init(&L.full[s], 1);
      L.done[s] = 0;
    }
    for (int s = 0; s < kXSlots; ++s) mbar_init(&L.xbar[s], 1);
    if (group_red)  // one arrival per warp of the row group
      for (int g = 0; g < pl.rps; ++g)
        for (int j = 0; j < kGroupRed; ++j) mbar_init(&L.gbar[g * kGroupRed + j], pl.G >> 5);
    fence_mbar_init();
  }
  __syncthreads();
  if (pl.P > 1 && pl.xmode == kXCluster) cluster_sync_all();
}

// Called by every lane of a warp after its last read of slot s. Returns true on lane 0 of
// the warp that finishes the slot last; that lane refills it.
__device__ __forceinline__ bool release_slot(const SmemLayout& L, int s, int nwarps) {
  __syncwarp();
  bool last = false;
  if ((threadIdx.x & 31) == 0) {
    __threadfence_block();
    if (atomicAdd(&L.done[s], 1) == nwarps - 1) {
      L.done[s] = 0;  // no warp can finish the slot's next tile before it is issued below
      __threadfence_block();
      last = true;
    }
  }
  return last;
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

// Split-phase row-group reduction (pipelined rows): group_post stores the warp's partial
// for reduction slot j and arrives on the group's mbarrier without waiting; group_take
// waits (bounded) for all warps of the group and sums their partials in warp order (same
// bits in every thread). The slot's k-th use completes phase k. Slots are reused only
// after every warp has read them: LayerNorm uses slots {mean, variance} x row parity (its
// two reductions per row order the warps); the one-reduction loops, where a warp posts row
// q before it takes row q-1, use row mod 4 (a warp posts row q+4 after taking row q+2,
// which needed every warp's post of row q+2, made after its take of row q).
__device__ __forceinline__ void group_post(float v, const SmemLayout& L, int gid, int warp, int lane, int j) {
  v = warp_sum(v);
  if (lane == 0) {
    L.gpart[j * 16 + warp] = v;
    mbar_arrive(&L.gbar[gid * kGroupRed + j]);
  }
}

__device__ __forceinline__ float group_take(const StreamPlan& pl, const SmemLayout& L, int gid, int lane, int j,
                                            uint32_t use) {
  mbar_wait(&L.gbar[gid * kGroupRed + j], use & 1u, kSiteFwdCluster);
  const int nw = pl.G >> 5;
  return warp_sum(lane < nw ? L.gpart[j * 16 + gid * nw + lane] : 0.f);
}

// Combining (mean, M2 = sum of squared deviations) of two sets of c samples each (Chan et
// al.'s parallel variance update with equal counts): mean = (m_a + m_b) / 2, M2 = M2_a +
// M2_b + (m_b - m_a)^2 c / 2. It is symmetric in its two operands (a + b, the square of a
// difference), so the lanes of an xor butterfly all end with identical bits, and it needs
// no division. `c` doubles at every level.
__device__ __forceinline__ void stats_combine_equal(float& m, float& M2, float mo, float M2o, float c) {
  const float d = mo - m;
  M2 = (M2 + M2o) + d * d * (0.5f * c);
  m = (m + mo) * 0.5f;
}

// Butterfly over lanes [0, width) (width a power of two): every lane ends with the (mean,
// M2) of the width lanes' sets of c samples each.
__device__ __forceinline__ void lanes_stats(float& m, float& M2, float c, int width) {
  for (int off = width >> 1; off > 0; off >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, off);
    const float M2o = __shfl_xor_sync(0xffffffffu, M2, off);
    stats_combine_equal(m, M2, mo, M2o, c);
    c *= 2.f;
  }
}

// Cluster exchange of a row total (rows split over the P CTAs of a cluster, one row group
// per CTA). cluster_send (warp 0): lane 0 stores this CTA's total locally and arms the
// slot's mbarrier for the P-1 peer totals; lane q != rank stores it into peer q's slot with
// st.async, completing 4 tx-bytes on the peer's mbarrier. cluster_recv (every warp): waits
// (bounded) for the slot and sums the P totals with one shuffle tree, so every warp of
// every CTA of the cluster gets the same bits. With an exchange lag of L rows (row r is
// received in iteration r + L), kXSlots >= 2L + 2 slots (row number mod kXSlots) are
// enough: a peer posts row r in iteration r, after it received this CTA's row r - L - 1,
// which warp 0 sends in iteration r - L - 1 only after every warp of this CTA has
// finished iteration r - L - 2 (the row group's named barrier in group_sum orders them)
// and so has read row r - 2L - 2 <= r - kXSlots out of the slot.
// Where the exchange goes through global memory (kXGlobal), the group's CTAs are CTAs
// cta0 .. cta0+P-1 of one cooperative grid (all resident at once). cluster_send: lane 0 of
// warp 0 writes the CTA's total and the row's tag as one 64-bit word into its record for
// the slot. Every warp reads the P records itself (lane q reads rank q's): xrec_load is
// issued a whole pass ahead (at the top of the iteration that receives the row), and
// cluster_recv re-reads (bounded) until all P words carry the row's tag, then sums the
// totals with the same shuffle tree as above. The slot argument above covers the records:
// with lag <= kMaxLag a CTA rewrites its record for row r only after every warp of every
// peer has read its row r - kXSlots, so a reader finds row r's word or row r - kXSlots's.
// Across executions: records are never cleared, so every execution tags its words with a
// generation of its own (xgen_begin). A host-side value baked into the launch parameters
// would not do: a CUDA graph replays the same parameters, and a reader running ahead of its
// peer would then take the previous replay's word for the same row as this one's.
struct XCtx {
  XRecord* rec;      // this launch's record set
  int64_t cta0;      // first CTA of the group
};

// Tag of row `seq`: the execution's tag base (0x80000000 | generation << 1, stored in
// shared memory by xgen_begin and addressed from the plan, so no register holds it across
// the kernel) | bit 0 of seq / kXSlots.
__device__ __forceinline__ uint32_t xrec_tag(const StreamPlan& pl, uint32_t seq) {
  const uint32_t base =
      *reinterpret_cast<const uint32_t*>(rmsb_dyn_smem + static_cast<size_t>(pl.S) * pl.stage_bytes + kXTagOff);
  return base | ((seq / kXSlots) & 1u);
}

// Draws this execution's generation for CTA group `cid` (kXGlobal; every thread of the
// CTA calls it, after pdl_wait). The group's counter (one per group of this P) gets one
// increment from each of its P CTAs per execution, so the P CTAs of one execution all read
// old values in [g * P, (g + 1) * P): the same generation g, with no wait among them. This
// holds as long as two executions that share a record set and a group do not run at the
// same time on the GPU (launches of one stream never do; the host hands consecutive
// launches different record sets). The tag base is kept in shared memory, not in a
// register for the whole kernel.
__device__ __forceinline__ void xgen_begin(const StreamPlan& pl, const SmemLayout& L, uint32_t* xgen, int64_t cid) {
  if (pl.P <= 1 || pl.xmode != kXGlobal) return;
  if (threadIdx.x == 0) {
    const uint32_t g = atomicAdd(xgen + cid, 1u) / static_cast<uint32_t>(pl.P);
    *L.xgen = 0x80000000u | ((g & 0x3fffffffu) << 1);
  }
  __syncthreads();
}

__device__ __forceinline__ XRecord xrec_load(const StreamPlan& pl, const XCtx& xc, int lane, uint32_t seq) {
  if (pl.xmode != kXGlobal || lane >= pl.P) return 0ull;
  return ld_relaxed_u64(xc.rec + (xc.cta0 + lane) * kXSlots + (seq & (kXSlots - 1)));
}

__device__ __forceinline__ void cluster_send(float v, const StreamPlan& pl, const SmemLayout& L, const XCtx& xc,
                                             int warp, int lane, uint32_t seq, uint32_t rank) {
  if (warp != 0) return;
  const uint32_t slot = seq & (kXSlots - 1);
  if (pl.xmode == kXGlobal) {
    if (lane == 0)
      st_relaxed_u64(xc.rec + (xc.cta0 + rank) * kXSlots + slot,
                     (static_cast<unsigned long long>(xrec_tag(pl, seq)) << 32) | __float_as_uint(v));
    return;
  }
  float* xp = L.xpart + slot * kMaxCluster;
  if (lane == 0) {
    xp[rank] = v;
    mbar_arrive_expect_tx(&L.xbar[slot], static_cast<uint32_t>(pl.P - 1) * 4u);
  }
  if (lane < pl.P && lane != static_cast<int>(rank))
    st_async_peer(map_peer(smem_u32(&xp[rank]), lane), v, map_peer(smem_u32(&L.xbar[slot]), lane));
}

// `pre`: this lane's xrec_load for the row (kXGlobal). With pl.xbcast, warp 0 alone polls
// the records and posts the total into the slot's xpart word, arriving on its xbar (both
// otherwise unused by the global exchange); the other warps wait there. The slot's k-th use
// completes phase k; the CTA-wide row sum before every exchange keeps the warps within a
// row of each other, so no warp is a whole slot cycle (8 rows) behind.
// kBcast = false compiles the broadcast out (kernels the planner never gives pl.xbcast).
template <bool kBcast = true>
__device__ __forceinline__ float cluster_recv(const StreamPlan& pl, const SmemLayout& L, const XCtx& xc, int warp,
                                              int lane, uint32_t seq, XRecord pre, int site) {
  const uint32_t slot = seq & (kXSlots - 1);
  if (pl.xmode == kXGlobal) {
    if (kBcast && pl.xbcast && warp != 0) {
      mbar_wait(&L.xbar[slot], (seq / kXSlots) & 1u, site);
      return L.xpart[slot * kMaxCluster];
    }
    const uint32_t want = xrec_tag(pl, seq);
    XRecord w = pre;
    uint64_t t0 = 0;
    while (!__all_sync(0xffffffffu, lane >= pl.P || static_cast<uint32_t>(w >> 32) == want)) {
      if (abort_requested()) break;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > g_wait_timeout_ns) {
        if (lane == 0) record_error(RMSNORM_B200_ERR_DEVICE_TIMEOUT, site);
        break;
      }
      __nanosleep(20);
      w = xrec_load(pl, xc, lane, seq);
    }
    const float tot = warp_sum(lane < pl.P ? __uint_as_float(static_cast<uint32_t>(w)) : 0.f);
    if (kBcast && pl.xbcast && lane == 0) {
      L.xpart[slot * kMaxCluster] = tot;
      mbar_arrive(&L.xbar[slot]);
    }
    return tot;
  }
  mbar_wait<true>(&L.xbar[slot], (seq / kXSlots) & 1u, site);
  const float* xp = L.xpart + slot * kMaxCluster;
  return warp_sum(lane < pl.P ? xp[lane] : 0.f);
}

// Row pairs (forward split rows, P <= 16): the records of rows seq_a (lanes 0..15) and
// seq_a + 1 (lanes 16..31), lane q of each half reading CTA q's record.
__device__ __forceinline__ XRecord xrec_load2(const StreamPlan& pl, const XCtx& xc, int lane, uint32_t seq_a) {
  const int q = lane & 15;
  if (pl.xmode != kXGlobal || q >= pl.P) return 0ull;
  const uint32_t seq = seq_a + static_cast<uint32_t>(lane >> 4);
  return ld_relaxed_u64(xc.rec + (xc.cta0 + q) * kXSlots + (seq & (kXSlots - 1)));
}

// Group totals of rows seq_a and (hb) seq_a + 1. Global records: one bounded poll of both
// rows' records (`pre`: this lane's xrec_load2), then the half-warp sums. warp_sum over a
// row's P values in lanes 0..P-1 adds zeros at its first level (offset 16) and then runs
// offsets 8..1 over the 16 lanes, so the 16-lane sums here give the same bits as
// cluster_recv. Cluster exchange: the two rows one after the other.
// With pl.xbcast, warp 0 alone polls and posts both totals as cluster_recv does.
__device__ __forceinline__ void cluster_recv2(const StreamPlan& pl, const SmemLayout& L, const XCtx& xc, int warp,
                                              int lane, uint32_t seq_a, bool hb, XRecord pre, int site, float& ta,
                                              float& tb) {
  if (pl.xmode == kXGlobal) {
    const uint32_t slot_a = seq_a & (kXSlots - 1);
    const uint32_t slot_b = (seq_a + 1) & (kXSlots - 1);
    if (pl.xbcast && warp != 0) {
      mbar_wait(&L.xbar[slot_a], (seq_a / kXSlots) & 1u, site);
      ta = L.xpart[slot_a * kMaxCluster];
      tb = 0.f;
      if (hb) {
        mbar_wait(&L.xbar[slot_b], ((seq_a + 1) / kXSlots) & 1u, site);
        tb = L.xpart[slot_b * kMaxCluster];
      }
      return;
    }
    const bool mine = (lane & 15) < pl.P && (lane < 16 || hb);
    const uint32_t want = xrec_tag(pl, seq_a + static_cast<uint32_t>(lane >> 4));
    XRecord w = pre;
    uint64_t t0 = 0;
    while (!__all_sync(0xffffffffu, !mine || static_cast<uint32_t>(w >> 32) == want)) {
      if (abort_requested()) break;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > g_wait_timeout_ns) {
        if (lane == 0) record_error(RMSNORM_B200_ERR_DEVICE_TIMEOUT, site);
        break;
      }
      __nanosleep(20);
      w = xrec_load2(pl, xc, lane, seq_a);
    }
    float v = mine ? __uint_as_float(static_cast<uint32_t>(w)) : 0.f;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    ta = __shfl_sync(0xffffffffu, v, 0);
    tb = __shfl_sync(0xffffffffu, v, 16);
    if (pl.xbcast && lane == 0) {
      L.xpart[slot_a * kMaxCluster] = ta;
      mbar_arrive(&L.xbar[slot_a]);
      if (hb) {
        L.xpart[slot_b * kMaxCluster] = tb;
        mbar_arrive(&L.xbar[slot_b]);
      }
    }
    return;
  }
  ta = cluster_recv<false>(pl, L, xc, 0, lane, seq_a, 0ull, site);  // cluster exchange
  tb = hb ? cluster_recv<false>(pl, L, xc, 0, lane, seq_a + 1, 0ull, site) : 0.f;
}

// Two rows' CTA-wide sums behind one barrier (split rows: one row group, gid 0). `buf`
// holds 64 floats (row a's warp partials, then row b's), double-buffered by the caller.
// The arithmetic is group_sum's, row by row.
__device__ __forceinline__ void group_sum2(float& a, float& b, const StreamPlan& pl, float* buf, int gl) {
  a = warp_sum(a);
  b = warp_sum(b);
  if (pl.G > 32) {
    const int nw = pl.G >> 5;
    const int lane = gl & 31;
    if (lane == 0) {
      buf[gl >> 5] = a;
      buf[32 + (gl >> 5)] = b;
    }
    named_barrier(1, pl.G);
    a = warp_sum(lane < nw ? buf[lane] : 0.f);
    b = warp_sum(lane < nw ? buf[32 + lane] : 0.f);
  }
}

// xor-shuffle sum over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float seg_sum(float v, int width, unsigned mask) {
  for (int off = width >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(mask, v, off);
  return v;
}

// Sums each of a thread's kV values over its aligned segment of `vs` lanes (the lanes own
// the same position in kV different segments) and applies `post` to each sum. For kV = 4
// or 2 and vs >= kV the reduction is transposed: the first butterfly levels split the
// values between lane halves, so log2(vs) shuffles finish all kV sums, each lane applies
// `post` to the one sum it holds, and kV shuffles hand every lane all kV results (instead
// of kV * log2(vs) shuffles and kV posts). Lanes holding the same sum combined the same
// partials by commutative additions, so every lane of a segment gets the same bits.
template <int kV, typename Post>
__device__ __forceinline__ void seg_reduce(const float (&v)[kV], float (&out)[kV], int vs, unsigned mask, Post post) {
  const int lane = threadIdx.x & 31;
  if constexpr (kV == 4 || kV == 2) {
    if (vs >= kV) {
      const int h1 = vs >> 1;
      const bool b1 = (lane & h1) != 0;
      float a;
      int done;  // butterfly levels left to run with plain exchanges
      if constexpr (kV == 4) {
        const int h2 = vs >> 2;
        const bool b2 = (lane & h2) != 0;
        // level 1: keep values {0,1} (b1 = 0) or {2,3} (b1 = 1) and send the other pair
        const float p0 = (b1 ? v[2] : v[0]) + __shfl_xor_sync(mask, b1 ? v[0] : v[2], h1);
        const float p1 = (b1 ? v[3] : v[1]) + __shfl_xor_sync(mask, b1 ? v[1] : v[3], h1);
        // level 2: keep one of the two; this lane now sums value 2*b1 + b2
        a = (b2 ? p1 : p0) + __shfl_xor_sync(mask, b2 ? p0 : p1, h2);
        done = h2 >> 1;
      } else {
        a = (b1 ? v[1] : v[0]) + __shfl_xor_sync(mask, b1 ? v[0] : v[1], h1);
        done = h1 >> 1;
      }
      for (int off = done; off > 0; off >>= 1) a += __shfl_xor_sync(mask, a, off);
      const float mine = post(a);
      const int base = lane & ~(vs - 1);
      const int low = lane & ((kV == 4 ? (vs >> 2) : (vs >> 1)) - 1);
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const int sel = kV == 4 ? (((k >> 1) ? (vs >> 1) : 0) | ((k & 1) ? (vs >> 2) : 0)) : (k ? (vs >> 1) : 0);
        out[k] = __shfl_sync(mask, mine, base | sel | low);
      }
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < kV; ++k) out[k] = post(seg_sum(v[k], vs, mask));
}

// After a failure: let every copy still in flight land before the CTA exits (waits bounded
// by time only). The ring held n_units loads (tiles, or row-slice chunks); slot s last held
// unit u_last(s).
__device__ __forceinline__ void drain_after_failure(const StreamPlan& pl, const SmemLayout& L, int64_t n_units) {
  for (int s = 0; s < pl.S && s < n_units; ++s) {
    const int64_t u_last = s + ((n_units - 1 - s) / pl.S) * pl.S;
    mbar_wait(&L.full[s], static_cast<uint32_t>(u_last / pl.S) & 1u, kSiteDrain, false);
  }
}

// Split rows (P > 1) stream as K chunks per row slice: local row i occupies ring units
// i*K .. i*K+K-1 (slot = unit mod S), and thread vector k lies in chunk k >> kpc_shift at
// chunk vector (k & kpc_mask) * G + gl. Chunk j of the row whose first chunk is in slot sb
// (phase phb) is in slot sb + j, wrapping once at most (K <= S).
__device__ __forceinline__ int chunk_slot(int sb, uint32_t phb, int j, int S, uint32_t* ph) {
  int s = sb + j;
  *ph = phb;
  if (s >= S) { s -= S; *ph ^= 1u; }
  return s;
}

template <typename T>
using Elt = typename std::conditional<Present<T>::value, T, float>::type;

// =======================================================================================
// Forward
// =======================================================================================
// Tile `tile` into slot s: R rows (P == 1, contiguous), or chunk j of the row slice of this
// CTA (P > 1; a chunk holds row_bytes[0] / sizeof(X) elements of the slice).
// With pf_tile >= 0, also prefetches tile pf_tile (chunk pf_j) into L2.
template <typename X, typename RT>
__device__ __forceinline__ void fwd_issue(const FwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                          unsigned char* smem, int64_t tile, int j, int s, int64_t slice_elt0,
                                          uint64_t pol, int64_t pf_tile = -1, int pf_j = 0) {
  unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
  const int64_t row0 = tile * pl.R;
  const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
  fence_proxy_async_smem();
  const uint32_t bx = static_cast<uint32_t>(rows) * pl.row_bytes[0];
  const uint32_t br = Present<RT>::value ? static_cast<uint32_t>(rows) * pl.row_bytes[1] : 0u;
  mbar_arrive_expect_tx(&L.full[s], bx + br);
  // P > 1 implies R == 1
  const int64_t e0 = row0 * pl.W + slice_elt0 + static_cast<int64_t>(j) * (pl.row_bytes[0] / sizeof(X));
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, bx, &L.full[s], pol);
  if constexpr (Present<RT>::value)
    bulk_load(st + pl.off[1], static_cast<const RT*>(p.res) + e0, br, &L.full[s], pol);
  if (pf_tile >= 0) {
    const int64_t prow0 = pf_tile * pl.R;
    const uint32_t prows = static_cast<uint32_t>(min(static_cast<int64_t>(pl.R), pl.nrows - prow0));
    const int64_t pe0 = prow0 * pl.W + slice_elt0 + static_cast<int64_t>(pf_j) * (pl.row_bytes[0] / sizeof(X));
    bulk_prefetch_l2(static_cast<const X*>(p.x) + pe0, prows * pl.row_bytes[0]);
    if constexpr (Present<RT>::value)
      bulk_prefetch_l2(static_cast<const RT*>(p.res) + pe0, prows * pl.row_bytes[1]);
  }
}

// X: input dtype; RT: residual dtype (NoT = none); OT: output dtype; ROT: residual_out
// dtype (NoT = not written); kBias: a bias is added (without one, its registers and adds
// are gone: out = h * rstd * w rounds exactly like the fma with a zero bias); kLN:
// LayerNorm instead of RMSNorm (no residual; mean, then the mean of squared deviations
// from the staged tile, out = (x - mean) * rstd * w + b; rows are never split).
template <typename X, typename RT, typename OT, typename ROT, bool kBias, bool kLN, int kVecs, int kBlock,
          int kMinBlocks, int kCols = kVecs>
__global__ void __launch_bounds__(kBlock, kMinBlocks) fwd_stream_kernel(const FwdParams p) {
  // kCols < kVecs: per-head column mode (thread vector k = column k % kCols of super-row
  // k / kCols of the thread's group in the sweep); only the tile loop runs in that mode
  static_assert(kVecs % kCols == 0 && (kCols == kVecs || !kLN), "column mode: RMSNorm tiles only");
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr bool kRes = Present<RT>::value;
  constexpr bool kRO = Present<ROT>::value;
  using RTe = Elt<RT>;
  using ROe = Elt<ROT>;
  const StreamPlan& pl = p.pl;
  const SmemLayout L = carve_smem(smem, pl);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  uint32_t rank = 0;
  int64_t cid = blockIdx.x;
  int64_t ncl = gridDim.x;
  if (pl.P > 1) {
    if (pl.xmode == kXCluster) {
      rank = cluster_ctarank();
      cid = cluster_id_x();
      ncl = cluster_count_x();
    } else {
      rank = blockIdx.x % pl.P;
      cid = blockIdx.x / pl.P;
      ncl = gridDim.x / pl.P;
    }
  }
  constexpr bool kLNMode = kLN;
  // LayerNorm row mode: rows pipelined tile by tile (the planner gives one row per group
  // per tile and at least two slots)
  const bool ln_rows = kLNMode && !pl.seg_mode && pl.R == pl.rps && pl.S >= 2;
  // RMSNorm row mode pipelined the same way (one reduction) when the planner asked for it
  const bool rms_rows = !kLNMode && pl.pipe_rows && !pl.seg_mode && pl.P == 1 && pl.R == pl.rps && pl.S >= 3;
  init_barriers(L, pl, ln_rows || rms_rows);
  pdl_wait();  // every global access of the launch follows this point
  pdl_launch_dependents();
  xgen_begin(pl, L, p.xgen, cid);
  const XCtx xc{p.xrec, cid * pl.P};

  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const uint64_t pol = l2_policy_evict_first();
  const int64_t n_local = cid < pl.ntiles ? (pl.ntiles - 1 - cid) / ncl + 1 : 0;
  const int S = pl.S;
  const int K = pl.K;
  const int kshift = __ffs(K) - 1;
  const int64_t n_units = n_local * K;
  // loads unit u into slot s and prefetches unit u + pf into L2
  auto issue_unit = [&](int64_t u, int s) {
    const int64_t v = u + pl.pf;
    const bool pf = pl.pf > 0 && v < n_units;
    fwd_issue<X, RT>(p, pl, L, smem, cid + (u >> kshift) * ncl, static_cast<int>(u & (K - 1)), s, slice_elt0, pol,
                     pf ? cid + (v >> kshift) * ncl : -1, static_cast<int>(v & (K - 1)));
  };
  if (tid == 0)
    for (int u = 0; u < S && u < n_units; ++u) issue_unit(u, u);

  const int G = pl.G;
  const int G8 = G * 8;
  const int gid = tid / G;
  const int gl = tid - gid * G;
  const bool in_group = gid < pl.rps;
  const int nwarps = (pl.rps * G + 31) >> 5;  // warps with work; the others idle to the end
  const bool active_warp = warp < nwarps;
  const float inv_n = 1.f / static_cast<float>(pl.N);  // mean = sum * (1/N), exact for N a power of two
  unsigned vmask = 0;
#pragma unroll
  for (int k = 0; k < kVecs; ++k)
    if (in_group && gl + (k % kCols) * G < pl.vslice) vmask |= 1u << k;

  // weight / bias of the thread's columns, as float pairs (element 2i in .x, 2i+1 in .y)
  float2 wr[kCols][4];
  float2 br[kBias ? kCols : 1][4];
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int64_t c = slice_elt0 + static_cast<int64_t>(gl + k * G) * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) wr[k][i] = splat2(1.f);
    if constexpr (kBias) {
#pragma unroll
      for (int i = 0; i < 4; ++i) br[kBias ? k : 0][i] = splat2(0.f);
    }
    if ((vmask >> k) & 1u) {
      if (p.w != nullptr) load8p_rt(p.w, p.w_dt, p.w_per_head ? c : c % pl.N, wr[k]);
      if constexpr (kBias) load8p_rt(p.b, p.b_dt, p.b_per_head ? c : c % pl.N, br[kBias ? k : 0]);
    }
  }
  const int xs_stride = static_cast<int>(pl.row_bytes[0] / sizeof(X));  // elements per staged row

  // Per-vector arithmetic. Without a residual the paired fp32 instructions are used; with
  // one (x + residual, residual_out stored) the scalar form measured faster on B200. Both
  // round every operation the same way; only the order of the sum of squares differs.
  constexpr bool kPaired = !kRes;
  // pass 1 of one vector: sum of squares of the pre-norm values h = x (+ residual)
  auto sumsq = [&](const X* xp, const RTe* rp) {
    if constexpr (kPaired) {
      float2 h[4];
      Pair8<X>::load(xp, h);
      float2 acc = mul2(h[0], h[0]);
#pragma unroll
      for (int i = 1; i < 4; ++i) acc = fma2(h[i], h[i], acc);
      return acc.x + acc.y;
    } else {
      float h[8];
      Vec8<X>::load(xp, h);
      if constexpr (kRes) {  // the stage holds a residual slice only when there is a residual
        float r[8];
        Vec8<RTe>::load(rp, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] += r[e];
      }
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(h[e], h[e], acc);
      return acc;
    }
  };
  // pass 2 of thread vector k: residual_out = h, out = h * rstd * w + b
  auto emit = [&](const X* xp, const RTe* rp, OT* op, ROe* rop, float rstd, int k) {
    if constexpr (kPaired) {
      float2 h[4], y[4];
      Pair8<X>::load(xp, h);
      if constexpr (kRO) Pair8<ROe>::store(rop, h);
      const float2 r2 = splat2(rstd);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (kBias) y[i] = fma2(mul2(h[i], r2), wr[k % kCols][i], br[kBias ? k % kCols : 0][i]);
        else y[i] = mul2(mul2(h[i], r2), wr[k % kCols][i]);
      }
      Pair8<OT>::store(op, y);
    } else {
      float h[8], y[8];
      Vec8<X>::load(xp, h);
      if constexpr (kRes) {
        float r[8];
        Vec8<RTe>::load(rp, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] += r[e];
      }
      if constexpr (kRO) Vec8<ROe>::store(rop, h);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float2 w2 = wr[k % kCols][e >> 1];
        const float w = (e & 1) ? w2.y : w2.x;
        if constexpr (kBias) {
          const float2 b2 = br[kBias ? k % kCols : 0][e >> 1];
          y[e] = fmaf(h[e] * rstd, w, (e & 1) ? b2.y : b2.x);
        } else {
          y[e] = (h[e] * rstd) * w;
        }
      }
      Vec8<OT>::store(op, y);
    }
  };

  // pass 2 of one staged row: writes residual_out, out and (row mode) rstd
  auto pass2 = [&](const X* xs, const RTe* rs, int64_t row, const float (&rstd_k)[kVecs]) {
    const int64_t g0 = row * pl.W + slice_elt0 + gl * 8;
    OT* op = static_cast<OT*>(p.out) + g0;
    ROe* rop = static_cast<ROe*>(p.ro) + g0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k)
      if ((vmask >> k) & 1u) emit(xs + k * G8, rs + k * G8, op + k * G8, rop + k * G8, rstd_k[k], k);
  };
  auto pass1 = [&](const X* xs, const RTe* rs, float (&part)[kVecs]) {
#pragma unroll
    for (int k = 0; k < kVecs; ++k) part[k] = ((vmask >> k) & 1u) ? sumsq(xs + k * G8, rs + k * G8) : 0.f;
  };
  auto stage_x = [&](int s) {
    return reinterpret_cast<const X*>(smem + static_cast<size_t>(s) * pl.stage_bytes + pl.off[0]) + gl * 8;
  };
  auto stage_r = [&](int s) {
    return reinterpret_cast<const RTe*>(smem + static_cast<size_t>(s) * pl.stage_bytes + pl.off[1]) + gl * 8;
  };
  // LayerNorm per-vector passes: sum, sum of squared deviations from the mean, output
  auto ln_sum = [&](const X* xp) {
    float2 h[4];
    Pair8<X>::load(xp, h);
    const float2 a = add2(add2(h[0], h[1]), add2(h[2], h[3]));
    return a.x + a.y;
  };
  auto ln_dev = [&](const X* xp, float mean) {
    float2 h[4];
    Pair8<X>::load(xp, h);
    const float2 nm = splat2(-mean);
    float2 d = add2(h[0], nm);
    float2 a = mul2(d, d);
#pragma unroll
    for (int i = 1; i < 4; ++i) {
      d = add2(h[i], nm);
      a = fma2(d, d, a);
    }
    return a.x + a.y;
  };
  auto ln_emit = [&](const X* xp, OT* op, float mean, float rstd, int k) {
    float2 h[4], y[4];
    Pair8<X>::load(xp, h);
    const float2 nm = splat2(-mean), r2 = splat2(rstd);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xh = mul2(add2(h[i], nm), r2);
      if constexpr (kBias) y[i] = fma2(xh, wr[k % kCols][i], br[kBias ? k % kCols : 0][i]);
      else y[i] = mul2(xh, wr[k % kCols][i]);
    }
    Pair8<OT>::store(op, y);
  };
  // the same two passes over a split row held as K > 1 chunks, first chunk in slot sb
  const int kpc_shift = pl.kpc_shift;
  const int kpc_mask = (1 << kpc_shift) - 1;
  auto chunk_off = [&](int sb, int k) {  // byte offset of thread vector k's slot
    int s = sb + (k >> kpc_shift);
    if (s >= S) s -= S;
    return static_cast<size_t>(s) * pl.stage_bytes;
  };
  auto pass1c = [&](int sb, float (&part)[kVecs]) {
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      part[k] = 0.f;
      if ((vmask >> k) & 1u) {
        const size_t so = chunk_off(sb, k);
        const int o = (k & kpc_mask) * G8 + gl * 8;
        part[k] = sumsq(reinterpret_cast<const X*>(smem + so + pl.off[0]) + o,
                        reinterpret_cast<const RTe*>(smem + so + pl.off[1]) + o);
      }
    }
  };
  auto pass2c = [&](int sb, int64_t row, float rstd) {
    const int64_t g0 = row * pl.W + slice_elt0 + gl * 8;
    OT* op = static_cast<OT*>(p.out) + g0;
    ROe* rop = static_cast<ROe*>(p.ro) + g0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      if ((vmask >> k) & 1u) {
        const size_t so = chunk_off(sb, k);
        const int o = (k & kpc_mask) * G8 + gl * 8;
        emit(reinterpret_cast<const X*>(smem + so + pl.off[0]) + o,
             reinterpret_cast<const RTe*>(smem + so + pl.off[1]) + o, op + k * G8, rop + k * G8, rstd, k);
      }
    }
  };

  if constexpr (kCols < kVecs) {
    // --------- per-head column mode: kVecs / kCols super-rows per thread per sweep ---------
    // Thread vector k is column k % kCols (vector gl + (k % kCols) * G of the super-row) of
    // tile row sweep + gid + (k / kCols) * rps: the thread keeps the weight / bias of only
    // kCols columns in registers, and one transposed segment reduction serves all kVecs
    // (row, head) pairs. The planner picks this mode for per-head rows of at most
    // kCols * T vectors; every tile row is a whole super-row (P = 1).
    constexpr int kRpt = kVecs / kCols;
    if (active_warp) {
      int s = 0;
      uint32_t ph = 0;
      const int rstep = pl.rps * kRpt;
      for (int64_t q = 0; q < n_local; ++q) {
        const int64_t tile = cid + q * ncl;
        mbar_wait(&L.full[s], ph, kSiteFwdFull);
        const X* xs0 = stage_x(s);
        const RTe* rs0 = stage_r(s);
        const int64_t row0 = tile * pl.R;
        const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
        for (int sw = 0; sw < pl.R; sw += rstep) {
          const int lr0 = sw + gid;
          const bool active = in_group && lr0 < rows;
          const unsigned amask = __ballot_sync(0xffffffffu, active);
          if (!active) continue;
          unsigned ok = 0;  // vectors whose column is in the slice and whose row is in the tile
#pragma unroll
          for (int k = 0; k < kVecs; ++k)
            if (((vmask >> k) & 1u) && lr0 + (k / kCols) * pl.rps < rows) ok |= 1u << k;
          auto xoff = [&](int k) { return (lr0 + (k / kCols) * pl.rps) * xs_stride + (k % kCols) * G8; };
          float part[kVecs];
#pragma unroll
          for (int k = 0; k < kVecs; ++k) part[k] = ((ok >> k) & 1u) ? sumsq(xs0 + xoff(k), rs0 + xoff(k)) : 0.f;
          float rstd_k[kVecs];
          seg_reduce<kVecs>(part, rstd_k, pl.vs, amask, [&](float t) { return rsqrtf(fmaf(t, inv_n, p.eps)); });
          const int64_t g0 = (row0 + lr0) * pl.W + slice_elt0 + gl * 8;
          OT* op = static_cast<OT*>(p.out) + g0;
          ROe* rop = static_cast<ROe*>(p.ro) + g0;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            if ((ok >> k) & 1u) {
              const int64_t o = static_cast<int64_t>((k / kCols) * pl.rps) * pl.W + (k % kCols) * G8;
              emit(xs0 + xoff(k), rs0 + xoff(k), op + o, rop + o, rstd_k[k], k);
            }
          }
          // rstd per (row, head): lane i < kVecs of each segment stores the segment's value
          // i, so one store instruction per sweep writes them all (the segment's lanes agree
          // on which of its vectors are valid)
          if (p.rstd != nullptr) {
            const int i = gl & (pl.vs - 1);
            if (pl.vs >= kVecs) {
              if (i < kVecs && ((ok >> i) & 1u)) {
                float v = rstd_k[0];
#pragma unroll
                for (int k = 1; k < kVecs; ++k)
                  if (i == k) v = rstd_k[k];
                st1(&p.rstd[(row0 + lr0 + (i / kCols) * pl.rps) * pl.heads + ((gl + (i % kCols) * G) >> pl.vs_shift)], v);
              }
            } else if (i == 0) {
#pragma unroll
              for (int k = 0; k < kVecs; ++k)
                if ((ok >> k) & 1u)
                  st1(&p.rstd[(row0 + lr0 + (k / kCols) * pl.rps) * pl.heads + ((gl + (k % kCols) * G) >> pl.vs_shift)], rstd_k[k]);
            }
          }
        }
        if (release_slot(L, s, nwarps) && q + S < n_local) issue_unit(q + S, s);
        if (++s == S) { s = 0; ph ^= 1u; }
      }
    }
  } else if (active_warp && ln_rows && pl.vslice == G * kVecs && ((G >> 5) & ((G >> 5) - 1)) == 0) {
    // --------- LayerNorm rows, pipelined, statistics in one pass ---------
    // Every thread holds whole vectors of the row (a full slice, so every thread and every
    // warp of the group has the same sample count; a power-of-two number of warps) and
    // computes the mean and the sum of squared deviations (M2) of its 8 * kVecs values in
    // one read of shared memory; the warp and then the row group combine them
    // (stats_combine_equal). Iteration
    // q: statistics of row q, posted; output of row q-1 once its statistics are in. Slots
    // are used by row mod 4 (a warp posts row q after taking row q-1, as in the RMSNorm
    // pipelined loop); the mean of each warp goes to gpart, its M2 to xpart (unused:
    // LayerNorm rows are never split).
    int s = 0, sp = 0;
    uint32_t ph = 0;
    bool act_p = false;
    int64_t row_p = 0;
    const X* xs_p = nullptr;
    const int nw = G >> 5;
    const float n_warp = static_cast<float>(8 * kVecs * 32);
    for (int64_t q = 0; q <= n_local; ++q) {
      bool act_q = false;
      int64_t row_q = 0;
      const X* xs_q = nullptr;
      const uint32_t slot = static_cast<uint32_t>(q) & 3u;
      if (q < n_local) {
        mbar_wait(&L.full[s], ph, kSiteFwdFull);
        const int64_t row0 = (cid + q * ncl) * pl.R;
        act_q = in_group && row0 + gid < pl.nrows;
        row_q = row0 + gid;
        xs_q = stage_x(s) + gid * xs_stride;
        float m = 0.f, M2 = 0.f;
        if (act_q) {
          // one read of the thread's 8 * kVecs values: sums of d = x - x0 and d^2, shifted
          // by the thread's first value x0 so that M2 = S2 - S1^2 / n cancels at most within
          // the thread's own values (every deviation is measured from one of them)
          float2 h[4];
          Pair8<X>::load(xs_q, h);
          const float x0 = h[0].x;
          const float2 sh = splat2(-x0);
          float2 s1 = splat2(0.f), s2 = splat2(0.f);
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            if (k > 0) Pair8<X>::load(xs_q + k * G8, h);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 d = add2(h[i], sh);
              s1 = add2(s1, d);
              s2 = fma2(d, d, s2);
            }
          }
          const float S1 = s1.x + s1.y;
          const float S2 = s2.x + s2.y;
          constexpr float kInvN = 1.f / static_cast<float>(8 * kVecs);
          m = fmaf(S1, kInvN, x0);
          M2 = fmaxf(fmaf(-S1, S1 * kInvN, S2), 0.f);
        }
        lanes_stats(m, M2, static_cast<float>(8 * kVecs), 32);
        if (lane == 0) {
          L.gpart[slot * 16 + warp] = m;
          L.xpart[slot * 16 + warp] = M2;
          mbar_arrive(&L.gbar[gid * kGroupRed + slot]);
        }
      }
      if (q >= 1) {
        const uint32_t ps = (slot + 3u) & 3u;
        mbar_wait(&L.gbar[gid * kGroupRed + ps], static_cast<uint32_t>((q - 1) >> 2) & 1u, kSiteFwdCluster);
        float m = L.gpart[ps * 16 + gid * nw + (lane & (nw - 1))];
        float M2 = L.xpart[ps * 16 + gid * nw + (lane & (nw - 1))];
        lanes_stats(m, M2, n_warp, nw);  // every lane combines the group's nw warps
        const float rstd = rsqrtf(M2 * inv_n + p.eps);  // m, M2: row q-1's mean and M2
        if (act_p) {
          OT* op = static_cast<OT*>(p.out) + row_p * pl.W + gl * 8;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) ln_emit(xs_p + k * G8, op + k * G8, m, rstd, k);
          if (gl == 0) {
            if (p.rstd != nullptr) st1(&p.rstd[row_p], rstd);
            if (p.mean != nullptr) st1(&p.mean[row_p], m);
          }
        }
        if (release_slot(L, sp, nwarps) && q - 1 + S < n_local) issue_unit(q - 1 + S, sp);
      }
      if (q < n_local) {
        sp = s;
        if (++s == S) { s = 0; ph ^= 1u; }
      }
      act_p = act_q;
      row_p = row_q;
      xs_p = xs_q;
    }
  } else if (active_warp && ln_rows) {
    // --------- LayerNorm rows, pipelined one tile deep (tiles hold one row per group) ---------
    // Iteration q: A(q) = sum of row q, posted; C(q-1) = output of row q-1 once its
    // variance is in; B(q) = squared deviations of row q once its mean is in, posted.
    // Every wait is covered by a pass of independent work. Needs S >= 2.
    int s = 0, sp = 0;
    uint32_t ph = 0;
    float mean_p = 0.f;
    bool act_p = false;
    int64_t row_p = 0;
    const X* xs_p = nullptr;
    for (int64_t q = 0; q <= n_local; ++q) {
      float mean_q = 0.f;
      bool act_q = false;
      int64_t row_q = 0;
      const X* xs_q = nullptr;
      const uint32_t par = static_cast<uint32_t>(q) & 1u;
      if (q < n_local) {
        mbar_wait(&L.full[s], ph, kSiteFwdFull);
        const int64_t row0 = (cid + q * ncl) * pl.R;
        act_q = in_group && row0 + gid < pl.nrows;
        row_q = row0 + gid;
        xs_q = stage_x(s) + gid * xs_stride;
        float part = 0.f;
        if (act_q) {
#pragma unroll
          for (int k = 0; k < kVecs; ++k)
            if ((vmask >> k) & 1u) part += ln_sum(xs_q + k * G8);
        }
        group_post(part, L, gid, warp, lane, 0 + par);
      }
      if (q >= 1) {
        const float var = group_take(pl, L, gid, lane, 2 + (par ^ 1u), static_cast<uint32_t>((q - 1) >> 1)) * inv_n;
        const float rstd = rsqrtf(var + p.eps);
        if (act_p) {
          OT* op = static_cast<OT*>(p.out) + row_p * pl.W + gl * 8;
#pragma unroll
          for (int k = 0; k < kVecs; ++k)
            if ((vmask >> k) & 1u) ln_emit(xs_p + k * G8, op + k * G8, mean_p, rstd, k);
          if (gl == 0) {
            if (p.rstd != nullptr) st1(&p.rstd[row_p], rstd);
            if (p.mean != nullptr) st1(&p.mean[row_p], mean_p);
          }
        }
        if (release_slot(L, sp, nwarps) && q - 1 + S < n_local) issue_unit(q - 1 + S, sp);
      }
      if (q < n_local) {
        mean_q = group_take(pl, L, gid, lane, 0 + par, static_cast<uint32_t>(q >> 1)) * inv_n;
        float part = 0.f;
        if (act_q) {
#pragma unroll
          for (int k = 0; k < kVecs; ++k)
            if ((vmask >> k) & 1u) part += ln_dev(xs_q + k * G8, mean_q);
        }
        group_post(part, L, gid, warp, lane, 2 + par);
        sp = s;
        if (++s == S) { s = 0; ph ^= 1u; }
      }
      mean_p = mean_q;
      act_p = act_q;
      row_p = row_q;
      xs_p = xs_q;
    }
  } else if (active_warp && rms_rows) {
    // --------- RMSNorm rows, pipelined one tile deep ---------
    // Iteration q: sum of squares of row q, posted; output of row q-1 once its sum is in.
    int s = 0, sp = 0;
    uint32_t ph = 0;
    bool act_p = false;
    int64_t row_p = 0;
    const X* xs_p = nullptr;
    const RTe* rs_p = nullptr;
    for (int64_t q = 0; q <= n_local; ++q) {
      bool act_q = false;
      int64_t row_q = 0;
      const X* xs_q = nullptr;
      const RTe* rs_q = nullptr;
      const uint32_t slot = static_cast<uint32_t>(q) & 3u;
      if (q < n_local) {
        mbar_wait(&L.full[s], ph, kSiteFwdFull);
        const int64_t row0 = (cid + q * ncl) * pl.R;
        act_q = in_group && row0 + gid < pl.nrows;
        row_q = row0 + gid;
        xs_q = stage_x(s) + gid * xs_stride;
        rs_q = stage_r(s) + gid * xs_stride;
        float part[kVecs];
        float ss = 0.f;
        if (act_q) {
          pass1(xs_q, rs_q, part);
#pragma unroll
          for (int k = 0; k < kVecs; ++k) ss += part[k];
        }
        group_post(ss, L, gid, warp, lane, slot);
      }
      if (q >= 1) {
        const float tot = group_take(pl, L, gid, lane, (slot + 3u) & 3u, static_cast<uint32_t>((q - 1) >> 2));
        const float r = rsqrtf(fmaf(tot, inv_n, p.eps));
        if (act_p) {
          float rstd_k[kVecs];
#pragma unroll
          for (int k = 0; k < kVecs; ++k) rstd_k[k] = r;
          pass2(xs_p, rs_p, row_p, rstd_k);
          if (p.rstd != nullptr && gl == 0) st1(&p.rstd[row_p], r);
        }
        if (release_slot(L, sp, nwarps) && q - 1 + S < n_local) issue_unit(q - 1 + S, sp);
      }
      if (q < n_local) {
        sp = s;
        if (++s == S) { s = 0; ph ^= 1u; }
      }
      act_p = act_q;
      row_p = row_q;
      xs_p = xs_q;
      rs_p = rs_q;
    }
  } else if (active_warp && pl.P == 1) {
    // ------------------------------- tile loop -------------------------------
    int s = 0;
    uint32_t ph = 0;
    uint32_t seq = 0;
    for (int64_t q = 0; q < n_local; ++q) {
      const int64_t tile = cid + q * ncl;
      mbar_wait(&L.full[s], ph, kSiteFwdFull);
      const X* xs0 = stage_x(s);
      const RTe* rs0 = stage_r(s);
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
        float part[kVecs];
        float rstd_k[kVecs];
        float mean_k[kVecs];
        // segment (seg mode) or row-group (row mode) sum of part[], scaled by `scale`
        auto reduce_k = [&](const float (&pt)[kVecs], float (&res)[kVecs], float scale) {
          if (pl.seg_mode) {
            seg_reduce<kVecs>(pt, res, pl.vs, amask, [&](float t) { return t * scale; });
          } else {
            float t = 0.f;
#pragma unroll
            for (int k = 0; k < kVecs; ++k) t += pt[k];
            t = group_sum(t, pl, L, gid, gl, seq++) * scale;
#pragma unroll
            for (int k = 0; k < kVecs; ++k) res[k] = t;
          }
        };
        if constexpr (kLN) {
#pragma unroll
          for (int k = 0; k < kVecs; ++k) part[k] = ((vmask >> k) & 1u) ? ln_sum(xs + k * G8) : 0.f;
          reduce_k(part, mean_k, inv_n);
#pragma unroll
          for (int k = 0; k < kVecs; ++k) part[k] = ((vmask >> k) & 1u) ? ln_dev(xs + k * G8, mean_k[k]) : 0.f;
          reduce_k(part, rstd_k, inv_n);
#pragma unroll
          for (int k = 0; k < kVecs; ++k) rstd_k[k] = rsqrtf(rstd_k[k] + p.eps);
          if (p.out != nullptr) {
            OT* op = static_cast<OT*>(p.out) + row * pl.W + gl * 8;
#pragma unroll
            for (int k = 0; k < kVecs; ++k)
              if ((vmask >> k) & 1u) ln_emit(xs + k * G8, op + k * G8, mean_k[k], rstd_k[k], k);
          }
        } else {
          pass1(xs, rs, part);
          if (pl.seg_mode) {
            seg_reduce<kVecs>(part, rstd_k, pl.vs, amask, [&](float t) { return rsqrtf(fmaf(t, inv_n, p.eps)); });
          } else {
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < kVecs; ++k) ss += part[k];
            ss = group_sum(ss, pl, L, gid, gl, seq++);
            const float r = rsqrtf(fmaf(ss, inv_n, p.eps));
#pragma unroll
            for (int k = 0; k < kVecs; ++k) rstd_k[k] = r;
          }
          pass2(xs, rs, row, rstd_k);
        }
        // per-row (per-segment) statistics: one lane of each segment or row group stores
        auto store_stat = [&](float* dst, const float (&v_k)[kVecs]) {
          if (pl.seg_mode) {
#pragma unroll
            for (int k = 0; k < kVecs; ++k) {
              const int v = gl + k * G;
              if (((vmask >> k) & 1u) && (v & (pl.vs - 1)) == 0) dst[row * pl.heads + (v >> pl.vs_shift)] = v_k[k];
            }
          } else if (gl == 0) {
            dst[row] = v_k[0];
          }
        };
        if (p.rstd != nullptr) store_stat(p.rstd, rstd_k);
        if constexpr (kLN) {
          if (p.mean != nullptr) store_stat(p.mean, mean_k);
        }
      }
      if (release_slot(L, s, nwarps) && q + S < n_local)
        issue_unit(q + S, s);
      if (++s == S) { s = 0; ph ^= 1u; }
    }
  } else if (!kRes && !kRO && active_warp && !kLN && pl.xpair) {
    // --------- split-row loop over row pairs (one row per tile, K = 1) ---------
    // Iteration j: pass 1 of local rows 2j and 2j+1, both CTA sums behind one barrier, both
    // sent; then both totals of pair j-1 received in one poll and their pass 2. A row slice
    // of 32 KB streams in about 1.5 us per SM at full HBM bandwidth, about what the fixed
    // per-row costs (CTA barrier, exchange round trip, record poll) took by themselves;
    // pairs pay them once per two rows. Sums are formed as in the row-by-row loop, so the
    // results are the same. The ring holds pairs j and j-1 (planned for S >= 6; compiled
    // into the residual-free kernels only, whose registers leave room for it). Record
    // slots (row mod 8): a CTA sends pair j after receiving pair j-2, which needed every
    // peer's send of pair j-2, made after that peer received pair j-4 (the rows whose
    // slots pair j reuses).
    int s1 = 0, s2 = 0;
    uint32_t ph1 = 0;
    const int64_t npairs = (n_local + 1) >> 1;
    for (int64_t j = 0; j <= npairs; ++j) {
      const int64_t ra2 = 2 * (j - 1);  // pair j-1's first row
      const XRecord pre =
          j >= 1 && (!pl.xbcast || warp == 0) ? xrec_load2(pl, xc, lane, static_cast<uint32_t>(ra2)) : 0ull;
      if (j < npairs) {
        const int64_t ra = 2 * j;
        const bool hb = ra + 1 < n_local;
        float pa[kVecs], pb[kVecs];
        mbar_wait(&L.full[s1], ph1, kSiteFwdFull);
        pass1(stage_x(s1), stage_r(s1), pa);
        if (++s1 == S) { s1 = 0; ph1 ^= 1u; }
        if (hb) {
          mbar_wait(&L.full[s1], ph1, kSiteFwdFull);
          pass1(stage_x(s1), stage_r(s1), pb);
          if (++s1 == S) { s1 = 0; ph1 ^= 1u; }
        } else {
#pragma unroll
          for (int k = 0; k < kVecs; ++k) pb[k] = 0.f;
        }
        float ssa = 0.f, ssb = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
          ssa += pa[k];
          ssb += pb[k];
        }
        group_sum2(ssa, ssb, pl, (j & 1) ? L.gpart : L.red, gl);
        cluster_send(ssa, pl, L, xc, warp, lane, static_cast<uint32_t>(ra), rank);
        if (hb) cluster_send(ssb, pl, L, xc, warp, lane, static_cast<uint32_t>(ra + 1), rank);
      }
      if (j >= 1) {
        const bool hb = ra2 + 1 < n_local;
        float tot[2];
        cluster_recv2(pl, L, xc, warp, lane, static_cast<uint32_t>(ra2), hb, pre, kSiteFwdCluster, tot[0], tot[1]);
        for (int h = 0; h < (hb ? 2 : 1); ++h) {
          const int64_t r2 = ra2 + h;
          const int64_t row = cid + r2 * ncl;
          float rstd_k[kVecs];
          const float rs = rsqrtf(fmaf(tot[h], inv_n, p.eps));
#pragma unroll
          for (int k = 0; k < kVecs; ++k) rstd_k[k] = rs;
          if (in_group) pass2(stage_x(s2), stage_r(s2), row, rstd_k);
          if (p.rstd != nullptr && tid == 0 && rank == 0) st1(&p.rstd[row], rs);
          if (release_slot(L, s2, nwarps) && r2 + S < n_local) issue_unit(r2 + S, s2);
          if (++s2 == S) s2 = 0;
        }
      }
    }
  } else if (active_warp && !kLN) {
    // --------- split-row loop (rows split over the cluster, one row per tile) ---------
    // Iteration i: pass 1 of row i and its exchange, then pass 2 of row i - lag.
    const int lag = pl.lag;
    int s1 = 0, s2 = 0;
    uint32_t ph1 = 0;
    for (int64_t i = 0; i < n_local + lag; ++i) {
      const int64_t r2 = i - lag;
      const XRecord pre =
          r2 >= 0 && (!pl.xbcast || warp == 0) ? xrec_load(pl, xc, lane, static_cast<uint32_t>(r2)) : 0ull;
      if (i < n_local) {
        float part[kVecs];
        if (K == 1) {
          mbar_wait(&L.full[s1], ph1, kSiteFwdFull);
          pass1(stage_x(s1), stage_r(s1), part);
        } else {
          for (int j = 0; j < K; ++j) {
            uint32_t ph;
            const int s = chunk_slot(s1, ph1, j, S, &ph);
            mbar_wait(&L.full[s], ph, kSiteFwdFull);
          }
          pass1c(s1, part);
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) ss += part[k];
        ss = group_sum(ss, pl, L, 0, gl, static_cast<uint32_t>(i));
        cluster_send(ss, pl, L, xc, warp, lane, static_cast<uint32_t>(i), rank);
        s1 += K;
        if (s1 >= S) { s1 -= S; ph1 ^= 1u; }
      }
      if (r2 >= 0 && r2 < n_local) {
        const float tot =
            cluster_recv<!kRes && !kRO>(pl, L, xc, warp, lane, static_cast<uint32_t>(r2), pre, kSiteFwdCluster);
        const int64_t row = cid + r2 * ncl;
        float rstd_k[kVecs];
        const float rs = rsqrtf(fmaf(tot, inv_n, p.eps));
#pragma unroll
        for (int k = 0; k < kVecs; ++k) rstd_k[k] = rs;
        if (in_group) {
          if (K == 1) pass2(stage_x(s2), stage_r(s2), row, rstd_k);
          else pass2c(s2, row, rs);
        }
        if (p.rstd != nullptr && tid == 0 && rank == 0) st1(&p.rstd[row], rs);
        if (K == 1) {
          if (release_slot(L, s2, nwarps) && r2 + S < n_local)
            issue_unit(r2 + S, s2);
          if (++s2 == S) s2 = 0;
        } else {
          for (int j = 0; j < K; ++j) {
            uint32_t ph;
            const int s = chunk_slot(s2, 0u, j, S, &ph);
            const int64_t un = r2 * K + j + S;  // unit that refills the slot
            if (release_slot(L, s, nwarps) && un < n_units)
              issue_unit(un, s);
          }
          s2 += K;
          if (s2 >= S) s2 -= S;
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0 && abort_requested()) drain_after_failure(pl, L, n_units);
  // no CTA leaves while a peer may still store into its shared memory (after a failure a
  // peer can be rows behind)
  if (pl.P > 1 && pl.xmode == kXCluster) cluster_sync_all();
}

// =======================================================================================
// Backward: dx in one pass from the saved rstd; dweight / dbias per-CTA partial rows.
// =======================================================================================
// Tile `tile` (or chunk j of this CTA's slice of row `tile`) into slot s; every chunk of a
// split row carries the row's rstd. kRstdBulk (per-head kernels): the tile's rstd block
// (rows x heads floats) comes with one bulk copy when it is 16-byte aligned and sized.
template <typename X, typename DY, typename DROT, bool kRstdBulk>
__device__ __forceinline__ void bwd_issue(const BwdParams& p, const StreamPlan& pl, const SmemLayout& L,
                                          unsigned char* smem, int64_t tile, int j, int s, int64_t slice_elt0,
                                          int rstd_per_row, uint64_t pol, int64_t pf_tile = -1, int pf_j = 0) {
  unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
  const int64_t row0 = tile * pl.R;
  const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
  fence_proxy_async_smem();
  // rstd of the tile's rows, tracked by the same mbarrier: one bulk copy when the block
  // is 16-byte aligned and sized (per-head tiles: rows x heads floats), else plain async
  // copies (a row-mode tile needs only a few floats)
  float* rdst = reinterpret_cast<float*>(st + pl.off[3]);
  const float* rsrc = p.rstd + row0 * rstd_per_row;
  const int cnt = rows * rstd_per_row;
  const uint32_t rbytes = static_cast<uint32_t>(cnt) * 4u;
  const bool rbulk = kRstdBulk && (reinterpret_cast<uintptr_t>(rsrc) & 15u) == 0 && (rbytes & 15u) == 0;
  if (!rbulk) {
    // the bounds-checked build checks the whole run once, before the first copy
    if (RMSB_DBG_OK(rsrc, rbytes, kDbgAsyncCopy) && RMSB_DBG_OK(rdst, rbytes, kDbgAsyncCopy)) {
      int c = 0;
      if ((reinterpret_cast<uintptr_t>(rsrc) & 15u) == 0)
        for (; c + 4 <= cnt; c += 4) cp_async_16(rdst + c, rsrc + c);
      for (; c < cnt; ++c) cp_async_4(rdst + c, rsrc + c);
    }
    cp_async_arrive(&L.full[s]);
  }
  const uint32_t b0 = static_cast<uint32_t>(rows) * pl.row_bytes[0];
  const uint32_t b1 = static_cast<uint32_t>(rows) * pl.row_bytes[1];
  const uint32_t b2 = Present<DROT>::value ? static_cast<uint32_t>(rows) * pl.row_bytes[2] : 0u;
  mbar_arrive_expect_tx(&L.full[s], b0 + b1 + b2 + (rbulk ? rbytes : 0u));
  if (rbulk) bulk_load(rdst, rsrc, rbytes, &L.full[s], pol);
  const int64_t e0 = row0 * pl.W + slice_elt0 + static_cast<int64_t>(j) * (pl.row_bytes[0] / sizeof(X));
  bulk_load(st + pl.off[0], static_cast<const X*>(p.x) + e0, b0, &L.full[s], pol);
  bulk_load(st + pl.off[1], static_cast<const DY*>(p.dy) + e0, b1, &L.full[s], pol);
  if constexpr (Present<DROT>::value)
    bulk_load(st + pl.off[2], static_cast<const DROT*>(p.dro) + e0, b2, &L.full[s], pol);
  if (pf_tile >= 0) {
    const int64_t prow0 = pf_tile * pl.R;
    const uint32_t prows = static_cast<uint32_t>(min(static_cast<int64_t>(pl.R), pl.nrows - prow0));
    const int64_t pe0 = prow0 * pl.W + slice_elt0 + static_cast<int64_t>(pf_j) * (pl.row_bytes[0] / sizeof(X));
    bulk_prefetch_l2(static_cast<const X*>(p.x) + pe0, prows * pl.row_bytes[0]);
    bulk_prefetch_l2(static_cast<const DY*>(p.dy) + pe0, prows * pl.row_bytes[1]);
    if constexpr (Present<DROT>::value)
      bulk_prefetch_l2(static_cast<const DROT*>(p.dro) + pe0, prows * pl.row_bytes[2]);
  }
}

// X: saved input dtype; DY: dout dtype; DXT: dx dtype; DROT: dresidual_out dtype (NoT =
// none); DREST: dresidual dtype (NoT = not written); kRstdBulk: see bwd_issue; kCols <
// kVecs: per-head column mode, as in the forward (the thread's weight and dweight / dbias
// accumulators cover kCols columns). kTmemAcc: the dweight / dbias accumulators live in
// tensor memory instead of registers (16 columns of the thread's TMEM lane per vector:
// dweight pairs, then dbias pairs). Weight, dweight and dbias of 4 vectors per thread
// need 96 registers, more than 128-register threads can spare beside the passes' working
// set; with the sums in TMEM a dbias backward keeps 4 vectors per thread, so a 16384-wide
// row fits one CTA instead of a 2-CTA cluster. Planned for unsplit rows in row mode only
// (thread groups of whole warps, so every warp issues its TMEM accesses together); the
// split-row loop is compiled out of these kernels.
template <typename X, typename DY, typename DXT, typename DROT, typename DREST, bool kHasDb, int kVecs,
          int kBlock, int kMinBlocks, bool kRstdBulk = false, int kCols = kVecs, bool kTmemAcc = false>
__global__ void __launch_bounds__(kBlock, kMinBlocks) bwd_stream_kernel(const BwdParams p) {
  static_assert(kVecs % kCols == 0, "column mode: whole rows per thread");
  static_assert(!kTmemAcc || (kHasDb && kCols == kVecs && kVecs == 4), "TMEM accumulators: 4-vector dbias rows");
  // TMEM columns of the CTA: 64 per warp (4 vectors x 16), the warps of a lane quarter
  // side by side
  constexpr uint32_t kTmemCols = static_cast<uint32_t>(kBlock / 128) * 64u;
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr bool kDro = Present<DROT>::value;
  constexpr bool kDres = Present<DREST>::value;
  using DROe = Elt<DROT>;
  using DRESe = Elt<DREST>;
  const StreamPlan& pl = p.pl;
  const SmemLayout L = carve_smem(smem, pl);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  uint32_t rank = 0;
  int64_t cid = blockIdx.x;
  int64_t ncl = gridDim.x;
  if (pl.P > 1) {
    if (pl.xmode == kXCluster) {
      rank = cluster_ctarank();
      cid = cluster_id_x();
      ncl = cluster_count_x();
    } else {
      rank = blockIdx.x % pl.P;
      cid = blockIdx.x / pl.P;
      ncl = gridDim.x / pl.P;
    }
  }
  // row mode with one row per group per tile: rows pipelined one tile deep (when planned)
  const bool rows_pipe = pl.pipe_rows && !pl.seg_mode && pl.P == 1 && pl.R == pl.rps && pl.S >= 3;
  if constexpr (kTmemAcc) {
    if (warp == 0) tmem_alloc_warp(L.tmem, kTmemCols);
    tmem_fence_before_sync();
  }
  init_barriers(L, pl, rows_pipe);
  // this thread's accumulators: TMEM lane 32 * (warp % 4) + lane, 64 columns per warp
  uint32_t tacc = 0;
  if constexpr (kTmemAcc) {
    tmem_fence_after_sync();
    tacc = *L.tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>(warp >> 2) * 64u;
    float2 z[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) z[i] = splat2(0.f);
#pragma unroll
    for (int k = 0; k < kVecs; ++k) tmem_st16(tacc + 16u * k, z);
    tmem_wait_st();
  }
  pdl_wait();  // every global access of the launch follows this point
  pdl_launch_dependents();
  xgen_begin(pl, L, p.xgen, cid);
  const XCtx xc{p.xrec, cid * pl.P};

  const int64_t slice_elt0 = static_cast<int64_t>(rank) * pl.vslice * 8;
  const int rstd_per_row = pl.seg_mode ? pl.heads : 1;
  const uint64_t pol = l2_policy_evict_first();
  const int64_t n_local = cid < pl.ntiles ? (pl.ntiles - 1 - cid) / ncl + 1 : 0;
  const int S = pl.S;
  const int K = pl.K;
  const int kshift = __ffs(K) - 1;
  const int64_t n_units = n_local * K;
  // loads unit u into slot s and prefetches unit u + pf into L2
  auto issue_unit = [&](int64_t u, int s) {
    const int64_t v = u + pl.pf;
    const bool pf = pl.pf > 0 && v < n_units;
    bwd_issue<X, DY, DROT, kRstdBulk>(p, pl, L, smem, cid + (u >> kshift) * ncl, static_cast<int>(u & (K - 1)), s, slice_elt0,
                           rstd_per_row, pol, pf ? cid + (v >> kshift) * ncl : -1, static_cast<int>(v & (K - 1)));
  };
  if (tid == 0)
    for (int u = 0; u < S && u < n_units; ++u) issue_unit(u, u);

  const int G = pl.G;
  const int G8 = G * 8;
  const int gid = tid / G;
  const int gl = tid - gid * G;
  const bool in_group = gid < pl.rps;
  const int nwarps = (pl.rps * G + 31) >> 5;
  const bool active_warp = warp < nwarps;
  const float inv_n = 1.f / static_cast<float>(pl.N);  // mean = sum * (1/N), exact for N a power of two
  unsigned vmask = 0;
#pragma unroll
  for (int k = 0; k < kVecs; ++k)
    if (in_group && gl + (k % kCols) * G < pl.vslice) vmask |= 1u << k;

  // weight of the thread's columns and its dweight / dbias accumulators, as float pairs
  // (the accumulators are in TMEM instead for kTmemAcc)
  constexpr int kAcc = kTmemAcc ? 1 : kCols;
  float2 wr[kCols][4];
  float2 dw[kAcc][4];
  float2 db[(kHasDb && !kTmemAcc) ? kCols : 1][4];
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int64_t c = slice_elt0 + static_cast<int64_t>(gl + k * G) * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) wr[k][i] = splat2(1.f);
    if constexpr (!kTmemAcc) {
#pragma unroll
      for (int i = 0; i < 4; ++i) dw[k % kAcc][i] = splat2(0.f);
      if constexpr (kHasDb) {
#pragma unroll
        for (int i = 0; i < 4; ++i) db[kHasDb ? k : 0][i] = splat2(0.f);
      }
    }
    if (((vmask >> k) & 1u) && p.w != nullptr) load8p_rt(p.w, p.w_dt, p.w_per_head ? c : c % pl.N, wr[k]);
  }
  const int x_stride = static_cast<int>(pl.row_bytes[0] / sizeof(X));

  // pass 1 of thread vector k with row rstd r: returns r * sum(x * dy * w) over the
  // vector and adds dy * x * r to dweight (dy to dbias)
  auto dot_acc = [&](const X* xp, const DY* dp, float r, int k) {
    float2 xv[4], dv[4];
    Pair8<X>::load(xp, xv);
    Pair8<DY>::load(dp, dv);
    const float2 r2 = splat2(r);
    float2 acc = splat2(0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = mul2(xv[i], dv[i]);
      acc = fma2(t, wr[k % kCols][i], acc);
      if constexpr (!kTmemAcc) {
        dw[k % kAcc][i] = fma2(t, r2, dw[k % kAcc][i]);
        if constexpr (kHasDb) db[kHasDb ? k % kCols : 0][i] = add2(db[kHasDb ? k % kCols : 0][i], dv[i]);
      }
    }
    return (acc.x + acc.y) * r;
  };
  // the same with the vector's dweight / dbias sums held in TMEM: `valid` false (a vector
  // outside the slice) still loads and stores them, since every lane of the warp issues
  // the TMEM accesses together
  auto dot_acc_tmem = [&](const X* xp, const DY* dp, float r, int k, bool valid) {
    float2 a[8];  // dweight pairs 0..3, dbias pairs 4..7
    tmem_ld16(tacc + 16u * k, a);
    float d = 0.f;
    float2 xv[4], dv[4];
    if (valid) {
      Pair8<X>::load(xp, xv);
      Pair8<DY>::load(dp, dv);
    }
    tmem_wait_ld();
    if (valid) {
      const float2 r2 = splat2(r);
      float2 acc = splat2(0.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = mul2(xv[i], dv[i]);
        acc = fma2(t, wr[k % kCols][i], acc);
        a[i] = fma2(t, r2, a[i]);
        a[4 + i] = add2(a[4 + i], dv[i]);
      }
      d = (acc.x + acc.y) * r;
    }
    tmem_st16(tacc + 16u * k, a);
    return d;
  };
  // pass 2 of thread vector k: dx = r * dy * w - r^2 c x (+ dresidual_out), stored to dx
  // and dresidual
  auto dx_emit = [&](const X* xp, const DY* dp, const DROe* ap, DXT* dxo, DRESe* dro, float r, float c, int k) {
    float2 xv[4], dv[4], g[4];
    Pair8<X>::load(xp, xv);
    Pair8<DY>::load(dp, dv);
    const float2 rr = splat2(r);
    const float2 nb = splat2(-(r * r) * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = fma2(mul2(dv[i], wr[k % kCols][i]), rr, mul2(xv[i], nb));
    if constexpr (kDro) {
      float2 a[4];
      Pair8<DROe>::load(ap, a);
#pragma unroll
      for (int i = 0; i < 4; ++i) g[i] = add2(g[i], a[i]);
    }
    Pair8<DXT>::store(dxo, g);
    if constexpr (kDres) Pair8<DRESe>::store(dro, g);
  };

  struct RowPtrs {
    const X* x;
    const DY* dy;
    const DROe* dro;
    const float* rstd;  // this row's rstd block (one per segment in seg mode)
  };
  auto row_ptrs = [&](int s, int lr) -> RowPtrs {
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    RowPtrs r;
    r.x = reinterpret_cast<const X*>(st + pl.off[0]) + lr * x_stride + gl * 8;
    r.dy = reinterpret_cast<const DY*>(st + pl.off[1]) + lr * x_stride + gl * 8;
    r.dro = reinterpret_cast<const DROe*>(st + pl.off[2]) + lr * x_stride + gl * 8;
    r.rstd = reinterpret_cast<const float*>(st + pl.off[3]) + lr * rstd_per_row;
    return r;
  };
  // pass 1: partial dot products per vector, dweight / dbias accumulation
  auto pass1 = [&](const RowPtrs& rp, float (&part)[kVecs], float (&rstd_k)[kVecs]) {
    if constexpr (kTmemAcc) {
      tmem_wait_st();  // the previous row's sums are in TMEM before they are read again
      const float r = ld1(&rp.rstd[0]);  // row mode: one rstd per row
#pragma unroll
      for (int k = 0; k < kVecs; ++k) {
        rstd_k[k] = r;
        part[k] = dot_acc_tmem(rp.x + k * G8, rp.dy + k * G8, r, k, (vmask >> k) & 1u);
      }
      return;
    }
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      part[k] = 0.f;
      rstd_k[k] = 0.f;
      if ((vmask >> k) & 1u) {
        const float r = ld1(&rp.rstd[pl.seg_mode ? ((gl + k * G) >> pl.vs_shift) : 0]);
        rstd_k[k] = r;
        part[k] = dot_acc(rp.x + k * G8, rp.dy + k * G8, r, k);
      }
    }
  };
  // pass 2: dx (+ dresidual_out), written to dx and dresidual
  auto pass2 = [&](const RowPtrs& rp, int64_t row, const float (&rstd_k)[kVecs], const float (&c_k)[kVecs]) {
    const int64_t g0 = row * pl.W + slice_elt0 + gl * 8;
    DXT* dxp = static_cast<DXT*>(p.dx) + g0;
    DRESe* drp = static_cast<DRESe*>(p.dres) + g0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k)
      if ((vmask >> k) & 1u)
        dx_emit(rp.x + k * G8, rp.dy + k * G8, rp.dro + k * G8, dxp + k * G8, drp + k * G8, rstd_k[k], c_k[k], k);
  };
  // the same two passes over a split row held as K > 1 chunks, first chunk in slot sb
  // (every chunk carries the row's rstd; the first chunk's copy is used)
  const int kpc_shift = pl.kpc_shift;
  const int kpc_mask = (1 << kpc_shift) - 1;
  auto chunk_ptrs = [&](int sb, int k) -> RowPtrs {
    int s = sb + (k >> kpc_shift);
    if (s >= S) s -= S;
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const int o = (k & kpc_mask) * G8 + gl * 8;
    RowPtrs r;
    r.x = reinterpret_cast<const X*>(st + pl.off[0]) + o;
    r.dy = reinterpret_cast<const DY*>(st + pl.off[1]) + o;
    r.dro = reinterpret_cast<const DROe*>(st + pl.off[2]) + o;
    r.rstd = nullptr;
    return r;
  };
  auto pass1c = [&](int sb, float r, float (&part)[kVecs]) {
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      part[k] = 0.f;
      if ((vmask >> k) & 1u) {
        const RowPtrs cp = chunk_ptrs(sb, k);
        part[k] = dot_acc(cp.x, cp.dy, r, k);
      }
    }
  };
  auto pass2c = [&](int sb, int64_t row, float r, float c) {
    const int64_t g0 = row * pl.W + slice_elt0 + gl * 8;
    DXT* dxp = static_cast<DXT*>(p.dx) + g0;
    DRESe* drp = static_cast<DRESe*>(p.dres) + g0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      if ((vmask >> k) & 1u) {
        const RowPtrs cp = chunk_ptrs(sb, k);
        dx_emit(cp.x, cp.dy, cp.dro, dxp + k * G8, drp + k * G8, r, c, k);
      }
    }
  };

  if constexpr (kCols < kVecs) {
    // --------- per-head column mode: kVecs / kCols super-rows per thread per sweep ---------
    // (see the forward): thread vector k is column k % kCols of tile row
    // sweep + gid + (k / kCols) * rps, with that (row, head)'s rstd from the staged block
    if (active_warp) {
      int s = 0;
      uint32_t ph = 0;
      const int rstep = pl.rps * (kVecs / kCols);
      for (int64_t q = 0; q < n_local; ++q) {
        const int64_t tile = cid + q * ncl;
        mbar_wait(&L.full[s], ph, kSiteBwdFull);
        const int64_t row0 = tile * pl.R;
        const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
        const RowPtrs rp = row_ptrs(s, 0);
        for (int sw = 0; sw < pl.R; sw += rstep) {
          const int lr0 = sw + gid;
          const bool active = in_group && lr0 < rows;
          const unsigned amask = __ballot_sync(0xffffffffu, active);
          if (!active) continue;
          unsigned ok = 0;  // vectors whose column is in the slice and whose row is in the tile
#pragma unroll
          for (int k = 0; k < kVecs; ++k)
            if (((vmask >> k) & 1u) && lr0 + (k / kCols) * pl.rps < rows) ok |= 1u << k;
          auto eoff = [&](int k) { return (lr0 + (k / kCols) * pl.rps) * x_stride + (k % kCols) * G8; };
          float part[kVecs], rstd_k[kVecs], c_k[kVecs];
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            part[k] = 0.f;
            rstd_k[k] = 0.f;
            if ((ok >> k) & 1u) {
              const float r = ld1(&rp.rstd[(lr0 + (k / kCols) * pl.rps) * rstd_per_row +
                                      ((gl + (k % kCols) * G) >> pl.vs_shift)]);
              rstd_k[k] = r;
              part[k] = dot_acc(rp.x + eoff(k), rp.dy + eoff(k), r, k);
            }
          }
          seg_reduce<kVecs>(part, c_k, pl.vs, amask, [&](float t) { return t * inv_n; });
          const int64_t g0 = (row0 + lr0) * pl.W + slice_elt0 + gl * 8;
          DXT* dxp = static_cast<DXT*>(p.dx) + g0;
          DRESe* drp = static_cast<DRESe*>(p.dres) + g0;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) {
            if ((ok >> k) & 1u) {
              const int64_t o = static_cast<int64_t>((k / kCols) * pl.rps) * pl.W + (k % kCols) * G8;
              dx_emit(rp.x + eoff(k), rp.dy + eoff(k), rp.dro + eoff(k), dxp + o, drp + o, rstd_k[k], c_k[k], k);
            }
          }
        }
        if (release_slot(L, s, nwarps) && q + S < n_local) issue_unit(q + S, s);
        if (++s == S) { s = 0; ph ^= 1u; }
      }
    }
  } else if (active_warp && rows_pipe) {
    // --------- rows pipelined one tile deep ---------
    // Iteration q: dot products (and dweight / dbias) of row q, posted; dx of row q-1
    // once its dot product is in.
    int s = 0, sp = 0;
    uint32_t ph = 0;
    bool act_p = false;
    int64_t row_p = 0;
    float rstd_p = 0.f;
    for (int64_t q = 0; q <= n_local; ++q) {
      bool act_q = false;
      int64_t row_q = 0;
      float rstd_q = 0.f;
      const uint32_t slot = static_cast<uint32_t>(q) & 3u;
      if (q < n_local) {
        mbar_wait(&L.full[s], ph, kSiteBwdFull);
        const int64_t row0 = (cid + q * ncl) * pl.R;
        act_q = in_group && row0 + gid < pl.nrows;
        row_q = row0 + gid;
        float dot = 0.f;
        if (act_q) {
          const RowPtrs rp = row_ptrs(s, gid);
          float part[kVecs], rstd_k[kVecs];
          pass1(rp, part, rstd_k);
          rstd_q = ld1(&rp.rstd[0]);
#pragma unroll
          for (int k = 0; k < kVecs; ++k) dot += part[k];
        }
        group_post(dot, L, gid, warp, lane, slot);
      }
      if (q >= 1) {
        const float c = group_take(pl, L, gid, lane, (slot + 3u) & 3u, static_cast<uint32_t>((q - 1) >> 2)) * inv_n;
        if (act_p) {
          float rstd_k[kVecs], c_k[kVecs];
#pragma unroll
          for (int k = 0; k < kVecs; ++k) { rstd_k[k] = rstd_p; c_k[k] = c; }
          pass2(row_ptrs(sp, gid), row_p, rstd_k, c_k);
        }
        if (release_slot(L, sp, nwarps) && q - 1 + S < n_local) issue_unit(q - 1 + S, sp);
      }
      if (q < n_local) {
        sp = s;
        if (++s == S) { s = 0; ph ^= 1u; }
      }
      act_p = act_q;
      row_p = row_q;
      rstd_p = rstd_q;
    }
  } else if (active_warp && pl.P == 1) {
    // ------------------------------- tile loop -------------------------------
    int s = 0;
    uint32_t ph = 0;
    uint32_t seq = 0;
    for (int64_t q = 0; q < n_local; ++q) {
      const int64_t tile = cid + q * ncl;
      mbar_wait(&L.full[s], ph, kSiteBwdFull);
      const int64_t row0 = tile * pl.R;
      const int rows = static_cast<int>(min(static_cast<int64_t>(pl.R), pl.nrows - row0));
      for (int sw = 0; sw < pl.R; sw += pl.rps) {
        const int lr = sw + gid;
        const bool active = in_group && lr < rows;
        const unsigned amask = __ballot_sync(0xffffffffu, active);
        if (!active) continue;
        const RowPtrs rp = row_ptrs(s, lr);
        float part[kVecs], rstd_k[kVecs], c_k[kVecs];
        pass1(rp, part, rstd_k);
        if (pl.seg_mode) {
          seg_reduce<kVecs>(part, c_k, pl.vs, amask, [&](float t) { return t * inv_n; });
        } else {
          float dot = 0.f;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) dot += part[k];
          const float c = group_sum(dot, pl, L, gid, gl, seq++) * inv_n;
#pragma unroll
          for (int k = 0; k < kVecs; ++k) c_k[k] = c;
        }
        pass2(rp, row0 + lr, rstd_k, c_k);
      }
      if (release_slot(L, s, nwarps) && q + S < n_local)
        issue_unit(q + S, s);
      if (++s == S) { s = 0; ph ^= 1u; }
    }
  } else if (active_warp && !kTmemAcc) {  // (TMEM-accumulator kernels are planned for P == 1 only)
    // --------- split-row loop (rows split over the cluster, one row per tile) ---------
    const int lag = pl.lag;
    int s1 = 0, s2 = 0;
    uint32_t ph1 = 0;
    for (int64_t i = 0; i < n_local + lag; ++i) {
      const int64_t r2 = i - lag;
      const XRecord pre =
          r2 >= 0 && (!pl.xbcast || warp == 0) ? xrec_load(pl, xc, lane, static_cast<uint32_t>(r2)) : 0ull;
      if (i < n_local) {
        float part[kVecs];
        if (K == 1) {
          mbar_wait(&L.full[s1], ph1, kSiteBwdFull);
          float rstd_k[kVecs];
          pass1(row_ptrs(s1, 0), part, rstd_k);
        } else {
          for (int j = 0; j < K; ++j) {
            uint32_t ph;
            const int s = chunk_slot(s1, ph1, j, S, &ph);
            mbar_wait(&L.full[s], ph, kSiteBwdFull);
          }
          pass1c(s1, row_ptrs(s1, 0).rstd[0], part);
        }
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) dot += part[k];
        dot = group_sum(dot, pl, L, 0, gl, static_cast<uint32_t>(i));
        cluster_send(dot, pl, L, xc, warp, lane, static_cast<uint32_t>(i), rank);
        s1 += K;
        if (s1 >= S) { s1 -= S; ph1 ^= 1u; }
      }
      if (r2 >= 0 && r2 < n_local) {
        const float c = cluster_recv(pl, L, xc, warp, lane, static_cast<uint32_t>(r2), pre, kSiteBwdCluster) * inv_n;
        const int64_t row = cid + r2 * ncl;
        const RowPtrs rp = row_ptrs(s2, 0);
        if (in_group) {
          if (K == 1) {
            float rstd_k[kVecs], c_k[kVecs];
#pragma unroll
            for (int k = 0; k < kVecs; ++k) { rstd_k[k] = ld1(&rp.rstd[0]); c_k[k] = c; }
            pass2(rp, row, rstd_k, c_k);
          } else {
            pass2c(s2, row, ld1(&rp.rstd[0]), c);
          }
        }
        for (int j = 0; j < K; ++j) {
          uint32_t ph;
          const int s = chunk_slot(s2, 0u, j, S, &ph);
          const int64_t un = r2 * K + j + S;  // unit that refills the slot
          if (release_slot(L, s, nwarps) && un < n_units)
            issue_unit(un, s);
        }
        s2 += K;
        if (s2 >= S) s2 -= S;
      }
    }
  }
  __syncthreads();
  if (tid == 0 && abort_requested()) drain_after_failure(pl, L, n_units);
  if (pl.P > 1 && pl.xmode == kXCluster) cluster_sync_all();

  // one partial row per (cluster, row group): the groups of a CTA own the same columns.
  // Every owned column is written, zeros included, so the reduction reads no stale data.
  const int64_t pbase = (cid * pl.rps + gid) * pl.W + slice_elt0 + gl * 8;
  if constexpr (kTmemAcc) {
    tmem_wait_st();
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      float2 a[8];
      tmem_ld16(tacc + 16u * k, a);
      tmem_wait_ld();
      if ((vmask >> k) & 1u) {
        if (p.dw_part != nullptr) Pair8<float>::store(p.dw_part + pbase + k * G8, *reinterpret_cast<float2(*)[4]>(a));
        if (p.db_part != nullptr)
          Pair8<float>::store(p.db_part + pbase + k * G8, *reinterpret_cast<float2(*)[4]>(a + 4));
      }
    }
    // every warp's TMEM accesses are done before warp 0 frees the columns
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
    if (warp == 0) tmem_dealloc_warp(*L.tmem, kTmemCols);
  } else {
#pragma unroll
    for (int k = 0; k < kCols; ++k) {
      if ((vmask >> k) & 1u) {
        if (p.dw_part != nullptr) Pair8<float>::store(p.dw_part + pbase + k * G8, dw[k % kAcc]);
        if constexpr (kHasDb) {
          if (p.db_part != nullptr) Pair8<float>::store(p.db_part + pbase + k * G8, db[kHasDb ? k : 0]);
        }
      }
    }
  }
}

}  // namespace rmsb200
