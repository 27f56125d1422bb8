// peer_allreduce.cuh -- the backward's last step across the GPUs of one node: the
// fixed-order column sums of the partial dweight / dbias rows (the work of
// reduce_partials_kernel) fused with the all-reduce of those sums over NVLink peer memory,
// in ONE kernel per rank.
//
// Every rank's buffer holds a receive area of 64-bit words [2 parities][world sources]
// [stride]; word = (call tag << 32) | float bits, written and read whole (single-copy
// atomic for aligned 8-byte accesses), so a value and its tag always arrive together and
// no fence or flag is needed. A call:
//   * draws its tag c >= 1 from this rank's device-side counter (every one of the
//     kARBlocks CTAs adds 1, so all CTAs of a call read the same c; a graph replay draws a
//     new one) -- every rank makes the same sequence of calls, so the ranks' tags agree;
//   * phase 1: each CTA reduces its column blocks of this rank's partial rows (fixed order)
//     and stores each column's value, tagged, into slot [c & 1][rank] of EVERY rank's
//     receive area (its own included) -- plain stores over NVLink, no TMA, no multicast;
//   * phase 2: each CTA waits (bounded) until slot [c & 1][q] holds tag c for every rank q
//     and each of its columns, then sums the ranks' values in rank order, so every rank
//     writes the same bits.
// Two parities suffice: a rank starts call c + 2 (overwriting parity c & 1 of its peers)
// only after its call c + 1 completed, which needed every peer's call-(c + 1) words, which
// each peer pushed only after its own call c (and all its reads of parity c & 1) ended.
// Column ownership depends only on the column count and kARBlocks, the same on every rank,
// so CTA i of one rank waits only on CTA i of the others; the grid (kARBlocks CTAs of
// kARThreads) fits a B200 at once, so those CTAs are resident together.
#pragma once

#include "device_common.cuh"
#include "generic_kernels.cuh"

namespace rmsb200 {

constexpr int kARBlocks = 128;   // CTAs of every call (the tag derivation relies on a fixed grid)
constexpr int kARThreads = 512;
constexpr int kARWarps = kARThreads / 32;
constexpr int kARCols = 128;     // output columns per column block (4 per lane)
constexpr int kARUnroll = 16;    // partial rows in flight per warp
constexpr int kMaxPeers = 8;
constexpr unsigned long long kPeerBufferHeader = 256;  // bytes before the receive area (the call counter)

__device__ unsigned long long g_peer_timeout_ns = 10000000000ull;  // 10 s: ranks may start a call apart

struct PeerParams {
  unsigned long long* recv[kMaxPeers];  // receive area of each rank, as this device addresses it
  uint32_t* seq;                        // this rank's call counter
  int32_t rank;
  int32_t world;
  int64_t stride;                       // words per (parity, source) slot
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  if (!RMSB_DBG_OK(p, 8, kDbgPeerWord)) return;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  if (!RMSB_DBG_OK(p, 8, kDbgPeerWord)) return 0ull;
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kARThreads, 1) reduce_allreduce_kernel(const ReduceParams rp, const PeerParams pp) {
  __shared__ float acc_s[kARWarps][kARCols];
  __shared__ float val_s[kARCols];
  __shared__ uint32_t tag_s;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) tag_s = atomicAdd(pp.seq, 1u) / static_cast<uint32_t>(kARBlocks) + 1u;
  __syncthreads();
  const uint32_t tag = tag_s;
  const int par = static_cast<int>(tag & 1u);
  const int64_t w0 = rp.job[0].wout;
  const int64_t w1 = rp.job[1].wout;
  const int64_t nb0 = (w0 + kARCols - 1) / kARCols;
  const int64_t nblocks = nb0 + (w1 + kARCols - 1) / kARCols;
  const unsigned long long tag_hi = static_cast<unsigned long long>(tag) << 32;

  // ---- phase 1: local column sums of the owned blocks, pushed to every rank ----
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const int jidx = b < nb0 ? 0 : 1;
    const ReduceJob& jb = jidx == 0 ? rp.job[0] : rp.job[1];
    const int64_t base = (b < nb0 ? b : b - nb0) * kARCols;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const bool vec = reduce_vectorised(jb, rp.W);
    if (vec) {
      // lane l: columns base + 4l .. base + 4l + 3 (whole or none: W and wout are multiples of 4)
      const int64_t j = base + 4 * lane;
      if (j < jb.wout) {
        const float* col = jb.part + j;
        for (int64_t c0 = warp; c0 < rp.C; c0 += kARWarps * kARUnroll) {
          float4 v[kARUnroll];  // all of a warp's rows in flight at once (typically one batch)
#pragma unroll
          for (int u = 0; u < kARUnroll; ++u) {
            const int64_t c = c0 + u * kARWarps;
            v[u] = c < rp.C ? ld_partial4(col + c * rp.W) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < kARUnroll; ++u) {
            acc[0] += v[u].x; acc[1] += v[u].y; acc[2] += v[u].z; acc[3] += v[u].w;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) acc_s[warp][4 * lane + e] = acc[e];
    } else {
      // lane l: columns base + l + 32 m (m < 4), heads folded where asked
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int64_t j = base + lane + 32 * m;
        float t = 0.f;
        if (j < jb.wout) {
          for (int64_t c = warp; c < rp.C; c += kARWarps) {
            const float* row = jb.part + c * rp.W + j;
            if (jb.fold == 1) {
              t += ld1(&row[0]);
            } else {
              float f = 0.f;
              for (int h = 0; h < jb.fold; ++h) f += ld1(&row[h * rp.N]);
              t += f;
            }
          }
        }
        acc_s[warp][lane + 32 * m] = t;
      }
    }
    __syncthreads();
    if (tid < kARCols) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kARWarps; ++w) t += acc_s[w][tid];
      val_s[tid] = t;
    }
    __syncthreads();
    // push: thread t stores column t % kARCols to ranks t / kARCols, + 4, ...
    {
      const int col = tid % kARCols;
      const int64_t j = base + col;
      if (j < jb.wout) {
        const int64_t idx = (jidx == 0 ? 0 : w0) + j;
        const unsigned long long word = tag_hi | __float_as_uint(val_s[col]);
        for (int q = tid / kARCols; q < pp.world; q += kARThreads / kARCols)
          st_relaxed_sys_u64(pp.recv[q] + (static_cast<int64_t>(par) * pp.world + pp.rank) * pp.stride + idx, word);
      }
    }
    __syncthreads();  // acc_s / val_s are reused by the next block
  }

  // ---- phase 2: every rank's values of the owned columns, summed in rank order ----
  const unsigned long long* mine = pp.recv[pp.rank] + static_cast<int64_t>(par) * pp.world * pp.stride;
  const uint64_t limit = g_peer_timeout_ns;
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const int jidx = b < nb0 ? 0 : 1;
    const ReduceJob& jb = jidx == 0 ? rp.job[0] : rp.job[1];
    const int64_t base = (b < nb0 ? b : b - nb0) * kARCols;
    if (tid < kARCols && base + tid < jb.wout) {
      const int64_t j = base + tid;
      const int64_t idx = (jidx == 0 ? 0 : w0) + j;
      float sum = 0.f;
      uint64_t t0 = 0;
      for (int q = 0; q < pp.world; ++q) {
        unsigned long long wd = ld_relaxed_sys_u64(mine + q * pp.stride + idx);
        while (static_cast<uint32_t>(wd >> 32) != tag) {
          if (abort_requested()) break;
          const uint64_t now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > limit) {
            record_error(RMSNORM_B200_ERR_DEVICE_TIMEOUT, kSitePeer);
            break;
          }
          __nanosleep(64);
          wd = ld_relaxed_sys_u64(mine + q * pp.stride + idx);
        }
        sum += __uint_as_float(static_cast<uint32_t>(wd));
      }
      store1_rt(jb.out, jb.out_dt, j, sum);
    }
  }
}

}  // namespace rmsb200
