// generic_kernels.cuh -- kernels for every case the streaming kernels do not take:
// hidden sizes that are not a multiple of 8, pointers that are not 16-byte aligned,
// dtype combinations outside the specialised set, per-head segments whose length is not
// a power of two <= 32 vectors, and rows too long for the cluster split. They compute
// the same fp32 math with scalar runtime-typed loads (one CTA per row, grid-stride) and
// keep dweight/dbias deterministic with fixed-order chunked column sums.
#pragma once

#include "device_common.cuh"

namespace rmsb200 {

constexpr int kGenericThreads = 256;

struct GenFwdParams {
  int64_t rows, N;
  int32_t H;
  const void* x; int32_t x_dt;
  const void* res; int32_t res_dt;
  const void* w; int32_t w_dt, w_ph;
  const void* b; int32_t b_dt, b_ph;
  void* out; int32_t out_dt;
  void* ro; int32_t ro_dt;
  float* rstd;
  float eps;
};

struct GenBwdParams {
  int64_t rows, N;
  int32_t H;
  const void* x; int32_t x_dt;
  const void* dy; int32_t dy_dt;
  const float* rstd;
  const void* w; int32_t w_dt, w_ph;
  const void* dro; int32_t dro_dt;
  void* dx; int32_t dx_dt;
  void* dres; int32_t dres_dt;
};

// Block-wide sum, summed in warp order so every thread gets the same bits.
__device__ __forceinline__ float block_sum_fixed(float v, float* red) {
  v = warp_sum(v);
  const int nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int j = 0; j < nw; ++j) t += red[j];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kGenericThreads) fwd_generic_kernel(const GenFwdParams p) {
  __shared__ float red[32];
  const int64_t N = p.N;
  for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const int64_t base = r * N;
    const int64_t head = r % p.H;
    float acc = 0.f;
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
      float v = load1_rt(p.x, p.x_dt, base + n);
      if (p.res) v += load1_rt(p.res, p.res_dt, base + n);
      acc = fmaf(v, v, acc);
    }
    acc = block_sum_fixed(acc, red);
    const float rs = rsqrtf(acc / static_cast<float>(N) + p.eps);
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
      float v = load1_rt(p.x, p.x_dt, base + n);
      if (p.res) v += load1_rt(p.res, p.res_dt, base + n);
      if (p.ro) store1_rt(p.ro, p.ro_dt, base + n, v);
      const float w = p.w ? load1_rt(p.w, p.w_dt, (p.w_ph ? head * N : 0) + n) : 1.f;
      const float b = p.b ? load1_rt(p.b, p.b_dt, (p.b_ph ? head * N : 0) + n) : 0.f;
      store1_rt(p.out, p.out_dt, base + n, fmaf(v * rs, w, b));
    }
    if (threadIdx.x == 0 && p.rstd) st1(&p.rstd[r], rs);
  }
}

// LayerNorm forward, generic path: mean, then the mean of squared deviations (two passes,
// so the variance has no cancellation), then out = (x - mean) * rstd * w + b. `out` may be
// null (statistics only); w null = ones, b null = zeros.
struct GenLnParams {
  int64_t rows, N;
  const void* x; int32_t x_dt;
  const void* w; int32_t w_dt;
  const void* b; int32_t b_dt;
  void* out; int32_t out_dt;
  float* mean;
  float* rstd;
  float eps;
};

__global__ void __launch_bounds__(kGenericThreads) ln_generic_kernel(const GenLnParams p) {
  __shared__ float red[32];
  const int64_t N = p.N;
  const float inv_n = 1.f / static_cast<float>(N);
  for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const int64_t base = r * N;
    float acc = 0.f;
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) acc += load1_rt(p.x, p.x_dt, base + n);
    const float mean = block_sum_fixed(acc, red) * inv_n;
    acc = 0.f;
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
      const float d = load1_rt(p.x, p.x_dt, base + n) - mean;
      acc = fmaf(d, d, acc);
    }
    const float rs = rsqrtf(fmaf(block_sum_fixed(acc, red), inv_n, p.eps));
    if (p.out) {
      for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
        const float d = load1_rt(p.x, p.x_dt, base + n) - mean;
        const float w = p.w ? load1_rt(p.w, p.w_dt, n) : 1.f;
        const float b = p.b ? load1_rt(p.b, p.b_dt, n) : 0.f;
        store1_rt(p.out, p.out_dt, base + n, fmaf(d * rs, w, b));
      }
    }
    if (threadIdx.x == 0) {
      if (p.mean) st1(&p.mean[r], mean);
      if (p.rstd) st1(&p.rstd[r], rs);
    }
  }
}

__global__ void __launch_bounds__(kGenericThreads) bwd_generic_dx_kernel(const GenBwdParams p) {
  __shared__ float red[32];
  const int64_t N = p.N;
  for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const int64_t base = r * N;
    const int64_t woff = p.w_ph ? (r % p.H) * N : 0;
    const float rs = ld1(&p.rstd[r]);
    float acc = 0.f;
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
      const float xh = load1_rt(p.x, p.x_dt, base + n) * rs;
      const float w = p.w ? load1_rt(p.w, p.w_dt, woff + n) : 1.f;
      acc = fmaf(xh, load1_rt(p.dy, p.dy_dt, base + n) * w, acc);
    }
    acc = block_sum_fixed(acc, red);
    const float c = acc / static_cast<float>(N);
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
      const float xh = load1_rt(p.x, p.x_dt, base + n) * rs;
      const float w = p.w ? load1_rt(p.w, p.w_dt, woff + n) : 1.f;
      float g = (load1_rt(p.dy, p.dy_dt, base + n) * w - xh * c) * rs;
      if (p.dro) g += load1_rt(p.dro, p.dro_dt, base + n);
      store1_rt(p.dx, p.dx_dt, base + n, g);
      if (p.dres) store1_rt(p.dres, p.dres_dt, base + n, g);
    }
  }
}

// partial[chunk][j] = sum over super-rows t of chunk (in order) of dout * xhat (and dout),
// for super-row column j in [0, H*N). Row of (t, j) is t*H + j/N.
__global__ void __launch_bounds__(kGenericThreads) bwd_generic_partials_kernel(
    const GenBwdParams p, int64_t chunk_rows, float* dw_part, float* db_part) {
  const int64_t W = p.N * p.H;
  const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= W) return;
  const int64_t nsup = p.rows / p.H;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * chunk_rows;
  const int64_t t1 = min(nsup, t0 + chunk_rows);
  const int64_t head = j / p.N;
  float dw = 0.f, db = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = t * W + j;
    const float dy = load1_rt(p.dy, p.dy_dt, e);
    const float xh = load1_rt(p.x, p.x_dt, e) * ld1(&p.rstd[t * p.H + head]);
    dw = fmaf(dy, xh, dw);
    db += dy;
  }
  if (dw_part) st1(&dw_part[static_cast<int64_t>(blockIdx.y) * W + j], dw);
  if (db_part) st1(&db_part[static_cast<int64_t>(blockIdx.y) * W + j], db);
}

// out[j] = sum over partial rows c < C and heads h < fold of part[c][h * N + j], in a fixed
// order: warp w of the block sums rows c = w, w + 16, w + 32, ... (eight rows' loads in
// flight per step, added in row order; heads innermost), then the 16 warp sums are added in
// warp order. fold = H folds a per-head super-row back onto a shared [N] parameter; fold = 1
// keeps all W = H*N columns. One lane per column (32 columns per block), so every warp load
// is a coalesced 128-byte row segment. blockIdx.y selects the job (dweight, dbias), so one
// launch reduces both. Narrow rows (per-head backwards: 1024-4096 columns, 148-600 partial
// rows) have few column blocks, so the rows are spread over 16 warps with eight loads in
// flight each, which keeps the number of dependent memory round trips per warp small.
constexpr int kReduceCols = 32;    // scalar path: columns per block (one per lane)
constexpr int kReduceVCols = 128;  // vectorised path: columns per block (four per lane)
constexpr int kReduceWarps = 16;
constexpr int kReduceThreads = kReduceCols * kReduceWarps;
constexpr int kReduceUnroll = 8;   // scalar path: partial rows in flight per warp
constexpr int kReduceBatch = 16;   // vectorised path: partial rows in flight per warp

struct ReduceJob {
  const float* part;  // [C][W] partial rows
  void* out;          // [wout]
  int64_t wout;       // output columns: N when heads are folded, else W
  int32_t fold;       // heads summed into each output column (1 = none)
  int32_t out_dt;
};

struct ReduceParams {
  ReduceJob job[2];
  int64_t C;  // partial rows
  int64_t W;  // columns of a partial row (H * N)
  int64_t N;  // columns of one head
};

// The vectorised path applies to a job without folded heads whose partial rows are
// 16-byte aligned and a multiple of 4 columns wide (the streaming kernels' partials).
__host__ __device__ __forceinline__ bool reduce_vectorised(const ReduceJob& jb, int64_t W) {
  return jb.fold == 1 && (W & 3) == 0 && (reinterpret_cast<uintptr_t>(jb.part) & 15u) == 0;
}

// Fixed-order column sums of the partial rows: warp w sums rows w, w + 16, ... in
// ascending order, then the 16 warp sums are added in warp order -- the same bits every
// run. Vectorised path: lane l owns columns 4l .. 4l + 3 of a 128-column block and a warp
// keeps up to kReduceBatch partial rows' loads in flight (the partial rows were just
// written by the backward and mostly sit in L2, so the sum is latency-bound; one batch
// covers the 148-600 rows of a streaming backward in about one round trip).
__global__ void __launch_bounds__(kReduceThreads) reduce_partials_kernel(const ReduceParams p) {
  __shared__ float acc_w[kReduceWarps][kReduceVCols];
  const ReduceJob& jb = blockIdx.y == 0 ? p.job[0] : p.job[1];  // no dynamic index into the parameters
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (reduce_vectorised(jb, p.W)) {
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kReduceVCols;
    if (base >= jb.wout) return;  // whole block idle
    const int64_t j = base + 4 * lane;  // all four columns valid or none (wout % 4 == 0)
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < jb.wout) {
      const float* col = jb.part + j;
      for (int64_t c0 = warp; c0 < p.C; c0 += kReduceWarps * kReduceBatch) {
        float4 v[kReduceBatch];
#pragma unroll
        for (int u = 0; u < kReduceBatch; ++u) {
          const int64_t c = c0 + u * kReduceWarps;
          v[u] = c < p.C ? ld_partial4(col + c * p.W) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kReduceBatch; ++u) {
          acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w;
        }
      }
    }
    *reinterpret_cast<float4*>(&acc_w[warp][4 * lane]) = acc;
    __syncthreads();
    if (threadIdx.x < kReduceVCols && base + threadIdx.x < jb.wout) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kReduceWarps; ++w) t += acc_w[w][threadIdx.x];
      store1_rt(jb.out, jb.out_dt, base + threadIdx.x, t);
    }
    return;
  }
  if (static_cast<int64_t>(blockIdx.x) * kReduceCols >= jb.wout) return;  // whole block idle
  const int64_t j = static_cast<int64_t>(blockIdx.x) * kReduceCols + lane;
  float acc = 0.f;
  if (j < jb.wout) {
    const float* col = jb.part + j;
    int64_t c = warp;
    if (jb.fold == 1) {
#pragma unroll 1
      for (; c + (kReduceUnroll - 1) * kReduceWarps < p.C; c += kReduceUnroll * kReduceWarps) {
        float v[kReduceUnroll];
#pragma unroll
        for (int u = 0; u < kReduceUnroll; ++u) v[u] = ld1(&col[(c + u * kReduceWarps) * p.W]);
#pragma unroll
        for (int u = 0; u < kReduceUnroll; ++u) acc += v[u];
      }
      for (; c < p.C; c += kReduceWarps) acc += col[c * p.W];
    } else {
      for (; c < p.C; c += kReduceWarps) {
        const float* row = col + c * p.W;
        float t = 0.f;
        for (int h = 0; h < jb.fold; ++h) t += ld1(&row[h * p.N]);
        acc += t;
      }
    }
  }
  acc_w[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && j < jb.wout) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kReduceWarps; ++w) t += acc_w[w][lane];
    store1_rt(jb.out, jb.out_dt, j, t);
  }
}

// Failure-detection self test: one CTA waits on an mbarrier that nothing arrives at.
__global__ void selftest_wait_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&bar, 0)) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        record_error(RMSNORM_B200_ERR_DEVICE_TIMEOUT, kSiteSelftest);
        break;
      }
    }
  }
}

}  // namespace rmsb200
