// stream_plan.h -- launch plan shared by the host planner and the streaming kernels.
#pragma once

#include <cstdint>

namespace rmsb200 {

// Layout vocabulary used throughout the library:
//   super-row : the H*N elements of one token; H = 1 for a shared affine. A super-row of
//               a per-head tensor holds H rows of N elements (one per head).
//   segment   : one normalisation row (N elements) inside a super-row.
//   vector    : 8 consecutive elements (16 B for fp16/bf16, 32 B for fp32).
//   slice     : the part of a super-row one CTA owns. Equal to the super-row unless the
//               row is split across a group of P CTAs (P > 1): a thread-block cluster whose
//               CTAs exchange row totals through distributed shared memory, or -- where
//               clusters of P CTAs would leave SMs idle -- P CTAs of one cooperative grid
//               that exchange them through tagged records in global memory.
//   tile      : R consecutive super-rows staged into one shared-memory stage by TMA.
//   sweep     : rps super-rows processed concurrently by rps thread groups of G threads
//               (rps * kVecs / cols super-rows in per-head column mode).
struct StreamPlan {
  int32_t T;          // threads of the CTA (multiple of 32); thread 0 also issues the copies
  int32_t G;          // consumer threads per super-row
  int32_t rps;        // super-rows per sweep (T / G)
  int32_t R;          // super-rows per tile (multiple of rps)
  int32_t S;          // shared-memory stages
  int32_t P;          // CTAs per cluster = slices per super-row
  int32_t seg_mode;   // 1: segments of `vs` vectors reduced with xor shuffles; 0: whole slice
  int32_t vs;         // segment length in vectors (seg_mode)
  int32_t vs_shift;   // log2(vs)
  int32_t vslice;     // vectors per slice
  int32_t heads;      // H
  int32_t N;          // hidden size (segment length in elements)
  int32_t nclusters;  // clusters in the grid (= CTAs when P == 1)
  int32_t K;          // ring units (chunks) per row slice: 1, or 2 / 4 for split rows (P > 1)
  int32_t kpc_shift;  // log2(thread vectors per chunk) = log2(kVecs / K)
  int32_t xmode;      // P > 1: kXCluster (DSMEM exchange) or kXGlobal (global-memory records)
  int32_t pf;         // ring units between a refill and the L2 prefetch issued with it (0 = none)
  int32_t pipe_rows;  // RMSNorm row mode: rows pipelined one tile deep (ring holds one more slot)
  int32_t xbcast;     // kXGlobal: warp 0 alone polls the records and posts the row total to
                      // the other warps (xpart / xbar of the row's slot)
  int32_t lag;        // rows the cluster exchange lags pass 1 by (P > 1): pass 2 of row i-lag
                      // follows pass 1 of row i
  int32_t xpair;      // forward split rows: rows go in pairs (one CTA-wide sum, one exchange
                      // round and one record poll per two rows); lag = 1 pair, K = 1
  int32_t cols;       // thread vectors (columns) per super-row in a sweep: the kernel's vectors
                      // per thread, or fewer in per-head column mode (each thread then covers
                      // kVecs / cols super-rows of the sweep)
  int64_t nrows;      // super-rows
  int64_t ntiles;
  int64_t W;          // super-row width in elements (H * N)
  uint32_t stage_bytes;
  uint32_t off[4];    // byte offsets within a stage: input 0, input 1, input 2, rstd
  uint32_t row_bytes[3];  // bytes of one super-row slice of inputs 0..2 (0 = absent)
};

constexpr int kMaxVecs = 4;          // vectors per thread per super-row slice
// Launch shapes: 512 threads x 1 CTA per SM, or 256 threads x 2 CTAs per SM (both give
// each thread up to 128 registers).
constexpr int kBlockLarge = 512;
constexpr int kBlockSmall = 256;
constexpr int kMaxStages = 16;
constexpr int kMaxCluster = 16;
constexpr int kSmemReserve = 2048;   // barriers + reduction scratch after the stages

// Row-total exchange of split rows (StreamPlan::xmode).
constexpr int kXCluster = 0;
constexpr int kXGlobal = 1;

// One row total of one CTA in the global-memory exchange, in one 64-bit word written and
// read whole (single-copy atomic): high half = tag, low half = the float's bits. Tag =
// 0x80000000 | (execution generation << 1) | (bit 0 of row / kXSlots). Records are kept
// per record set and per group size P, so the records of CTA c belong to one CTA group
// (CTAs c - c % P .. c - c % P + P - 1) and only that group's executions write them; the
// group's generation counter gives every execution a generation of its own, drawn on the
// device (a graph replay of the same launch parameters draws a new one). A reader waiting
// for a row therefore finds that row's word, the one of the row kXSlots before it, or a
// word of an earlier execution of the same group (a smaller generation, modulo 2^30);
// never-written records (zero) carry no valid tag.
using XRecord = unsigned long long;
constexpr int kXRecSets = 4;        // record sets, used round-robin by launch epoch
constexpr int kXRecMaxCtas = 512;   // CTAs of a global-exchange grid
constexpr int kXGroupSizes = 4;     // P = 2, 4, 8, 16 (index log2(P) - 1)

struct FwdParams {
  StreamPlan pl;
  const void* x;
  const void* res;
  const void* w;
  const void* b;
  void* out;
  void* ro;
  float* rstd;
  int32_t w_dt, b_dt;
  int32_t w_per_head, b_per_head;  // 1 when the affine tensor is [H, N]
  float eps;
  float* mean;     // LayerNorm: per-row mean (null = not stored)
  XRecord* xrec;   // kXGlobal: this launch's records for its P ([kXRecMaxCtas][kXSlots])
  uint32_t* xgen;  // kXGlobal: the generation counters of its P, one per CTA group
};

struct BwdParams {
  StreamPlan pl;
  const void* x;
  const void* dy;
  const void* dro;
  const float* rstd;
  const void* w;
  void* dx;
  void* dres;
  float* dw_part;   // [nclusters][W] fp32 or null
  float* db_part;   // [nclusters][W] fp32 or null
  int32_t w_dt;
  int32_t w_per_head;
  XRecord* xrec;   // as in FwdParams
  uint32_t* xgen;
};

}  // namespace rmsb200
