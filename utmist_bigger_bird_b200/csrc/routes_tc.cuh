// tcgen05 routing passes (RDAttention.routes, modal_rd/attention.py:143-174) for head_dim 128.
#pragma once
#include "bb_common.cuh"

namespace bb {

// One routing call as the tcgen05 passes see it. Rows of a KV head are its query heads' routing
// queries, head-major, each head padded to r_pad rows (r_pad in {16, 32, 64}, groups * r_pad <=
// 256); row i of KV head kv is query head kv * groups + i / r_pad at position qpos[i % r_pad].
struct RtTcArgs {
  const void* q;
  int64_t sq_h, sq_t;
  const void* k;
  int64_t sk_h, sk_t;
  const int64_t* qpos;
  int64_t n, r, r_pad, groups, kv_heads;
  int64_t cpk;  // CTAs per KV head (each takes a contiguous range of 128-key tiles)
  float scaling;
  int pool;
  int dtype;
  int64_t lo_end, hi_start;  // col[:, :lo_end] = -1 and col[:, hi_start:] = -1
  float2* stats;             // [kv_heads][256][cpk]: per-row (max, sum of exp) over a CTA's keys
  const float2* merged;      // [kv_heads][256]: softmax max and sum over all keys
  float* col;                // [heads][n]
};

// True when the tcgen05 passes handle this call (they take the row max on unscaled scores,
// so the scale must be positive).
bool routes_tc_eligible(int64_t d, int64_t r_pad, int64_t groups, int dtype, float scaling);
// CTAs per KV head for this device.
int64_t routes_tc_cpk(int64_t kv_heads, int64_t n);
// Pass 1: per-row softmax statistics of each CTA's key range.
int routes_tc_stats(const RtTcArgs& a, cudaStream_t stream);
// Pass 2: column scores (pooled softmax) and the -1 sink/window columns.
int routes_tc_col(const RtTcArgs& a, cudaStream_t stream);

}  // namespace bb
