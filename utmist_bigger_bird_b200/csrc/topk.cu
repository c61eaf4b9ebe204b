// Row-wise top-k with positions ascending, one thread-block cluster per row.
//
// The routing top-k (RDAttention.routes, modal_rd/attention.py:180-181: torch.topk of the pooled
// column scores, then sorted), the KV-eviction selection (:252) and the decode routing top-k
// (kernels/bigger_bird_route.py:115) all pick the k largest of a few rows of up to ~1M fp32 values.
// With one CTA per row, 8 rows keep 8 of 148 SMs busy; here each row is cut into C contiguous
// segments, one CTA each, grouped in a cluster of C CTAs (C up to 16) that cooperates through
// distributed shared memory:
//
//   load     each CTA reads its segment once (coalesced) into shared memory as order-preserving
//            uint32 keys (padded one word per 32 so per-thread runs are conflict-free)
//   select   radix select, 8 bits a pass from the top: per-CTA histograms of the keys that match
//            the prefix so far, summed over the cluster through DSMEM, and the digit of the k-th
//            largest key is chosen by every CTA alike; stops early once the chosen bin is taken
//            whole
//   compact  every key above the threshold and the first `rem` keys equal to it (lowest
//            positions first, as the single-CTA kernel does), written in position order: CTA
//            offsets from a cluster-wide exclusive sum of the per-CTA counts, thread offsets from
//            block scans
//
// The result is bit-identical to the single-CTA kernel (same order keys, same tie rule).
//
// Rows longer than a 16-CTA cluster holds (16 x 49152 keys, e.g. 1M-token prompts) take two
// levels: the row is cut into S segments of ~32K keys whose top-k are selected independently (the
// same kernel on "virtual rows", positions kept absolute), the S*k candidates are gathered in
// position order, and a second top-k over them picks the final k. Every key of the row's top-k is
// in its segment's top-k (ties at a segment's cut also go to the lowest positions), and candidate
// order is position order, so the result equals the one-level selection exactly.
#include <algorithm>
#include <cooperative_groups.h>

#include "bb_common.cuh"

namespace cg = cooperative_groups;

namespace bb {

int topk_single(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                cudaStream_t stream);

namespace {

constexpr int TC_THREADS = 512;
constexpr int TC_WARPS = TC_THREADS / 32;
constexpr int TC_MAX_CLUSTER = 16;
constexpr int64_t TC_SEG_MAX = 49152;  // keys a CTA: 49152 * 4 * 33 / 32 = 198 KB of shared memory

__device__ __forceinline__ uint32_t okey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ int pad(int i) { return i + (i >> 5); }

// Exclusive block scan of one int per thread (TC_THREADS threads); total in `total`.
__device__ __forceinline__ int excl_scan(int v, int* wsum, int& total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += o;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < TC_WARPS ? wsum[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    if (lane < TC_WARPS) wsum[lane] = w;
  }
  __syncthreads();
  const int res = x - v + (warp > 0 ? wsum[warp - 1] : 0);
  total = wsum[TC_WARPS - 1];
  __syncthreads();
  return res;
}

struct TcSmem {
  unsigned int whist[TC_WARPS][256];  // per-warp histograms of one pass
  unsigned int hist[2][256];          // this CTA's histogram, double-buffered across passes
  unsigned int total[256];            // cluster-wide histogram
  int wsum[32];
  int counts[2];                      // this CTA's keys above / equal to the threshold
  uint32_t sel_bin;
  int64_t sel_rem, sel_cnt;
};

// Rows of the selection: value row r (stride n) is cut into `segs` virtual rows of `len` keys (the
// last one shorter); virtual row vr selects from keys [s * len, s * len + len) of value row
// vr / segs (s = vr % segs) and writes absolute positions to output row vr. segs = 1, len = n is a
// plain row-wise selection.
struct TkRows {
  int64_t n, len, segs;
};

template <typename OutT>
__global__ void __launch_bounds__(TC_THREADS) topk_cluster_kernel(const float* __restrict__ vals, TkRows rw,
                                                                  int64_t k, OutT* __restrict__ out,
                                                                  int64_t so_h, int64_t seg) {
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  const int64_t row = blockIdx.x / C;
  __shared__ TcSmem sm;
  extern __shared__ uint32_t keys[];  // pad(seg) words
  const int64_t vbase = (row % rw.segs) * rw.len;
  const int64_t vlen = std::min<int64_t>(rw.len, rw.n - vbase);
  const float* v = vals + (row / rw.segs) * rw.n + vbase;
  const int64_t lo = (int64_t)cr * seg;
  const int cnt = (int)std::max<int64_t>(0, std::min<int64_t>(seg, vlen - lo));
  for (int i = threadIdx.x; i < cnt; i += TC_THREADS) keys[pad(i)] = okey(__ldg(v + lo + i));
  // Thread t owns keys [t * E, t * E + E) of the segment.
  const int E = (cnt + TC_THREADS - 1) / TC_THREADS;
  const int t0 = min(cnt, (int)threadIdx.x * E), t1 = min(cnt, t0 + E);
  const int warp = threadIdx.x / 32;
  __syncthreads();

  uint32_t prefix = 0, pmask = 0;
  int64_t rem = k;
  int buf = 0;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < TC_WARPS * 256; i += TC_THREADS) (&sm.whist[0][0])[i] = 0;
    __syncthreads();
    // Scores of a row are close in magnitude, so most keys share the high digits: count hits on
    // the current bin in a register and add them once.
    uint32_t hot = 0xFFFFFFFFu;
    unsigned int hot_cnt = 0;
    for (int i = t0; i < t1; ++i) {
      const uint32_t u = keys[pad(i)];
      if ((u & pmask) == prefix) {
        const uint32_t bin = (u >> shift) & 255u;
        if (bin == hot) {
          ++hot_cnt;
        } else {
          if (hot_cnt) atomicAdd(&sm.whist[warp][hot], hot_cnt);
          hot = bin;
          hot_cnt = 1;
        }
      }
    }
    if (hot_cnt) atomicAdd(&sm.whist[warp][hot], hot_cnt);
    __syncthreads();
    if (threadIdx.x < 256) {
      unsigned int s = 0;
#pragma unroll
      for (int w = 0; w < TC_WARPS; ++w) s += sm.whist[w][threadIdx.x];
      sm.hist[buf][threadIdx.x] = s;
    }
    cluster.sync();  // every CTA's histogram of this pass is visible
    if (threadIdx.x < 256) {
      unsigned int s = 0;
      for (int c = 0; c < C; ++c) s += cluster.map_shared_rank(&sm.hist[buf][0], c)[threadIdx.x];
      sm.total[threadIdx.x] = s;
    }
    __syncthreads();
    if (warp == 0) {
      // Bins from the top: lane l sums bins 255 - 8l .. 248 - 8l, an inclusive warp scan of those
      // sums finds the lane whose range holds the rem-th key, then that lane walks its 8 bins.
      const int lane = threadIdx.x;
      int64_t part = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) part += sm.total[255 - 8 * lane - j];
      int64_t incl = part;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const bool hit = incl >= rem && incl - part < rem;
      const unsigned who = __ballot_sync(0xffffffffu, hit);
      const int64_t all = __shfl_sync(0xffffffffu, incl, 31);
      if (who == 0u) {
        // Fewer than rem keys match (k above the row length): the lowest bin, as the
        // single-CTA kernel ends up choosing.
        if (lane == 0) {
          sm.sel_bin = 0;
          sm.sel_cnt = sm.total[0];
          sm.sel_rem = rem - (all - (int64_t)sm.total[0]);
        }
      } else if (lane == __ffs(who) - 1) {
        int64_t cum = incl - part;
        int b = 255 - 8 * lane;
        for (int j = 0; j < 8; ++j, --b) {
          if (cum + sm.total[b] >= rem || j == 7) break;
          cum += sm.total[b];
        }
        sm.sel_bin = (uint32_t)b;
        sm.sel_cnt = sm.total[b];
        sm.sel_rem = rem - cum;
      }
    }
    __syncthreads();
    prefix |= sm.sel_bin << shift;
    pmask |= 255u << shift;
    rem = sm.sel_rem;
    const bool whole = sm.sel_cnt == rem;
    buf ^= 1;
    __syncthreads();
    if (whole) break;  // every key of the chosen bin is taken: the prefix alone decides
  }

  // Compaction: keys above the threshold, then the first `rem` equal keys in position order.
  int gt = 0, eq = 0;
  for (int i = t0; i < t1; ++i) {
    const uint32_t u = keys[pad(i)] & pmask;
    gt += u > prefix;
    eq += u == prefix;
  }
  int gt_cta, eq_cta;
  excl_scan(gt, sm.wsum, gt_cta);
  const int eq_before_t = excl_scan(eq, sm.wsum, eq_cta);
  if (threadIdx.x == 0) {
    sm.counts[0] = gt_cta;
    sm.counts[1] = eq_cta;
  }
  cluster.sync();
  int64_t off = 0, eq_before = 0;
  for (int c = 0; c < cr; ++c) {
    const int* rc = cluster.map_shared_rank(&sm.counts[0], c);
    const int64_t g = rc[0], e = rc[1];
    off += g + std::max<int64_t>(0, std::min<int64_t>(e, rem - eq_before));
    eq_before += e;
  }
  const int64_t cta_eq_take = std::max<int64_t>(0, std::min<int64_t>(eq_cta, rem - eq_before));
  const int eq_take_t = (int)std::max<int64_t>(0, std::min<int64_t>(eq, cta_eq_take - eq_before_t));
  int sel_total;
  const int sel_before = excl_scan(gt + eq_take_t, sm.wsum, sel_total);
  int64_t pos = off + sel_before;
  int eq_seen = 0;
  OutT* o = out + row * so_h;
  for (int i = t0; i < t1; ++i) {
    const uint32_t u = keys[pad(i)] & pmask;
    bool take = u > prefix;
    if (u == prefix) take = eq_seen++ < eq_take_t;
    if (take) {
      if (pos < k) o[pos] = (OutT)(vbase + lo + i);
      ++pos;
    }
  }
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace

namespace {

// Cluster size for `rows` rows of `n` keys: enough CTAs to cover the SMs, segments of at least
// 4096 keys, at most 16; 0 when a row does not fit one cluster's shared memory.
int cluster_size(int64_t rows, int64_t n) {
  int C = 1;
  while (C < TC_MAX_CLUSTER && rows * C < num_sms() && n / (2 * C) >= 4096) C *= 2;
  while (C < TC_MAX_CLUSTER && cdiv(n, C) > TC_SEG_MAX) C *= 2;
  return cdiv(n, C) > TC_SEG_MAX ? 0 : C;
}

// One cluster of C CTAs per (virtual) row. A launch the device refuses for its configuration
// (cluster shape or shared memory) falls back to the single-CTA kernel when the rows are plain
// rows; any other error is reported.
template <typename OutT>
int launch_cluster(const float* vals, int64_t vrows, TkRows rw, int64_t k, OutT* out, int64_t so_h, int C,
                   cudaStream_t stream) {
  const int64_t seg = cdiv(rw.len, C);
  const size_t smem = (size_t)(seg + seg / 32 + 1) * 4;
  cudaFuncSetAttribute(topk_cluster_kernel<OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (C > 8) cudaFuncSetAttribute(topk_cluster_kernel<OutT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(vrows * C));
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, topk_cluster_kernel<OutT>, vals, rw, k, out, so_h, seg);
  if (e != cudaSuccess) {
    const bool config_error = e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration ||
                              e == cudaErrorInvalidClusterSize || e == cudaErrorLaunchOutOfResources;
    if (!config_error || rw.segs != 1) return fail(BB_ERR_LAUNCH, "topk_cluster_kernel: %s", cudaGetErrorString(e));
    (void)cudaGetLastError();  // the refused launch's own error
    return topk_single(vals, vrows, rw.n, k, out, sizeof(OutT) == 8, so_h, stream);
  }
  count_launch();
  return BB_OK;
}

// Second level of a long-row selection: candidate values in position order.
__global__ void topk_gather_kernel(const float* __restrict__ vals, int64_t n, const int32_t* __restrict__ cpos,
                                   int64_t per_row, float* __restrict__ cval, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    cval[i] = __ldg(vals + (i / per_row) * n + cpos[i]);
}
template <typename OutT>
__global__ void topk_map_kernel(const int32_t* __restrict__ sel, const int32_t* __restrict__ cpos, int64_t per_row,
                                int64_t k, OutT* __restrict__ out, int64_t so_h, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k;
    out[r * so_h + i % k] = (OutT)cpos[r * per_row + sel[i]];
  }
}

// Segments of a two-level selection (0: the row fits one cluster).
int64_t long_row_segments(int64_t rows, int64_t n, int64_t k) {
  if (cluster_size(rows, n) != 0 || k > 4096 || rows * cdiv(n, 32768) * k > ((int64_t)1 << 31)) return 0;
  return std::max<int64_t>(2, n / 32768);
}

}  // namespace

size_t topk_scratch_bytes(int64_t rows, int64_t n, int64_t k) {
  const int64_t S = long_row_segments(rows, n, k);
  if (S == 0 || k <= 0) return 0;
  return align_up((size_t)rows * S * k * 4, 256) * 2 + align_up((size_t)rows * k * 4, 256);
}

// The k largest of each of `rows` rows of n fp32 values, positions ascending (ties at the cut in
// position order): the routing top-k, also used by KV eviction and decode routing. `out` holds
// int32 positions, or int64 when out64. Rows too long for one cluster use `scratch`
// (topk_scratch_bytes).
int topk_sorted(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (k <= 0 || rows <= 0 || n <= 0) return BB_OK;
  const int64_t S = long_row_segments(rows, n, k);
  if (S > 0) {
    if (!scratch || scratch_bytes < topk_scratch_bytes(rows, n, k))
      return fail(BB_ERR_WORKSPACE, "topk: scratch too small for rows of %lld keys", (long long)n);
    const int64_t per_row = S * k;
    char* w = static_cast<char*>(scratch);
    int32_t* cpos = reinterpret_cast<int32_t*>(w);
    float* cval = reinterpret_cast<float*>(w + align_up((size_t)rows * per_row * 4, 256));
    int32_t* sel = reinterpret_cast<int32_t*>(w + 2 * align_up((size_t)rows * per_row * 4, 256));
    const TkRows seg_rows{n, cdiv(n, S), S};
    const int C1 = cluster_size(rows * S, seg_rows.len);
    if (C1 == 0) return fail(BB_ERR_UNSUPPORTED, "topk: segment of %lld keys too long", (long long)seg_rows.len);
    int st = launch_cluster(vals, rows * S, seg_rows, k, cpos, k, C1, stream);
    if (st) return st;
    const int64_t total = rows * per_row;
    const int blocks = (int)std::min<int64_t>(cdiv(total, 256), 4 * num_sms());
    topk_gather_kernel<<<blocks, 256, 0, stream>>>(vals, n, cpos, per_row, cval, total);
    BB_CHECK_LAUNCH("topk_gather_kernel");
    const int C2 = cluster_size(rows, per_row);
    if (C2 == 0) return fail(BB_ERR_UNSUPPORTED, "topk: %lld candidates per row", (long long)per_row);
    st = C2 == 1 ? topk_single(cval, rows, per_row, k, sel, false, k, stream)
                 : launch_cluster(cval, rows, TkRows{per_row, per_row, 1}, k, sel, k, C2, stream);
    if (st) return st;
    const int64_t tk = rows * k;
    const int b2 = (int)std::min<int64_t>(cdiv(tk, 256), 4 * num_sms());
    if (out64)
      topk_map_kernel<<<b2, 256, 0, stream>>>(sel, cpos, per_row, k, static_cast<int64_t*>(out), so_h, tk);
    else
      topk_map_kernel<<<b2, 256, 0, stream>>>(sel, cpos, per_row, k, static_cast<int32_t*>(out), so_h, tk);
    BB_CHECK_LAUNCH("topk_map_kernel");
    return BB_OK;
  }
  const int C = cluster_size(rows, n);
  if (C <= 1 || rows * C > 65535) return topk_single(vals, rows, n, k, out, out64, so_h, stream);
  const TkRows rw{n, n, 1};
  return out64 ? launch_cluster(vals, rows, rw, k, static_cast<int64_t*>(out), so_h, C, stream)
               : launch_cluster(vals, rows, rw, k, static_cast<int32_t*>(out), so_h, C, stream);
}

}  // namespace bb
