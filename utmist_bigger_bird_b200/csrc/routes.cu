// Routing (RDAttention.routes, modal_rd/attention.py:143-174) as three kernels:
//
//   1. route_stats: per (key chunk, KV head, head block) CTA, S = Qsel . K^T on tensor cores,
//      each score rounded to the input dtype (the bf16/fp16 matmul output of :164) and scaled in
//      fp32, causal mask key > qpos -> -inf, then per-row running max/sum of exp over the chunk.
//   2. route_col: recomputes S for the chunk, p = exp(s - M) / L with the merged row statistics
//      (the fp32 softmax of :166), pools p over each query head's r routing rows (mean or max,
//      :167) and writes col[h, key]; sink columns and the Python slice [n - window:] get -1.
//   3. route_topk: per query head, an 8-bit radix select of the budget-th largest column score,
//      then an index-ordered compaction, so the routes come out sorted ascending (:173).
//
// For head_dim 128 the two score passes run on tcgen05 instead (routes_tc.cu); merge and top-k
// are shared. The mma.sync passes below serve the other head sizes and row paddings.
//
// Rows of a CTA are laid out head-major with each head's r routing queries padded to a multiple
// of 16, so every 16-row MMA tile belongs to exactly one query head and pooling is a fixed-order
// reduction (deterministic run to run).
#include <algorithm>
#include <mutex>

#include "bb_common.cuh"
#include "routes_tc.cuh"

namespace bb {

int topk_sorted(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                void* scratch, size_t scratch_bytes, cudaStream_t stream);
size_t topk_scratch_bytes(int64_t rows, int64_t n, int64_t k);
namespace {

constexpr int RT_THREADS = 256;   // 8 warps
constexpr int RT_ROWS = 256;      // rows per CTA (16 m-tiles, 2 per warp)
constexpr int RT_BN = 64;         // keys per tile
constexpr int RT_CHUNK = 1024;    // keys per CTA

template <int DP> struct RtSmem {
  static constexpr int LD = DP + 8;  // padded row (elements): conflict-free ldmatrix
  static constexpr size_t q_bytes = (size_t)RT_ROWS * LD * 2;
  static constexpr size_t k_bytes = (size_t)2 * RT_BN * LD * 2;
  static constexpr size_t red_bytes = (size_t)16 * RT_BN * 4;
  static constexpr size_t bytes = q_bytes + k_bytes + red_bytes + RT_ROWS * 8 + RT_ROWS * 8;
};

struct RtParams {
  const void* q; int64_t sq_h, sq_t;
  const void* k; int64_t sk_h, sk_t;
  const int64_t* qpos;
  int64_t n, d, r, r_pad, groups, heads_per_block, chunks;
  float scaling;
  int pool;
  int64_t lo_end, hi_start;          // col[:, :lo_end] = -1, col[:, hi_start:] = -1
  float2* stats;                     // [Hk][row_blocks][RT_ROWS][chunks]
  float2* merged;                    // [Hk][row_blocks][RT_ROWS]: softmax max and sum per row
  float* col;                        // [H][n]
  int64_t row_blocks;
};

// One warp per row: M = max_c m_c, L = sum_c l_c * exp(m_c - M) over the key chunks.
__global__ void __launch_bounds__(256) route_merge_kernel(const float2* __restrict__ stats,
                                                          float2* __restrict__ merged,
                                                          int64_t rows, int64_t chunks) {
  const int64_t row = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const float2* st = stats + row * chunks;
  float M = -INFINITY;
  for (int64_t c = lane; c < chunks; c += 32) M = fmaxf(M, st[c].x);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float L = 0.f;
  if (M != -INFINITY)
    for (int64_t c = lane; c < chunks; c += 32)
      if (st[c].x != -INFINITY) L += st[c].y * expf(st[c].x - M);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  if (lane == 0) merged[row] = make_float2(M, L);
}

// Loads the CTA's routing query rows into shared memory (zero rows for padding).
template <typename T, int DP>
__device__ __forceinline__ void rt_load_q(const RtParams& p, T* qs, int kv, int hb,
                                          int64_t* rowpos) {
  constexpr int LD = RtSmem<DP>::LD;
  const int nh = (int)min(p.heads_per_block, p.groups - (int64_t)hb * p.heads_per_block);
  const int rows = nh * (int)p.r_pad;
  const T* q = static_cast<const T*>(p.q);
  // A routing position outside [0, n) makes its row empty (never read).
  for (int i = threadIdx.x; i < RT_ROWS; i += RT_THREADS) {
    int64_t pos = -1;
    if (i < rows) {
      const int qi = i % (int)p.r_pad;
      if (qi < p.r) pos = p.qpos[qi];
      if (pos >= p.n) pos = -1;
    }
    rowpos[i] = pos < 0 ? -1 : pos;
  }
  constexpr int CH = DP / 8;  // 16-byte chunks per row
  for (int c = threadIdx.x; c < RT_ROWS * CH; c += RT_THREADS) {
    const int i = c / CH, ch = c % CH;
    bool valid = false;
    const T* src = q;
    if (i < rows && ch * 8 < p.d) {
      const int j = i / (int)p.r_pad, qi = i % (int)p.r_pad;
      if (qi < p.r && p.qpos[qi] >= 0 && p.qpos[qi] < p.n) {
        const int64_t head = (int64_t)kv * p.groups + (int64_t)hb * p.heads_per_block + j;
        src = q + head * p.sq_h + p.qpos[qi] * p.sq_t + ch * 8;
        valid = true;
      }
    }
    cp_async_16(smem_u32(qs + i * LD + ch * 8), src, valid);
  }
}

template <typename T, int DP>
__device__ __forceinline__ void rt_load_k(const RtParams& p, T* ks, int kv, int64_t key0) {
  constexpr int LD = RtSmem<DP>::LD;
  constexpr int CH = DP / 8;
  const T* k = static_cast<const T*>(p.k) + (int64_t)kv * p.sk_h;
  for (int c = threadIdx.x; c < RT_BN * CH; c += RT_THREADS) {
    const int i = c / CH, ch = c % CH;
    const int64_t key = key0 + i;
    const bool valid = key < p.n && ch * 8 < p.d;
    const T* src = valid ? k + key * p.sk_t + ch * 8 : k;
    cp_async_16(smem_u32(ks + i * LD + ch * 8), src, valid);
  }
}

// S tile (rows 32w..32w+31 of the CTA x 64 keys) into acc[2 m-tiles][8 n-tiles][4].
template <typename T, int DP>
__device__ __forceinline__ void rt_scores(const T* qs, const T* ks, float (&acc)[2][8][4]) {
  constexpr int LD = RtSmem<DP>::LD;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < DP / 16; ++kk) {
    uint32_t a[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int row = warp * 32 + mt * 16 + (lane % 16);
      const int col = kk * 16 + (lane / 16) * 8;
      ldmatrix_x4(a[mt][0], a[mt][1], a[mt][2], a[mt][3], smem_u32(qs + row * LD + col));
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of n8 tiles
      uint32_t b0, b1, b2, b3;
      const int key = np * 16 + (lane / 16) * 8 + (lane % 8);
      const int col = kk * 16 + ((lane / 8) % 2) * 8;
      ldmatrix_x4(b0, b1, b2, b3, smem_u32(ks + key * LD + col));
      const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        mma_16816<T>(acc[mt][np * 2], a[mt], bA);
        mma_16816<T>(acc[mt][np * 2 + 1], a[mt], bB);
      }
    }
  }
}

// Masked, dtype-rounded, scaled score of acc element e of (mt, nt) for this thread.
template <typename T>
__device__ __forceinline__ float rt_score(float acc, int64_t key, int64_t qpos, int64_t n,
                                          float scaling) {
  const float s = Elem<T>::round(acc) * scaling;
  return (qpos < 0 || key >= n || key > qpos) ? -INFINITY : s;
}

template <typename T, int DP>
__global__ void __launch_bounds__(RT_THREADS, 2) route_stats_kernel(RtParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  T* qs = reinterpret_cast<T*>(smem);
  T* ks = reinterpret_cast<T*>(smem + RtSmem<DP>::q_bytes);
  int64_t* rowpos = reinterpret_cast<int64_t*>(smem + RtSmem<DP>::q_bytes + RtSmem<DP>::k_bytes +
                                               RtSmem<DP>::red_bytes);
  const int chunk = blockIdx.x, kv = blockIdx.y, hb = blockIdx.z;
  const int64_t key_begin = (int64_t)chunk * RT_CHUNK;
  const int64_t key_end = min(p.n, key_begin + (int64_t)RT_CHUNK);
  const int tiles = (int)cdiv(key_end - key_begin, RT_BN);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  rt_load_q<T, DP>(p, qs, kv, hb, rowpos);
  rt_load_k<T, DP>(p, ks, kv, key_begin);
  cp_async_commit();

  // rows owned by this thread: r(mt, h) = warp*32 + mt*16 + lane/4 + 8h
  float m[2][2], l[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) { m[mt][h] = -INFINITY; l[mt][h] = 0.f; }

  for (int t = 0; t < tiles; ++t) {
    if (t + 1 < tiles) rt_load_k<T, DP>(p, ks + ((t + 1) & 1) * RT_BN * RtSmem<DP>::LD, kv,
                                        key_begin + (int64_t)(t + 1) * RT_BN);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    float acc[2][8][4];
    rt_scores<T, DP>(qs, ks + (t & 1) * RT_BN * RtSmem<DP>::LD, acc);
    const int64_t key0 = key_begin + (int64_t)t * RT_BN;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = warp * 32 + mt * 16 + lane / 4 + 8 * h;
        const int64_t qp = rowpos[row];
        float s[16];
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t key = key0 + nt * 8 + (lane % 4) * 2 + e;
            s[nt * 2 + e] = rt_score<T>(acc[mt][nt][h * 2 + e], key, qp, p.n, p.scaling);
            mx = fmaxf(mx, s[nt * 2 + e]);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(m[mt][h], mx);
        float sum = 0.f;
        if (mnew != -INFINITY) {
#pragma unroll
          for (int i = 0; i < 16; ++i) sum += __expf(s[i] - mnew);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (mnew != -INFINITY) {
          l[mt][h] = (m[mt][h] == -INFINITY ? 0.f : l[mt][h] * __expf(m[mt][h] - mnew)) + sum;
          m[mt][h] = mnew;
        }
      }
    }
    __syncthreads();
  }
  if (lane % 4 == 0) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = warp * 32 + mt * 16 + lane / 4 + 8 * h;
        const int64_t idx = (((int64_t)kv * p.row_blocks + hb) * RT_ROWS + row) * p.chunks + chunk;
        p.stats[idx] = make_float2(m[mt][h], l[mt][h]);
      }
  }
}

template <typename T, int DP>
__global__ void __launch_bounds__(RT_THREADS, 2) route_col_kernel(RtParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  T* qs = reinterpret_cast<T*>(smem);
  T* ks = reinterpret_cast<T*>(smem + RtSmem<DP>::q_bytes);
  float* red = reinterpret_cast<float*>(smem + RtSmem<DP>::q_bytes + RtSmem<DP>::k_bytes);
  int64_t* rowpos = reinterpret_cast<int64_t*>(smem + RtSmem<DP>::q_bytes + RtSmem<DP>::k_bytes +
                                               RtSmem<DP>::red_bytes);
  float2* rowstat = reinterpret_cast<float2*>(rowpos + RT_ROWS);
  const int chunk = blockIdx.x, kv = blockIdx.y, hb = blockIdx.z;
  const int64_t key_begin = (int64_t)chunk * RT_CHUNK;
  const int64_t key_end = min(p.n, key_begin + (int64_t)RT_CHUNK);
  const int tiles = (int)cdiv(key_end - key_begin, RT_BN);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nh = (int)min(p.heads_per_block, p.groups - (int64_t)hb * p.heads_per_block);
  const int mt_per_head = (int)(p.r_pad / 16);

  rt_load_q<T, DP>(p, qs, kv, hb, rowpos);
  rt_load_k<T, DP>(p, ks, kv, key_begin);
  cp_async_commit();

  for (int row = threadIdx.x; row < RT_ROWS; row += RT_THREADS) {
    // (max, 1 / sum): p = exp(s - max) / sum is evaluated as exp(s - max) * (1 / sum).
    const float2 ml = p.merged[((int64_t)kv * p.row_blocks + hb) * RT_ROWS + row];
    rowstat[row] = make_float2(ml.x, ml.y > 0.f ? 1.f / ml.y : 0.f);
  }

  for (int t = 0; t < tiles; ++t) {
    if (t + 1 < tiles) rt_load_k<T, DP>(p, ks + ((t + 1) & 1) * RT_BN * RtSmem<DP>::LD, kv,
                                        key_begin + (int64_t)(t + 1) * RT_BN);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    float acc[2][8][4];
    rt_scores<T, DP>(qs, ks + (t & 1) * RT_BN * RtSmem<DP>::LD, acc);
    const int64_t key0 = key_begin + (int64_t)t * RT_BN;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float pooled[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) pooled[i] = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = warp * 32 + mt * 16 + lane / 4 + 8 * h;
        const int64_t qp = rowpos[row];
        const float2 st = rowstat[row];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t key = key0 + nt * 8 + (lane % 4) * 2 + e;
            const float s = rt_score<T>(acc[mt][nt][h * 2 + e], key, qp, p.n, p.scaling);
            const float pr = s == -INFINITY ? 0.f : __expf(s - st.x) * st.y;
            const int i = nt * 2 + e;
            pooled[i] = p.pool == BB_POOL_MAX ? fmaxf(pooled[i], pr) : pooled[i] + pr;
          }
      }
      // Reduce over the 8 row groups of the m-tile (lane bits 2..4).
#pragma unroll
      for (int i = 0; i < 16; ++i) {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          const float o = __shfl_xor_sync(0xffffffffu, pooled[i], off);
          pooled[i] = p.pool == BB_POOL_MAX ? fmaxf(pooled[i], o) : pooled[i] + o;
        }
      }
      if (lane < 4) {
        const int mtile = warp * 2 + mt;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) red[mtile * RT_BN + nt * 8 + lane * 2 + e] = pooled[nt * 2 + e];
      }
    }
    __syncthreads();
    // Column scores of this tile for the block's heads: fixed-order sum over each head's m-tiles.
    for (int c = threadIdx.x; c < nh * RT_BN; c += RT_THREADS) {
      const int j = c / RT_BN, col = c % RT_BN;
      const int64_t key = key0 + col;
      if (key >= p.n) continue;
      float v = 0.f;
      for (int mtile = j * mt_per_head; mtile < (j + 1) * mt_per_head; ++mtile) {
        const float x = red[mtile * RT_BN + col];
        v = p.pool == BB_POOL_MAX ? fmaxf(v, x) : v + x;
      }
      if (p.pool != BB_POOL_MAX) v = v / (float)p.r;
      if (key < p.lo_end || key >= p.hi_start) v = -1.f;
      const int64_t head = (int64_t)kv * p.groups + (int64_t)hb * p.heads_per_block + j;
      p.col[head * p.n + key] = v;
    }
    __syncthreads();
  }
}

// ----------------------------------------------------------------------------- top-k
constexpr int TK_THREADS = 1024;
constexpr int TK_VEC = 16;  // scores per thread per chunk

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Inclusive block-wide scan of one int per thread (TK_THREADS threads); returns the total.
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  const int res = v + (warp > 0 ? warp_sums[warp - 1] : 0);
  total = warp_sums[31];
  __syncthreads();
  return res;
}

// Scores of elements [i0, i0 + 16) as order keys; bit e of the result marks element i0 + e < n.
__device__ __forceinline__ unsigned load16_keys(const float* __restrict__ c, int64_t i0, int64_t n, bool vec,
                                                uint32_t (&u)[TK_VEC]) {
  if (vec && i0 + TK_VEC <= n) {
    const float4* p4 = reinterpret_cast<const float4*>(c + i0);
#pragma unroll
    for (int v = 0; v < TK_VEC / 4; ++v) {
      const float4 f = __ldg(p4 + v);
      u[4 * v] = order_key(f.x);
      u[4 * v + 1] = order_key(f.y);
      u[4 * v + 2] = order_key(f.z);
      u[4 * v + 3] = order_key(f.w);
    }
    return 0xFFFFu;
  }
  unsigned valid = 0;
#pragma unroll
  for (int e = 0; e < TK_VEC; ++e) {
    const bool ok = i0 + e < n;
    u[e] = ok ? order_key(__ldg(c + i0 + e)) : 0u;
    valid |= (ok ? 1u : 0u) << e;
  }
  return valid;
}

// The lowest k set bits of m.
__device__ __forceinline__ unsigned lowest_bits(unsigned m, int k) {
  unsigned r = 0;
  for (int i = 0; i < k && m; ++i) {
    const unsigned b = m & (0u - m);
    r |= b;
    m ^= b;
  }
  return r;
}

// One CTA per query head. Each thread owns 16 consecutive scores of a 16K-score chunk (vector
// loads, 16x fewer dependent iterations than one score per thread).
template <typename OutT>
__global__ void __launch_bounds__(TK_THREADS) route_topk_kernel(const float* __restrict__ col,
                                                                int64_t n, int64_t budget,
                                                                OutT* __restrict__ out,
                                                                int64_t so_h) {
  __shared__ unsigned int hist[256];
  __shared__ int warp_sums[32];
  __shared__ uint32_t sel_bin;
  __shared__ int64_t sel_rem;
  const int64_t h = blockIdx.x;
  const float* c = col + h * n;
  OutT* o = out + h * so_h;
  if (budget <= 0) return;
  const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15) == 0);
  constexpr int64_t CHUNK = (int64_t)TK_THREADS * TK_VEC;
  uint32_t prefix = 0, pmask = 0;
  int64_t rem = budget;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += TK_THREADS) hist[i] = 0;
    __syncthreads();
    // Column scores are close in magnitude, so one digit is often shared by most keys (the top
    // byte always is): each thread counts hits on the bin of its first key in a register and adds
    // them once, instead of one shared-memory atomic per key on the same word.
    uint32_t hot = 0xFFFFFFFFu;
    unsigned int hot_cnt = 0;
    for (int64_t base = 0; base < n; base += CHUNK) {
      uint32_t u[TK_VEC];
      const unsigned valid = load16_keys(c, base + (int64_t)threadIdx.x * TK_VEC, n, vec, u);
#pragma unroll
      for (int e = 0; e < TK_VEC; ++e) {
        if (((valid >> e) & 1u) && (u[e] & pmask) == prefix) {
          const uint32_t bin = (u[e] >> shift) & 255u;
          if (bin == hot) {
            ++hot_cnt;
          } else if (hot_cnt == 0) {
            hot = bin;
            hot_cnt = 1;
          } else {
            atomicAdd(&hist[bin], 1u);
          }
        }
      }
    }
    if (hot_cnt) atomicAdd(&hist[hot], hot_cnt);
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t cum = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (cum + hist[b] >= rem) break;
        cum += hist[b];
      }
      sel_bin = (uint32_t)b;
      sel_rem = rem - cum;
    }
    __syncthreads();
    prefix |= sel_bin << shift;
    pmask |= 255u << shift;
    rem = sel_rem;
    __syncthreads();
  }
  // prefix = key of the budget-th largest score; take every key above it and the first `rem`
  // keys equal to it, in index order.
  int64_t written = 0, eq_seen = 0;
  for (int64_t base = 0; base < n && written < budget; base += CHUNK) {
    const int64_t i0 = base + (int64_t)threadIdx.x * TK_VEC;
    uint32_t u[TK_VEC];
    const unsigned valid = load16_keys(c, i0, n, vec, u);
    unsigned gtm = 0, eqm = 0;
#pragma unroll
    for (int e = 0; e < TK_VEC; ++e) {
      if ((valid >> e) & 1u) {
        gtm |= (u[e] > prefix ? 1u : 0u) << e;
        eqm |= (u[e] == prefix ? 1u : 0u) << e;
      }
    }
    const int eq_cnt = __popc(eqm);
    int eq_total;
    const int eq_incl = block_scan(eq_cnt, warp_sums, eq_total);
    const int64_t eq_before = eq_seen + eq_incl - eq_cnt;
    const int64_t eq_take = rem - eq_before < 0 ? 0 : (rem - eq_before > eq_cnt ? eq_cnt : rem - eq_before);
    const unsigned takem = gtm | lowest_bits(eqm, (int)eq_take);
    const int tk = __popc(takem);
    int take_total;
    const int take_incl = block_scan(tk, warp_sums, take_total);
    int64_t pos = written + take_incl - tk;
#pragma unroll
    for (int e = 0; e < TK_VEC; ++e) {
      if ((takem >> e) & 1u) {
        if (pos < budget) o[pos] = (OutT)(i0 + e);
        ++pos;
      }
    }
    written += take_total;
    eq_seen += eq_total;
  }
}

int64_t slice_start(int64_t n, int64_t s) {  // Python slice start semantics for a[s:]
  if (s < 0) s = std::max<int64_t>(0, n + s);
  return std::min(s, n);
}

struct RtPlan {
  int64_t r_pad, heads_per_block, row_blocks, chunks, groups;
  bool tc;                                        // tcgen05 score passes (routes_tc.cu)
  size_t partial_bytes, stats_bytes, col_bytes;   // stats_bytes = partials + merged rows
  size_t topk_bytes;                              // long-row top-k scratch (after the column scores)
};

int plan_routes(const bb_routes_args* a, RtPlan* pl) {
  if (!a) return fail(BB_ERR_ARG, "routes: null args");
  if (a->dtype != BB_BF16 && a->dtype != BB_F16) return fail(BB_ERR_DTYPE, "routes: dtype must be f16 or bf16");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
    return fail(BB_ERR_SHAPE, "routes: heads must be a positive multiple of kv_heads");
  if (a->d <= 0 || a->d > 128 || a->d % 8) return fail(BB_ERR_UNSUPPORTED, "routes: head_dim must be a multiple of 8 and <= 128");
  if (a->n <= 0 || a->r <= 0 || a->r > a->n) return fail(BB_ERR_SHAPE, "routes: need 0 < r <= n");
  if (a->r > RT_ROWS) return fail(BB_ERR_UNSUPPORTED, "routes: n_route > %d not supported", RT_ROWS);
  if (a->budget < 0 || a->budget > a->n) return fail(BB_ERR_ARG, "routes: bad budget");
  pl->groups = a->heads / a->kv_heads;
  pl->r_pad = (a->r + 15) / 16 * 16;
  pl->tc = routes_tc_eligible(a->d, pl->r_pad, pl->groups, a->dtype, a->scaling);
  if (pl->tc) {
    // One row block of RT_ROWS rows per KV head; a statistics "chunk" per CTA of the KV head.
    pl->heads_per_block = pl->groups;
    pl->row_blocks = 1;
    pl->chunks = routes_tc_cpk(a->kv_heads, a->n);
  } else {
    pl->heads_per_block = std::max<int64_t>(1, std::min<int64_t>(pl->groups, RT_ROWS / pl->r_pad));
    pl->row_blocks = cdiv(pl->groups, pl->heads_per_block);
    pl->chunks = cdiv(a->n, RT_CHUNK);
  }
  pl->partial_bytes = align_up((size_t)a->kv_heads * pl->row_blocks * RT_ROWS * pl->chunks * sizeof(float2), 256);
  pl->stats_bytes = pl->partial_bytes + align_up((size_t)a->kv_heads * pl->row_blocks * RT_ROWS * sizeof(float2), 256);
  pl->col_bytes = a->out_col ? 0 : align_up((size_t)a->heads * a->n * sizeof(float), 256);
  pl->topk_bytes = align_up(topk_scratch_bytes(a->heads, a->n, a->budget), 256);
  return BB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T, int DP>
int launch_routes_t(const bb_routes_args* a, const RtPlan& pl, char* ws, cudaStream_t stream) {
  RtParams p;
  p.q = a->q; p.sq_h = a->sq_h; p.sq_t = a->sq_t;
  p.k = a->k; p.sk_h = a->sk_h; p.sk_t = a->sk_t;
  p.qpos = a->qpos;
  p.n = a->n; p.d = a->d; p.r = a->r; p.r_pad = pl.r_pad; p.groups = pl.groups;
  p.heads_per_block = pl.heads_per_block; p.chunks = pl.chunks; p.row_blocks = pl.row_blocks;
  p.scaling = a->scaling; p.pool = a->pool;
  p.lo_end = a->sink < 0 ? std::max<int64_t>(0, a->n + a->sink) : std::min(a->sink, a->n);
  p.hi_start = slice_start(a->n, a->n - a->window);
  p.stats = reinterpret_cast<float2*>(ws);
  p.merged = reinterpret_cast<float2*>(ws + pl.partial_bytes);
  p.col = a->out_col ? a->out_col : reinterpret_cast<float*>(ws + pl.stats_bytes);
  const int64_t rows = a->kv_heads * pl.row_blocks * RT_ROWS;
  if (pl.tc) {
    RtTcArgs t;
    t.q = a->q; t.sq_h = a->sq_h; t.sq_t = a->sq_t;
    t.k = a->k; t.sk_h = a->sk_h; t.sk_t = a->sk_t;
    t.qpos = a->qpos;
    t.n = a->n; t.r = a->r; t.r_pad = pl.r_pad; t.groups = pl.groups; t.kv_heads = a->kv_heads;
    t.cpk = pl.chunks;
    t.scaling = a->scaling; t.pool = a->pool; t.dtype = a->dtype;
    t.lo_end = p.lo_end; t.hi_start = p.hi_start;
    t.stats = p.stats; t.merged = p.merged; t.col = p.col;
    int st = routes_tc_stats(t, stream);
    if (st) return st;
    route_merge_kernel<<<(unsigned)cdiv(rows, 8), 256, 0, stream>>>(p.stats, p.merged, rows, pl.chunks);
    BB_CHECK_LAUNCH("route_merge_kernel");
    st = routes_tc_col(t, stream);
    if (st) return st;
  } else {
    const size_t smem = RtSmem<DP>::bytes;
    cudaFuncSetAttribute(route_stats_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(route_col_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)pl.chunks, (unsigned)a->kv_heads, (unsigned)pl.row_blocks);
    route_stats_kernel<T, DP><<<grid, RT_THREADS, smem, stream>>>(p);
    BB_CHECK_LAUNCH("route_stats_kernel");
    route_merge_kernel<<<(unsigned)cdiv(rows, 8), 256, 0, stream>>>(p.stats, p.merged, rows, pl.chunks);
    BB_CHECK_LAUNCH("route_merge_kernel");
    route_col_kernel<T, DP><<<grid, RT_THREADS, smem, stream>>>(p);
    BB_CHECK_LAUNCH("route_col_kernel");
  }
  if (a->budget > 0)
    return topk_sorted(p.col, a->heads, a->n, a->budget, a->out_idx, false, a->so_h,
                       ws + pl.stats_bytes + pl.col_bytes, pl.topk_bytes, stream);
  return BB_OK;
}

template <typename T>
int launch_routes_d(const bb_routes_args* a, const RtPlan& pl, char* ws, cudaStream_t s) {
  if (a->d <= 32) return launch_routes_t<T, 32>(a, pl, ws, s);
  if (a->d <= 64) return launch_routes_t<T, 64>(a, pl, ws, s);
  return launch_routes_t<T, 128>(a, pl, ws, s);
}

}  // namespace

// The k largest of each of `rows` rows of n fp32 values, positions ascending (ties at the cut in
// position order), one CTA a row: rows too long for the cluster kernel of topk.cu.
int topk_single(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                cudaStream_t stream) {
  if (k <= 0 || rows <= 0) return BB_OK;
  if (out64)
    route_topk_kernel<<<(unsigned)rows, TK_THREADS, 0, stream>>>(vals, n, k, static_cast<int64_t*>(out), so_h);
  else
    route_topk_kernel<<<(unsigned)rows, TK_THREADS, 0, stream>>>(vals, n, k, static_cast<int32_t*>(out), so_h);
  BB_CHECK_LAUNCH("route_topk_kernel");
  return BB_OK;
}

int routes_workspace_size(const bb_routes_args* a, size_t* bytes) {
  RtPlan pl;
  int st = plan_routes(a, &pl);
  if (st) return st;
  *bytes = pl.stats_bytes + pl.col_bytes + pl.topk_bytes;
  return BB_OK;
}

int routes(const bb_routes_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  RtPlan pl;
  int st = plan_routes(a, &pl);
  if (st) return st;
  const size_t need = pl.stats_bytes + pl.col_bytes + pl.topk_bytes;
  if (ws_bytes < need || (!ws && need))
    return fail(BB_ERR_WORKSPACE, "routes: workspace too small (%zu < %zu)", ws_bytes, need);
  if (!a->q || !a->k || !a->qpos || (a->budget > 0 && !a->out_idx)) return fail(BB_ERR_ARG, "routes: null pointer");
  if (!aligned16(a->q) || !aligned16(a->k) || (a->sq_h * 2) % 16 || (a->sq_t * 2) % 16 ||
      (a->sk_h * 2) % 16 || (a->sk_t * 2) % 16)
    return fail(BB_ERR_STRIDE, "routes: q/k rows must start on 16-byte boundaries");
  char* w = static_cast<char*>(ws);
  if (a->dtype == BB_BF16) return launch_routes_d<__nv_bfloat16>(a, pl, w, stream);
  return launch_routes_d<__half>(a, pl, w, stream);
}

}  // namespace bb

// ---------------------------------------------------------------------------------------------
// bb_routes_noalloc: routing with its scratch in a fixed device array instead of a caller
// workspace, for hosts that cannot hand out device memory (a program that has reserved the GPU
// for its own pool, or an FFI caller without a device allocator). The array is allocated when
// the library's module is loaded on a device and is held by that device until the process
// exits; nothing here calls cudaMalloc, cudaFree or an allocating library routine.
//
// Host code must not pass `g_routes_scratch` itself to a kernel: in host code the name is a
// host-side stand-in, not a device address. The device address is looked up once per device
// with cudaGetSymbolAddress, with that device current, on the first call made on it.
static __device__ __align__(256) unsigned char g_routes_scratch[BB_ROUTES_NOALLOC_SCRATCH_BYTES];

namespace bb {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int routes_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(BB_ERR_DEVICE, "routes_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(BB_ERR_DEVICE, "routes_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_routes_scratch);
    if (e != cudaSuccess || !p)
      return fail(BB_ERR_DEVICE, "routes_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return BB_OK;
}

}  // namespace
}  // namespace bb

extern "C" int bb_routes_noalloc(const bb_routes_args* a, bb_stream_t stream) {
  size_t need = 0;
  int st = bb::routes_workspace_size(a, &need);
  if (st) return st;
  if (need > BB_ROUTES_NOALLOC_SCRATCH_BYTES)
    return bb::fail(BB_ERR_WORKSPACE,
                    "routes_noalloc: this request needs %zu bytes of scratch, more than the library's "
                    "fixed %zu; use bb_routes with a caller workspace",
                    need, (size_t)BB_ROUTES_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  st = bb::routes_scratch_address(&scratch);
  if (st) return st;
  // Every scratch byte the routing kernels read is written earlier in the same call (row
  // statistics, merged statistics, column scores), so the previous call's contents need no clearing.
  return bb::routes(a, scratch, BB_ROUTES_NOALLOC_SCRATCH_BYTES, bb::as_stream(stream));
}
