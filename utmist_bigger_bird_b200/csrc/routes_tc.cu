// Routing on tcgen05 for head_dim 128 (RDAttention.routes, modal_rd/attention.py:143-174): the
// two score passes of routes.cu (row softmax statistics, then pooled column scores) as persistent,
// warp-specialised kernels. Each CTA owns a contiguous range of 128-key tiles of one KV head;
// its routing query rows (<= 256) stay in shared memory, K tiles arrive by TMA (128B swizzle) in
// a 4-slot ring, and the scores go to TMEM (two buffers, so the MMA of the next tile overlaps the
// exponentials of this one). 320 threads: producer (warp 0), MMA issuer (warp 1), 8 score warps.
//
//   pass 1  S = Q K^T with the routing rows on TMEM lanes (two M = 128 halves, N = 128 keys):
//           each score warp thread owns one row and keeps its running (max, sum of exp) over the
//           CTA's keys: score = dtype-rounded dot product * scaling (the bf16/fp16 matmul output
//           of :164, then fp32), key > qpos -> -inf (:165).
//   pass 2  S^T = K Q^T with the keys on TMEM lanes (M = 128 keys, N = 256 rows): each thread owns
//           one key and pools p = exp(s - M_row) / L_row over its heads' rows (mean or max, :167)
//           with the merged statistics; sink columns and the Python slice [n - window:] get -1
//           (:169-170) and are not computed.
//
// Both passes are bound by the SM's exponential unit (one exp per (row, key): 32768 per tile).
#include <algorithm>

#include "flash.cuh"
#include "routes_tc.cuh"
#include "tc_common.cuh"

namespace bb {
namespace rtc {
using namespace tc;

constexpr int THREADS = 320;
constexpr int ROWS = 256;
constexpr int NB = 4;
constexpr uint32_t SM_Q = 0;                    // routing rows, 64 KB
constexpr uint32_t SM_K = 2 * TILE;             // K ring, NB x 32 KB
constexpr uint32_t SM_ROWPOS = SM_K + NB * TILE;  // [256] int64 query position (-1: padding)
constexpr uint32_t SM_ROWSTAT = SM_ROWPOS + ROWS * 8;  // [256] float: pass-2 exponent bias
enum { B_Q = 0, B_KF = 1, B_KE = B_KF + NB, B_SF = B_KE + NB, B_SE = B_SF + 2, B_DONE = B_SE + 2,
       N_BARS = B_DONE + 1 };
constexpr uint32_t SM_BAR = SM_ROWSTAT + ROWS * 4;
constexpr uint32_t SM_MISC = SM_BAR + N_BARS * 8;  // [0] TMEM base, [1] abort flag
constexpr uint32_t SM_ALLOC = SM_MISC + 16 + 1024;
static_assert(SM_ALLOC <= 232448, "routing kernels exceed the 227 KB shared memory limit");

constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float LN2_F = 0.6931471805599453f;
// Lazy rescale of a row's running sum: the reference max moves only when a tile's max passes it
// by more than 8 (log2 units), so every exp2 argument stays <= 8.
constexpr float RESCALE = 8.0f;

// Fault codes (this unit's fault word): which wait gave up.
enum { F_RT_Q = 16, F_RT_K = 17, F_RT_S = 18, F_RT_SE = 19, F_RT_KE = 20 };

__device__ __forceinline__ void tile_range(int64_t first, int64_t count, int64_t cpk, int64_t c, int64_t& t0,
                                           int64_t& t1) {
  t0 = first + count * c / cpk;
  t1 = first + count * (c + 1) / cpk;
}

// Position of routing row i of a KV head, or -1 for a padding row / out-of-range position.
__device__ __forceinline__ int64_t row_position(const RtTcArgs& a, int i) {
  if (i >= (int)(a.groups * a.r_pad)) return -1;
  const int qi = i % (int)a.r_pad;
  if (qi >= a.r) return -1;
  const int64_t ps = a.qpos[qi];
  return (ps >= 0 && ps < a.n) ? ps : -1;
}

// Gathers the 256 routing rows of KV head `kv` into the 128B-swizzled K-major layout with
// cp.async (zero rows for padding). SPLIT: two 128-row halves, each [2 d-halves][128][64] (pass
// 1, A operand); otherwise [2 d-halves][256][64] (pass 2, B operand with N = 256).
template <typename T, bool SPLIT>
__device__ __forceinline__ void load_rows(const RtTcArgs& a, uint32_t qs, int64_t kv, int lane, const int64_t* rowpos) {
  const T* q = static_cast<const T*>(a.q);
  for (int idx = lane; idx < ROWS * 16; idx += 32) {
    const int i = idx >> 4, c = idx & 15;
    const int64_t ps = rowpos[i];
    const T* src = q;
    if (ps >= 0) src = q + (kv * a.groups + i / (int)a.r_pad) * a.sq_h + ps * a.sq_t + c * 8;
    uint32_t dst;
    if (SPLIT) {
      const int m = i >> 7, r = i & 127;
      dst = qs + (uint32_t)m * TILE + (uint32_t)(c >> 3) * HALF + (uint32_t)r * 128u + (uint32_t)(((c & 7) ^ (r & 7)) << 4);
    } else {
      dst = qs + (uint32_t)(c >> 3) * (2u * HALF) + (uint32_t)i * 128u + (uint32_t)(((c & 7) ^ (i & 7)) << 4);
    }
    cp_async_16(dst, src, ps >= 0);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
}

// Producer: the CTA's K tiles [t0, t1) of KV head kv into the ring (TMA, zero fill past n).
__device__ __forceinline__ void produce_k(const CUtensorMap* kmap, int kswap, int64_t kv, int64_t t0, int nt,
                                          uint32_t sbase, Abort abort_flag, uint32_t bars) {
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  int fills[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) fills[i] = 0;
  for (int it = 0; it < nt; ++it) {
    const int b = it % NB, round = it / NB;
    if (round > 0 && !mbar_wait_warp(bar(B_KE + b), (round - 1) & 1, abort_flag, F_RT_KE)) break;
    const int key = (int)((t0 + it) * 128);
    const uint32_t dst = sbase + SM_K + (uint32_t)b * TILE;
    mbar_expect_tx_one(bar(B_KF + b), TILE);
    if (kswap) {
      tma_load_3d_one(dst, kmap, 0, (int)kv, key, bar(B_KF + b));
      tma_load_3d_one(dst + HALF, kmap, 64, (int)kv, key, bar(B_KF + b));
    } else {
      tma_load_3d_one(dst, kmap, 0, key, (int)kv, bar(B_KF + b));
      tma_load_3d_one(dst + HALF, kmap, 64, key, (int)kv, bar(B_KF + b));
    }
    ++fills[b];
  }
  for (int b = 0; b < NB; ++b)
    if (fills[b] > 0) mbar_drain(bar(B_KF + b), (fills[b] - 1) & 1);
}

__device__ __forceinline__ void init_bars(uint32_t bars, volatile uint32_t* misc) {
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  mbar_init(bar(B_Q), 1);
  for (int i = 0; i < NB; ++i) {
    mbar_init(bar(B_KF + i), 1);
    mbar_init(bar(B_KE + i), 1);
  }
  for (int i = 0; i < 2; ++i) {
    mbar_init(bar(B_SF + i), 1);
    mbar_init(bar(B_SE + i), 256);
  }
  mbar_init(bar(B_DONE), 1);
  misc[1] = 0;
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ----------------------------------------------------------------------------- pass 1
template <typename T>
__global__ void __launch_bounds__(THREADS, 1) rt_stats_kernel(const __grid_constant__ CUtensorMap kmap, int kswap,
                                                              RtTcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  unsigned char* sptr = smem_raw + (sbase - raw);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sptr + SM_MISC);
  const Abort abort_flag{misc + 1, 0u};
  int64_t* rowpos = reinterpret_cast<int64_t*>(sptr + SM_ROWPOS);
  const uint32_t bars = sbase + SM_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t c = blockIdx.x, kv = blockIdx.y;
  int64_t t0, t1;
  tile_range(0, cdiv(a.n, (int64_t)128), a.cpk, c, t0, t1);
  const int nt = (int)(t1 - t0);

  for (int i = threadIdx.x; i < ROWS; i += THREADS) rowpos[i] = row_position(a, i);
  if (threadIdx.x == 0) init_bars(bars, misc);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + SM_MISC), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == 0) {
    if (nt > 0) {
      load_rows<T, true>(a, sbase + SM_Q, kv, lane, rowpos);
      mbar_arrive_one(bar(B_Q));
      produce_k(&kmap, kswap, kv, t0, nt, sbase, abort_flag, bars);
    }
  } else if (warp == 1) {
    if (nt > 0) {
      constexpr uint32_t ID = idesc<T>(false);
      bool ok = mbar_wait_warp(bar(B_Q), 0, abort_flag, F_RT_Q);
      for (int it = 0; ok && it < nt; ++it) {
        const int b = it % NB, sb = it & 1;
        if (!mbar_wait_warp(bar(B_KF + b), (it / NB) & 1, abort_flag, F_RT_K)) break;
        if (it >= 2 && !mbar_wait_warp(bar(B_SE + sb), ((it >> 1) - 1) & 1, abort_flag, F_RT_SE)) break;
        tc_fence_after();
        const uint64_t kd = desc_k(sbase + SM_K + (uint32_t)b * TILE);
        gemm_ss8(tmem + (uint32_t)sb * 256u, desc_k(sbase + SM_Q), kd, ID, 0u);
        gemm_ss8(tmem + (uint32_t)sb * 256u + 128u, desc_k(sbase + SM_Q + TILE), kd, ID, 0u);
        mma_commit_one(bar(B_SF + sb));
        mma_commit_one(bar(B_KE + b));
      }
      mma_commit_one(bar(B_DONE));
      mbar_drain(bar(B_DONE), 0);
    }
  } else {
    // Score warps: warp w reads TMEM lanes 32 * (w % 4) ..; warps 2-5 hold rows 0-127, 6-9 rows 128-255.
    const int half = (warp - 2) >> 2, wq = warp & 3;
    const int row = 128 * half + 32 * wq + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16) + 128u * (uint32_t)half;
    const int64_t qp = rowpos[row];
    const float c2 = a.scaling * LOG2E_F;  // scores in log2 units
    float m = -INFINITY, l = 0.f;
    for (int it = 0; it < nt; ++it) {
      const int sb = it & 1;
      if (!mbar_wait_warp(bar(B_SF + sb), (it >> 1) & 1, abort_flag, F_RT_S)) break;
      tc_fence_after();
      float s[128];
      tmem_ld128(tl + (uint32_t)sb * 256u, s);
      tc_fence_before();
      mbar_arrive(bar(B_SE + sb));
      if (qp < 0) continue;
      const int64_t key0 = (t0 + it) * 128;
      // Dtype-rounded dot products; the (positive) scale is applied inside the exponent below,
      // so the row max is taken on the unscaled values.
#pragma unroll
      for (int i = 0; i < 128; i += 2) round2<T>(s[i], s[i + 1]);
      if (!(key0 + 127 <= qp && key0 + 128 <= a.n)) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (key0 + i > qp || key0 + i >= a.n) s[i] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(s[k], s[8 + k]);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], s[i + k], s[i + 8 + k]);
      const float mt =
          c2 * fmaxf(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], fmax3(mx8[5], mx8[6], mx8[7])));
      if (mt > m + RESCALE) {
        if (m > -INFINITY) l *= fast_exp2(m - mt);
        m = mt;
      }
      if (m == -INFINITY) continue;
      // l += sum_i exp2(s_i * c2 - m), two lanes of the sum per packed add.
      const uint64_t c22 = f2_pack(c2, c2), nm2 = f2_pack(-m, -m);
      uint64_t l01 = f2_pack(0.f, 0.f), l23 = f2_pack(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 128; i += 4) {
        float x0, x1, x2, x3;
        f2_unpack(f2_fma(f2_pack(s[i], s[i + 1]), c22, nm2), x0, x1);
        f2_unpack(f2_fma(f2_pack(s[i + 2], s[i + 3]), c22, nm2), x2, x3);
        l01 = f2_add(l01, f2_pack(fast_exp2(x0), fast_exp2(x1)));
        l23 = f2_add(l23, f2_pack(fast_exp2(x2), fast_exp2(x3)));
      }
      float ls[4];
      f2_unpack(l01, ls[0], ls[1]);
      f2_unpack(l23, ls[2], ls[3]);
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
    }
    // Natural-log statistics for the merge: sum_j exp(s_j - m * ln 2) = l.
    a.stats[((int64_t)kv * ROWS + row) * a.cpk + c] = make_float2(m == -INFINITY ? -INFINITY : m * LN2_F, l);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

// ----------------------------------------------------------------------------- pass 2
template <typename T, int RP>
__global__ void __launch_bounds__(THREADS, 1) rt_col_kernel(const __grid_constant__ CUtensorMap kmap, int kswap,
                                                            RtTcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  unsigned char* sptr = smem_raw + (sbase - raw);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sptr + SM_MISC);
  const Abort abort_flag{misc + 1, 0u};
  int64_t* rowpos = reinterpret_cast<int64_t*>(sptr + SM_ROWPOS);
  float* rowbias = reinterpret_cast<float*>(sptr + SM_ROWSTAT);
  const uint32_t bars = sbase + SM_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t c = blockIdx.x, kv = blockIdx.y;
  // Only tiles that hold a column outside the -1 regions [0, lo_end) and [hi_start, n).
  const int64_t tlo = a.lo_end / 128;
  const int64_t thi = a.hi_start > a.lo_end ? cdiv(a.hi_start, (int64_t)128) : tlo;
  int64_t t0, t1;
  tile_range(tlo, thi - tlo, a.cpk, c, t0, t1);
  const int nt = (int)(t1 - t0);

  // Row data: position, and the exponent bias -(M log2 e + log2 L) so that
  // p = exp(s - M) / L = exp2(s log2 e - M log2 e - log2 L); padding rows get -inf (p = 0).
  for (int i = threadIdx.x; i < ROWS; i += THREADS) {
    const int64_t ps = row_position(a, i);
    rowpos[i] = ps;
    float bias = -INFINITY;
    if (ps >= 0) {
      const float2 ml = a.merged[kv * ROWS + i];
      if (ml.y > 0.f && ml.x > -INFINITY) bias = -(ml.x * LOG2E_F + __log2f(ml.y));
    }
    rowbias[i] = bias;
  }
  if (threadIdx.x == 0) init_bars(bars, misc);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + SM_MISC), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == 0) {
    if (nt > 0) {
      load_rows<T, false>(a, sbase + SM_Q, kv, lane, rowpos);
      mbar_arrive_one(bar(B_Q));
      produce_k(&kmap, kswap, kv, t0, nt, sbase, abort_flag, bars);
    }
  } else if (warp == 1) {
    if (nt > 0) {
      constexpr uint32_t ID = idesc<T>(false, 256, 128);
      bool ok = mbar_wait_warp(bar(B_Q), 0, abort_flag, F_RT_Q);
      for (int it = 0; ok && it < nt; ++it) {
        const int b = it % NB, sb = it & 1;
        if (!mbar_wait_warp(bar(B_KF + b), (it / NB) & 1, abort_flag, F_RT_K)) break;
        if (it >= 2 && !mbar_wait_warp(bar(B_SE + sb), ((it >> 1) - 1) & 1, abort_flag, F_RT_SE)) break;
        tc_fence_after();
        // A = 128 keys (K-major, d halves 16 KB apart), B = 256 rows (K-major, d halves 32 KB apart).
        gemm_ss8<1024, 2048>(tmem + (uint32_t)sb * 256u, desc_k(sbase + SM_K + (uint32_t)b * TILE), desc_k(sbase + SM_Q),
                             ID, 0u);
        mma_commit_one(bar(B_SF + sb));
        mma_commit_one(bar(B_KE + b));
      }
      mma_commit_one(bar(B_DONE));
      mbar_drain(bar(B_DONE), 0);
    }
  } else {
    // Score warps: thread = key (TMEM lane 32 * (warp % 4) + lane); warps 2-5 pool rows 0-127,
    // warps 6-9 rows 128-255 (128 / RP whole query heads each).
    const int half = (warp - 2) >> 2, wq = warp & 3;
    const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16) + 128u * (uint32_t)half;
    const float c2 = a.scaling * LOG2E_F;
    const float inv_r = 1.f / (float)a.r;
    const bool max_pool = a.pool == BB_POOL_MAX;
    int64_t min_qp = (int64_t)1 << 62;
    for (int i = 0; i < ROWS; ++i)
      if (rowpos[i] >= 0 && rowpos[i] < min_qp) min_qp = rowpos[i];
    constexpr int HPH = 128 / RP;  // query heads per half
    for (int it = 0; it < nt; ++it) {
      const int sb = it & 1;
      if (!mbar_wait_warp(bar(B_SF + sb), (it >> 1) & 1, abort_flag, F_RT_S)) break;
      tc_fence_after();
      float s[128];
      tmem_ld128(tl + (uint32_t)sb * 256u, s);
      tc_fence_before();
      mbar_arrive(bar(B_SE + sb));
      const int64_t key0 = (t0 + it) * 128;
      const int64_t key = key0 + 32 * wq + lane;
      const bool causal_free = key0 + 127 <= min_qp;  // no routing row sees a key after its query
      const uint64_t c22 = f2_pack(c2, c2);
#pragma unroll
      for (int hh = 0; hh < HPH; ++hh) {
        const int rbase = 128 * half + hh * RP;
        if (rbase >= (int)(a.groups * a.r_pad)) break;
        // p_j = exp2(round(s_j) * c2 + bias_j) for the head's RP rows, two rows per packed FMA.
        uint64_t sum2 = f2_pack(0.f, 0.f);
        float mx = 0.f;
#pragma unroll
        for (int j = 0; j < RP; j += 2) {
          float r0 = s[hh * RP + j], r1 = s[hh * RP + j + 1];
          round2<T>(r0, r1);
          const float2 bias = *reinterpret_cast<const float2*>(rowbias + rbase + j);
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(r0, r1), c22, f2_pack(bias.x, bias.y)), x0, x1);
          float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          if (!causal_free) {
            if (key > rowpos[rbase + j]) p0 = 0.f;
            if (key > rowpos[rbase + j + 1]) p1 = 0.f;
          }
          if (max_pool)
            mx = fmax3(mx, p0, p1);
          else
            sum2 = f2_add(sum2, f2_pack(p0, p1));
        }
        float acc = mx;
        if (!max_pool) {
          float a0, a1;
          f2_unpack(sum2, a0, a1);
          acc = a0 + a1;
        }
        if (key < a.n) {
          float v = max_pool ? acc : acc * inv_r;
          if (key < a.lo_end || key >= a.hi_start) v = -1.f;
          const int64_t head = kv * a.groups + rbase / (int)a.r_pad;
          a.col[head * a.n + key] = v;
        }
      }
    }
  }
  // The -1 columns outside this KV head's computed tiles, shared by its cpk CTAs.
  {
    const int64_t a_end = tlo * 128 < a.n ? tlo * 128 : a.n;  // [0, a_end)
    const int64_t b_beg = thi * 128 < a.n ? thi * 128 : a.n;  // [b_beg, n)
    const int64_t nfill = a_end + (a.n - b_beg);
    const int64_t total = nfill * a.groups;
    for (int64_t idx = c * THREADS + threadIdx.x; idx < total; idx += a.cpk * THREADS) {
      const int64_t j = idx / nfill, o = idx % nfill;
      const int64_t key = o < a_end ? o : b_beg + (o - a_end);
      a.col[(kv * a.groups + j) * a.n + key] = -1.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

template <typename T>
int launch_stats(const RtTcArgs& a, const CUtensorMap& kmap, int kswap, cudaStream_t stream) {
  cudaFuncSetAttribute(rt_stats_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM_ALLOC);
  dim3 grid((unsigned)a.cpk, (unsigned)a.kv_heads);
  rt_stats_kernel<T><<<grid, THREADS, SM_ALLOC, stream>>>(kmap, kswap, a);
  BB_CHECK_LAUNCH("rt_stats_kernel");
  return BB_OK;
}

template <typename T, int RP>
int launch_col_rp(const RtTcArgs& a, const CUtensorMap& kmap, int kswap, cudaStream_t stream) {
  cudaFuncSetAttribute(rt_col_kernel<T, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM_ALLOC);
  dim3 grid((unsigned)a.cpk, (unsigned)a.kv_heads);
  rt_col_kernel<T, RP><<<grid, THREADS, SM_ALLOC, stream>>>(kmap, kswap, a);
  BB_CHECK_LAUNCH("rt_col_kernel");
  return BB_OK;
}

template <typename T>
int launch_col(const RtTcArgs& a, const CUtensorMap& kmap, int kswap, cudaStream_t stream) {
  if (a.r_pad == 16) return launch_col_rp<T, 16>(a, kmap, kswap, stream);
  if (a.r_pad == 32) return launch_col_rp<T, 32>(a, kmap, kswap, stream);
  return launch_col_rp<T, 64>(a, kmap, kswap, stream);
}

int k_map(const RtTcArgs& a, CUtensorMap* m, int* swap) {
  return make_map(m, swap, a.k, a.dtype, a.kv_heads, a.n, a.sk_h, a.sk_t);
}

}  // namespace rtc

bool routes_tc_eligible(int64_t d, int64_t r_pad, int64_t groups, int dtype, float scaling) {
  return d == 128 && scaling > 0.f && (dtype == BB_BF16 || dtype == BB_F16) && (r_pad == 16 || r_pad == 32 || r_pad == 64) &&
         groups * r_pad <= rtc::ROWS && tc::encode_fn() != nullptr;
}

int64_t routes_tc_cpk(int64_t kv_heads, int64_t n) {
  const int64_t tiles = cdiv(n, (int64_t)128);
  return std::max<int64_t>(1, std::min<int64_t>(tiles, num_sms() / std::max<int64_t>(1, kv_heads)));
}

int routes_tc_stats(const RtTcArgs& a, cudaStream_t stream) {
  CUtensorMap m;
  int swap = 0;
  int st = rtc::k_map(a, &m, &swap);
  if (st) return st;
  return a.dtype == BB_BF16 ? rtc::launch_stats<__nv_bfloat16>(a, m, swap, stream)
                            : rtc::launch_stats<__half>(a, m, swap, stream);
}

int routes_tc_col(const RtTcArgs& a, cudaStream_t stream) {
  CUtensorMap m;
  int swap = 0;
  int st = rtc::k_map(a, &m, &swap);
  if (st) return st;
  return a.dtype == BB_BF16 ? rtc::launch_col<__nv_bfloat16>(a, m, swap, stream)
                            : rtc::launch_col<__half>(a, m, swap, stream);
}

int routes_set_wait_limit(unsigned long long ns) { return tc::unit_set_wait_limit(ns); }

int routes_fault_take(int* code) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tc::g_tc_fault, sizeof(int));
  if (e != cudaSuccess) return fail(BB_ERR_LAUNCH, "device_fault: %s", cudaGetErrorString(e));
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(tc::g_tc_fault, &zero, sizeof(int));
  }
  *code = v;
  return BB_OK;
}

}  // namespace bb
