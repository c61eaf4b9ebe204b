// Sparse flash attention for head_dim 128 on B200: tcgen05 MMA with TMEM accumulators, TMA tile
// loads, warp-specialised.
//
// Semantics are those of bigger_bird_flash (kernels/bigger_bird_flash.py:42-96): one online
// softmax per query over the disjoint union of the sink keys [0, front), the causal window
// [q-W+1, q] and the routed keys idx[h, group(q), :] in [front, q-W]; scores q.k*scale*log2(e),
// exp2, P rounded to the input dtype before P.V, output acc / max(l, 1e-20), fully masked rows 0.
//
// flash_tc_kernel: one CTA computes a 128-query tile of one query head (grid.z splits the tile's
// key range for the exact tail); used for odd GQA groups. flash_tc_pair_kernel (further below)
// computes two query heads of one KV head per CTA and is used otherwise. flash_tc_kernel, 192
// threads:
//   warp 0      producer: Q and every K/V tile by TMA (128B swizzle): sink/window tiles from K/V,
//               routed tiles from the call's gathered routed rows (route_gather_kernel).
//   warp 1      allocates TMEM and issues the MMAs (one elected lane):
//                 S_j = Q K_j^T   (SS: A = Q smem K-major, B = K smem K-major) into S[j % 2]
//                 O  += P_j V_j   (TS: A = P in TMEM over S[j % 2], B = V smem MN-major) into O
//               S_{j+1} is issued before O += P_j V_j so the tensor core overlaps the softmax.
//   warps 2-5   softmax: thread i owns query row i = TMEM lane i. It reads S with tcgen05.ld,
//               masks edge tiles, updates the running max lazily (O in TMEM is rescaled only
//               when the max grows by more than 2^8, so P <= 256), writes P as packed 16-bit
//               pairs over S with tcgen05.st, and finally normalises O into the output.
// TMEM: S[0] = columns 0-127, S[1] = 128-255, O = 256-383 (512 allocated; one CTA per SM).
// Shared memory: Q 32 KB + a ring of NB = 4 tiles of 32 KB that alternately hold K_j and V_j.
//
// Every mbarrier wait is bounded (~2 s): on expiry the CTA raises an abort flag and the device
// fault word, every role leaves its loop, in-flight copies and MMAs are drained (bounded), TMEM is
// freed and the kernel returns.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "flash.cuh"
#include "tc_common.cuh"

namespace bb {


namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int THREADS = 192;
constexpr int NB = 4;
constexpr float RESCALE_LOG2 = 8.0f;

// In the pair kernel's softmax every EXP2_POLY_EVERY-th pair of exponentials of a row is computed on
// the FMA pipe (exp2_poly2) instead of the special-function unit, so the two pipes share the row's
// exponentials.
constexpr int EXP2_POLY_EVERY = 8;

// 2^x of a packed pair on the FMA pipe, x = j + f with j = floor(x) and f in [0, 1): adding 1.5 * 2^23
// rounded toward minus infinity leaves j in the low mantissa bits of t, 2^f comes from a degree-3
// polynomial with p(0) = 1 fitted here for minimax relative error on [0, 1) (8.6e-5, below the
// rounding step of the 16-bit P it feeds), and 2^j is added into p's exponent field (t's bits shifted
// left by 23 are j << 23, since every higher bit of t shifts out). x is clamped at -127, where f = 0
// and p = 1, so the sum clears the exponent field exactly: scores that far below the reference (and
// masked ones, -inf) give exactly 0, as the special-function unit's flush-to-zero exponential does.
// x = 0 gives exactly 1; x never exceeds the lazy-rescale bound, far inside the exponent range.
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& a, float& b) {
  float xa, xb;
  f2_unpack(x2, xa, xb);
  const uint64_t xc = f2_pack(fmaxf(xa, -127.f), fmaxf(xb, -127.f));
  const uint64_t big = f2_pack(12582912.f, 12582912.f);
  const uint64_t t = f2_add_rm(xc, big);
  const uint64_t fr = f2_sub(xc, f2_sub(t, big));
  uint64_t p = f2_fma(f2_pack(0.07706707f, 0.07706707f), fr, f2_pack(0.22764495f, 0.22764495f));
  p = f2_fma(p, fr, f2_pack(0.6951168f, 0.6951168f));
  p = f2_fma(p, fr, f2_pack(1.f, 1.f));
  float pa, pb, ta, tb;
  f2_unpack(p, pa, pb);
  f2_unpack(t, ta, tb);
  a = __uint_as_float(__float_as_uint(pa) + (__float_as_uint(ta) << 23));
  b = __uint_as_float(__float_as_uint(pb) + (__float_as_uint(tb) << 23));
}

constexpr uint32_t SM_Q = 0;
constexpr uint32_t SM_KV = TILE;
enum { B_Q = 0, B_FULL = 1, B_EMPTY = B_FULL + NB, B_S = B_EMPTY + NB, B_P = B_S + 2, B_O = B_P + 2,
       B_DONE = B_O + 1, N_BARS = B_DONE + 1 };
constexpr uint32_t SM_BAR = SM_KV + NB * TILE;
constexpr uint32_t SM_MISC = SM_BAR + N_BARS * 8;  // [0] TMEM base, [1] abort flag
constexpr uint32_t SM_BYTES = SM_MISC + 16;
constexpr uint32_t SM_ALLOC = SM_BYTES + 1024;     // slack to align the base to 1024 bytes

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 256;

// Fault codes written to this unit's fault word (which wait gave up).
enum { F_SOFTMAX_S = 1, F_SOFTMAX_O = 2, F_MMA_Q = 3, F_MMA_K = 4, F_MMA_P = 5, F_MMA_V = 6,
       F_PROD_EMPTY = 7, F_EPI_O = 8, F_MMA_STALL = 9 };

// Test hook of the abort path (bb_debug_stall_attention): when non-zero, the MMA issuer of every
// CTA first waits for a barrier that nothing completes, so its bounded wait runs out.
static __device__ int g_tc_stall = 0;


// ----------------------------------------------------------------------------- tile schedule
// Tiles of one query tile, in order: contiguous key tiles (aligned to 128, covering the sink
// [0, front) and the window [q_first - W + 1, q_last]; two ranges, merged when they touch), then
// cdiv(route_k, 128) routed tiles for each route group touched by the query rows.
struct Sched {
  int64_t q_first, q_last;
  int n_a, w_lo, n_w, n_contig;   // contiguous tile indices: [0, n_a) and [w_lo, w_lo + n_w)
  int64_t g_lo;
  int n_rpg, n_groups, total;
  // Routed tiles k = (group - g_lo) * n_rpg + r kept in the schedule (bit k), when the call's
  // per-tile minimum positions are known and there are at most 64 routed tiles; else all are kept.
  bool skip;
  uint64_t live;
};

struct Tile {
  int kind;        // 0 contiguous, 1 routed
  int64_t k0;      // first key (contiguous)
  int64_t group, slot0;
  bool masked;
};

// h0, nh: the query heads of the CTA (a routed step holds tile r of each of them).
__device__ __forceinline__ Sched make_sched(const FlashParams& p, int64_t row0, int64_t row1, int64_t h0, int nh) {
  Sched s;
  s.q_first = p.offset + row0;
  s.q_last = p.offset + row1 - 1;
  const int64_t sink_end = min(p.front, s.q_last + 1);
  int n_a = sink_end > 0 ? (int)cdiv(sink_end, BN) : 0;
  const int64_t wl = max(s.q_first - p.window + 1, (int64_t)0) / BN;
  const int64_t wh = s.q_last / BN + 1;
  int w_lo = (int)wl, n_w = (int)(wh - wl);
  if (w_lo <= n_a) {  // ranges touch: one range [0, wh)
    n_a = (int)max((int64_t)n_a, wh);
    n_w = 0;
    w_lo = n_a;
  }
  s.n_a = n_a;
  s.w_lo = w_lo;
  s.n_w = n_w;
  s.n_contig = n_a + n_w;
  s.n_rpg = (int)cdiv(p.route_k, BN);
  s.g_lo = s.q_first / p.route_chunk;
  const int64_t g_hi = min(s.q_last / p.route_chunk, p.route_groups - 1);
  // A routed key ps is attended by row q only if front <= ps <= q - W: query tiles whose last row
  // is within W of the sink's end have no routed steps at all.
  s.n_groups = (p.route_k > 0 && g_hi >= s.g_lo && s.q_last - p.window >= p.front) ? (int)(g_hi - s.g_lo + 1) : 0;
  s.total = s.n_contig + s.n_groups * s.n_rpg;
  // A routed tile none of whose keys any row of the query tile can attend (its smallest key at or
  // after the sink, from route_gather_kernel, lies beyond q_last - W for every head of the CTA) is
  // left out of the schedule: its step would be masked entirely.
  s.skip = false;
  s.live = 0;
  const int nrt = s.n_groups * s.n_rpg;
  if (p.tile_min && nrt > 0 && nrt <= 64) {
    const int64_t lim = s.q_last - p.window;
    uint64_t m = 0;
    for (int k = 0; k < nrt; ++k) {
      const int64_t g = s.g_lo + k / s.n_rpg;
      const int r = k % s.n_rpg;
      bool live = false;
      for (int e = 0; e < nh; ++e)
        live |= (int64_t)(uint32_t)p.tile_min[((h0 + e) * p.route_groups + g) * s.n_rpg + r] <= lim;
      if (live) m |= 1ull << k;
    }
    s.skip = true;
    s.live = m;
    s.total = s.n_contig + __popcll(m);
  }
  return s;
}

// Index of the r-th set bit of m (r < popcount(m)).
__device__ __forceinline__ int nth_bit(uint64_t m, int r) {
  const uint32_t lo = (uint32_t)m;
  const int c = __popc(lo);
  return r < c ? (int)__fns(lo, 0, r + 1) : 32 + (int)__fns((uint32_t)(m >> 32), 0, r - c + 1);
}

__device__ __forceinline__ Tile tile_at(const FlashParams& p, const Sched& s, int t) {
  Tile tl;
  tl.group = 0;
  tl.slot0 = 0;
  if (t < s.n_contig) {
    tl.kind = 0;
    tl.k0 = (int64_t)(t < s.n_a ? t : s.w_lo + (t - s.n_a)) * BN;
    // Unmasked iff every key of the tile is valid for every row of the query tile.
    const bool causal_ok = tl.k0 + BN - 1 <= s.q_first;
    const bool sink_all = tl.k0 + BN <= p.front;
    const bool window_all = tl.k0 >= s.q_last - p.window + 1;
    tl.masked = !(causal_ok && (sink_all || window_all)) || p.mask != nullptr;
  } else {
    const int r = s.skip ? nth_bit(s.live, t - s.n_contig) : t - s.n_contig;
    tl.kind = 1;
    tl.k0 = 0;
    tl.group = s.g_lo + r / s.n_rpg;
    tl.slot0 = (int64_t)(r % s.n_rpg) * BN;
    tl.masked = true;
  }
  return tl;
}

// Position of routed slot `slot` of `group` for head h, or -1 when empty / out of range.
__device__ __forceinline__ int64_t routed_pos(const FlashParams& p, int64_t h, int64_t group, int64_t slot) {
  if (slot >= p.route_k) return -1;
  const int64_t ps = p.idx[h * p.si_h + group * p.si_g + slot * p.si_k];
  return (ps < 0 || ps >= p.n) ? -1 : ps;
}

// Routed positions of one 128-slot tile, held by a warp: lane l keeps the positions of slots l,
// l + 32, l + 64 and l + 96 (-1 = empty or out of range) and the mask reads slot i with a shuffle.
// Each warp loads its own copy (the four warps of a softmax group read the same 512 bytes, L1
// hits), so no barrier between warps is needed: a barrier there could strand the other warps of
// the group when one warp leaves on an abort.
struct RoutedPos {
  int32_t v[4];
};
__device__ __forceinline__ RoutedPos load_routed(const FlashParams& p, int64_t h, int64_t group, int64_t slot0,
                                                 int lane) {
  RoutedPos r;
#pragma unroll
  for (int k = 0; k < 4; ++k) r.v[k] = (int32_t)routed_pos(p, h, group, slot0 + lane + 32 * k);
  return r;
}

// Per-row mask limits of a tile. Contiguous tiles (kind 0, first key k0): key k0 + i is valid iff
// k0 + i <= q and (k0 + i < front or k0 + i >= q - W + 1), i.e. i <= hi && (i < f || i >= lo).
// Routed tiles (kind 1): slot i's key ps (-1 = empty) is valid iff front <= ps <= q - W and the
// row's route group is the tile's, i.e. f <= ps <= hi. Bounds are folded into per-row int32
// limits first (positions are < 2^31), so the per-element work is two compares and a select.
// (Calls with a token mask run on the mma.sync kernel.)
struct MaskLimits {
  int hi, f, lo;
};
__device__ __forceinline__ MaskLimits mask_limits(int kind, int64_t k0, int64_t group, const FlashParams& p,
                                                  int64_t qpos, int64_t qgroup) {
  MaskLimits m;
  if (kind == 0) {
    m.hi = (int)max(min(qpos - k0, (int64_t)128), (int64_t)-1);
    m.f = (int)max(min(p.front - k0, (int64_t)128), (int64_t)0);
    m.lo = (int)max(min(qpos - p.window + 1 - k0, (int64_t)129), (int64_t)0);
  } else {
    m.hi = qgroup == group ? (int)max(min(qpos - p.window, (int64_t)0x7fffffff), (int64_t)-1) : -1;
    m.f = (int)min(p.front, (int64_t)0x7fffffff);
    m.lo = 0;
  }
  return m;
}
// Masks the 128 columns of a row held in s[0..127] (warp-uniform call: routed tiles shuffle).
__device__ __forceinline__ void mask_cols128(float* s, int kind, const MaskLimits& m, const RoutedPos& rp) {
  if (kind == 0) {
#pragma unroll
    for (int i = 0; i < 128; ++i)
      if (!(i <= m.hi && (i < m.f || i >= m.lo))) s[i] = -INFINITY;
  } else {
#pragma unroll
    for (int i = 0; i < 128; ++i) {
      const int ps = __shfl_sync(0xffffffffu, rp.v[i >> 5], i & 31);
      if (!(ps >= m.f && ps <= m.hi)) s[i] = -INFINITY;
    }
  }
}

struct TcMaps {
  CUtensorMap q, k, v;
  CUtensorMap kg, vg;   // gathered routed rows [bh * route_groups * route_kpad][128] (when routed)
  int q_swap, kv_swap;  // 1: the map's dims are {d, heads, rows} (coordinates swapped)
};

// Routed K/V rows of every (head, route group, slot), gathered once per call into two contiguous
// [bh][route_groups][route_kpad][128] arrays, so that the attention kernels load a routed tile
// with two tiled TMA boxes like a window tile instead of gathering the same rows again for every
// query tile. One thread per 16-byte chunk; empty slots and the padding to 128 are zero rows
// (the kernels mask them by position anyway). It also records, per 128-slot routed tile, the
// smallest position at or after the sink (tile_min, preset to all ones), which lets the
// attention kernels leave out routed tiles that no row of a query tile can attend.
template <typename T>
__global__ void __launch_bounds__(256) route_gather_kernel(FlashParams p) {
  const int64_t rows = p.bh * p.route_groups * p.route_kpad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * 16;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i >> 4, c = i & 15;
    const int64_t slot = r % p.route_kpad, g = (r / p.route_kpad) % p.route_groups;
    const int64_t h = r / (p.route_kpad * p.route_groups);
    const int64_t kvh = (h / p.num_heads) * (p.num_heads / p.kv_groups) + (h % p.num_heads) / p.kv_groups;
    const int64_t ps = routed_pos(p, h, g, slot);
    if (c == 0 && ps >= p.front)
      atomicMin(reinterpret_cast<unsigned int*>(p.tile_min) + (r >> 7), (unsigned int)ps);
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (ps >= 0) {
      kv = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.k) + kvh * p.sk_h + ps * p.sk_t) + c);
      vv = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.v) + kvh * p.sv_h + ps * p.sv_t) + c);
    }
    reinterpret_cast<uint4*>(p.kg)[i] = kv;
    reinterpret_cast<uint4*>(p.vg)[i] = vv;
  }
}

// Row of the gathered arrays where head h's 128-slot routed tile starting at slot0 of group g
// begins.
__device__ __forceinline__ int gathered_row(const FlashParams& p, int64_t h, int64_t g, int64_t slot0) {
  return (int)((h * p.route_groups + g) * p.route_kpad + slot0);
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1) flash_tc_kernel(const __grid_constant__ TcMaps maps, FlashParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  unsigned char* sptr = smem_raw + (sbase - raw);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sptr + SM_MISC);
  const Abort abort_flag{misc + 1, p.serial};
  auto bar = [&](int i) { return sbase + SM_BAR + 8u * (uint32_t)i; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t h = blockIdx.y;
  const int split = blockIdx.z;
  const int64_t row0 = p.row_begin + (int64_t)blockIdx.x * BM;
  const int64_t row1 = min(row0 + BM, p.row_end);
  const int64_t kvh = (h / p.num_heads) * (p.num_heads / p.kv_groups) + (h % p.num_heads) / p.kv_groups;
  const int64_t batch = h / p.num_heads;
  const Sched sc = make_sched(p, row0, row1, h, 1);
  const int t_begin = (int)((int64_t)sc.total * split / p.splits);
  const int nt = (int)((int64_t)sc.total * (split + 1) / p.splits) - t_begin;

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int i = 0; i < NB; ++i) {
      mbar_init(bar(B_FULL + i), 1);
      mbar_init(bar(B_EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_S + i), 1);
      mbar_init(bar(B_P + i), 128);
    }
    mbar_init(bar(B_O), 1);
    mbar_init(bar(B_DONE), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + SM_MISC),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    int fills[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) fills[i] = 0;
    bool q_issued = false;
    if (nt > 0) {
      {
        const int qc1 = (int)row0, qc2 = (int)h;
        mbar_expect_tx_one(bar(B_Q), TILE);
        if (maps.q_swap) {
          tma_load_3d_one(sbase + SM_Q, &maps.q, 0, qc2, qc1, bar(B_Q));
          tma_load_3d_one(sbase + SM_Q + HALF, &maps.q, 64, qc2, qc1, bar(B_Q));
        } else {
          tma_load_3d_one(sbase + SM_Q, &maps.q, 0, qc1, qc2, bar(B_Q));
          tma_load_3d_one(sbase + SM_Q + HALF, &maps.q, 64, qc1, qc2, bar(B_Q));
        }
      }
      q_issued = true;
      for (int it = 0; it < 2 * nt; ++it) {
        const int j = it >> 1;
        const bool is_v = it & 1;
        const int b = it % NB;
        const int round = it / NB;
        if (round > 0 && !mbar_wait_warp(bar(B_EMPTY + b), (round - 1) & 1, abort_flag, F_PROD_EMPTY)) break;
        const Tile tl = tile_at(p, sc, t_begin + j);
        const uint32_t dst = sbase + SM_KV + (uint32_t)b * TILE;
        if (tl.kind == 0) {
          {
            const CUtensorMap* m = is_v ? &maps.v : &maps.k;
            const int c1 = (int)tl.k0, c2 = (int)kvh;
            mbar_expect_tx_one(bar(B_FULL + b), TILE);
            if (maps.kv_swap) {
              tma_load_3d_one(dst, m, 0, c2, c1, bar(B_FULL + b));
              tma_load_3d_one(dst + HALF, m, 64, c2, c1, bar(B_FULL + b));
            } else {
              tma_load_3d_one(dst, m, 0, c1, c2, bar(B_FULL + b));
              tma_load_3d_one(dst + HALF, m, 64, c1, c2, bar(B_FULL + b));
            }
          }
        } else {
          const CUtensorMap* m = is_v ? &maps.vg : &maps.kg;
          const int row = gathered_row(p, h, tl.group, tl.slot0);
          mbar_expect_tx_one(bar(B_FULL + b), TILE);
          tma_load_3d_one(dst, m, 0, row, 0, bar(B_FULL + b));
          tma_load_3d_one(dst + HALF, m, 64, row, 0, bar(B_FULL + b));
        }
        ++fills[b];
      }
    }
    // Drain: no copy may still be writing this CTA's shared memory when it exits.
    {
      if (q_issued) mbar_drain(bar(B_Q), 0);
      for (int b = 0; b < NB; ++b)
        if (fills[b] > 0) mbar_drain(bar(B_FULL + b), (fills[b] - 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (nt > 0) {
      constexpr uint32_t ID_QK = idesc<T>(false), ID_PV = idesc<T>(true);
      bool ok = mbar_wait_warp(bar(B_Q), 0, abort_flag, F_MMA_Q);
      // Test hook (bb_debug_stall_attention): see flash_tc_pair_kernel.
      if (ok && *(volatile int*)&g_tc_stall) ok = mbar_wait_warp(bar(B_DONE), 0, abort_flag, F_MMA_STALL);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait_warp(bar(B_P + (i & 1)), (i >> 1) & 1, abort_flag, F_MMA_P)) return false;
        const int itv = 2 * i + 1, bv = itv % NB;
        if (!mbar_wait_warp(bar(B_FULL + bv), (itv / NB) & 1, abort_flag, F_MMA_V)) return false;
        tc_fence_after();
        const uint32_t vb = sbase + SM_KV + (uint32_t)bv * TILE;
        gemm_ts8(tmem + COL_O, tmem + (uint32_t)(i & 1) * 128u, desc_mn(vb), ID_PV, i > 0 ? 1u : 0u);
        mma_commit_one(bar(B_O));
        mma_commit_one(bar(B_EMPTY + bv));
        return true;
      };
      for (int j = 0; ok && j < nt; ++j) {
        const int itk = 2 * j, bk = itk % NB;
        if (!mbar_wait_warp(bar(B_FULL + bk), (itk / NB) & 1, abort_flag, F_MMA_K)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sbase + SM_KV + (uint32_t)bk * TILE;
        const uint32_t ds = tmem + (uint32_t)(j & 1) * 128u;
        gemm_ss8(ds, desc_k(sbase + SM_Q), desc_k(kb), ID_QK, 0u);
        mma_commit_one(bar(B_S + (j & 1)));
        mma_commit_one(bar(B_EMPTY + bk));
        if (j > 0) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(nt - 1);
      mma_commit_one(bar(B_DONE));
      mbar_drain(bar(B_DONE), 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t tl_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const int64_t qpos = p.offset + row0 + row;
    const int64_t qgroup = qpos / p.route_chunk;
    const float c = p.scale_log2;
    float m_ref = -1.0e20f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const Tile tl = tile_at(p, sc, t_begin + j);
      const MaskLimits ml = tl.masked ? mask_limits(tl.kind, tl.k0, tl.group, p, qpos, qgroup)
                                      : MaskLimits{127, 128, 0};
      if (!mbar_wait_warp(bar(B_S + (j & 1)), (j >> 1) & 1, abort_flag, F_SOFTMAX_S)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      const uint32_t scol = tl_lane + (uint32_t)(j & 1) * 128u;
      tmem_ld128(scol, s);
      if (tl.masked)
        mask_cols128(s, tl.kind, ml, tl.kind == 1 ? load_routed(p, h, tl.group, tl.slot0, lane)
                                                  : RoutedPos{{-1, -1, -1, -1}});
      // Row max as a tree (short dependency chains).
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = s[k];
#pragma unroll
      for (int i = 8; i < 128; i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(mx8[k], s[i + k]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mt = mx * c;
      // The wait for P_{j-1} V_{j-1} (completion j of B_O) is taken in order every tile: here when
      // O must be rescaled, otherwise after the exponentials, by when it has normally completed.
      bool o_waited = j == 0;
      float alpha = 1.f;
      bool rescale_o = false;
      if (mt > m_ref + RESCALE_LOG2) {
        alpha = fast_exp2(m_ref - mt);
        rescale_o = j > 0 && m_ref > -1.0e20f;
        l *= alpha;
        m_ref = mt;
      }
      // The O rescale uses warp-wide TMEM loads/stores, so it is decided per warp: lanes that
      // keep their reference multiply by exactly 1.
      if (!rescale_o) alpha = 1.f;
      if (__any_sync(0xffffffffu, rescale_o)) {
        if (!o_waited) {
          if (!mbar_wait_warp(bar(B_O), (j - 1) & 1, abort_flag, F_SOFTMAX_O)) {
            ok = false;
            break;
          }
          o_waited = true;
        }
        tc_fence_after();
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          float o[32];
          tmem_ld32(tl_lane + COL_O + q4 * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tl_lane + COL_O + q4 * 32, o);
        }
        tmem_wait_st();
      }
      uint32_t pk[64];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg = -m_ref;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float a = fast_exp2(fmaf(s[2 * i], c, neg));
        const float b = fast_exp2(fmaf(s[2 * i + 1], c, neg));
        ls[i & 3] += a + b;
        pk[i] = pack2<T>(a, b);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      if (!o_waited && !mbar_wait_warp(bar(B_O), (j - 1) & 1, abort_flag, F_SOFTMAX_O)) {
        ok = false;
        break;
      }
      tmem_st64(scol, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(B_P + (j & 1)));
    }
    // Epilogue: wait for the last P.V, normalise, store.
    bool have_o = false;
    if (ok && nt > 0) have_o = mbar_wait_warp(bar(B_O), (nt - 1) & 1, abort_flag, F_EPI_O);
    tc_fence_after();
    const int64_t lrow = row0 + row;
    const bool store = lrow < row1;
    if (p.splits > 1) {
      float* acc = p.part_acc + (((int64_t)split * p.bh + h) * p.t + lrow) * 128;
      if (store) p.part_ml[((int64_t)split * p.bh + h) * p.t + lrow] = make_float2(have_o ? m_ref : -1.0e20f, have_o ? l : 0.f);
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float o[32];
        if (have_o) {
          tmem_ld32(tl_lane + COL_O + q4 * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (store) {
          float4* dst = reinterpret_cast<float4*>(acc + q4 * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
    } else {
      float inv = (have_o && l > 0.f) ? 1.f / fmaxf(l, 1.0e-20f) : 0.f;
      if (p.mask && store && qpos < p.n && !p.mask[batch * p.sm_b + qpos * p.sm_t]) inv = 0.f;
      T* out = static_cast<T*>(p.out) + h * p.so_h + lrow * p.so_t;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float o[32];
        if (have_o) {
          tmem_ld32(tl_lane + COL_O + q4 * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (store) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack2<T>(o[2 * i] * inv, o[2 * i + 1] * inv);
          uint4* dst = reinterpret_cast<uint4*>(out + q4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ============================================================================= paired kernel
// Two query heads of one KV head (a GQA pair, heads 2m and 2m+1) x 128 query rows per CTA. A step
// is one 128-key tile per head: the K/V tiles of the sink and window are shared by both heads
// and loaded once; in a routed step each head gets its own gathered K/V tile (its r-th routed
// tile), so the tensor core never multiplies a head by keys it does not attend. Each head has its
// own softmax warpgroup, S buffer and O accumulator in TMEM:
//   S_A = columns 0-127, S_B = 128-255, O_A = 256-383, O_B = 384-511.
// The single MMA thread alternates  P_A V -> S_A(next) -> P_B V -> S_B(next), so while one
// warpgroup runs its softmax the tensor core works for the other (ping-pong).
// 384 threads (12 warps, three per SM sub-partition): warpgroup 0 = producer (warp 0), MMA issuer
// (warp 1) and two idle warps; softmax of head A (warps 4-7) and of head B (warps 8-11), with more
// registers than the launch gives (P_REG_HIGH below) for the score row and its exponentials; warp w
// reads TMEM lanes 32 * (w % 4) .. 32 * (w % 4) + 31, so each softmax group covers all 128 rows.
constexpr int P_THREADS = 384;
// Register split (setmaxnreg): the launch gives every thread P_REG_LAUNCH registers (what ptxas
// reports for this kernel); warpgroup 0 (producer, MMA issuer, two idle warps) drops to P_REG_LOW so
// that the two softmax warpgroups can rise to P_REG_HIGH. The shares must add up to at most the
// launch total (an increase waits for registers that a decrease frees), and every SM sub-partition
// holds one warp of each warpgroup.
constexpr int P_REG_LAUNCH = 168, P_REG_LOW = 104, P_REG_HIGH = 200;
static_assert(128 * P_REG_LOW + 256 * P_REG_HIGH <= P_THREADS * P_REG_LAUNCH, "register split exceeds the launch");
static_assert(32 * (P_REG_LOW + 2 * P_REG_HIGH) <= 16384, "register split exceeds a sub-partition");
// K/V ring: 5 slots of 32 KB, the most that fits beside the two Q tiles in 227 KB. Fill order:
// a shared step loads K_j then V_j (two fills), a routed step K_A, K_B, V_A, V_B (four fills). At
// most four filled slots are in use at once (V_A, V_B of the previous step and K_A, K_B of this
// one), so the fifth gives the loads of the next tiles lead over the MMA issuer.
constexpr int PNB = 5;
constexpr uint32_t P_SM_QA = 0;
constexpr uint32_t P_SM_QB = TILE;
constexpr uint32_t P_SM_KV = 2 * TILE;
// PB_P + 2w: P_w columns for keys 0-63 stored, PB_P + 2w + 1: keys 64-127 stored.
enum { PB_Q = 0, PB_FULL = 1, PB_EMPTY = PB_FULL + PNB, PB_S = PB_EMPTY + PNB, PB_P = PB_S + 2, PB_O = PB_P + 4,
       PB_DONE = PB_O + 2, PN_BARS = PB_DONE + 1 };
constexpr uint32_t P_SM_BAR = P_SM_KV + PNB * TILE;
constexpr uint32_t P_SM_MISC = P_SM_BAR + PN_BARS * 8;
constexpr uint32_t P_SM_ALLOC = P_SM_MISC + 16 + 1024;
static_assert(P_SM_ALLOC <= 232448, "pair kernel shared memory exceeds the 227 KB per-block limit");

// Ring fills of a split whose first `shared` steps are shared: step j < shared fills 2j (K) and
// 2j + 1 (V); a routed step j fills F, F+1, F+2, F+3 = K_A, K_B, V_A, V_B with
// F = 2 * shared + 4 * (j - shared). Fill f uses slot f % PNB in round f / PNB.
struct PairFills {
  int shared;
};

template <typename T>
__global__ void __launch_bounds__(P_THREADS, 1) flash_tc_pair_kernel(const __grid_constant__ TcMaps maps,
                                                                      FlashParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  unsigned char* sptr = smem_raw + (sbase - raw);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sptr + P_SM_MISC);
  const Abort abort_flag{misc + 1, p.serial};
  auto bar = [&](int i) { return sbase + P_SM_BAR + 8u * (uint32_t)i; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t hA = 2 * (int64_t)blockIdx.y;
  const int split = blockIdx.z;
  const int64_t row0 = p.row_begin + (int64_t)blockIdx.x * BM;
  const int64_t row1 = min(row0 + BM, p.row_end);
  const int64_t kvh = (hA / p.num_heads) * (p.num_heads / p.kv_groups) + (hA % p.num_heads) / p.kv_groups;
  const Sched sc = make_sched(p, row0, row1, hA, 2);
  const int t_begin = (int)((int64_t)sc.total * split / p.splits);
  const int nt = (int)((int64_t)sc.total * (split + 1) / p.splits) - t_begin;
  const PairFills fl{max(0, min(sc.n_contig - t_begin, nt))};

  if (threadIdx.x == 0) {
    mbar_init(bar(PB_Q), 1);
    for (int i = 0; i < PNB; ++i) {
      mbar_init(bar(PB_FULL + i), 1);
      mbar_init(bar(PB_EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(PB_S + i), 1);
      mbar_init(bar(PB_P + 2 * i), 128);
      mbar_init(bar(PB_P + 2 * i + 1), 128);
      mbar_init(bar(PB_O + i), 1);
    }
    mbar_init(bar(PB_DONE), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + P_SM_MISC),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(P_REG_LOW));
    if (warp == 0) {
      // ---------------------------------------------------------------- producer
      int fills[PNB];
#pragma unroll
      for (int i = 0; i < PNB; ++i) fills[i] = 0;
      if (nt > 0) {
        {
          mbar_expect_tx_one(bar(PB_Q), 2 * TILE);
          for (int w = 0; w < 2; ++w) {
            const uint32_t dq = sbase + (w ? P_SM_QB : P_SM_QA);
            const int c1 = (int)row0, c2 = (int)(hA + w);
            if (maps.q_swap) {
              tma_load_3d_one(dq, &maps.q, 0, c2, c1, bar(PB_Q));
              tma_load_3d_one(dq + HALF, &maps.q, 64, c2, c1, bar(PB_Q));
            } else {
              tma_load_3d_one(dq, &maps.q, 0, c1, c2, bar(PB_Q));
              tma_load_3d_one(dq + HALF, &maps.q, 64, c1, c2, bar(PB_Q));
            }
          }
        }
        int it = 0;
        // One loop over the fills: a shared step loads K_j then V_j from the K/V maps, a routed step
        // K_A, K_B, V_A, V_B from the gathered routed rows (route_gather_kernel); each fill is two
        // tiled TMA boxes.
        const int n_fills = 2 * fl.shared + 4 * (nt - fl.shared);
        for (; it < n_fills; ++it) {
          const int b = it % PNB;
          const int round = it / PNB;
          if (round > 0 && !mbar_wait_warp(bar(PB_EMPTY + b), (round - 1) & 1, abort_flag, F_PROD_EMPTY)) break;
          const bool routed = it >= 2 * fl.shared;
          const int f = routed ? (it - 2 * fl.shared) & 3 : it & 1;
          const int j = routed ? fl.shared + ((it - 2 * fl.shared) >> 2) : it >> 1;
          const Tile tl = tile_at(p, sc, t_begin + j);
          const CUtensorMap* m = routed ? (f >= 2 ? &maps.vg : &maps.kg) : (f ? &maps.v : &maps.k);
          int c1, c2;
          if (routed) {
            c1 = gathered_row(p, hA + (f & 1), tl.group, tl.slot0);
            c2 = 0;
          } else if (maps.kv_swap) {
            c1 = (int)kvh;
            c2 = (int)tl.k0;
          } else {
            c1 = (int)tl.k0;
            c2 = (int)kvh;
          }
          const uint32_t dst = sbase + P_SM_KV + (uint32_t)b * TILE;
          mbar_expect_tx_one(bar(PB_FULL + b), TILE);
          tma_load_3d_one(dst, m, 0, c1, c2, bar(PB_FULL + b));
          tma_load_3d_one(dst + HALF, m, 64, c1, c2, bar(PB_FULL + b));
          ++fills[b];
        }
      }
      {
        if (nt > 0) mbar_drain(bar(PB_Q), 0);
        for (int b = 0; b < PNB; ++b)
          if (fills[b] > 0) mbar_drain(bar(PB_FULL + b), (fills[b] - 1) & 1);
      }
    } else if (warp == 1 && nt > 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t ID_QK = idesc<T>(false), ID_PV = idesc<T>(true);
      auto slot_of = [](int f) { return (uint32_t)(f % PNB); };
      auto full_wait = [&](int f, int code) {
        return mbar_wait_warp(bar(PB_FULL + f % PNB), (uint32_t)((f / PNB) & 1), abort_flag, code);
      };
      auto s_mma = [&](int w, uint32_t kb) {
        const uint32_t qs = sbase + (w ? P_SM_QB : P_SM_QA);
        gemm_ss8(tmem + (uint32_t)w * 128u, desc_k(qs), desc_k(kb), ID_QK, 0u);
        mma_commit_one(bar(PB_S + w));
      };
      // O_w += P_w(i) V in two K halves (keys 0-63, 64-127), each issued as soon as the softmax has
      // stored that half of P. `fv` is V's fill number; `wait_v`: wait for it (head A always, head B
      // only for its own routed V).
      auto pv = [&](int w, int i, int fv, bool wait_v) -> bool {
        if (!mbar_wait_warp(bar(PB_P + 2 * w), i & 1, abort_flag, F_MMA_P)) return false;
        if (wait_v && !full_wait(fv, F_MMA_V)) return false;
        tc_fence_after();
        const uint32_t vb = sbase + P_SM_KV + slot_of(fv) * TILE;
        const uint32_t od = tmem + 256u + (uint32_t)w * 128u, pa = tmem + (uint32_t)w * 128u;
        gemm_ts4(od, pa, desc_mn(vb), ID_PV, i > 0 ? 1u : 0u);
        if (!mbar_wait_warp(bar(PB_P + 2 * w + 1), i & 1, abort_flag, F_MMA_P)) return false;
        tc_fence_after();
        gemm_ts4(od, pa + 32u, desc_mn(vb + 4u * 2048u), ID_PV, 1u);
        mma_commit_one(bar(PB_O + w));
        return true;
      };
      bool ok = mbar_wait_warp(bar(PB_Q), 0, abort_flag, F_MMA_Q);
      // Test hook (bb_debug_stall_attention): wait for the end-of-kernel barrier, which only this
      // warp completes, so the bounded wait runs out and the launch takes its abort path.
      if (ok && *(volatile int*)&g_tc_stall) ok = mbar_wait_warp(bar(PB_DONE), 0, abort_flag, F_MMA_STALL);
      const int c = fl.shared;
      int j = 0;
      // Shared steps (kept as one short loop: its code is the hot path).
      for (; ok && j < c; ++j) {
        const int fk = 2 * j;
        if (!full_wait(fk, F_MMA_K)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sbase + P_SM_KV + slot_of(fk) * TILE;
        if (j > 0) {
          if (!(ok = pv(0, j - 1, fk - 1, true))) break;
          s_mma(0, kb);
          if (!(ok = pv(1, j - 1, fk - 1, false))) break;
          mma_commit_one(bar(PB_EMPTY + slot_of(fk - 1)));  // V_{j-1} consumed by both heads
          s_mma(1, kb);
        } else {
          s_mma(0, kb);
          s_mma(1, kb);
        }
        mma_commit_one(bar(PB_EMPTY + slot_of(fk)));  // K_j consumed by both heads
      }
      // Routed steps: each head its own K and V (fills F, F+1, F+2, F+3 = K_A, K_B, V_A, V_B).
      for (; ok && j < nt; ++j) {
        const int F = 2 * c + 4 * (j - c);
        if (!full_wait(F, F_MMA_K)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (j > 0) {
          const bool prev_routed = j - 1 >= c;
          const int fva = prev_routed ? F - 2 : F - 1, fvb = F - 1;
          if (!(ok = pv(0, j - 1, fva, true))) break;
          if (prev_routed) mma_commit_one(bar(PB_EMPTY + slot_of(fva)));
          s_mma(0, sbase + P_SM_KV + slot_of(F) * TILE);
          mma_commit_one(bar(PB_EMPTY + slot_of(F)));
          if (!(ok = pv(1, j - 1, fvb, prev_routed))) break;
          mma_commit_one(bar(PB_EMPTY + slot_of(fvb)));
        } else {
          s_mma(0, sbase + P_SM_KV + slot_of(F) * TILE);
          mma_commit_one(bar(PB_EMPTY + slot_of(F)));
        }
        if (!full_wait(F + 1, F_MMA_K)) {
          ok = false;
          break;
        }
        tc_fence_after();
        s_mma(1, sbase + P_SM_KV + slot_of(F + 1) * TILE);
        mma_commit_one(bar(PB_EMPTY + slot_of(F + 1)));
      }
      if (ok) {
        const int last = nt - 1;
        if (last < c) {
          const int fv = 2 * last + 1;
          if (pv(0, last, fv, true) && pv(1, last, fv, false))
            mma_commit_one(bar(PB_EMPTY + slot_of(fv)));
        } else {
          const int F = 2 * c + 4 * (last - c);
          if (pv(0, last, F + 2, true)) {
            mma_commit_one(bar(PB_EMPTY + slot_of(F + 2)));
            if (pv(1, last, F + 3, true)) mma_commit_one(bar(PB_EMPTY + slot_of(F + 3)));
          }
        }
      }
      mma_commit_one(bar(PB_DONE));
      mbar_drain(bar(PB_DONE), 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(P_REG_HIGH));
    const int w = (warp - 4) >> 2;  // 0: head A (warps 4-7), 1: head B (warps 8-11)
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int64_t h = hA + w;
    const int64_t batch = h / p.num_heads;
    const uint32_t tl_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t scol = tl_lane + (uint32_t)w * 128u;
    const uint32_t ocol = tl_lane + 256u + (uint32_t)w * 128u;
    const int64_t qpos = p.offset + row0 + row;
    const int64_t qgroup = qpos / p.route_chunk;
    const float c = p.scale_log2;
    float m_ref = -1.0e20f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const Tile tl = tile_at(p, sc, t_begin + j);
      const MaskLimits ml = tl.masked ? mask_limits(tl.kind, tl.k0, tl.group, p, qpos, qgroup)
                                      : MaskLimits{127, 128, 0};
      if (!mbar_wait_warp(bar(PB_S + w), j & 1, abort_flag, F_SOFTMAX_S)) {
        ok = false;
        break;
      }
      // P_w(j-1) V_{j-1} was issued before S_w(j), and the commit that completed S_w(j) tracks every
      // earlier MMA of the issuer, so O(j-1) is complete now (the rescale below may read it). The O
      // barrier is therefore waited only once, for the last tile: it is then at most one phase
      // behind, which a parity wait resolves.
      tc_fence_after();
      // The whole S row in registers (one TMEM load), its exact max, then P = exp2(s * c - m_ref)
      // written as packed 16-bit pairs over S columns [0, 64) in four 16-column stores.
      float s[128];
      tmem_ld128(scol, s);
      if (tl.masked)
        mask_cols128(s, tl.kind, ml, tl.kind == 1 ? load_routed(p, h, tl.group, tl.slot0, lane)
                                                  : RoutedPos{{-1, -1, -1, -1}});
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(s[k], s[8 + k]);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], s[i + k], s[i + 8 + k]);
      const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], fmax3(mx8[5], mx8[6], mx8[7])));
      const float mt = mx * c;
      // Lazy rescale: the reference max moves only when the tile max passes it by more than
      // 2^RESCALE_LOG2, so P stays below 2^RESCALE_LOG2 and most tiles leave O untouched.
      float alpha = 1.f;
      bool rescale_o = false;
      if (mt > m_ref + RESCALE_LOG2) {
        alpha = fast_exp2(m_ref - mt);
        rescale_o = j > 0 && m_ref > -1.0e20f;
        l *= alpha;
        m_ref = mt;
      }
      // The O rescale uses warp-wide TMEM loads/stores, so it is decided per warp: lanes that
      // keep their reference multiply by exactly 1. A warp that rescales holds back its
      // first-half arrive until O is rescaled (the first P.V half accumulates into O).
      if (!rescale_o) alpha = 1.f;
      const bool warp_rescale = __any_sync(0xffffffffu, rescale_o);
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg = -m_ref;
      const uint64_t c2 = f2_pack(c, c), n2 = f2_pack(neg, neg);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint64_t x2 = f2_fma(f2_pack(s[32 * q + 2 * i], s[32 * q + 2 * i + 1]), c2, n2);
          float a, b;
          if (i % EXP2_POLY_EVERY == EXP2_POLY_EVERY - 1) {
            exp2_poly2(x2, a, b);
          } else {
            float xa, xb;
            f2_unpack(x2, xa, xb);
            a = fast_exp2(xa);
            b = fast_exp2(xb);
          }
          ls[i & 3] += a + b;
          pk[i] = pack2<T>(a, b);
        }
        tmem_st16(scol + 16u * q, pk);
        if (q == 1 && !warp_rescale) {
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(bar(PB_P + 2 * w));
        }
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // O(j-1) is complete (waited above) and no part of P(j).V(j) is issued before this warp's
      // first-half arrive below.
      if (warp_rescale) {
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          float o[32];
          tmem_ld32(ocol + q4 * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(ocol + q4 * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      if (warp_rescale) mbar_arrive(bar(PB_P + 2 * w));
      mbar_arrive(bar(PB_P + 2 * w + 1));
    }
    bool have_o = false;
    if (ok && nt > 0) have_o = mbar_wait_warp(bar(PB_O + w), (nt - 1) & 1, abort_flag, F_EPI_O);
    tc_fence_after();
    const int64_t lrow = row0 + row;
    const bool store = lrow < row1;
    if (p.splits > 1) {
      float* acc = p.part_acc + (((int64_t)split * p.bh + h) * p.t + lrow) * 128;
      if (store)
        p.part_ml[((int64_t)split * p.bh + h) * p.t + lrow] =
            make_float2(have_o ? m_ref : -1.0e20f, have_o ? l : 0.f);
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float o[32];
        if (have_o) {
          tmem_ld32(ocol + q4 * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (store) {
          float4* dst = reinterpret_cast<float4*>(acc + q4 * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
    } else {
      float inv = (have_o && l > 0.f) ? 1.f / fmaxf(l, 1.0e-20f) : 0.f;
      if (p.mask && store && qpos < p.n && !p.mask[batch * p.sm_b + qpos * p.sm_t]) inv = 0.f;
      T* out = static_cast<T*>(p.out) + h * p.so_h + lrow * p.so_t;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float o[32];
        if (have_o) {
          tmem_ld32(ocol + q4 * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (store) {
          uint32_t q16[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) q16[i] = pack2<T>(o[2 * i] * inv, o[2 * i + 1] * inv);
          uint4* dst = reinterpret_cast<uint4*>(out + q4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(q16[4 * i], q16[4 * i + 1], q16[4 * i + 2], q16[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// Merges the split partials of a 128-wide head: one warp per row, 4 columns per lane.
template <typename T>
__global__ void __launch_bounds__(128) tc_combine_kernel(FlashParams p) {
  using E = Elem<T>;
  const int64_t h = blockIdx.y;
  const int64_t row = p.row_begin + (int64_t)blockIdx.x * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= p.row_end) return;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_ml[((int64_t)s * p.bh + h) * p.t + row].x);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < p.splits; ++s) {
    const int64_t base = ((int64_t)s * p.bh + h) * p.t + row;
    const float2 ml = p.part_ml[base];
    const float w = fast_exp2(ml.x - M);
    L += ml.y * w;
    const float4 a = reinterpret_cast<const float4*>(p.part_acc + base * 128)[lane];
    acc.x += a.x * w;
    acc.y += a.y * w;
    acc.z += a.z * w;
    acc.w += a.w * w;
  }
  float inv = 1.f / fmaxf(L, 1.0e-20f);
  const int64_t qpos = p.offset + row;
  const int64_t batch = h / p.num_heads;
  if (p.mask && !p.mask[batch * p.sm_b + qpos * p.sm_t]) inv = 0.f;
  T* ob = static_cast<T*>(p.out) + h * p.so_h + row * p.so_t + lane * 4;
  uint2 v;
  v.x = pack2<T>(acc.x * inv, acc.y * inv);
  v.y = pack2<T>(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(ob) = v;
}

// ----------------------------------------------------------------------------- host side
// Two query heads per CTA when consecutive heads share a KV head (even GQA group size).
bool pair_mode(const bb_flash_args* a) {
  return a->kv_groups % 2 == 0 && a->num_heads % 2 == 0 && a->bh % 2 == 0;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 3-D map over a [heads][rows][128] view with element strides (s_head, s_row); the two outer
// dimensions are ordered by stride (swap = 1 when the head stride is the smaller one).
int make_map(CUtensorMap* m, int* swap, const void* base, int dtype, int64_t heads, int64_t rows,
             int64_t s_head, int64_t s_row) {
  auto fn = encode_fn();
  if (!fn) return fail(BB_ERR_DEVICE, "flash: cuTensorMapEncodeTiled is unavailable");
  if (heads == 1) s_head = s_row * rows;
  const bool sw = s_head < s_row;
  *swap = sw ? 1 : 0;
  cuuint64_t dims[3] = {128, (cuuint64_t)(sw ? heads : rows), (cuuint64_t)(sw ? rows : heads)};
  cuuint64_t strides[2] = {(cuuint64_t)((sw ? s_head : s_row) * 2), (cuuint64_t)((sw ? s_row : s_head) * 2)};
  cuuint32_t box[3] = {64, sw ? 1u : 128u, sw ? 128u : 1u};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dtype == BB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BB_ERR_LAUNCH, "flash: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BB_OK;
}

// Bytes of one of the two gathered routed-row arrays.
size_t gather_kv_bytes(const bb_flash_args* a) {
  return align_up((size_t)a->bh * a->route_groups * cdiv(a->route_k, BN) * BN * 128 * 2, 256);
}

template <typename T>
int launch(const bb_flash_args* a, FlashParams& p, cudaStream_t stream) {
  p.serial = unit_next_serial();
  TcMaps maps;
  const int64_t hk = a->bh / a->kv_groups;
  int st = make_map(&maps.q, &maps.q_swap, a->q, a->dtype, a->bh, a->t, a->sq_h, a->sq_t);
  if (st) return st;
  int sk = 0, sv = 0;
  st = make_map(&maps.k, &sk, a->k, a->dtype, hk, a->n, a->sk_h, a->sk_t);
  if (st) return st;
  st = make_map(&maps.v, &sv, a->v, a->dtype, hk, a->n, a->sv_h, a->sv_t);
  if (st) return st;
  if (sk != sv) return fail(BB_ERR_STRIDE, "flash: K and V views must have the same dimension order");
  maps.kv_swap = sk;
  maps.kg = maps.k;  // unused without routes
  maps.vg = maps.v;
  if (p.kg) {
    const int64_t rows = p.bh * p.route_groups * p.route_kpad;
    if (rows > 0x7fffffffLL) return fail(BB_ERR_UNSUPPORTED, "flash: too many routed rows (%lld)", (long long)rows);
    const size_t half = gather_kv_bytes(a);
    p.vg = static_cast<char*>(p.kg) + half;
    p.tile_min = reinterpret_cast<int32_t*>(static_cast<char*>(p.vg) + half);
    if (cudaMemsetAsync(p.tile_min, 0xff, (size_t)(rows / BN) * 4, stream) != cudaSuccess)
      return fail(BB_ERR_LAUNCH, "flash: %s", cudaGetErrorString(cudaGetLastError()));
    int unused = 0;
    st = make_map(&maps.kg, &unused, p.kg, a->dtype, 1, rows, 0, 128);
    if (st) return st;
    st = make_map(&maps.vg, &unused, p.vg, a->dtype, 1, rows, 0, 128);
    if (st) return st;
    const int64_t grid = std::min<int64_t>(cdiv(rows * 16, 256), (int64_t)num_sms() * 8);
    route_gather_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(p);
    BB_CHECK_LAUNCH("route_gather_kernel");
  }
  if (pair_mode(a)) {
    // The kernel's register split only works if the launch hands out at least what its warpgroups
    // ask for; an increase beyond that would wait forever, so refuse to launch instead.
    static int launch_regs = -1;
    if (launch_regs < 0) {
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, flash_tc_pair_kernel<T>) != cudaSuccess)
        return fail(BB_ERR_LAUNCH, "flash: %s", cudaGetErrorString(cudaGetLastError()));
      launch_regs = fa.numRegs;
    }
    if (launch_regs * P_THREADS < 128 * P_REG_LOW + 256 * P_REG_HIGH)
      return fail(BB_ERR_LAUNCH, "flash: the pair kernel launches with %d registers a thread, fewer than its split needs",
                  launch_regs);
    cudaFuncSetAttribute(flash_tc_pair_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SM_ALLOC);
    dim3 grid((unsigned)cdiv(a->row_end - a->row_begin, BM), (unsigned)(a->bh / 2), (unsigned)p.splits);
    flash_tc_pair_kernel<T><<<grid, P_THREADS, P_SM_ALLOC, stream>>>(maps, p);
    BB_CHECK_LAUNCH("flash_tc_pair_kernel");
  } else {
    cudaFuncSetAttribute(flash_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM_ALLOC);
    dim3 grid((unsigned)cdiv(a->row_end - a->row_begin, BM), (unsigned)a->bh, (unsigned)p.splits);
    flash_tc_kernel<T><<<grid, THREADS, SM_ALLOC, stream>>>(maps, p);
    BB_CHECK_LAUNCH("flash_tc_kernel");
  }
  if (p.splits > 1) {
    dim3 g2((unsigned)cdiv(a->row_end - a->row_begin, 4), (unsigned)a->bh);
    tc_combine_kernel<T><<<g2, 128, 0, stream>>>(p);
    BB_CHECK_LAUNCH("tc_combine_kernel");
  }
  return BB_OK;
}

}  // namespace tc

int flash_tc_splits(const bb_flash_args* a, int sms) {
  const int64_t rows = a->row_end - a->row_begin;
  const bool pair = tc::pair_mode(a);
  const int64_t ctas = cdiv(rows, tc::BM) * (pair ? a->bh / 2 : a->bh);
  const int64_t tiles = cdiv(std::min(a->n, a->window + tc::BM), tc::BN) + cdiv(a->front, tc::BN) +
                        cdiv(a->route_k, tc::BN);
  if (ctas <= 0 || ctas >= 2LL * sms || tiles < 16) return 1;
  // Cost of s splits in key-tile steps: whole waves of CTAs times each CTA's steps plus its fixed
  // cost (start-up to the first S, epilogue, the partial-result write and its share of the combine),
  // which timings of the exact tail over explicit split counts put at about ten steps.
  constexpr int64_t CTA_FIXED_STEPS = 10;
  int best = 1;
  int64_t best_cost = cdiv(ctas, sms) * (tiles + CTA_FIXED_STEPS);
  for (int s = 2; s <= 32 && s * 4 <= tiles; ++s) {
    const int64_t cost = cdiv(ctas * s, sms) * (cdiv(tiles, s) + CTA_FIXED_STEPS);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

size_t flash_tc_gather_bytes(const bb_flash_args* a) {
  if (a->route_k <= 0) return 0;
  return 2 * tc::gather_kv_bytes(a) + align_up((size_t)a->bh * a->route_groups * cdiv(a->route_k, tc::BN) * 4, 256);
}

int flash_tc_launch(const bb_flash_args* a, FlashParams& p, cudaStream_t stream) {
  if (a->dtype == BB_BF16) return tc::launch<__nv_bfloat16>(a, p, stream);
  return tc::launch<__half>(a, p, stream);
}

int flash_set_wait_limit(unsigned long long ns) { return tc::unit_set_wait_limit(ns); }

int flash_set_stall(int on) {
  const int v = on ? 1 : 0;
  return cudaMemcpyToSymbol(tc::g_tc_stall, &v, sizeof(int)) == cudaSuccess ? 0 : -1;
}

int flash_fault_take(int* code) {
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
