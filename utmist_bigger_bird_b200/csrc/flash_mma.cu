// Sparse flash attention, warp-level tensor-core version (mma.sync m16n8k16).
//
// Semantics of bigger_bird_flash (kernels/bigger_bird_flash.py:42-96): one online softmax per
// query over three disjoint key sets -- sink [0, front), causal window [q-W+1, q] restricted to
// keys >= front, and routed keys idx[h, group(q), :] in [front, q-W] -- with scores
// q.k * scale * log2(e), exp2, a finite running-max floor of -1e20 (so a fully masked row gives
// 0) and P rounded to the input dtype before the PV product (:37); output acc / max(l, 1e-20).
//
// One CTA = 64 query rows of one query head (4 warps x 16 rows). Key tiles of 64 rows are
// gathered with cp.async from their positions (contiguous for sink/window, indexed for routes),
// double-buffered in shared memory. The per-CTA tile list is [sink tiles][window tiles]
// [routed tiles per route group]; for short query ranges over long key ranges (the exact tail)
// the list is split across grid.z and the partial (acc, max, sum) are merged by
// flash_combine_kernel.
#include <algorithm>

#include "flash.cuh"

namespace bb {

constexpr int FM_BM = 64;
constexpr int FM_BN = 64;
constexpr int FM_THREADS = 128;


namespace {

template <int DP> struct FmSmem {
  static constexpr int LD = DP + 8;
  static constexpr size_t q_bytes = (size_t)FM_BM * LD * 2;
  static constexpr size_t kv_bytes = (size_t)FM_BN * LD * 2;  // one K (or V) stage
  static constexpr size_t bytes = q_bytes + 4 * kv_bytes + 2 * FM_BN * 8;
};

// Tile list of one CTA.
struct TileList {
  int64_t q_first, q_last;     // absolute positions of the CTA's first/last valid rows
  int64_t win_lo, win_hi;      // window keys [win_lo, win_hi]
  int64_t g_lo;                // first route group
  int n_sink, n_win, n_route_per_group, n_groups, total;
};

__device__ __forceinline__ TileList make_tiles(const FlashParams& p, int64_t row0, int64_t row1) {
  TileList tl;
  tl.q_first = p.offset + row0;
  tl.q_last = p.offset + row1 - 1;
  const int64_t sink_end = min(p.front, tl.q_last + 1);
  tl.n_sink = sink_end > 0 ? (int)cdiv(sink_end, FM_BN) : 0;
  tl.win_lo = max(max(p.front, tl.q_first - p.window + 1), (int64_t)0);
  tl.win_hi = tl.q_last;
  tl.n_win = tl.win_hi >= tl.win_lo ? (int)cdiv(tl.win_hi - tl.win_lo + 1, FM_BN) : 0;
  tl.n_route_per_group = (int)cdiv(p.route_k, FM_BN);
  tl.g_lo = tl.q_first / p.route_chunk;
  const int64_t g_hi = min(tl.q_last / p.route_chunk, p.route_groups - 1);
  tl.n_groups = p.route_k > 0 && g_hi >= tl.g_lo ? (int)(g_hi - tl.g_lo + 1) : 0;
  tl.total = tl.n_sink + tl.n_win + tl.n_groups * tl.n_route_per_group;
  return tl;
}

// Kind of tile t: 0 sink, 1 window, 2 routed. For routed tiles *group and *slot0 are set.
__device__ __forceinline__ int tile_kind(const TileList& tl, int t, int64_t* key0, int64_t* group,
                                         int64_t* slot0) {
  if (t < tl.n_sink) { *key0 = (int64_t)t * FM_BN; return 0; }
  t -= tl.n_sink;
  if (t < tl.n_win) { *key0 = tl.win_lo + (int64_t)t * FM_BN; return 1; }
  t -= tl.n_win;
  *group = tl.g_lo + t / tl.n_route_per_group;
  *slot0 = (int64_t)(t % tl.n_route_per_group) * FM_BN;
  return 2;
}

// Loads key/value rows of tile t into one stage and records each row's position (-1: none).
template <typename T, int DP>
__device__ __forceinline__ void load_tile(const FlashParams& p, const TileList& tl, int t,
                                          int64_t h, int64_t kvh, T* ks, T* vs, int64_t* pos) {
  constexpr int LD = FmSmem<DP>::LD;
  constexpr int CH = DP / 8;
  int64_t key0 = 0, group = 0, slot0 = 0;
  const int kind = tile_kind(tl, t, &key0, &group, &slot0);
  for (int i = threadIdx.x; i < FM_BN; i += FM_THREADS) {
    int64_t ps = -1;
    if (kind == 0) {
      ps = key0 + i;
      if (ps >= p.front) ps = -1;
    } else if (kind == 1) {
      ps = key0 + i;
      if (ps > tl.win_hi) ps = -1;
    } else {
      const int64_t slot = slot0 + i;
      if (slot < p.route_k) {
        ps = p.idx[h * p.si_h + group * p.si_g + slot * p.si_k];
        if (ps < 0 || ps >= p.n) ps = -1;
      }
    }
    pos[i] = ps;
  }
  __syncthreads();
  const T* kb = static_cast<const T*>(p.k) + kvh * p.sk_h;
  const T* vb = static_cast<const T*>(p.v) + kvh * p.sv_h;
  for (int c = threadIdx.x; c < FM_BN * CH; c += FM_THREADS) {
    const int i = c / CH, ch = c % CH;
    const int64_t ps = pos[i];
    const bool valid = ps >= 0 && ch * 8 < p.d;
    cp_async_16(smem_u32(ks + i * LD + ch * 8), valid ? kb + ps * p.sk_t + ch * 8 : kb, valid);
    cp_async_16(smem_u32(vs + i * LD + ch * 8), valid ? vb + ps * p.sv_t + ch * 8 : vb, valid);
  }
}

template <typename T, int DP>
__global__ void __launch_bounds__(FM_THREADS, 2) flash_mma_kernel(FlashParams p) {
  using E = Elem<T>;
  constexpr int LD = FmSmem<DP>::LD;
  constexpr int NT_O = DP / 8;  // n8 tiles of the output
  extern __shared__ __align__(128) unsigned char smem[];
  T* qs = reinterpret_cast<T*>(smem);
  T* kst[2] = {reinterpret_cast<T*>(smem + FmSmem<DP>::q_bytes),
               reinterpret_cast<T*>(smem + FmSmem<DP>::q_bytes + FmSmem<DP>::kv_bytes)};
  T* vst[2] = {reinterpret_cast<T*>(smem + FmSmem<DP>::q_bytes + 2 * FmSmem<DP>::kv_bytes),
               reinterpret_cast<T*>(smem + FmSmem<DP>::q_bytes + 3 * FmSmem<DP>::kv_bytes)};
  int64_t* post[2] = {reinterpret_cast<int64_t*>(smem + FmSmem<DP>::q_bytes + 4 * FmSmem<DP>::kv_bytes),
                      reinterpret_cast<int64_t*>(smem + FmSmem<DP>::q_bytes + 4 * FmSmem<DP>::kv_bytes) + FM_BN};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t h = blockIdx.y;
  const int split = blockIdx.z;
  const int64_t row0 = p.row_begin + (int64_t)blockIdx.x * FM_BM;
  const int64_t row1 = min(row0 + FM_BM, p.row_end);
  const int64_t kvh = (h / p.num_heads) * (p.num_heads / p.kv_groups) + (h % p.num_heads) / p.kv_groups;
  const int64_t batch = h / p.num_heads;
  const TileList tl = make_tiles(p, row0, row1);
  const int t_begin = (int)((int64_t)tl.total * split / p.splits);
  const int t_end = (int)((int64_t)tl.total * (split + 1) / p.splits);

  // Q tile.
  {
    constexpr int CH = DP / 8;
    const T* qb = static_cast<const T*>(p.q) + h * p.sq_h;
    for (int c = threadIdx.x; c < FM_BM * CH; c += FM_THREADS) {
      const int i = c / CH, ch = c % CH;
      const int64_t row = row0 + i;
      const bool valid = row < row1 && ch * 8 < p.d;
      cp_async_16(smem_u32(qs + i * LD + ch * 8), valid ? qb + row * p.sq_t + ch * 8 : qb, valid);
    }
  }
  if (t_begin < t_end) load_tile<T, DP>(p, tl, t_begin, h, kvh, kst[0], vst[0], post[0]);
  cp_async_commit();

  // Per-thread rows: r0 = warp*16 + lane/4, r1 = r0 + 8.
  const int64_t qpos0 = tl.q_first + warp * 16 + lane / 4;
  const int64_t qpos1 = qpos0 + 8;
  const int64_t grp0 = qpos0 / p.route_chunk, grp1 = qpos1 / p.route_chunk;
  float o[NT_O][4];
#pragma unroll
  for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -1.0e20f, m1 = -1.0e20f, l0 = 0.f, l1 = 0.f;
  uint32_t qf[DP / 16][4];
  bool q_loaded = false;

  for (int t = t_begin; t < t_end; ++t) {
    const int st = (t - t_begin) & 1;
    if (t + 1 < t_end) {
      __syncthreads();  // the other stage's previous readers are done
      load_tile<T, DP>(p, tl, t + 1, h, kvh, kst[st ^ 1], vst[st ^ 1], post[st ^ 1]);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (!q_loaded) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk)
        ldmatrix_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3],
                    smem_u32(qs + (warp * 16 + (lane % 16)) * LD + kk * 16 + (lane / 16) * 8));
      q_loaded = true;
    }
    const T* ks = kst[st];
    const T* vs = vst[st];
    const int64_t* pos = post[st];
    int64_t key0 = 0, group = 0, slot0 = 0;
    const int kind = tile_kind(tl, t, &key0, &group, &slot0);

    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3,
                    smem_u32(ks + (np * 16 + (lane / 16) * 8 + (lane % 8)) * LD + kk * 16 + ((lane / 8) % 2) * 8));
        const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
        mma_16816<T>(s[np * 2], qf[kk], bA);
        mma_16816<T>(s[np * 2 + 1], qf[kk], bB);
      }
    }
    // Mask + scale, row max.
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t ps = pos[nt * 8 + (lane % 4) * 2 + e];
        bool ok0, ok1;
        if (ps < 0) {
          ok0 = ok1 = false;
        } else if (kind == 0) {
          ok0 = ps <= qpos0;
          ok1 = ps <= qpos1;
        } else if (kind == 1) {
          ok0 = ps <= qpos0 && ps >= qpos0 - p.window + 1;
          ok1 = ps <= qpos1 && ps >= qpos1 - p.window + 1;
        } else {
          ok0 = ps >= p.front && ps <= qpos0 && ps < qpos0 - p.window + 1 && grp0 == group;
          ok1 = ps >= p.front && ps <= qpos1 && ps < qpos1 - p.window + 1 && grp1 == group;
        }
        if (p.mask && ps >= 0 && !p.mask[batch * p.sm_b + ps * p.sm_t]) ok0 = ok1 = false;
        s[nt][e] = ok0 ? s[nt][e] * p.scale_log2 : -INFINITY;
        s[nt][2 + e] = ok1 ? s[nt][2 + e] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[nt][e]);
        mx1 = fmaxf(mx1, s[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(fmaxf(m0, mx0), -1.0e20f);
    const float mn1 = fmaxf(fmaxf(m1, mx1), -1.0e20f);
    const float a0 = fast_exp2(m0 - mn0), a1 = fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = fast_exp2(s[nt][0] - mn0), p1 = fast_exp2(s[nt][1] - mn0);
      const float p2 = fast_exp2(s[nt][2] - mn1), p3 = fast_exp2(s[nt][3] - mn1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pf[nt / 2][(nt % 2) * 2 + 0] = pack2<T>(p0, p1);
      pf[nt / 2][(nt % 2) * 2 + 1] = pack2<T>(p2, p3);
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int i = 0; i < NT_O; ++i) {
      o[i][0] *= a0; o[i][1] *= a0;
      o[i][2] *= a1; o[i][3] *= a1;
    }
    // O += P V.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      // A fragment order: (r0,k0-7), (r1,k0-7), (r0,k8-15), (r1,k8-15)
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dp = 0; dp < DP / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3,
                          smem_u32(vs + (kk * 16 + ((lane / 8) % 2) * 8 + (lane % 8)) * LD + dp * 16 + (lane / 16) * 8));
        const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
        mma_16816<T>(o[dp * 2], a, bA);
        mma_16816<T>(o[dp * 2 + 1], a, bB);
      }
    }
  }
  if (!q_loaded) {
    // No tiles: rows keep acc = 0, l = 0 (fully masked -> 0).
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  const int64_t lr0 = row0 + warp * 16 + lane / 4, lr1 = lr0 + 8;  // local rows (of T)
  if (p.splits > 1) {
    float* acc = p.part_acc + ((int64_t)split * p.bh + h) * p.t * DP;
    float2* ml = p.part_ml + ((int64_t)split * p.bh + h) * p.t;
#pragma unroll
    for (int i = 0; i < NT_O; ++i) {
      const int c = i * 8 + (lane % 4) * 2;
      if (lr0 < row1) { acc[lr0 * DP + c] = o[i][0]; acc[lr0 * DP + c + 1] = o[i][1]; }
      if (lr1 < row1) { acc[lr1 * DP + c] = o[i][2]; acc[lr1 * DP + c + 1] = o[i][3]; }
    }
    if (lane % 4 == 0) {
      if (lr0 < row1) ml[lr0] = make_float2(m0, l0);
      if (lr1 < row1) ml[lr1] = make_float2(m1, l1);
    }
    return;
  }
  float inv0 = 1.f / fmaxf(l0, 1.0e-20f), inv1 = 1.f / fmaxf(l1, 1.0e-20f);
  if (p.mask) {
    if (qpos0 < p.n && !p.mask[batch * p.sm_b + qpos0 * p.sm_t]) inv0 = 0.f;
    if (qpos1 < p.n && !p.mask[batch * p.sm_b + qpos1 * p.sm_t]) inv1 = 0.f;
  }
  T* ob = static_cast<T*>(p.out) + h * p.so_h;
#pragma unroll
  for (int i = 0; i < NT_O; ++i) {
    const int c = i * 8 + (lane % 4) * 2;
    if (c < p.d) {
      if (lr0 < row1) {
        ob[lr0 * p.so_t + c] = E::from_f(o[i][0] * inv0);
        ob[lr0 * p.so_t + c + 1] = E::from_f(o[i][1] * inv0);
      }
      if (lr1 < row1) {
        ob[lr1 * p.so_t + c] = E::from_f(o[i][2] * inv1);
        ob[lr1 * p.so_t + c + 1] = E::from_f(o[i][3] * inv1);
      }
    }
  }
}

// Merges split partials: out = sum_s acc_s 2^(m_s - M) / max(sum_s l_s 2^(m_s - M), 1e-20).
template <typename T>
__global__ void __launch_bounds__(128) flash_combine_kernel(FlashParams p, int dp) {
  using E = Elem<T>;
  const int64_t h = blockIdx.y;
  const int64_t row = p.row_begin + blockIdx.x;
  const int64_t batch = h / p.num_heads;
  if (row >= p.row_end) return;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_ml[((int64_t)s * p.bh + h) * p.t + row].x);
  float L = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float2 ml = p.part_ml[((int64_t)s * p.bh + h) * p.t + row];
    L += ml.y * fast_exp2(ml.x - M);
  }
  float inv = 1.f / fmaxf(L, 1.0e-20f);
  const int64_t qpos = p.offset + row;
  if (p.mask && !p.mask[batch * p.sm_b + qpos * p.sm_t]) inv = 0.f;
  T* ob = static_cast<T*>(p.out) + h * p.so_h + row * p.so_t;
  for (int c = threadIdx.x; c < p.d; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float2 ml = p.part_ml[((int64_t)s * p.bh + h) * p.t + row];
      acc += p.part_acc[(((int64_t)s * p.bh + h) * p.t + row) * dp + c] * fast_exp2(ml.x - M);
    }
    ob[c] = E::from_f(acc * inv);
  }
}

int dpad_of(int64_t d) { return d <= 32 ? 32 : (d <= 64 ? 64 : 128); }

// Split factor: spread long key ranges of few CTAs over the machine.
int choose_splits(const bb_flash_args* a) {
  const int64_t rows = a->row_end - a->row_begin;
  const int64_t ctas = cdiv(rows, FM_BM) * a->bh;
  const int64_t keys = std::min(a->n, a->window + FM_BM) + a->front + a->route_k;
  const int64_t tiles = cdiv(keys, FM_BN);
  const int64_t target = 2LL * num_sms() * 2;
  if (ctas >= target || tiles < 16) return 1;
  return (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(cdiv(target, ctas), tiles / 8), 32));
}

template <typename T, int DP>
int launch_flash_t(const bb_flash_args* a, FlashParams& p, cudaStream_t stream) {
  const size_t smem = FmSmem<DP>::bytes;
  cudaFuncSetAttribute(flash_mma_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)cdiv(a->row_end - a->row_begin, FM_BM), (unsigned)a->bh, (unsigned)p.splits);
  flash_mma_kernel<T, DP><<<grid, FM_THREADS, smem, stream>>>(p);
  BB_CHECK_LAUNCH("flash_mma_kernel");
  if (p.splits > 1) {
    dim3 g2((unsigned)(a->row_end - a->row_begin), (unsigned)a->bh);
    flash_combine_kernel<T><<<g2, 128, 0, stream>>>(p, DP);
    BB_CHECK_LAUNCH("flash_combine_kernel");
  }
  return BB_OK;
}

}  // namespace

// head_dim 128 without a token mask (every Llama-shaped layer) runs on the tcgen05/TMEM kernels;
// smaller head dims and token-masked calls (the reference's exp 19 caller) run on the mma.sync kernel.
bool use_tc(const bb_flash_args* a) { return a->d == 128 && a->token_mask == nullptr; }

int flash_check(const bb_flash_args* a) {
  if (!a) return fail(BB_ERR_ARG, "flash: null args");
  if (a->dtype != BB_BF16 && a->dtype != BB_F16) return fail(BB_ERR_DTYPE, "flash: dtype must be f16 or bf16");
  if (a->kv_groups <= 0 || a->num_heads <= 0 || a->num_heads % a->kv_groups || a->bh % a->num_heads)
    return fail(BB_ERR_SHAPE, "flash: heads must be multiples of kv_groups / num_heads");
  if (a->d <= 0 || a->d > 128 || a->d % 8) return fail(BB_ERR_UNSUPPORTED, "flash: head_dim must be a multiple of 8 and <= 128");
  if (a->front < 0 || a->window < 1) return fail(BB_ERR_ARG, "front >= 0 and window >= 1 required");
  if (a->n < a->t) return fail(BB_ERR_SHAPE, "Key sequence must be at least as long as query sequence");
  if (a->n > 0x7fffffffLL) return fail(BB_ERR_UNSUPPORTED, "flash: sequences longer than 2^31 - 1 keys are not supported");
  if (a->route_chunk <= 0 || a->route_groups < 1 || a->route_k < 0) return fail(BB_ERR_SHAPE, "flash: bad route groups");
  if (a->row_begin < 0 || a->row_end > a->t || a->row_begin > a->row_end) return fail(BB_ERR_ARG, "flash: bad row range");
  return BB_OK;
}

int flash_check_pointers(const bb_flash_args* a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a->q || !a->k || !a->v || !a->out || (a->route_k > 0 && !a->idx)) return fail(BB_ERR_ARG, "flash: null pointer");
  if (!al(a->q) || !al(a->k) || !al(a->v) || (a->sq_h * 2) % 16 || (a->sq_t * 2) % 16 ||
      (a->sk_h * 2) % 16 || (a->sk_t * 2) % 16 || (a->sv_h * 2) % 16 || (a->sv_t * 2) % 16)
    return fail(BB_ERR_STRIDE, "flash: q/k/v rows must start on 16-byte boundaries");
  if (use_tc(a) && (!al(a->out) || (a->so_h * 2) % 16 || (a->so_t * 2) % 16))
    return fail(BB_ERR_STRIDE, "flash: output rows must start on 16-byte boundaries");
  return BB_OK;
}



int splits_of(const bb_flash_args* a) { return use_tc(a) ? flash_tc_splits(a, num_sms()) : choose_splits(a); }

int flash_workspace_size(const bb_flash_args* a, size_t* bytes) {
  int st = flash_check(a);
  if (st) return st;
  const int splits = splits_of(a);
  *bytes = splits > 1 ? align_up((size_t)splits * a->bh * a->t * dpad_of(a->d) * 4, 256) +
                            align_up((size_t)splits * a->bh * a->t * 8, 256)
                      : 0;
  if (use_tc(a)) *bytes += flash_tc_gather_bytes(a);
  return BB_OK;
}

int flash(const bb_flash_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  int st = flash_check(a);
  if (st) return st;
  if (a->row_end == a->row_begin || a->bh == 0) return BB_OK;
  st = flash_check_pointers(a);
  if (st) return st;
  size_t need = 0;
  flash_workspace_size(a, &need);
  if (ws_bytes < need || (need && !ws)) return fail(BB_ERR_WORKSPACE, "flash: workspace too small (%zu < %zu)", ws_bytes, need);
  FlashParams p;
  p.q = a->q; p.sq_h = a->sq_h; p.sq_t = a->sq_t;
  p.k = a->k; p.sk_h = a->sk_h; p.sk_t = a->sk_t;
  p.v = a->v; p.sv_h = a->sv_h; p.sv_t = a->sv_t;
  p.idx = a->idx; p.si_h = a->si_h; p.si_g = a->si_g; p.si_k = a->si_k;
  p.mask = a->token_mask; p.sm_b = a->sm_b; p.sm_t = a->sm_t;
  p.out = a->out; p.so_h = a->so_h; p.so_t = a->so_t;
  p.t = a->t; p.n = a->n; p.d = a->d; p.offset = a->n - a->t;
  p.num_heads = a->num_heads; p.kv_groups = a->kv_groups;
  p.front = std::min(a->front, a->n); p.window = a->window;
  p.route_k = a->route_k; p.route_groups = a->route_groups; p.route_chunk = a->route_chunk;
  p.row_begin = a->row_begin; p.row_end = a->row_end;
  p.scale_log2 = a->scale * LOG2E;
  p.splits = splits_of(a);
  p.bh = a->bh;
  p.serial = 0;
  const int dp = dpad_of(a->d);
  char* w = static_cast<char*>(ws);
  p.part_acc = reinterpret_cast<float*>(w);
  const size_t split_bytes = p.splits > 1 ? align_up((size_t)p.splits * a->bh * a->t * dp * 4, 256) +
                                                align_up((size_t)p.splits * a->bh * a->t * 8, 256)
                                          : 0;
  p.part_ml = reinterpret_cast<float2*>(w + (p.splits > 1 ? align_up((size_t)p.splits * a->bh * a->t * dp * 4, 256) : 0));
  p.route_kpad = cdiv(a->route_k, 128) * 128;
  p.kg = use_tc(a) && a->route_k > 0 ? w + split_bytes : nullptr;  // the tcgen05 launch lays out the rest
  p.vg = nullptr;
  p.tile_min = nullptr;
  if (use_tc(a)) return flash_tc_launch(a, p, stream);
  if (a->dtype == BB_BF16) {
    if (dp == 32) return launch_flash_t<__nv_bfloat16, 32>(a, p, stream);
    if (dp == 64) return launch_flash_t<__nv_bfloat16, 64>(a, p, stream);
    return launch_flash_t<__nv_bfloat16, 128>(a, p, stream);
  }
  if (dp == 32) return launch_flash_t<__half, 32>(a, p, stream);
  if (dp == 64) return launch_flash_t<__half, 64>(a, p, stream);
  return launch_flash_t<__half, 128>(a, p, stream);
}

}  // namespace bb
