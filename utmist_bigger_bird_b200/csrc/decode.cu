// Decode after a sparse prefill (one new query token per head):
//
//   decode_partial_kernel  split-K sparse flash decoding (kernels/bigger_bird_decode.py:21-64): the
//                          virtual key list front | window | routed of each route group is cut into
//                          `splits` chunks; per chunk, each query head's partial softmax (running max,
//                          sum, P.V with P rounded to the cache dtype) goes to the workspace.
//   decode_combine_kernel  merges the chunks (:103-107): w_s = exp2(m_s - max_s m_s),
//                          out = sum_s w_s acc_s / sum_s w_s l_s, in the query dtype.
//   droute_scores_kernel   decode routing pass 1 (kernels/bigger_bird_route.py:24-53): log2-scaled
//                          scores of every cached key for all query heads of a KV head, stored, plus
//                          per-chunk softmax statistics.
//   droute_pool_kernel     pass 2 (:56-77): merged statistics, probabilities averaged over the group,
//                          -1 outside [front, n - window).
//
// Keys and values are read in place from the cache (any head/row strides, rows 16-byte aligned).
// The cache length can come from a device int64 (`n_dev`), so a captured CUDA graph stays valid as
// the cache grows inside a fixed-capacity buffer. All of it is bound by HBM (each cache row is read
// once per route group); the dot products run on CUDA cores.
#include <algorithm>

#include "bb_common.cuh"

namespace bb {

int topk_sorted(const float* vals, int64_t rows, int64_t n, int64_t k, int32_t* out, int64_t so_h,
                cudaStream_t stream);

namespace {

constexpr int DK_THREADS = 128;  // 4 warps
constexpr int DK_BN = 64;        // keys per block
constexpr int DK_MAXROWS = 16;   // query heads per route group
constexpr float LOG2E_F_DK = 1.4426950408889634f;

struct DecodeParams {
  const void* q; int64_t sq_h;
  const void* k; int64_t sk_h, sk_t;
  const void* v; int64_t sv_h, sv_t;
  const int32_t* idx; int64_t si_r;  // [route rows][route_k]
  const int64_t* n_dev;
  int64_t n, cap, d, heads, kv_heads, groups, rows, route_rows, route_k, front, window;
  int64_t splits, split_len;
  float scale_log2;
  float* part_m;    // [route_rows][splits][rows]
  float* part_l;
  float* part_acc;  // [route_rows][splits][rows][d]
  void* out; int64_t so_h;
  // decode routing
  float* scores;    // [heads][cap]
  float* probs;     // [kv_heads][cap]
};

template <int DP> struct DkSmem {
  static constexpr int LD = DP + 8;  // padded row (elements): conflict-free 16-byte reads
  static constexpr size_t kv_bytes = (size_t)DK_BN * LD * 2;  // one 64-key block of K or V
};

__device__ __forceinline__ int64_t cache_len(const DecodeParams& p) {
  if (!p.n_dev) return p.n;
  const int64_t n = *p.n_dev;
  return n < 0 ? 0 : (n > p.cap ? p.cap : n);
}

// Position of virtual key j of route row r (front | window | routed), or -1 when it is not a key.
__device__ __forceinline__ int64_t virtual_pos(const DecodeParams& p, int64_t r, int64_t j, int64_t n) {
  int64_t pos;
  if (j < p.front) pos = j;
  else if (j < p.front + p.window) pos = n - p.window + (j - p.front);
  else pos = p.idx[r * p.si_r + (j - p.front - p.window)];
  return (pos >= 0 && pos < n) ? pos : -1;
}

// 64 rows of a K or V block (rows at positions pos_s[i]; -1 -> zero row) into padded shared memory.
template <typename T, int DP>
__device__ __forceinline__ void load_block(const T* base, int64_t s_t, const int64_t* pos_s, T* dst, int64_t d) {
  constexpr int LD = DkSmem<DP>::LD;
  constexpr int CH = DP / 8;
  for (int c = threadIdx.x; c < DK_BN * CH; c += DK_THREADS) {
    const int i = c / CH, ch = c % CH;
    const int64_t pos = pos_s[i];
    const bool ok = pos >= 0 && ch * 8 < d;
    const T* src = ok ? base + pos * s_t + ch * 8 : base;
    cp_async_16(smem_u32(dst + i * LD + ch * 8), src, ok);
  }
}

// Scores of this lane's two keys (lane, lane + 32) of the block for one query row (fp32 q in smem).
template <typename T, int DP>
__device__ __forceinline__ void row_scores(const float* qrow, const T* ks, int lane, float& s0, float& s1) {
  constexpr int LD = DkSmem<DP>::LD;
  float a0 = 0.f, a1 = 0.f;
  const T* k0 = ks + lane * LD;
  const T* k1 = ks + (lane + 32) * LD;
#pragma unroll 4
  for (int c = 0; c < DP; c += 8) {
    const uint4 u0 = *reinterpret_cast<const uint4*>(k0 + c);
    const uint4 u1 = *reinterpret_cast<const uint4*>(k1 + c);
    const T* e0 = reinterpret_cast<const T*>(&u0);
    const T* e1 = reinterpret_cast<const T*>(&u1);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float qv = qrow[c + e];
      a0 = fmaf(qv, Elem<T>::to_f(e0[e]), a0);
      a1 = fmaf(qv, Elem<T>::to_f(e1[e]), a1);
    }
  }
  s0 = a0;
  s1 = a1;
}

template <typename T, int DP>
__global__ void __launch_bounds__(DK_THREADS) decode_partial_kernel(DecodeParams p) {
  constexpr int LD = DkSmem<DP>::LD;
  extern __shared__ __align__(128) unsigned char smem[];
  T* ks = reinterpret_cast<T*>(smem);                                   // [2][64][LD]
  T* vs = ks + 2 * DK_BN * LD;                                          // [2][64][LD]
  float* qs = reinterpret_cast<float*>(vs + 2 * DK_BN * LD);            // [rows][DP]
  float* ps = qs + DK_MAXROWS * DP;                                     // [rows][64] P (dtype-rounded)
  int64_t* pos_s = reinterpret_cast<int64_t*>(ps + DK_MAXROWS * DK_BN);  // [2][64]
  const int64_t r = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int64_t kv = (r * p.rows) / p.groups;
  const int rows = (int)p.rows;
  const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
  const T* V = static_cast<const T*>(p.v) + kv * p.sv_h;
  // query rows (fp32, pre-scaled to log2 units as scores * scale * log2 e)
  const T* Q = static_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < rows * DP; i += DK_THREADS) {
    const int row = i / DP, c = i % DP;
    qs[i] = c < p.d ? Elem<T>::to_f(Q[(r * p.rows + row) * p.sq_h + c]) : 0.f;
  }
  const int64_t total = p.front + p.window + p.route_k;
  const int64_t j0 = split * p.split_len;
  const int64_t j1 = min(j0 + p.split_len, total);
  const int nblocks = j0 < j1 ? (int)cdiv(j1 - j0, (int64_t)DK_BN) : 0;
  // per-warp state for its rows (warp w owns rows w, w + 4, ...), lane owns dims 4*lane .. 4*lane+3
  constexpr int RPW = DK_MAXROWS / 4;
  constexpr int DPL = DP / 32;  // dims per lane
  float m[RPW], l[RPW], acc[RPW][DPL];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    m[i] = -1.0e20f;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[i][e] = 0.f;
  }
  auto positions = [&](int b, int buf) {
    for (int i = threadIdx.x; i < DK_BN; i += DK_THREADS) {
      const int64_t j = j0 + (int64_t)b * DK_BN + i;
      pos_s[buf * DK_BN + i] = j < j1 ? virtual_pos(p, r, j, n) : -1;
    }
  };
  if (nblocks > 0) {
    positions(0, 0);
    __syncthreads();
    load_block<T, DP>(K, p.sk_t, pos_s, ks, p.d);
    load_block<T, DP>(V, p.sv_t, pos_s, vs, p.d);
    cp_async_commit();
  }
  for (int b = 0; b < nblocks; ++b) {
    const int buf = b & 1;
    if (b + 1 < nblocks) {
      positions(b + 1, buf ^ 1);
      __syncthreads();
      load_block<T, DP>(K, p.sk_t, pos_s + (buf ^ 1) * DK_BN, ks + (buf ^ 1) * DK_BN * LD, p.d);
      load_block<T, DP>(V, p.sv_t, pos_s + (buf ^ 1) * DK_BN, vs + (buf ^ 1) * DK_BN * LD, p.d);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* kb = ks + buf * DK_BN * LD;
    const T* vb = vs + buf * DK_BN * LD;
    const bool ok0 = pos_s[buf * DK_BN + lane] >= 0, ok1 = pos_s[buf * DK_BN + lane + 32] >= 0;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int row = warp + 4 * i;
      if (row >= rows) break;
      float s0, s1;
      row_scores<T, DP>(qs + row * DP, kb, lane, s0, s1);
      s0 = ok0 ? s0 * p.scale_log2 : -INFINITY;
      s1 = ok1 ? s1 * p.scale_log2 : -INFINITY;
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(fmaxf(m[i], mx), -1.0e20f);
      const float alpha = fast_exp2(m[i] - mnew);
      // P rounded to the cache dtype before P.V (kernels/bigger_bird_decode.py:58); the sum uses
      // the unrounded values (:59).
      const float p0 = fast_exp2(s0 - mnew), p1 = fast_exp2(s1 - mnew);
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      ps[row * DK_BN + lane] = Elem<T>::round(p0);
      ps[row * DK_BN + lane + 32] = Elem<T>::round(p1);
      __syncwarp();
      float a[DPL];
#pragma unroll
      for (int e = 0; e < DPL; ++e) a[e] = 0.f;
      for (int key = 0; key < DK_BN; ++key) {
        const float pk = ps[row * DK_BN + key];
        const T* vr = vb + key * LD + lane * DPL;
#pragma unroll
        for (int e = 0; e < DPL; ++e) a[e] = fmaf(pk, Elem<T>::to_f(vr[e]), a[e]);
      }
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[i][e] = acc[i][e] * alpha + a[e];
      l[i] = l[i] * alpha + sum;
      m[i] = mnew;
      __syncwarp();
    }
    __syncthreads();
  }
  // partials: (m, l, acc) per row of this chunk
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int row = warp + 4 * i;
    if (row >= rows) break;
    const int64_t at = (r * p.splits + split) * p.rows + row;
    if (lane == 0) {
      p.part_m[at] = m[i];
      p.part_l[at] = l[i];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e)
      if (lane * DPL + e < p.d) p.part_acc[at * p.d + lane * DPL + e] = acc[i][e];
  }
}

// One warp per query head: merges its splits.
template <typename T>
__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeParams p) {
  const int64_t h = (int64_t)blockIdx.x * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (h >= p.heads) return;
  const int64_t r = h / p.rows, row = h % p.rows;
  float M = -INFINITY;
  for (int64_t s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_m[(r * p.splits + s) * p.rows + row]);
  float L = 0.f;
  for (int64_t s = 0; s < p.splits; ++s) {
    const int64_t at = (r * p.splits + s) * p.rows + row;
    L += p.part_l[at] * fast_exp2(p.part_m[at] - M);
  }
  T* o = static_cast<T*>(p.out) + h * p.so_h;
  for (int64_t c = lane; c < p.d; c += 32) {
    float a = 0.f;
    for (int64_t s = 0; s < p.splits; ++s) {
      const int64_t at = (r * p.splits + s) * p.rows + row;
      a += p.part_acc[at * p.d + c] * fast_exp2(p.part_m[at] - M);
    }
    o[c] = Elem<T>::from_f(a / L);
  }
}

// Decode routing pass 1: grid (kv_heads, splits); chunk of contiguous cached keys.
template <typename T, int DP>
__global__ void __launch_bounds__(DK_THREADS) droute_scores_kernel(DecodeParams p) {
  constexpr int LD = DkSmem<DP>::LD;
  extern __shared__ __align__(128) unsigned char smem[];
  T* ks = reinterpret_cast<T*>(smem);                         // [2][64][LD]
  float* qs = reinterpret_cast<float*>(ks + 2 * DK_BN * LD);  // [rows][DP]
  int64_t* pos_s = reinterpret_cast<int64_t*>(qs + DK_MAXROWS * DP);
  const int64_t kv = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int rows = (int)p.groups;
  const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
  const T* Q = static_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < rows * DP; i += DK_THREADS) {
    const int row = i / DP, c = i % DP;
    qs[i] = c < p.d ? Elem<T>::to_f(Q[(kv * p.groups + row) * p.sq_h + c]) : 0.f;
  }
  const int64_t j0 = split * p.split_len;
  const int64_t j1 = min(j0 + p.split_len, n);
  const int nblocks = j0 < j1 ? (int)cdiv(j1 - j0, (int64_t)DK_BN) : 0;
  constexpr int RPW = DK_MAXROWS / 4;
  float m[RPW], l[RPW];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    m[i] = -1.0e20f;
    l[i] = 0.f;
  }
  auto positions = [&](int b, int buf) {
    for (int i = threadIdx.x; i < DK_BN; i += DK_THREADS) {
      const int64_t j = j0 + (int64_t)b * DK_BN + i;
      pos_s[buf * DK_BN + i] = j < j1 ? j : -1;
    }
  };
  if (nblocks > 0) {
    positions(0, 0);
    __syncthreads();
    load_block<T, DP>(K, p.sk_t, pos_s, ks, p.d);
    cp_async_commit();
  }
  for (int b = 0; b < nblocks; ++b) {
    const int buf = b & 1;
    if (b + 1 < nblocks) {
      positions(b + 1, buf ^ 1);
      __syncthreads();
      load_block<T, DP>(K, p.sk_t, pos_s + (buf ^ 1) * DK_BN, ks + (buf ^ 1) * DK_BN * LD, p.d);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* kb = ks + buf * DK_BN * LD;
    const int64_t pos0 = pos_s[buf * DK_BN + lane], pos1 = pos_s[buf * DK_BN + lane + 32];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int row = warp + 4 * i;
      if (row >= rows) break;
      float s0, s1;
      row_scores<T, DP>(qs + row * DP, kb, lane, s0, s1);
      s0 = pos0 >= 0 ? s0 * p.scale_log2 : -INFINITY;
      s1 = pos1 >= 0 ? s1 * p.scale_log2 : -INFINITY;
      float* srow = p.scores + (kv * p.groups + row) * p.cap;
      if (pos0 >= 0) srow[pos0] = s0;
      if (pos1 >= 0) srow[pos1] = s1;
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(fmaxf(m[i], mx), -1.0e20f);
      float sum = fast_exp2(s0 - mnew) + fast_exp2(s1 - mnew);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[i] = l[i] * fast_exp2(m[i] - mnew) + sum;
      m[i] = mnew;
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int row = warp + 4 * i;
    if (row >= rows) break;
    if (lane == 0) {
      const int64_t at = (kv * p.splits + split) * p.groups + row;
      p.part_m[at] = m[i];
      p.part_l[at] = l[i];
    }
  }
}

// Decode routing pass 2: grid (kv_heads, cdiv(cap, 256)); one thread per cached position.
__global__ void __launch_bounds__(256) droute_pool_kernel(DecodeParams p) {
  const int64_t kv = blockIdx.x;
  const int64_t pos = (int64_t)blockIdx.y * 256 + threadIdx.x;
  const int64_t n = cache_len(p);
  __shared__ float sm[DK_MAXROWS], sinv[DK_MAXROWS];
  if (threadIdx.x < p.groups) {
    const int row = threadIdx.x;
    float M = -1.0e20f;
    for (int64_t s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_m[(kv * p.splits + s) * p.groups + row]);
    float L = 0.f;
    for (int64_t s = 0; s < p.splits; ++s) {
      const int64_t at = (kv * p.splits + s) * p.groups + row;
      L += p.part_l[at] * fast_exp2(p.part_m[at] - M);
    }
    sm[row] = M;
    sinv[row] = 1.f / fmaxf(L, 1.0e-30f);
  }
  __syncthreads();
  if (pos >= p.cap) return;
  float acc = 0.f;
  if (pos < n)
    for (int64_t row = 0; row < p.groups; ++row)
      acc += fast_exp2(p.scores[(kv * p.groups + row) * p.cap + pos] - sm[row]) * sinv[row];
  const bool keep = pos >= p.front && pos < n - p.window;
  p.probs[kv * p.cap + pos] = keep ? acc / (float)p.groups : -1.f;
}

struct DecodePlan {
  int64_t splits, split_len;
  size_t m_bytes, l_bytes, acc_bytes, total;
};

int dpad(int64_t d) { return d <= 32 ? 32 : (d <= 64 ? 64 : 128); }

int check_common(const bb_decode_args* a, int64_t rows_per_group_max) {
  if (!a) return fail(BB_ERR_ARG, "decode: null args");
  if (a->dtype != BB_F16 && a->dtype != BB_BF16) return fail(BB_ERR_DTYPE, "decode requires fp16 or bf16");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
    return fail(BB_ERR_SHAPE, "decode: heads must be a positive multiple of kv_heads");
  if (a->d <= 0 || a->d > 128 || a->d % 8) return fail(BB_ERR_UNSUPPORTED, "decode: head_dim must be a multiple of 8 and <= 128");
  if (a->cap <= 0) return fail(BB_ERR_SHAPE, "decode: empty cache");
  if (a->n < 0 || a->n > a->cap) return fail(BB_ERR_ARG, "decode: n must lie in [0, cap]");
  if (a->heads / a->kv_heads > rows_per_group_max)
    return fail(BB_ERR_UNSUPPORTED, "decode: at most %d query heads per KV head", (int)rows_per_group_max);
  if (a->front < 0 || a->window < 0) return fail(BB_ERR_ARG, "decode: front and window must be >= 0");
  return BB_OK;
}

int plan_decode(const bb_decode_args* a, DecodePlan* pl) {
  int st = check_common(a, DK_MAXROWS);
  if (st) return st;
  if (a->route_k < 0) return fail(BB_ERR_ARG, "decode: bad route count");
  if (a->route_k > 0 && a->route_rows != a->kv_heads && a->route_rows != a->heads)
    return fail(BB_ERR_SHAPE, "decode: indices must be [Hkv, R] (pooled) or [H, R] (per head)");
  const int64_t rr = a->route_k > 0 ? a->route_rows : a->kv_heads;
  const int64_t rows = a->heads / rr;
  const int64_t total = a->front + a->window + a->route_k;
  int64_t splits = a->splits;
  if (splits <= 0) splits = std::max<int64_t>(1, std::min<int64_t>(cdiv(total, (int64_t)4 * DK_BN), cdiv((int64_t)4 * num_sms(), rr)));
  int64_t split_len = cdiv(cdiv(std::max<int64_t>(total, 1), splits), (int64_t)DK_BN) * DK_BN;
  splits = cdiv(std::max<int64_t>(total, 1), split_len);
  pl->splits = splits;
  pl->split_len = split_len;
  const size_t parts = (size_t)rr * splits * rows;
  pl->m_bytes = align_up(parts * 4, 256);
  pl->l_bytes = align_up(parts * 4, 256);
  pl->acc_bytes = align_up(parts * a->d * 4, 256);
  pl->total = pl->m_bytes + pl->l_bytes + pl->acc_bytes;
  return BB_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_kv(const bb_decode_args* a, bool need_v) {
  if (!a->q || !a->k || (need_v && !a->v)) return fail(BB_ERR_ARG, "decode: null pointer");
  if (!al16(a->k) || (a->sk_h * 2) % 16 || (a->sk_t * 2) % 16 ||
      (need_v && (!al16(a->v) || (a->sv_h * 2) % 16 || (a->sv_t * 2) % 16)))
    return fail(BB_ERR_STRIDE, "decode: k/v rows must start on 16-byte boundaries");
  return BB_OK;
}

DecodeParams make_params(const bb_decode_args* a) {
  DecodeParams p{};
  p.q = a->q; p.sq_h = a->sq_h;
  p.k = a->k; p.sk_h = a->sk_h; p.sk_t = a->sk_t;
  p.v = a->v; p.sv_h = a->sv_h; p.sv_t = a->sv_t;
  p.idx = a->idx; p.si_r = a->si_r;
  p.n_dev = a->n_dev;
  p.n = a->n; p.cap = a->cap; p.d = a->d; p.heads = a->heads; p.kv_heads = a->kv_heads;
  p.groups = a->heads / a->kv_heads;
  p.route_k = a->route_k;
  p.front = a->front; p.window = a->window;
  p.scale_log2 = a->scale * LOG2E_F_DK;
  p.out = a->out; p.so_h = a->so_h;
  return p;
}

template <typename T, int DP>
int launch_decode(const bb_decode_args* a, const DecodePlan& pl, char* ws, cudaStream_t stream) {
  DecodeParams p = make_params(a);
  const int64_t rr = a->route_k > 0 ? a->route_rows : a->kv_heads;
  p.route_rows = rr;
  p.rows = a->heads / rr;
  p.splits = pl.splits;
  p.split_len = pl.split_len;
  p.part_m = reinterpret_cast<float*>(ws);
  p.part_l = reinterpret_cast<float*>(ws + pl.m_bytes);
  p.part_acc = reinterpret_cast<float*>(ws + pl.m_bytes + pl.l_bytes);
  const size_t smem = 4 * DkSmem<DP>::kv_bytes + (size_t)DK_MAXROWS * DP * 4 + (size_t)DK_MAXROWS * DK_BN * 4 +
                      2 * DK_BN * 8;
  cudaFuncSetAttribute(decode_partial_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  decode_partial_kernel<T, DP><<<dim3((unsigned)rr, (unsigned)pl.splits), DK_THREADS, smem, stream>>>(p);
  BB_CHECK_LAUNCH("decode_partial_kernel");
  decode_combine_kernel<T><<<(unsigned)cdiv(a->heads, (int64_t)4), 128, 0, stream>>>(p);
  BB_CHECK_LAUNCH("decode_combine_kernel");
  return BB_OK;
}

struct DroutePlan {
  int64_t splits, split_len;
  size_t scores_bytes, m_bytes, l_bytes, probs_bytes, total;
};

int plan_droute(const bb_decode_args* a, DroutePlan* pl) {
  int st = check_common(a, DK_MAXROWS);
  if (st) return st;
  if (a->route_k < 0 || a->route_k > a->cap) return fail(BB_ERR_ARG, "decode_route: k_route must lie in [0, cap]");
  int64_t splits = a->splits;
  if (splits <= 0)
    splits = std::max<int64_t>(1, std::min<int64_t>({cdiv(a->cap, (int64_t)4 * DK_BN), cdiv((int64_t)4 * num_sms(), a->kv_heads), (int64_t)256}));
  int64_t split_len = cdiv(cdiv(a->cap, splits), (int64_t)DK_BN) * DK_BN;
  splits = cdiv(a->cap, split_len);
  pl->splits = splits;
  pl->split_len = split_len;
  const size_t parts = (size_t)a->kv_heads * splits * (a->heads / a->kv_heads);
  pl->scores_bytes = align_up((size_t)a->heads * a->cap * 4, 256);
  pl->m_bytes = align_up(parts * 4, 256);
  pl->l_bytes = align_up(parts * 4, 256);
  pl->probs_bytes = a->out_probs ? 0 : align_up((size_t)a->kv_heads * a->cap * 4, 256);
  pl->total = pl->scores_bytes + pl->m_bytes + pl->l_bytes + pl->probs_bytes;
  return BB_OK;
}

template <typename T, int DP>
int launch_droute(const bb_decode_args* a, const DroutePlan& pl, char* ws, cudaStream_t stream) {
  DecodeParams p = make_params(a);
  p.splits = pl.splits;
  p.split_len = pl.split_len;
  p.scores = reinterpret_cast<float*>(ws);
  p.part_m = reinterpret_cast<float*>(ws + pl.scores_bytes);
  p.part_l = reinterpret_cast<float*>(ws + pl.scores_bytes + pl.m_bytes);
  p.probs = a->out_probs ? a->out_probs : reinterpret_cast<float*>(ws + pl.scores_bytes + pl.m_bytes + pl.l_bytes);
  const size_t smem = 2 * DkSmem<DP>::kv_bytes + (size_t)DK_MAXROWS * DP * 4 + 2 * DK_BN * 8;
  cudaFuncSetAttribute(droute_scores_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  droute_scores_kernel<T, DP><<<dim3((unsigned)a->kv_heads, (unsigned)pl.splits), DK_THREADS, smem, stream>>>(p);
  BB_CHECK_LAUNCH("droute_scores_kernel");
  droute_pool_kernel<<<dim3((unsigned)a->kv_heads, (unsigned)cdiv(a->cap, (int64_t)256)), 256, 0, stream>>>(p);
  BB_CHECK_LAUNCH("droute_pool_kernel");
  if (a->route_k > 0 && a->out_idx) {
    int st = topk_sorted(p.probs, a->kv_heads, a->cap, a->route_k, a->out_idx, a->so_i, stream);
    if (st) return st;
  }
  return BB_OK;
}

}  // namespace

int decode_workspace_size(const bb_decode_args* a, size_t* bytes) {
  DecodePlan pl;
  int st = plan_decode(a, &pl);
  if (st) return st;
  *bytes = pl.total;
  return BB_OK;
}

int decode(const bb_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  DecodePlan pl;
  int st = plan_decode(a, &pl);
  if (st) return st;
  if (!ws || ws_bytes < pl.total) return fail(BB_ERR_WORKSPACE, "decode: workspace too small (%zu < %zu)", ws_bytes, pl.total);
  st = check_kv(a, true);
  if (st) return st;
  if (!a->out || (a->route_k > 0 && !a->idx)) return fail(BB_ERR_ARG, "decode: null pointer");
  char* w = static_cast<char*>(ws);
  const int dp = dpad(a->d);
  if (a->dtype == BB_BF16) {
    if (dp == 32) return launch_decode<__nv_bfloat16, 32>(a, pl, w, stream);
    if (dp == 64) return launch_decode<__nv_bfloat16, 64>(a, pl, w, stream);
    return launch_decode<__nv_bfloat16, 128>(a, pl, w, stream);
  }
  if (dp == 32) return launch_decode<__half, 32>(a, pl, w, stream);
  if (dp == 64) return launch_decode<__half, 64>(a, pl, w, stream);
  return launch_decode<__half, 128>(a, pl, w, stream);
}

int decode_route_workspace_size(const bb_decode_args* a, size_t* bytes) {
  DroutePlan pl;
  int st = plan_droute(a, &pl);
  if (st) return st;
  *bytes = pl.total;
  return BB_OK;
}

int decode_route(const bb_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  DroutePlan pl;
  int st = plan_droute(a, &pl);
  if (st) return st;
  if (!ws || ws_bytes < pl.total) return fail(BB_ERR_WORKSPACE, "decode_route: workspace too small (%zu < %zu)", ws_bytes, pl.total);
  st = check_kv(a, false);
  if (st) return st;
  if (a->route_k > 0 && !a->out_idx && !a->out_probs) return fail(BB_ERR_ARG, "decode_route: no output");
  char* w = static_cast<char*>(ws);
  const int dp = dpad(a->d);
  if (a->dtype == BB_BF16) {
    if (dp == 32) return launch_droute<__nv_bfloat16, 32>(a, pl, w, stream);
    if (dp == 64) return launch_droute<__nv_bfloat16, 64>(a, pl, w, stream);
    return launch_droute<__nv_bfloat16, 128>(a, pl, w, stream);
  }
  if (dp == 32) return launch_droute<__half, 32>(a, pl, w, stream);
  if (dp == 64) return launch_droute<__half, 64>(a, pl, w, stream);
  return launch_droute<__half, 128>(a, pl, w, stream);
}

}  // namespace bb
