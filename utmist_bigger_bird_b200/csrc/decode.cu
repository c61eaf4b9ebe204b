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
// Keys and values are read in place from the cache (any head/row strides, rows 16-byte aligned):
// each cache row is one bulk copy (cp.async.bulk, d * 2 bytes) into a padded shared-memory row,
// completing on the stage's mbarrier, so gathering routed rows costs one instruction a row. The
// cache length can come from a device int64 (`n_dev`), so a captured CUDA graph stays valid as
// the cache grows inside a fixed-capacity buffer. All of it is bound by HBM (each cache row is read
// once per route group); the dot products run on the tensor cores (mma.sync m16n8k16, the group's
// query heads as the 16 rows), so the instruction stream stays far below the copy time. Every
// wait on a stage is bounded (about 2 s): a CTA that gives up records a fault code (40, 41) for
// bb_device_fault, drains its copies in flight and returns.
#include <algorithm>
#include <climits>

#include "tc_common.cuh"

namespace bb {

int topk_sorted(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                void* scratch, size_t scratch_bytes, cudaStream_t stream);
size_t topk_scratch_bytes(int64_t rows, int64_t n, int64_t k);

namespace {

constexpr int DK_THREADS = 128;  // 4 warps
constexpr int DK_WARPS = 4;
constexpr int DK_BN = 64;        // keys per stage: 16 per warp
constexpr int DK_NST = 3;        // stages in the ring (two in flight while one is used); 2 CTAs a SM
constexpr int DK_MAXROWS = 16;   // query heads per route group: one m16 tile
constexpr float LOG2E_F_DK = 1.4426950408889634f;

struct DecodeParams {
  const void* q; int64_t sq_h;
  const void* k; int64_t sk_h, sk_t;
  const void* v; int64_t sv_h, sv_t;
  const void* idx; int64_t si_r;  // [route rows][route_k], int32 or (idx64) int64
  int idx64;
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

// Shared-memory plan of one CTA: a ring of DK_NST stages of 64 K rows (and 64 V rows), padded to
// DP + 8 elements so that ldmatrix reads are free of bank conflicts; 16 query rows; 64 positions a
// stage. After the key loop the ring is reused for the cross-warp merge (m, l and O per warp).
template <int DP> struct DkSmem {
  static constexpr int LD = DP + 8;
  static constexpr size_t tile = (size_t)DK_BN * LD * 2;                  // one stage of K (or V)
  static constexpr size_t q_bytes = (size_t)DK_MAXROWS * LD * 2;
  static constexpr size_t pos_bytes = (size_t)DK_NST * DK_BN * 4 + DK_NST * 8 + 16;  // + full barriers, abort flag
  static constexpr size_t merge_bytes = (size_t)DK_WARPS * DK_MAXROWS * (DP + 2) * 4;
  static constexpr size_t ring(bool with_v) {
    return DK_NST * tile * (with_v ? 2 : 1) > merge_bytes ? DK_NST * tile * (with_v ? 2 : 1) : merge_bytes;
  }
  static constexpr size_t bytes(bool with_v) { return ring(with_v) + q_bytes + pos_bytes; }
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
  else {
    const int64_t o = r * p.si_r + (j - p.front - p.window);
    pos = p.idx64 ? static_cast<const int64_t*>(p.idx)[o] : (int64_t) static_cast<const int32_t*>(p.idx)[o];
  }
  return (pos >= 0 && pos < n) ? pos : -1;
}

// Row gather: thread t copies row t % 64 of the stage's K (t < 64) or V (t >= 64) with one bulk
// copy (d * 2 bytes) that completes on the stage's full barrier; a row that is not a key is
// zero-filled instead. Every thread arrives on the barrier once a stage (count DK_THREADS).
__device__ __forceinline__ void bulk_row(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
template <typename T>
__device__ __forceinline__ void stage_row(T* row, const T* src, bool valid, int64_t d, uint32_t bar) {
  if (valid) {
    tc::mbar_expect_tx(bar, (uint32_t)(d * 2));
    bulk_row(smem_u32(row), src, (uint32_t)(d * 2), bar);
  } else {
    for (int64_t c = 0; c < d; c += 8) *reinterpret_cast<uint4*>(row + c) = make_uint4(0u, 0u, 0u, 0u);
    // This thread's later bulk copies into the row (async proxy) must land after these stores.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::mbar_arrive(bar);
  }
}

// The query rows of a route group into shared memory (zero past `rows` and past d), as bf16/f16.
template <typename T, int DP>
__device__ __forceinline__ void load_q(const DecodeParams& p, int64_t first_head, int rows, T* qs) {
  constexpr int LD = DkSmem<DP>::LD;
  const T* Q = static_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < DK_MAXROWS * DP; i += DK_THREADS) {
    const int row = i / DP, c = i % DP;
    qs[row * LD + c] = (row < rows && c < p.d) ? Q[(first_head + row) * p.sq_h + c] : Elem<T>::from_f(0.f);
  }
}

// A fragments of the 16 x DP query tile (m16n8k16 row-major A).
template <typename T, int DP>
__device__ __forceinline__ void q_frags(const T* qs, uint32_t (&qf)[DP / 16][4]) {
  constexpr int LD = DkSmem<DP>::LD;
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int kk = 0; kk < DP / 16; ++kk)
    ldmatrix_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], smem_u32(qs + (lane % 16) * LD + kk * 16 + (lane / 16) * 8));
}

// S (16 rows x this warp's 16 keys) = Q K^T: two n8 tiles.
template <typename T, int DP>
__device__ __forceinline__ void warp_scores(const uint32_t (&qf)[DP / 16][4], const T* kb, int key0, float (&s)[2][4]) {
  constexpr int LD = DkSmem<DP>::LD;
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int t = 0; t < 2; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < DP / 16; ++kk) {
    uint32_t b0, b1, b2, b3;
    ldmatrix_x4(b0, b1, b2, b3, smem_u32(kb + (key0 + (lane / 16) * 8 + (lane % 8)) * LD + kk * 16 + ((lane / 8) % 2) * 8));
    const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
    mma_16816<T>(s[0], qf[kk], bA);
    mma_16816<T>(s[1], qf[kk], bB);
  }
}

// Split-K sparse decoding, one CTA per (route row, split). Each warp runs its own online softmax
// over 16 keys of every 64-key stage (S and P.V on mma.sync m16n8k16, rows = the group's query
// heads); the four warps' states are merged once at the end.
template <typename T, int DP>
__global__ void __launch_bounds__(DK_THREADS, 2) decode_partial_kernel(DecodeParams p) {
  using S = DkSmem<DP>;
  constexpr int LD = S::LD;
  extern __shared__ __align__(128) unsigned char smem[];
  T* ks = reinterpret_cast<T*>(smem);                        // [NST][64][LD]
  T* vs = ks + DK_NST * DK_BN * LD;                          // [NST][64][LD]
  constexpr size_t ring = S::ring(true);
  T* qs = reinterpret_cast<T*>(smem + ring);                 // [16][LD]
  int32_t* pos_s = reinterpret_cast<int32_t*>(smem + ring + S::q_bytes);  // [NST][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(pos_s + DK_NST * DK_BN);   // [NST]
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(full + DK_NST);
  const int64_t r = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int rows = (int)p.rows;
  const int64_t kv = (r * p.rows) / p.groups;
  const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
  const T* V = static_cast<const T*>(p.v) + kv * p.sv_h;
  const int64_t total = p.front + p.window + p.route_k;
  const int64_t j0 = split * p.split_len;
  const int64_t j1 = min(j0 + p.split_len, total);
  const int nblocks = j0 < j1 ? (int)cdiv(j1 - j0, (int64_t)DK_BN) : 0;
  if (p.d < DP)  // columns past d are never copied: keep them zero
    for (int i = threadIdx.x; i < (int)(2 * DK_NST * S::tile / 16); i += DK_THREADS)
      reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before any bulk copy into the ring
  load_q<T, DP>(p, r * p.rows, rows, qs);
  if (threadIdx.x == 0) {
    for (int i = 0; i < DK_NST; ++i) tc::mbar_init(smem_u32(full + i), DK_THREADS);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // Thread t moves row t % 64 of K (t < 64) or V (t >= 64); `pf` holds the position of its row in
  // the next stage to issue (looked up one stage early, so a route's index load is off the path).
  const int lrow = threadIdx.x % DK_BN;
  const bool is_k = threadIdx.x < DK_BN;
  const T* src_base = is_k ? K : V;
  const int64_t src_t = is_k ? p.sk_t : p.sv_t;
  T* dst_ring = is_k ? ks : vs;
  auto fetch = [&](int blk) -> int32_t {
    const int64_t j = j0 + (int64_t)blk * DK_BN + lrow;
    return (blk < nblocks && j < j1) ? (int32_t)virtual_pos(p, r, j, n) : -1;
  };
  auto issue = [&](int blk, int32_t pos) {
    if (blk >= nblocks) return;
    const int slot = blk % DK_NST;
    if (is_k) pos_s[slot * DK_BN + lrow] = pos;
    stage_row<T>(dst_ring + (slot * DK_BN + lrow) * LD, src_base + (int64_t)(pos < 0 ? 0 : pos) * src_t, pos >= 0,
                 p.d, smem_u32(full + slot));
  };
#pragma unroll 1
  for (int s = 0; s < DK_NST - 1; ++s) issue(s, fetch(s));
  int32_t pf = fetch(DK_NST - 1);
  uint32_t qf[DP / 16][4];
  q_frags<T, DP>(qs, qf);

  float o[DP / 8][4];
#pragma unroll
  for (int i = 0; i < DP / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -1.0e20f, m1 = -1.0e20f, l0 = 0.f, l1 = 0.f;
  const int key0 = warp * 16;
  const bool two = rows > 8;  // query rows 8..15 in use (c2/c3 of the fragments)
  int b = 0;
#pragma unroll 1
  for (; b < nblocks; ++b) {
    const int slot = b % DK_NST;
    const bool ok = tc::mbar_wait(smem_u32(full + slot), (uint32_t)((b / DK_NST) & 1), tc::Abort{abort_flag, 0u}, 40);
    if (!__syncthreads_and(ok)) break;  // stage b landed for all; stage b - 1 is free
    issue(b + DK_NST - 1, pf);
    pf = fetch(b + DK_NST);
    const T* kb = ks + slot * DK_BN * LD;
    const T* vb = vs + slot * DK_BN * LD;
    const int32_t* ps = pos_s + slot * DK_BN;
    float s[2][4];
    warp_scores<T, DP>(qf, kb, key0, s);
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int kk = key0 + t * 8 + 2 * (lane % 4);
      const bool v0 = ps[kk] >= 0, v1 = ps[kk + 1] >= 0;
      s[t][0] = v0 ? s[t][0] * p.scale_log2 : -INFINITY;
      s[t][1] = v1 ? s[t][1] * p.scale_log2 : -INFINITY;
      s[t][2] = v0 ? s[t][2] * p.scale_log2 : -INFINITY;
      s[t][3] = v1 ? s[t][3] * p.scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
      mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    const float n0 = fmaxf(m0, mx0);  // m starts at the -1e20 floor
    const float a0 = fast_exp2(m0 - n0);
    m0 = n0;
    float pr[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      pr[t][0] = fast_exp2(s[t][0] - n0);
      pr[t][1] = fast_exp2(s[t][1] - n0);
      pr[t][2] = pr[t][3] = 0.f;
    }
    float a1 = 1.f;
    if (two) {
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n1 = fmaxf(m1, mx1);
      a1 = fast_exp2(m1 - n1);
      m1 = n1;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        pr[t][2] = fast_exp2(s[t][2] - n1);
        pr[t][3] = fast_exp2(s[t][3] - n1);
      }
      l1 = l1 * a1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
    }
    // l from the unrounded probabilities (kernels/bigger_bird_decode.py:59); P.V with P rounded
    // to the cache dtype (:58), which the A fragment packing does.
    l0 = l0 * a0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
    const uint32_t a[4] = {pack2<T>(pr[0][0], pr[0][1]), pack2<T>(pr[0][2], pr[0][3]),
                           pack2<T>(pr[1][0], pr[1][1]), pack2<T>(pr[1][2], pr[1][3])};
    if (!__all_sync(0xffffffffu, a0 == 1.f && a1 == 1.f)) {  // running max moved: rescale O
#pragma unroll
      for (int i = 0; i < DP / 8; ++i) {
        o[i][0] *= a0;
        o[i][1] *= a0;
        o[i][2] *= a1;
        o[i][3] *= a1;
      }
    }
#pragma unroll
    for (int dp = 0; dp < DP / 16; ++dp) {
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3,
                        smem_u32(vb + (key0 + ((lane / 8) % 2) * 8 + (lane % 8)) * LD + dp * 16 + (lane / 16) * 8));
      const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
      mma_16816<T>(o[dp * 2], a, bA);
      mma_16816<T>(o[dp * 2 + 1], a, bB);
    }
  }
  if (b < nblocks) {
    // A wait gave up (fault recorded): let the copies still in flight land, then leave.
    for (int blk = b; blk < min(nblocks, b + DK_NST - 1); ++blk)
      tc::mbar_drain(smem_u32(full + blk % DK_NST), (uint32_t)((blk / DK_NST) & 1));
    return;
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  // Merge the four warps: [warp][row] m and l, then [warp][row][DP] O, in the ring's space.
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);
  float* wl = wm + DK_WARPS * DK_MAXROWS;
  float* wo = wl + DK_WARPS * DK_MAXROWS;
  const int g = lane / 4, c = 2 * (lane % 4);
  if (lane % 4 == 0) {
    wm[warp * DK_MAXROWS + g] = m0;
    wl[warp * DK_MAXROWS + g] = l0;
    wm[warp * DK_MAXROWS + g + 8] = m1;
    wl[warp * DK_MAXROWS + g + 8] = l1;
  }
#pragma unroll
  for (int i = 0; i < DP / 8; ++i) {
    *reinterpret_cast<float2*>(wo + (warp * DK_MAXROWS + g) * DP + i * 8 + c) = make_float2(o[i][0], o[i][1]);
    *reinterpret_cast<float2*>(wo + (warp * DK_MAXROWS + g + 8) * DP + i * 8 + c) = make_float2(o[i][2], o[i][3]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * DP; i += DK_THREADS) {
    const int row = i / DP, col = i % DP;
    float M = -1.0e20f;
#pragma unroll
    for (int w = 0; w < DK_WARPS; ++w) M = fmaxf(M, wm[w * DK_MAXROWS + row]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < DK_WARPS; ++w) {
      const float f = fast_exp2(wm[w * DK_MAXROWS + row] - M);
      L += wl[w * DK_MAXROWS + row] * f;
      A += wo[(w * DK_MAXROWS + row) * DP + col] * f;
    }
    const int64_t at = (r * p.splits + split) * p.rows + row;
    if (col == 0) {
      p.part_m[at] = M;
      p.part_l[at] = L;
    }
    if (col < p.d) p.part_acc[at * p.d + col] = A;
  }
}

// One CTA per query head merges its splits: w_s = exp2(m_s - max m), out = sum w_s acc_s / sum w_s l_s.
template <typename T>
__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeParams p) {
  extern __shared__ float wsm[];  // [splits] weights, then [splits] l
  __shared__ float red[4];
  __shared__ float4 part[4][32];   // per warp: its splits' share of the 128 columns
  const int64_t h = blockIdx.x;
  const int64_t r = h / p.rows, row = h % p.rows;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int S = (int)p.splits;
  float* lsm = wsm + S;
  auto at = [&](int s) { return (r * p.splits + s) * p.rows + row; };
  // m and l of every split in one round of loads
  float M = -INFINITY;
  for (int s = threadIdx.x; s < S; s += 128) {
    const float m = p.part_m[at(s)];
    wsm[s] = m;
    lsm[s] = p.part_l[at(s)];
    M = fmaxf(M, m);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  float L = 0.f;
  for (int s = threadIdx.x; s < S; s += 128) {
    const float w = fast_exp2(wsm[s] - M);
    wsm[s] = w;
    L += lsm[s] * w;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  __syncthreads();
  L = (red[0] + red[1]) + (red[2] + red[3]);
  // Warp w sums splits w, w + 4, ...; lane holds 4 columns (16-byte loads, independent of each other).
  const bool live = 4 * lane < p.d;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (live) {
#pragma unroll 4
    for (int sp = warp; sp < S; sp += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p.part_acc + at(sp) * p.d + 4 * lane);
      const float wv = wsm[sp];
      acc.x += v.x * wv;
      acc.y += v.y * wv;
      acc.z += v.z * wv;
      acc.w += v.w * wv;
    }
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && live) {
    const float4 a0 = part[0][lane], a1 = part[1][lane], a2 = part[2][lane], a3 = part[3][lane];
    T* o = static_cast<T*>(p.out) + h * p.so_h + 4 * lane;
    o[0] = Elem<T>::from_f(((a0.x + a1.x) + (a2.x + a3.x)) / L);
    o[1] = Elem<T>::from_f(((a0.y + a1.y) + (a2.y + a3.y)) / L);
    o[2] = Elem<T>::from_f(((a0.z + a1.z) + (a2.z + a3.z)) / L);
    o[3] = Elem<T>::from_f(((a0.w + a1.w) + (a2.w + a3.w)) / L);
  }
}

// Decode routing pass 1: one CTA per (KV head, chunk of contiguous cached keys). Scores of the
// group's query heads on mma.sync, stored log2-scaled, plus the chunk's softmax statistics.
template <typename T, int DP>
__global__ void __launch_bounds__(DK_THREADS) droute_scores_kernel(DecodeParams p) {
  using S = DkSmem<DP>;
  constexpr int LD = S::LD;
  extern __shared__ __align__(128) unsigned char smem[];
  T* ks = reinterpret_cast<T*>(smem);  // [NST][64][LD]
  constexpr size_t ring = S::ring(false);
  T* qs = reinterpret_cast<T*>(smem + ring);
  int32_t* pos_s = reinterpret_cast<int32_t*>(smem + ring + S::q_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(pos_s + DK_NST * DK_BN);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(full + DK_NST);
  const int64_t kv = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int rows = (int)p.groups;
  const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
  const int64_t j0 = split * p.split_len;
  const int64_t j1 = min(j0 + p.split_len, n);
  const int nblocks = j0 < j1 ? (int)cdiv(j1 - j0, (int64_t)DK_BN) : 0;
  if (p.d < DP)
    for (int i = threadIdx.x; i < (int)(DK_NST * S::tile / 16); i += DK_THREADS)
      reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before any bulk copy into the ring
  load_q<T, DP>(p, kv * p.groups, rows, qs);
  if (threadIdx.x == 0) {
    for (int i = 0; i < DK_NST; ++i) tc::mbar_init(smem_u32(full + i), DK_THREADS);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int lrow = threadIdx.x % DK_BN;
  const bool loader = threadIdx.x < DK_BN;
  auto issue = [&](int blk) {
    if (blk >= nblocks) return;
    const int slot = blk % DK_NST;
    if (!loader) {
      tc::mbar_arrive(smem_u32(full + slot));
      return;
    }
    const int64_t j = j0 + (int64_t)blk * DK_BN + lrow;
    const int32_t pos = j < j1 ? (int32_t)j : -1;
    pos_s[slot * DK_BN + lrow] = pos;
    stage_row<T>(ks + (slot * DK_BN + lrow) * LD, K + (int64_t)(pos < 0 ? 0 : pos) * p.sk_t, pos >= 0, p.d,
                 smem_u32(full + slot));
  };
#pragma unroll 1
  for (int s = 0; s < DK_NST - 1; ++s) issue(s);
  uint32_t qf[DP / 16][4];
  q_frags<T, DP>(qs, qf);
  float m0 = -1.0e20f, m1 = -1.0e20f, l0 = 0.f, l1 = 0.f;
  const int key0 = warp * 16;
  const int g = lane / 4, c = 2 * (lane % 4);
  const bool two = rows > 8;
  float* srow0 = p.scores + (kv * p.groups + g) * p.cap;
  float* srow1 = p.scores + (kv * p.groups + (two ? g + 8 : g)) * p.cap;
  int b = 0;
#pragma unroll 1
  for (; b < nblocks; ++b) {
    const int slot = b % DK_NST;
    const bool ok = tc::mbar_wait(smem_u32(full + slot), (uint32_t)((b / DK_NST) & 1), tc::Abort{abort_flag, 0u}, 41);
    if (!__syncthreads_and(ok)) break;
    issue(b + DK_NST - 1);
    const int32_t* ps = pos_s + slot * DK_BN;
    float s[2][4];
    warp_scores<T, DP>(qf, ks + slot * DK_BN * LD, key0, s);
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int kk = key0 + t * 8 + c;
      const int32_t q0 = ps[kk], q1 = ps[kk + 1];
      s[t][0] = q0 >= 0 ? s[t][0] * p.scale_log2 : -INFINITY;
      s[t][1] = q1 >= 0 ? s[t][1] * p.scale_log2 : -INFINITY;
      s[t][2] = q0 >= 0 ? s[t][2] * p.scale_log2 : -INFINITY;
      s[t][3] = q1 >= 0 ? s[t][3] * p.scale_log2 : -INFINITY;
      if (g < rows) {
        if (q0 >= 0) srow0[q0] = s[t][0];
        if (q1 >= 0) srow0[q1] = s[t][1];
      }
      if (two && g + 8 < rows) {
        if (q0 >= 0) srow1[q0] = s[t][2];
        if (q1 >= 0) srow1[q1] = s[t][3];
      }
      mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
      mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    const float n0 = fmaxf(m0, mx0);
    l0 = l0 * fast_exp2(m0 - n0) + (fast_exp2(s[0][0] - n0) + fast_exp2(s[0][1] - n0)) +
         (fast_exp2(s[1][0] - n0) + fast_exp2(s[1][1] - n0));
    m0 = n0;
    if (two) {
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n1 = fmaxf(m1, mx1);
      l1 = l1 * fast_exp2(m1 - n1) + (fast_exp2(s[0][2] - n1) + fast_exp2(s[0][3] - n1)) +
           (fast_exp2(s[1][2] - n1) + fast_exp2(s[1][3] - n1));
      m1 = n1;
    }
  }
  if (b < nblocks) {
    for (int blk = b; blk < min(nblocks, b + DK_NST - 1); ++blk)
      tc::mbar_drain(smem_u32(full + blk % DK_NST), (uint32_t)((blk / DK_NST) & 1));
    return;
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);
  float* wl = wm + DK_WARPS * DK_MAXROWS;
  if (lane % 4 == 0) {
    wm[warp * DK_MAXROWS + g] = m0;
    wl[warp * DK_MAXROWS + g] = l0;
    wm[warp * DK_MAXROWS + g + 8] = m1;
    wl[warp * DK_MAXROWS + g + 8] = l1;
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    const int row = threadIdx.x;
    float M = -1.0e20f;
#pragma unroll
    for (int w = 0; w < DK_WARPS; ++w) M = fmaxf(M, wm[w * DK_MAXROWS + row]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < DK_WARPS; ++w) L += wl[w * DK_MAXROWS + row] * fast_exp2(wm[w * DK_MAXROWS + row] - M);
    const int64_t at = (kv * p.splits + split) * p.groups + row;
    p.part_m[at] = M;
    p.part_l[at] = L;
  }
}

// Decode routing pass 2: grid (kv_heads, cdiv(cap, 1024)); four positions a thread. The group's
// merged statistics come first, 16 threads a query head.
__global__ void __launch_bounds__(256) droute_pool_kernel(DecodeParams p) {
  const int64_t kv = blockIdx.x;
  const int64_t n = cache_len(p);
  __shared__ float sm[DK_MAXROWS], sinv[DK_MAXROWS];
  {
    const int row = threadIdx.x / 16, sub = threadIdx.x % 16;
    const bool live = row < p.groups;
    float M = -1.0e20f;
    if (live)
      for (int64_t s = sub; s < p.splits; s += 16) M = fmaxf(M, p.part_m[(kv * p.splits + s) * p.groups + row]);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    if (live)
      for (int64_t s = sub; s < p.splits; s += 16) {
        const int64_t at = (kv * p.splits + s) * p.groups + row;
        L += p.part_l[at] * fast_exp2(p.part_m[at] - M);
      }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (live && sub == 0) {
      sm[row] = M;
      sinv[row] = 1.f / fmaxf(L, 1.0e-30f);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t pos = (int64_t)blockIdx.y * 1024 + i * 256 + threadIdx.x;
    if (pos >= p.cap) break;
    float acc = 0.f;
    if (pos < n)
      for (int64_t row = 0; row < p.groups; ++row)
        acc += fast_exp2(p.scores[(kv * p.groups + row) * p.cap + pos] - sm[row]) * sinv[row];
    const bool keep = pos >= p.front && pos < n - p.window;
    p.probs[kv * p.cap + pos] = keep ? acc / (float)p.groups : -1.f;
  }
}

// ----------------------------------------------------------------------------- TMA variant
// Head dim 128 with each head's cache rows evenly strided (the [Hkv, cap, d] layout of a KV
// cache): a producer warp fills each 64-key stage either with four tiled TMA loads (K and V x two
// 64-column halves, 128-byte swizzle) when the stage's 64 positions are consecutive cache rows
// (front, window and dense stages), or with cp.async 16-byte chunks into the same swizzled
// layout (stages with routed or missing keys). Split s takes stages s, s + S, s + 2S, ... of the
// virtual key list (S splits), so the few routed stages spread over many CTAs instead of lining up
// in the last one. Four consumer warps compute as in the generic kernel on the swizzled tiles.
constexpr int DT_CONSUMERS = 4;
constexpr int DT_THREADS = 32 * (DT_CONSUMERS + 1);
constexpr int DT_NST = 3;
constexpr uint32_t DT_HALF = 64u * 128u;   // 64 rows x 128 bytes: one 64-column half
constexpr uint32_t DT_TILE = 2u * DT_HALF;  // 64 rows x 128 columns of K (or V)
constexpr int DT_LDQ = 136;                 // padded query rows (elements)

struct DtMaps {
  CUtensorMap k, v;           // 2-D row views [rows, 128]; head h starts at row h * head_rows
  int64_t k_head_rows, v_head_rows;
};

struct DtSmem {
  static constexpr uint32_t ring(bool with_v) { return DT_NST * DT_TILE * (with_v ? 2u : 1u); }
  static constexpr uint32_t merge = DT_CONSUMERS * DK_MAXROWS * (128 + 2) * 4;
  static constexpr uint32_t area(bool with_v) { return ring(with_v) > merge ? ring(with_v) : merge; }
  static constexpr uint32_t q_bytes = DK_MAXROWS * DT_LDQ * 2;
  static constexpr uint32_t ctl = DT_NST * 8 * 3 + 16;
  static constexpr size_t bytes(bool with_v) { return (size_t)area(with_v) + q_bytes + ctl + 1024; }  // + alignment
};

template <typename T> __device__ __forceinline__ void zero_row(T* row, int64_t d) {
  for (int64_t c = 0; c < d; c += 8) *reinterpret_cast<uint4*>(row + c) = make_uint4(0u, 0u, 0u, 0u);
}

__device__ __forceinline__ uint32_t sw_addr(uint32_t tile, int row, int chunk) {
  return tile + (uint32_t)(chunk >> 3) * DT_HALF + (uint32_t)row * 128u + ((uint32_t)((chunk & 7) ^ (row & 7)) << 4);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}

// One stage: positions p0 / p1 of rows `lane` / `lane + 32` (-1: not a key). A stage of 64
// consecutive cache rows is two (K) or four (K and V) tiled TMA loads; any other stage (routed
// keys, the cache's edges) is cp.async 16-byte chunks into the same 128B-swizzled layout, rows that
// are not keys zero-filled, completion through cp.async.mbarrier.arrive. The stage's full barrier
// expects 33 arrivals: every producer lane once, plus lane 0 once more after it has published the
// key mask (a release the consumers' wait acquires).
template <typename T>
__device__ __forceinline__ void dt_produce(uint64_t* mask_slot, uint32_t bar, int32_t p0, int32_t p1,
                                           const CUtensorMap* mk, const CUtensorMap* mv, int64_t k_row0,
                                           int64_t v_row0, const T* K, int64_t sk_t, const T* V, int64_t sv_t,
                                           uint32_t ktile, uint32_t vtile) {
  const int lane = threadIdx.x % 32;
  const unsigned m0 = __ballot_sync(0xffffffffu, p0 >= 0), m1 = __ballot_sync(0xffffffffu, p1 >= 0);
  const int32_t first = __shfl_sync(0xffffffffu, p0, 0);
  const bool contiguous =
      __all_sync(0xffffffffu, p0 >= 0 && p1 >= 0 && p0 == first + lane && p1 == first + 32 + lane);
  if (lane == 0) *mask_slot = ((uint64_t)m1 << 32) | m0;
  if (contiguous) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier cp.async fills of the slot first
    __syncwarp();
    if (lane == 0) {
      tc::mbar_expect_tx(bar, mv ? 2u * DT_TILE : DT_TILE);
      tma_load_2d(ktile, mk, 0, (int)(k_row0 + first), bar);
      tma_load_2d(ktile + DT_HALF, mk, 64, (int)(k_row0 + first), bar);
      if (mv) {
        tma_load_2d(vtile, mv, 0, (int)(v_row0 + first), bar);
        tma_load_2d(vtile + DT_HALF, mv, 64, (int)(v_row0 + first), bar);
      }
    }
    tc::mbar_arrive(bar);
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = lane + 32 * h;
      const int32_t pos = h ? p1 : p0;
      const bool ok = pos >= 0;
      const T* kr = K + (int64_t)(ok ? pos : 0) * sk_t;
      const T* vr = mv ? V + (int64_t)(ok ? pos : 0) * sv_t : nullptr;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        cp_async_16(sw_addr(ktile, row, c), kr + c * 8, ok);
        if (vr) cp_async_16(sw_addr(vtile, row, c), vr + c * 8, ok);
      }
    }
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
    if (lane == 0) tc::mbar_arrive(bar);
  }
}

// S = Q K^T for this warp's 16 keys of a swizzled K tile (two accumulator chains, as warp_scores).
template <typename T>
__device__ __forceinline__ void dt_scores(const uint32_t (&qf)[8][4], uint32_t kt, int key0, float (&s)[2][4]) {
  const int lane = threadIdx.x % 32;
  float e[2][4], o[2][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) e[t][i] = o[t][i] = 0.f;
  const int row = key0 + (lane / 16) * 8 + (lane % 8);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    uint32_t b0, b1, b2, b3;
    ldmatrix_x4(b0, b1, b2, b3, sw_addr(kt, row, kk * 2 + (lane / 8) % 2));
    const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
    float(&a0)[4] = (kk & 1) ? o[0] : e[0];
    float(&a1)[4] = (kk & 1) ? o[1] : e[1];
    mma_16816<T>(a0, qf[kk], bA);
    mma_16816<T>(a1, qf[kk], bB);
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[t][i] = e[t][i] + o[t][i];
}

struct DtCtl {
  uint64_t* mask;
  uint64_t* full;
  uint64_t* empty;
  volatile uint32_t* abort_flag;
};

template <typename T>
__device__ __forceinline__ void dt_setup(unsigned char* smem_raw, bool with_v, uint32_t& ring, T*& qs, DtCtl& c) {
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;  // the swizzled TMA tiles need 1024-byte alignment
  unsigned char* base = smem_raw + pad;
  ring = raw + pad;
  qs = reinterpret_cast<T*>(base + DtSmem::area(with_v));
  unsigned char* ctl = base + DtSmem::area(with_v) + DtSmem::q_bytes;
  c.mask = reinterpret_cast<uint64_t*>(ctl);
  c.full = c.mask + DT_NST;
  c.empty = c.full + DT_NST;
  c.abort_flag = reinterpret_cast<volatile uint32_t*>(c.empty + DT_NST);
  if (threadIdx.x == 0) {
    for (int i = 0; i < DT_NST; ++i) {
      tc::mbar_init(smem_u32(c.full + i), 33);
      tc::mbar_init(smem_u32(c.empty + i), DT_CONSUMERS);
    }
    *c.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
}

template <typename T>
__device__ __forceinline__ void dt_load_q(const DecodeParams& p, int64_t first_head, int rows, T* qs) {
  const T* Q = static_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < DK_MAXROWS * 128; i += DT_THREADS) {
    const int row = i / 128, col = i % 128;
    qs[row * DT_LDQ + col] = row < rows ? Q[(first_head + row) * p.sq_h + col] : Elem<T>::from_f(0.f);
  }
}

template <typename T>
__device__ __forceinline__ void dt_q_frags(const T* qs, uint32_t (&qf)[8][4]) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    ldmatrix_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3],
                smem_u32(qs + (lane % 16) * DT_LDQ + kk * 16 + (lane / 16) * 8));
}

template <typename T>
__global__ void __launch_bounds__(DT_THREADS, 2) decode_tma_kernel(const __grid_constant__ DtMaps maps, DecodeParams p) {
  extern __shared__ unsigned char smem_raw[];
  uint32_t ring;
  T* qs;
  DtCtl c;
  dt_setup<T>(smem_raw, true, ring, qs, c);
  const int64_t r = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int rows = (int)p.rows;
  const int64_t kv = (r * p.rows) / p.groups;
  const int64_t total = p.front + p.window + p.route_k;
  const int64_t stages = cdiv(total, (int64_t)DK_BN);
  const int nblocks = split < stages ? (int)cdiv(stages - split, p.splits) : 0;  // stages split + i * splits
  dt_load_q<T>(p, r * p.rows, rows, qs);
  __syncthreads();

  float o[16][4];
  float m0 = -1.0e20f, m1 = -1.0e20f, l0 = 0.f, l1 = 0.f;
  if (warp == DT_CONSUMERS) {
    const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
    const T* V = static_cast<const T*>(p.v) + kv * p.sv_h;
    auto fetch = [&](int blk, int row) -> int32_t {
      const int64_t j = (split + (int64_t)blk * p.splits) * DK_BN + row;
      return (blk < nblocks && j < total) ? (int32_t)virtual_pos(p, r, j, n) : -1;
    };
    int32_t f0 = fetch(0, lane), f1 = fetch(0, lane + 32);
    int slot = 0;
    uint32_t ph = 0;
    for (int blk = 0; blk < nblocks; ++blk) {
      if (blk >= DT_NST && !tc::mbar_wait_warp(smem_u32(c.empty + slot), ph ^ 1u, tc::Abort{c.abort_flag, 0u}, 44)) break;
      const int32_t p0 = f0, p1 = f1;
      f0 = fetch(blk + 1, lane);
      f1 = fetch(blk + 1, lane + 32);
      const uint32_t off = (uint32_t)slot * 2u * DT_TILE;
      dt_produce<T>(c.mask + slot, smem_u32(c.full + slot), p0, p1, &maps.k, &maps.v, kv * maps.k_head_rows,
                    kv * maps.v_head_rows, K, p.sk_t, V, p.sv_t, ring + off, ring + off + DT_TILE);
      if (++slot == DT_NST) {
        slot = 0;
        ph ^= 1u;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    uint32_t qf[8][4];
    dt_q_frags<T>(qs, qf);
    const int key0 = warp * 16;
    const bool two = rows > 8;
    const int kbit = key0 + 2 * (lane % 4);
    const int vrow = key0 + ((lane / 8) % 2) * 8 + (lane % 8);
    int slot = 0;
    uint32_t ph = 0;
    for (int b = 0; b < nblocks; ++b) {
      if (!tc::mbar_wait_warp(smem_u32(c.full + slot), ph, tc::Abort{c.abort_flag, 0u}, 45)) break;
      const uint64_t msk = c.mask[slot];
      const uint32_t kt = ring + (uint32_t)slot * 2u * DT_TILE, vt = kt + DT_TILE;
      float s[2][4];
      dt_scores<T>(qf, kt, key0, s);
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const bool v0 = (msk >> (kbit + t * 8)) & 1u, v1 = (msk >> (kbit + t * 8 + 1)) & 1u;
        s[t][0] = v0 ? s[t][0] * p.scale_log2 : -INFINITY;
        s[t][1] = v1 ? s[t][1] * p.scale_log2 : -INFINITY;
        s[t][2] = v0 ? s[t][2] * p.scale_log2 : -INFINITY;
        s[t][3] = v1 ? s[t][3] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
        mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      const float n0 = fmaxf(m0, mx0);
      const float a0 = fast_exp2(m0 - n0);
      m0 = n0;
      float pr[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        pr[t][0] = fast_exp2(s[t][0] - n0);
        pr[t][1] = fast_exp2(s[t][1] - n0);
        pr[t][2] = pr[t][3] = 0.f;
      }
      float a1 = 1.f;
      if (two) {
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float n1 = fmaxf(m1, mx1);
        a1 = fast_exp2(m1 - n1);
        m1 = n1;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          pr[t][2] = fast_exp2(s[t][2] - n1);
          pr[t][3] = fast_exp2(s[t][3] - n1);
        }
        l1 = l1 * a1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
      }
      l0 = l0 * a0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
      const uint32_t a[4] = {pack2<T>(pr[0][0], pr[0][1]), pack2<T>(pr[0][2], pr[0][3]),
                             pack2<T>(pr[1][0], pr[1][1]), pack2<T>(pr[1][2], pr[1][3])};
      if (!__all_sync(0xffffffffu, a0 == 1.f && a1 == 1.f)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i][0] *= a0;
          o[i][1] *= a0;
          o[i][2] *= a1;
          o[i][3] *= a1;
        }
      }
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, sw_addr(vt, vrow, dp * 2 + lane / 16));
        const uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
        mma_16816<T>(o[dp * 2], a, bA);
        mma_16816<T>(o[dp * 2 + 1], a, bB);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(c.empty + slot));
      if (++slot == DT_NST) {
        slot = 0;
        ph ^= 1u;
      }
    }
  }
  __syncthreads();
  if (*c.abort_flag) {
    if (warp == DT_CONSUMERS && lane == 0)
      for (int blk = max(0, nblocks - DT_NST); blk < nblocks; ++blk)
        tc::mbar_drain(smem_u32(c.full + blk % DT_NST), (uint32_t)((blk / DT_NST) & 1));
    return;
  }
  const uint32_t pad = ring - smem_u32(smem_raw);
  float* wm = reinterpret_cast<float*>(smem_raw + pad);
  float* wl = wm + DT_CONSUMERS * DK_MAXROWS;
  float* wo = wl + DT_CONSUMERS * DK_MAXROWS;
  if (warp < DT_CONSUMERS) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const int g = lane / 4, cc = 2 * (lane % 4);
    if (lane % 4 == 0) {
      wm[warp * DK_MAXROWS + g] = m0;
      wl[warp * DK_MAXROWS + g] = l0;
      wm[warp * DK_MAXROWS + g + 8] = m1;
      wl[warp * DK_MAXROWS + g + 8] = l1;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      *reinterpret_cast<float2*>(wo + (warp * DK_MAXROWS + g) * 128 + i * 8 + cc) = make_float2(o[i][0], o[i][1]);
      *reinterpret_cast<float2*>(wo + (warp * DK_MAXROWS + g + 8) * 128 + i * 8 + cc) = make_float2(o[i][2], o[i][3]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * 128; i += DT_THREADS) {
    const int row = i / 128, col = i % 128;
    float M = -1.0e20f;
#pragma unroll
    for (int w = 0; w < DT_CONSUMERS; ++w) M = fmaxf(M, wm[w * DK_MAXROWS + row]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < DT_CONSUMERS; ++w) {
      const float f = fast_exp2(wm[w * DK_MAXROWS + row] - M);
      L += wl[w * DK_MAXROWS + row] * f;
      A += wo[(w * DK_MAXROWS + row) * 128 + col] * f;
    }
    const int64_t at = (r * p.splits + split) * p.rows + row;
    if (col == 0) {
      p.part_m[at] = M;
      p.part_l[at] = L;
    }
    p.part_acc[at * 128 + col] = A;
  }
}

// Decode routing pass 1 on the TMA path: K stages only (contiguous positions, so every full stage
// is one pair of tiled loads).
template <typename T>
__global__ void __launch_bounds__(DT_THREADS) droute_tma_kernel(const __grid_constant__ DtMaps maps, DecodeParams p) {
  extern __shared__ unsigned char smem_raw[];
  uint32_t ring;
  T* qs;
  DtCtl c;
  dt_setup<T>(smem_raw, false, ring, qs, c);
  const int64_t kv = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n = cache_len(p);
  const int rows = (int)p.groups;
  const int64_t j0 = split * p.split_len;
  const int64_t j1 = min(j0 + p.split_len, n);
  const int nblocks = j0 < j1 ? (int)cdiv(j1 - j0, (int64_t)DK_BN) : 0;
  dt_load_q<T>(p, kv * p.groups, rows, qs);
  __syncthreads();
  float m0 = -1.0e20f, m1 = -1.0e20f, l0 = 0.f, l1 = 0.f;
  if (warp == DT_CONSUMERS) {
    const T* K = static_cast<const T*>(p.k) + kv * p.sk_h;
    int slot = 0;
    uint32_t ph = 0;
    for (int blk = 0; blk < nblocks; ++blk) {
      if (blk >= DT_NST && !tc::mbar_wait_warp(smem_u32(c.empty + slot), ph ^ 1u, tc::Abort{c.abort_flag, 0u}, 46)) break;
      const int64_t j = j0 + (int64_t)blk * DK_BN + lane;
      dt_produce<T>(c.mask + slot, smem_u32(c.full + slot), j < j1 ? (int32_t)j : -1,
                    j + 32 < j1 ? (int32_t)(j + 32) : -1, &maps.k, nullptr, kv * maps.k_head_rows, 0, K, p.sk_t,
                    static_cast<const T*>(nullptr), 0, ring + (uint32_t)slot * DT_TILE, 0u);
      if (++slot == DT_NST) {
        slot = 0;
        ph ^= 1u;
      }
    }
  } else {
    uint32_t qf[8][4];
    dt_q_frags<T>(qs, qf);
    const int key0 = warp * 16;
    const int g = lane / 4, cc = 2 * (lane % 4);
    const bool two = rows > 8;
    float* srow0 = p.scores + (kv * p.groups + g) * p.cap;
    float* srow1 = p.scores + (kv * p.groups + (two ? g + 8 : g)) * p.cap;
    int slot = 0;
    uint32_t ph = 0;
    for (int b = 0; b < nblocks; ++b) {
      if (!tc::mbar_wait_warp(smem_u32(c.full + slot), ph, tc::Abort{c.abort_flag, 0u}, 47)) break;
      const uint64_t msk = c.mask[slot];
      const int64_t jb = j0 + (int64_t)b * DK_BN;
      float s[2][4];
      dt_scores<T>(qf, ring + (uint32_t)slot * DT_TILE, key0, s);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(c.empty + slot));
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int kk = key0 + t * 8 + cc;
        const bool v0 = (msk >> kk) & 1u, v1 = (msk >> (kk + 1)) & 1u;
        s[t][0] = v0 ? s[t][0] * p.scale_log2 : -INFINITY;
        s[t][1] = v1 ? s[t][1] * p.scale_log2 : -INFINITY;
        s[t][2] = v0 ? s[t][2] * p.scale_log2 : -INFINITY;
        s[t][3] = v1 ? s[t][3] * p.scale_log2 : -INFINITY;
        if (g < rows) {
          if (v0) srow0[jb + kk] = s[t][0];
          if (v1) srow0[jb + kk + 1] = s[t][1];
        }
        if (two && g + 8 < rows) {
          if (v0) srow1[jb + kk] = s[t][2];
          if (v1) srow1[jb + kk + 1] = s[t][3];
        }
        mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
        mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      const float n0 = fmaxf(m0, mx0);
      l0 = l0 * fast_exp2(m0 - n0) + (fast_exp2(s[0][0] - n0) + fast_exp2(s[0][1] - n0)) +
           (fast_exp2(s[1][0] - n0) + fast_exp2(s[1][1] - n0));
      m0 = n0;
      if (two) {
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float n1 = fmaxf(m1, mx1);
        l1 = l1 * fast_exp2(m1 - n1) + (fast_exp2(s[0][2] - n1) + fast_exp2(s[0][3] - n1)) +
             (fast_exp2(s[1][2] - n1) + fast_exp2(s[1][3] - n1));
        m1 = n1;
      }
      if (++slot == DT_NST) {
        slot = 0;
        ph ^= 1u;
      }
    }
  }
  __syncthreads();
  if (*c.abort_flag) {
    if (warp == DT_CONSUMERS && lane == 0)
      for (int blk = max(0, nblocks - DT_NST); blk < nblocks; ++blk)
        tc::mbar_drain(smem_u32(c.full + blk % DT_NST), (uint32_t)((blk / DT_NST) & 1));
    return;
  }
  const uint32_t pad = ring - smem_u32(smem_raw);
  float* wm = reinterpret_cast<float*>(smem_raw + pad);
  float* wl = wm + DT_CONSUMERS * DK_MAXROWS;
  if (warp < DT_CONSUMERS) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const int g = lane / 4;
    if (lane % 4 == 0) {
      wm[warp * DK_MAXROWS + g] = m0;
      wl[warp * DK_MAXROWS + g] = l0;
      wm[warp * DK_MAXROWS + g + 8] = m1;
      wl[warp * DK_MAXROWS + g + 8] = l1;
    }
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    const int row = threadIdx.x;
    float M = -1.0e20f;
#pragma unroll
    for (int w = 0; w < DT_CONSUMERS; ++w) M = fmaxf(M, wm[w * DK_MAXROWS + row]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < DT_CONSUMERS; ++w) L += wl[w * DK_MAXROWS + row] * fast_exp2(wm[w * DK_MAXROWS + row] - M);
    const int64_t at = (kv * p.splits + split) * p.groups + row;
    p.part_m[at] = M;
    p.part_l[at] = L;
  }
}

struct DecodePlan {
  int64_t splits, split_len;
  size_t m_bytes, l_bytes, acc_bytes, total;
};

int dpad(int64_t d) { return d <= 32 ? 32 : (d <= 64 ? 64 : 128); }

size_t dk_smem(int dp, bool with_v) {
  return dp == 32 ? DkSmem<32>::bytes(with_v) : (dp == 64 ? DkSmem<64>::bytes(with_v) : DkSmem<128>::bytes(with_v));
}

// Splits that fill the GPU in one wave: resident CTAs a SM (from shared memory) x SMs, over the
// CTAs a split count multiplies (route rows); at least two stages of keys a split, at most 8192.
int64_t auto_splits(int64_t keys, int64_t ctas_per_split, size_t smem) {
  const int64_t per_sm = std::max<int64_t>(1, std::min<int64_t>(8, (int64_t)(233472 / (smem + 1024))));
  const int64_t wave = std::max<int64_t>(1, per_sm * num_sms() / ctas_per_split);
  return std::max<int64_t>(1, std::min<int64_t>({cdiv(keys, (int64_t)2 * DK_BN), wave, (int64_t)8192}));
}

// The TMA path: head_dim 128, fp16/bf16, each head's rows on one stride (s_t >= 128 elements)
// and heads a whole number of rows apart, so that a 2-D [rows, 128] view covers the cache.
bool dt_layout_ok(int64_t kv_heads, int64_t cap, int64_t s_h, int64_t s_t) {
  if (s_t < 128 || (s_t * 2) % 16) return false;
  if (kv_heads > 1 && (s_h <= 0 || s_h % s_t)) return false;
  const int64_t head_rows = kv_heads > 1 ? s_h / s_t : 0;
  return (kv_heads - 1) * head_rows + cap < ((int64_t)1 << 31);
}
bool dt_usable(const bb_decode_args* a, bool need_v) {
  return a->d == 128 && (a->dtype == BB_BF16 || a->dtype == BB_F16) && tc::encode_fn() != nullptr &&
         dt_layout_ok(a->kv_heads, a->cap, a->sk_h, a->sk_t) &&
         (!need_v || dt_layout_ok(a->kv_heads, a->cap, a->sv_h, a->sv_t));
}
int dt_map(CUtensorMap* m, int64_t* head_rows, const void* base, int dtype, int64_t kv_heads, int64_t cap,
           int64_t s_h, int64_t s_t) {
  auto fn = tc::encode_fn();
  *head_rows = kv_heads > 1 ? s_h / s_t : 0;
  cuuint64_t dims[2] = {128, (cuuint64_t)((kv_heads - 1) * *head_rows + cap)};
  cuuint64_t strides[1] = {(cuuint64_t)(s_t * 2)};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype == BB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BB_ERR_LAUNCH, "decode: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BB_OK;
}

int check_common(const bb_decode_args* a, int64_t rows_per_group_max) {
  if (!a) return fail(BB_ERR_ARG, "decode: null args");
  if (a->dtype != BB_F16 && a->dtype != BB_BF16) return fail(BB_ERR_DTYPE, "decode requires fp16 or bf16");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
    return fail(BB_ERR_SHAPE, "decode: heads must be a positive multiple of kv_heads");
  if (a->d <= 0 || a->d > 128 || a->d % 8) return fail(BB_ERR_UNSUPPORTED, "decode: head_dim must be a multiple of 8 and <= 128");
  if (a->cap <= 0) return fail(BB_ERR_SHAPE, "decode: empty cache");
  if (a->cap > INT32_MAX) return fail(BB_ERR_UNSUPPORTED, "decode: cache capacity above 2^31 - 1 keys");
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
  if (splits <= 0) splits = auto_splits(total, rr, dt_usable(a, true) ? DtSmem::bytes(true) : dk_smem(dpad(a->d), true));
  splits = std::min<int64_t>(splits, 4096);  // the combine keeps two floats a split in shared memory (32 KB)
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
  p.idx = a->idx; p.si_r = a->si_r; p.idx64 = a->idx_i64 != 0;
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
  if (DP == 128 && dt_usable(a, true)) {
    DtMaps maps;
    int st = dt_map(&maps.k, &maps.k_head_rows, a->k, a->dtype, a->kv_heads, a->cap, a->sk_h, a->sk_t);
    if (!st) st = dt_map(&maps.v, &maps.v_head_rows, a->v, a->dtype, a->kv_heads, a->cap, a->sv_h, a->sv_t);
    if (st) return st;
    const size_t smem = DtSmem::bytes(true);
    cudaFuncSetAttribute(decode_tma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    decode_tma_kernel<T><<<dim3((unsigned)rr, (unsigned)pl.splits), DT_THREADS, smem, stream>>>(maps, p);
    BB_CHECK_LAUNCH("decode_tma_kernel");
  } else {
    const size_t smem = DkSmem<DP>::bytes(true);
    cudaFuncSetAttribute(decode_partial_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    decode_partial_kernel<T, DP><<<dim3((unsigned)rr, (unsigned)pl.splits), DK_THREADS, smem, stream>>>(p);
    BB_CHECK_LAUNCH("decode_partial_kernel");
  }
  decode_combine_kernel<T><<<(unsigned)a->heads, 128, (size_t)pl.splits * 8, stream>>>(p);
  BB_CHECK_LAUNCH("decode_combine_kernel");
  return BB_OK;
}

struct DroutePlan {
  int64_t splits, split_len;
  size_t scores_bytes, m_bytes, l_bytes, probs_bytes, topk_bytes, total;
};

int plan_droute(const bb_decode_args* a, DroutePlan* pl) {
  int st = check_common(a, DK_MAXROWS);
  if (st) return st;
  if (a->route_k < 0 || a->route_k > a->cap) return fail(BB_ERR_ARG, "decode_route: k_route must lie in [0, cap]");
  int64_t splits = a->splits;
  if (splits <= 0)
    splits = auto_splits(a->cap, a->kv_heads, dt_usable(a, false) ? DtSmem::bytes(false) : dk_smem(dpad(a->d), false));
  splits = std::min<int64_t>(splits, 8192);
  int64_t split_len = cdiv(cdiv(a->cap, splits), (int64_t)DK_BN) * DK_BN;
  splits = cdiv(a->cap, split_len);
  pl->splits = splits;
  pl->split_len = split_len;
  const size_t parts = (size_t)a->kv_heads * splits * (a->heads / a->kv_heads);
  pl->scores_bytes = align_up((size_t)a->heads * a->cap * 4, 256);
  pl->m_bytes = align_up(parts * 4, 256);
  pl->l_bytes = align_up(parts * 4, 256);
  pl->probs_bytes = a->out_probs ? 0 : align_up((size_t)a->kv_heads * a->cap * 4, 256);
  pl->topk_bytes = align_up(topk_scratch_bytes(a->kv_heads, a->cap, a->route_k), 256);
  pl->total = pl->scores_bytes + pl->m_bytes + pl->l_bytes + pl->probs_bytes + pl->topk_bytes;
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
  if (DP == 128 && dt_usable(a, false)) {
    DtMaps maps;
    maps.v_head_rows = 0;
    int st = dt_map(&maps.k, &maps.k_head_rows, a->k, a->dtype, a->kv_heads, a->cap, a->sk_h, a->sk_t);
    if (st) return st;
    const size_t smem = DtSmem::bytes(false);
    cudaFuncSetAttribute(droute_tma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    droute_tma_kernel<T><<<dim3((unsigned)a->kv_heads, (unsigned)pl.splits), DT_THREADS, smem, stream>>>(maps, p);
    BB_CHECK_LAUNCH("droute_tma_kernel");
  } else {
    const size_t smem = DkSmem<DP>::bytes(false);
    cudaFuncSetAttribute(droute_scores_kernel<T, DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    droute_scores_kernel<T, DP><<<dim3((unsigned)a->kv_heads, (unsigned)pl.splits), DK_THREADS, smem, stream>>>(p);
    BB_CHECK_LAUNCH("droute_scores_kernel");
  }
  droute_pool_kernel<<<dim3((unsigned)a->kv_heads, (unsigned)cdiv(a->cap, (int64_t)1024)), 256, 0, stream>>>(p);
  BB_CHECK_LAUNCH("droute_pool_kernel");
  if (a->route_k > 0 && a->out_idx) {
    int st = topk_sorted(p.probs, a->kv_heads, a->cap, a->route_k, a->out_idx, a->out_idx_i64 != 0, a->so_i,
                         ws + pl.scores_bytes + pl.m_bytes + pl.l_bytes + pl.probs_bytes, pl.topk_bytes, stream);
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

int decode_set_wait_limit(unsigned long long ns) { return tc::unit_set_wait_limit(ns); }

int decode_fault_take(int* code) {
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
