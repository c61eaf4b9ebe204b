// KV eviction after a sparse prefill (RDAttention.evict, modal_rd/attention.py:226-259):
//
//   1. evict_member_kernel   marks, per KV head, every key that is a route of one of its query
//                            heads (the scatter of :240-241 reduced over the group, :247).
//   2. evict_score_kernel    score[kv, j] = max over the group's query heads of col[h, j] (:243).
//   3. evict_prio_kernel     prio = 2 * member + forward_pool(score) (:245-247, :70-75), with the
//                            sink keys and the last `window` keys at -inf (:249-250). Without a
//                            forward pool, steps 2-3 run as one pass (evict_prio_direct_kernel).
//   4. route_topk_kernel     the `keep` largest priorities per KV head, positions ascending
//                            (:252, shared with routing).
//   5. evict_gather_kernel   kept positions [sink | selected | window] and the K/V rows at them,
//                            16-byte vectors (:253-258).
// Steps 1-3 and 5 read or write each byte once and are HBM-bound; the score/priority buffers are
// fp32 [Hk, n] and the member mask one byte per (KV head, key).
#include <algorithm>

#include "bb_common.cuh"

namespace bb {

int topk_sorted(const float* vals, int64_t rows, int64_t n, int64_t k, void* out, bool out64, int64_t so_h,
                void* scratch, size_t scratch_bytes, cudaStream_t stream);
size_t topk_scratch_bytes(int64_t rows, int64_t n, int64_t k);

namespace {

struct EvictParams {
  const float* col; int64_t sc_h;
  const int32_t* idx; int64_t si_h; int64_t budget;
  int64_t heads, kv_heads, groups, n;
  int64_t sink, window, keep, pool, pool_back;
  uint8_t* member;  // [Hk][n]
  float* score;     // [Hk][n]
  float* prio;      // [Hk][n]
  int32_t* sel;     // [Hk][keep]
};

__global__ void evict_member_kernel(EvictParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.heads * p.budget) return;
  const int64_t h = t / p.budget, j = t % p.budget;
  const int64_t key = p.idx[h * p.si_h + j];
  if (key >= 0 && key < p.n) p.member[(h / p.groups) * p.n + key] = 1;
}

__global__ void evict_score_kernel(EvictParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.kv_heads * p.n) return;
  const int64_t kv = t / p.n, j = t % p.n;
  float s = -INFINITY;
  for (int64_t g = 0; g < p.groups; ++g) s = fmaxf(s, p.col[(kv * p.groups + g) * p.sc_h + j]);
  p.score[t] = s;
}

__global__ void evict_prio_kernel(EvictParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.kv_heads * p.n) return;
  const int64_t kv = t / p.n, j = t % p.n;
  float pr = -INFINITY;
  if (j >= p.sink && j < p.n - p.window) {
    const float* sc = p.score + kv * p.n;
    float s;
    if (p.pool > 1 || p.pool_back > 0) {
      const int64_t lo = j - (p.pool > 1 ? p.pool - 1 : 0), hi = j + p.pool_back;
      s = -INFINITY;
      for (int64_t i = lo < 0 ? 0 : lo; i <= hi && i < p.n; ++i) s = fmaxf(s, sc[i]);
    } else {
      s = sc[j];
    }
    pr = (p.member[t] ? 2.f : 0.f) + s;
  }
  p.prio[t] = pr;
}

// Steps 2-3 in one pass when there is no forward pool (the default policy): the group max of the
// column scores goes straight into the priority.
__global__ void evict_prio_direct_kernel(EvictParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.kv_heads * p.n) return;
  const int64_t kv = t / p.n, j = t % p.n;
  float pr = -INFINITY;
  if (j >= p.sink && j < p.n - p.window) {
    float s = -INFINITY;
    for (int64_t g = 0; g < p.groups; ++g) s = fmaxf(s, p.col[(kv * p.groups + g) * p.sc_h + j]);
    pr = (p.member[t] ? 2.f : 0.f) + s;
  }
  p.prio[t] = pr;
}

// One warp per kept row: its position and the K and V rows (d elements of esz bytes).
__global__ void evict_gather_kernel(EvictParams p, const char* __restrict__ k, int64_t sk_h, int64_t sk_t,
                                    const char* __restrict__ v, int64_t sv_h, int64_t sv_t, char* __restrict__ ok,
                                    int64_t sok_h, int64_t sok_t, char* __restrict__ ov, int64_t sov_h,
                                    int64_t sov_t, int64_t* __restrict__ out_pos, int64_t d, int esz) {
  const int64_t L = p.sink + p.keep + p.window;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= p.kv_heads * L) return;
  const int64_t kv = w / L, r = w % L;
  int64_t pos;
  if (r < p.sink) pos = r;
  else if (r < p.sink + p.keep) pos = p.sel[kv * p.keep + (r - p.sink)];
  else pos = p.n - p.window + (r - p.sink - p.keep);
  if (lane == 0) out_pos[w] = pos;
  const int64_t row_bytes = d * esz;
  const char* ks = k + (kv * sk_h + pos * sk_t) * esz;
  const char* vs = v + (kv * sv_h + pos * sv_t) * esz;
  char* kd = ok + (kv * sok_h + r * sok_t) * esz;
  char* vd = ov + (kv * sov_h + r * sov_t) * esz;
  for (int64_t b = (int64_t)lane * 16; b < row_bytes; b += 32 * 16) {
    *reinterpret_cast<uint4*>(kd + b) = *reinterpret_cast<const uint4*>(ks + b);
    *reinterpret_cast<uint4*>(vd + b) = *reinterpret_cast<const uint4*>(vs + b);
  }
}

struct EvictPlan {
  size_t member_bytes, score_bytes, prio_bytes, sel_bytes, topk_bytes, total;
};

int esize(int dtype) { return dtype == BB_F32 ? 4 : 2; }

int plan_evict(const bb_evict_args* a, EvictPlan* pl) {
  if (!a) return fail(BB_ERR_ARG, "kv_evict: null args");
  if (a->dtype != BB_F16 && a->dtype != BB_BF16 && a->dtype != BB_F32)
    return fail(BB_ERR_DTYPE, "kv_evict: dtype must be f16, bf16 or f32");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
    return fail(BB_ERR_SHAPE, "kv_evict: heads must be a positive multiple of kv_heads");
  if (a->n <= 0 || a->d <= 0) return fail(BB_ERR_SHAPE, "kv_evict: need n > 0 and d > 0");
  if (a->sink < 0 || a->window < 0 || a->sink + a->window > a->n)
    return fail(BB_ERR_ARG, "kv_evict: need 0 <= sink, 0 <= window and sink + window <= n");
  if (a->keep < 0 || a->keep > a->n - a->sink - a->window)
    return fail(BB_ERR_ARG, "kv_evict: keep must lie in [0, n - sink - window]");
  if (a->budget < 0) return fail(BB_ERR_ARG, "kv_evict: bad budget");
  if (a->pool < 0 || a->pool_back < 0) return fail(BB_ERR_ARG, "kv_evict: pool and pool_back must be >= 0");
  if ((a->d * esize(a->dtype)) % 16) return fail(BB_ERR_UNSUPPORTED, "kv_evict: rows must be a multiple of 16 bytes");
  const size_t cells = (size_t)a->kv_heads * a->n;
  pl->member_bytes = align_up(cells, 256);
  pl->score_bytes = align_up(cells * sizeof(float), 256);
  pl->prio_bytes = align_up(cells * sizeof(float), 256);
  pl->sel_bytes = align_up((size_t)a->kv_heads * std::max<int64_t>(a->keep, 1) * sizeof(int32_t), 256);
  pl->topk_bytes = align_up(topk_scratch_bytes(a->kv_heads, a->n, a->keep), 256);
  pl->total = pl->member_bytes + pl->score_bytes + pl->prio_bytes + pl->sel_bytes + pl->topk_bytes;
  return BB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int kv_evict_workspace_size(const bb_evict_args* a, size_t* bytes) {
  EvictPlan pl;
  int st = plan_evict(a, &pl);
  if (st) return st;
  *bytes = pl.total;
  return BB_OK;
}

int kv_evict(const bb_evict_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  EvictPlan pl;
  int st = plan_evict(a, &pl);
  if (st) return st;
  if (!ws || ws_bytes < pl.total) return fail(BB_ERR_WORKSPACE, "kv_evict: workspace too small (%zu < %zu)", ws_bytes, pl.total);
  if (!a->col || !a->k || !a->v || !a->out_k || !a->out_v || !a->out_pos || (a->budget > 0 && !a->idx))
    return fail(BB_ERR_ARG, "kv_evict: null pointer");
  const int es = esize(a->dtype);
  if (!aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out_k) || !aligned16(a->out_v) ||
      (a->sk_h * es) % 16 || (a->sk_t * es) % 16 || (a->sv_h * es) % 16 || (a->sv_t * es) % 16 ||
      (a->sok_h * es) % 16 || (a->sok_t * es) % 16 || (a->sov_h * es) % 16 || (a->sov_t * es) % 16)
    return fail(BB_ERR_STRIDE, "kv_evict: k/v rows must start on 16-byte boundaries");
  EvictParams p;
  p.col = a->col; p.sc_h = a->sc_h;
  p.idx = a->idx; p.si_h = a->si_h; p.budget = a->budget;
  p.heads = a->heads; p.kv_heads = a->kv_heads; p.groups = a->heads / a->kv_heads; p.n = a->n;
  p.sink = a->sink; p.window = a->window; p.keep = a->keep; p.pool = a->pool; p.pool_back = a->pool_back;
  char* w = static_cast<char*>(ws);
  p.member = reinterpret_cast<uint8_t*>(w);
  p.score = reinterpret_cast<float*>(w + pl.member_bytes);
  p.prio = reinterpret_cast<float*>(w + pl.member_bytes + pl.score_bytes);
  p.sel = reinterpret_cast<int32_t*>(w + pl.member_bytes + pl.score_bytes + pl.prio_bytes);
  const int64_t cells = a->kv_heads * a->n;
  cudaError_t e = cudaMemsetAsync(p.member, 0, (size_t)cells, stream);
  if (e != cudaSuccess) return fail(BB_ERR_LAUNCH, "kv_evict: memset: %s", cudaGetErrorString(e));
  if (a->budget > 0) {
    evict_member_kernel<<<(unsigned)cdiv(a->heads * a->budget, (int64_t)256), 256, 0, stream>>>(p);
    BB_CHECK_LAUNCH("evict_member_kernel");
  }
  if (p.pool > 1 || p.pool_back > 0) {
    evict_score_kernel<<<(unsigned)cdiv(cells, (int64_t)256), 256, 0, stream>>>(p);
    BB_CHECK_LAUNCH("evict_score_kernel");
    evict_prio_kernel<<<(unsigned)cdiv(cells, (int64_t)256), 256, 0, stream>>>(p);
    BB_CHECK_LAUNCH("evict_prio_kernel");
  } else {
    evict_prio_direct_kernel<<<(unsigned)cdiv(cells, (int64_t)256), 256, 0, stream>>>(p);
    BB_CHECK_LAUNCH("evict_prio_direct_kernel");
  }
  if (a->keep > 0) {
    st = topk_sorted(p.prio, a->kv_heads, a->n, a->keep, p.sel, false, a->keep,
                     w + pl.member_bytes + pl.score_bytes + pl.prio_bytes + pl.sel_bytes, pl.topk_bytes, stream);
    if (st) return st;
  }
  const int64_t L = a->sink + a->keep + a->window;
  if (L > 0) {
    evict_gather_kernel<<<(unsigned)cdiv(a->kv_heads * L * 32, (int64_t)256), 256, 0, stream>>>(
        p, static_cast<const char*>(a->k), a->sk_h, a->sk_t, static_cast<const char*>(a->v), a->sv_h, a->sv_t,
        static_cast<char*>(a->out_k), a->sok_h, a->sok_t, static_cast<char*>(a->out_v), a->sov_h, a->sov_t,
        a->out_pos, a->d, es);
    BB_CHECK_LAUNCH("evict_gather_kernel");
  }
  return BB_OK;
}

}  // namespace bb
