// extern "C" entry points of libbb_b200.so (declared in include/bb_b200.h).
#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>

#include "flash.cuh"

namespace bb {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int num_sms() {
  static thread_local int cached_dev = -1, cached = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cached;
  if (dev != cached_dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) cached = v;
    cached_dev = dev;
  }
  return cached;
}

int rope_inplace(void* x, int dtype, int64_t B, int64_t H, int64_t T_, int64_t D, int64_t sxb,
                 int64_t sxh, int64_t sxt, const void* cos, const void* sin, int64_t scb,
                 int64_t sct, cudaStream_t stream);
int rope_pair_inplace(void* q, int64_t hq, int64_t sqh, int64_t sqt, void* k, int64_t hk, int64_t skh, int64_t skt,
                      int dtype, int64_t T_, int64_t D, const void* cos, const void* sin, int64_t sct,
                      cudaStream_t stream);
int routes_workspace_size(const bb_routes_args* a, size_t* bytes);
int routes(const bb_routes_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int kv_evict_workspace_size(const bb_evict_args* a, size_t* bytes);
int kv_evict(const bb_evict_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int decode_workspace_size(const bb_decode_args* a, size_t* bytes);
int decode(const bb_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int decode_route_workspace_size(const bb_decode_args* a, size_t* bytes);
int decode_route(const bb_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int flash_workspace_size(const bb_flash_args* a, size_t* bytes);
int flash(const bb_flash_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int silu_mul(void* gate, int64_t s_gate, const void* up, int64_t s_up, int64_t rows, int64_t cols, int dtype,
             cudaStream_t stream);
int embed_gather(const void* table, int64_t vocab, int64_t row_bytes, const int64_t* ids, int64_t n, void* out,
                 int32_t* bad, cudaStream_t stream);
int rmsnorm(void* x, int64_t sx, const void* r, int64_t sr, const void* w, void* y, int64_t sy, int64_t rows,
            int64_t cols, float eps, int dtype, cudaStream_t stream);

namespace {

// routed[h][g][k] = idx[h][k] if query group g overlaps the final vertical_scope tokens else -1
// (modal_rd/attention.py:187-194).
__global__ void scope_routes_kernel(const int32_t* __restrict__ idx, int64_t si_h,
                                    int32_t* __restrict__ routed, int64_t H, int64_t G, int64_t K,
                                    int64_t chunk, int64_t n, int64_t scope) {
  const int64_t total = H * G * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = i % K, g = (i / K) % G, h = i / (K * G);
    const bool active = g * chunk + chunk > n - scope;
    routed[i] = active ? idx[h * si_h + k] : -1;
  }
}

struct PrefillPlan {
  bb_routes_args ra;
  bb_flash_args main, tail;
  size_t routes_ws, flash_ws, scope_bytes, total;
  int64_t r, groups;
};

int64_t next_pow2(int64_t x) {
  int64_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

int plan_prefill(const bb_prefill_args* a, PrefillPlan* pl) {
  if (!a) return fail(BB_ERR_ARG, "sparse_prefill: null args");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads) return fail(BB_ERR_SHAPE, "sparse_prefill: heads must be a multiple of kv_heads");
  bb_routes_args& r = pl->ra;
  memset(&r, 0, sizeof(r));
  r.q = a->q; r.sq_h = a->sq_h; r.sq_t = a->sq_t;
  r.k = a->k; r.sk_h = a->sk_h; r.sk_t = a->sk_t;
  r.qpos = a->qpos;
  r.heads = a->heads; r.kv_heads = a->kv_heads; r.n = a->n; r.d = a->d; r.r = a->r;
  r.sink = a->sink; r.window = a->window; r.budget = a->budget;
  r.scaling = a->scaling; r.pool = a->pool; r.dtype = a->dtype;
  r.out_idx = a->out_idx; r.so_h = a->si_h; r.out_col = nullptr;
  int st = routes_workspace_size(&r, &pl->routes_ws);
  if (st) return st;
  pl->r = std::min(a->exact_tail, a->n);
  const int64_t g = a->heads / a->kv_heads;
  bb_flash_args& m = pl->main;
  memset(&m, 0, sizeof(m));
  m.q = a->q; m.sq_h = a->sq_h; m.sq_t = a->sq_t;
  m.k = a->k; m.sk_h = a->sk_h; m.sk_t = a->sk_t;
  m.v = a->v; m.sv_h = a->sv_h; m.sv_t = a->sv_t;
  m.out = a->out; m.so_h = a->so_h; m.so_t = a->so_t;
  m.bh = a->heads; m.t = a->n; m.n = a->n; m.d = a->d;
  m.num_heads = a->heads; m.kv_groups = g;
  m.front = a->sink; m.window = a->window;
  m.route_k = a->budget;
  if (a->vertical_scope) {
    if (a->scope_chunk <= 0) return fail(BB_ERR_ARG, "sparse_prefill: scope_chunk must be positive");
    pl->groups = cdiv(a->n, a->scope_chunk);
    m.route_groups = pl->groups; m.route_chunk = a->scope_chunk;
    m.si_h = pl->groups * a->budget; m.si_g = a->budget; m.si_k = 1;
  } else {
    pl->groups = 1;
    m.route_groups = 1; m.route_chunk = std::max<int64_t>(64, next_pow2(a->n));
    m.idx = a->out_idx; m.si_h = a->si_h; m.si_g = 0; m.si_k = 1;
  }
  m.row_begin = 0; m.row_end = a->n - pl->r;
  m.scale = a->scaling; m.dtype = a->dtype;
  st = flash_workspace_size(&m, &pl->flash_ws);
  if (st) return st;
  bb_flash_args& t = pl->tail;
  t = m;
  const int64_t off = a->n - pl->r;
  t.q = static_cast<const char*>(a->q) + off * a->sq_t * 2;
  t.out = static_cast<char*>(a->out) + off * a->so_t * 2;
  t.t = pl->r; t.front = 0; t.window = std::max<int64_t>(a->n, 1); t.route_k = 0;
  t.route_groups = 1; t.route_chunk = std::max<int64_t>(64, next_pow2(a->n)); t.idx = nullptr;
  t.row_begin = 0; t.row_end = pl->r;
  if (pl->r > 0) {
    size_t tw = 0;
    st = flash_workspace_size(&t, &tw);
    if (st) return st;
    pl->flash_ws = std::max(pl->flash_ws, tw);
  }
  pl->scope_bytes = a->vertical_scope ? align_up((size_t)a->heads * pl->groups * a->budget * 4, 256) : 0;
  pl->routes_ws = align_up(pl->routes_ws, 256);
  pl->flash_ws = align_up(pl->flash_ws, 256);
  pl->total = pl->routes_ws + pl->flash_ws + pl->scope_bytes;
  return BB_OK;
}

}  // namespace
}  // namespace bb

extern "C" {

const char* bb_last_error(void) { return bb::g_last_error.c_str(); }

int bb_abi_version(void) { return BB_ABI_VERSION; }

uint64_t bb_kernel_launches(void) { return bb::g_launches.load(std::memory_order_relaxed); }

int bb_device_fault(int* code) {
  if (!code) return bb::fail(BB_ERR_ARG, "device_fault: null pointer");
  int a = 0, b = 0, c = 0;
  int st = bb::flash_fault_take(&a);
  if (st != BB_OK) return st;
  st = bb::routes_fault_take(&b);
  if (st != BB_OK) return st;
  st = bb::decode_fault_take(&c);
  if (st != BB_OK) return st;
  *code = a ? a : (b ? b : c);
  return BB_OK;
}

int bb_set_wait_limit_ns(uint64_t ns) {
  if (ns == 0) return bb::fail(BB_ERR_ARG, "set_wait_limit_ns: the limit must be positive");
  if (bb::flash_set_wait_limit(ns) || bb::routes_set_wait_limit(ns) || bb::decode_set_wait_limit(ns))
    return bb::fail(BB_ERR_LAUNCH, "set_wait_limit_ns: %s", cudaGetErrorString(cudaGetLastError()));
  return BB_OK;
}

int bb_debug_stall_attention(int on) {
  if (bb::flash_set_stall(on)) return bb::fail(BB_ERR_LAUNCH, "debug_stall_attention: %s", cudaGetErrorString(cudaGetLastError()));
  return BB_OK;
}

int bb_rope_inplace(void* x, int dtype, int64_t B, int64_t H, int64_t T, int64_t D, int64_t sxb,
                    int64_t sxh, int64_t sxt, const void* cos, const void* sin, int64_t scb,
                    int64_t sct, bb_stream_t stream) {
  return bb::rope_inplace(x, dtype, B, H, T, D, sxb, sxh, sxt, cos, sin, scb, sct, bb::as_stream(stream));
}

int bb_routes_workspace_size(const bb_routes_args* a, size_t* bytes) {
  return bb::routes_workspace_size(a, bytes);
}

int bb_routes(const bb_routes_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  return bb::routes(a, ws, ws_bytes, bb::as_stream(stream));
}

int bb_kv_evict_workspace_size(const bb_evict_args* a, size_t* bytes) {
  if (!bytes) return bb::fail(BB_ERR_ARG, "kv_evict: null bytes pointer");
  return bb::kv_evict_workspace_size(a, bytes);
}

int bb_kv_evict(const bb_evict_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  return bb::kv_evict(a, ws, ws_bytes, bb::as_stream(stream));
}

int bb_decode_workspace_size(const bb_decode_args* a, size_t* bytes) {
  if (!bytes) return bb::fail(BB_ERR_ARG, "decode: null bytes pointer");
  return bb::decode_workspace_size(a, bytes);
}

int bb_decode(const bb_decode_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  return bb::decode(a, ws, ws_bytes, bb::as_stream(stream));
}

int bb_decode_route_workspace_size(const bb_decode_args* a, size_t* bytes) {
  if (!bytes) return bb::fail(BB_ERR_ARG, "decode_route: null bytes pointer");
  return bb::decode_route_workspace_size(a, bytes);
}

int bb_decode_route(const bb_decode_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  return bb::decode_route(a, ws, ws_bytes, bb::as_stream(stream));
}

int bb_silu_mul(void* gate, int64_t s_gate, const void* up, int64_t s_up, int64_t rows, int64_t cols, int dtype,
                bb_stream_t stream) {
  return bb::silu_mul(gate, s_gate, up, s_up, rows, cols, dtype, bb::as_stream(stream));
}

int bb_embed_gather(const void* table, int64_t vocab, int64_t row_bytes, const int64_t* ids, int64_t n, void* out,
                    int32_t* bad, bb_stream_t stream) {
  return bb::embed_gather(table, vocab, row_bytes, ids, n, out, bad, bb::as_stream(stream));
}

int bb_rmsnorm(void* x, int64_t sx, const void* residual, int64_t sr, const void* weight, void* y, int64_t sy,
               int64_t rows, int64_t cols, float eps, int dtype, bb_stream_t stream) {
  return bb::rmsnorm(x, sx, residual, sr, weight, y, sy, rows, cols, eps, dtype, bb::as_stream(stream));
}

int bb_flash_workspace_size(const bb_flash_args* a, size_t* bytes) {
  return bb::flash_workspace_size(a, bytes);
}

int bb_flash(const bb_flash_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  return bb::flash(a, ws, ws_bytes, bb::as_stream(stream));
}

int bb_sparse_prefill_workspace_size(const bb_prefill_args* a, size_t* bytes) {
  bb::PrefillPlan pl;
  int st = bb::plan_prefill(a, &pl);
  if (st) return st;
  *bytes = pl.total;
  return BB_OK;
}

int bb_sparse_prefill(const bb_prefill_args* a, void* ws, size_t ws_bytes, bb_stream_t stream) {
  bb::PrefillPlan pl;
  int st = bb::plan_prefill(a, &pl);
  if (st) return st;
  if (ws_bytes < pl.total || (pl.total && !ws))
    return bb::fail(BB_ERR_WORKSPACE, "sparse_prefill: workspace too small (%zu < %zu)", ws_bytes, pl.total);
  cudaStream_t s = bb::as_stream(stream);
  char* w = static_cast<char*>(ws);
  if (a->cos || a->sin) {
    if (!a->cos || !a->sin) return bb::fail(BB_ERR_ARG, "sparse_prefill: cos and sin go together");
    st = bb::rope_pair_inplace(a->q, a->heads, a->sq_h, a->sq_t, a->k, a->kv_heads, a->sk_h, a->sk_t, a->dtype, a->n,
                               a->d, a->cos, a->sin, a->sc_t, s);
    if (st == BB_ERR_UNSUPPORTED) {
      st = bb::rope_inplace(a->q, a->dtype, 1, a->heads, a->n, a->d, 0, a->sq_h, a->sq_t, a->cos, a->sin, 0, a->sc_t, s);
      if (st) return st;
      st = bb::rope_inplace(a->k, a->dtype, 1, a->kv_heads, a->n, a->d, 0, a->sk_h, a->sk_t, a->cos, a->sin, 0, a->sc_t, s);
    }
    if (st) return st;
  }
  st = bb::routes(&pl.ra, w, pl.routes_ws, s);
  if (st) return st;
  char* fw = w + pl.routes_ws;
  if (a->vertical_scope && a->budget > 0) {
    int32_t* routed = reinterpret_cast<int32_t*>(fw + pl.flash_ws);
    const int64_t total = a->heads * pl.groups * a->budget;
    bb::scope_routes_kernel<<<(unsigned)std::min<int64_t>(bb::cdiv(total, 256), 4096), 256, 0, s>>>(
        a->out_idx, a->si_h, routed, a->heads, pl.groups, a->budget, a->scope_chunk, a->n, a->vertical_scope);
    BB_CHECK_LAUNCH("scope_routes_kernel");
    pl.main.idx = routed;
  }
  st = bb::flash(&pl.main, fw, pl.flash_ws, s);
  if (st) return st;
  if (pl.r > 0) {
    st = bb::flash(&pl.tail, fw, pl.flash_ws, s);
    if (st) return st;
  }
  return BB_OK;
}

}  // extern "C"
