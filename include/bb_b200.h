/*
 * bb_b200.h -- C ABI of the B200 (sm_100a) Bigger Bird v3 sparse-prefill library (libbb_b200.so).
 *
 * Plain pointers, sizes and element strides only; every tensor argument is a device pointer
 * (unless stated otherwise) and every launch goes on the caller's CUDA stream. No call blocks
 * the host or allocates device memory: scratch space is passed in by the caller, sized by the
 * matching *_workspace_size query. Calls return a bb_status; bb_last_error() gives the message
 * of the last failing call on the calling host thread.
 *
 * Reference interfaces replaced (paths inside derkychen/utmist-bigger-bird):
 *   bb_rope_inplace      modal_rd/attention.py:51-60      rope_inplace(x, cos, sin)
 *   bb_routes            modal_rd/attention.py:143-174    RDAttention.routes(q, k)
 *   bb_flash             kernels/bigger_bird_flash.py:99-138  bigger_bird_flash(q, k, v, indices, ...)
 *   bb_sparse_prefill    modal_rd/attention.py:176-206    RDAttention.sparse_prefill(q, k, v)
 *                        (+ the in-place RoPE of forward, modal_rd/attention.py:121, when cos/sin given)
 *   bb_kv_evict          modal_rd/attention.py:226-259    RDAttention.evict(cache, q, k, v)
 *                        (+ forward_pool, modal_rd/attention.py:70-75)
 *   bb_decode            kernels/bigger_bird_decode.py:67-107  bigger_bird_decode(q, k, v, indices, ...)
 *   bb_decode_route      kernels/bigger_bird_route.py:80-115   pooled_probs / bigger_bird_route(q, k, k_route)
 */
#ifndef BB_B200_H
#define BB_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BB_API __attribute__((visibility("default")))
#else
#define BB_API
#endif

typedef struct CUstream_st* bb_stream_t; /* == cudaStream_t; NULL = legacy default stream */

typedef enum {
  BB_OK = 0,
  BB_ERR_ARG = 1,          /* bad scalar argument (front < 0, window < 1, ...)          -> ValueError */
  BB_ERR_SHAPE = 2,        /* inconsistent shapes / heads / route groups                -> ValueError */
  BB_ERR_DTYPE = 3,        /* unsupported element type                                  -> ValueError */
  BB_ERR_STRIDE = 4,       /* innermost stride != 1 or misaligned base/stride           -> ValueError */
  BB_ERR_WORKSPACE = 5,    /* workspace missing or smaller than *_workspace_size        -> ValueError */
  BB_ERR_LAUNCH = 6,       /* CUDA launch / attribute error                             -> RuntimeError */
  BB_ERR_UNSUPPORTED = 7,  /* valid input outside what this build implements            -> ValueError */
  BB_ERR_DEVICE = 8        /* not an sm_100 device / driver entry point missing         -> RuntimeError */
} bb_status;

typedef enum { BB_F16 = 0, BB_BF16 = 1, BB_F32 = 2 } bb_dtype;
typedef enum { BB_POOL_MEAN = 0, BB_POOL_MAX = 1 } bb_pool;

/* Message of the last error on this host thread ("" if none). */
BB_API const char* bb_last_error(void);
/* Library ABI version (BB_ABI_VERSION). */
BB_API int bb_abi_version(void);
#define BB_ABI_VERSION 2
/* Number of CUDA kernels this library has launched in this process (all threads, all devices).
 * Instrumentation for benchmarks; no counterpart in the reference. */
BB_API uint64_t bb_kernel_launches(void);
/* Reads and clears the current device's fault word. Kernels bound every wait on another warp's
 * progress (about 2 s); a kernel that gives up a wait records a non-zero code here, drains its
 * copies, frees its tensor memory and returns instead of hanging. Synchronous (copies 4 bytes
 * from the device). No counterpart in the reference. */
BB_API int bb_device_fault(int* code);
/* Sets the limit of every bounded wait of this library's kernels on the current device (ns > 0;
 * 2e9 by default), for launches made after the call. A shorter limit makes a kernel give up
 * sooner when another warp stops making progress. Synchronous. No counterpart in the reference. */
BB_API int bb_set_wait_limit_ns(uint64_t ns);
/* Test hook of the attention kernels' abort path (off by default). While on, the MMA warp of
 * every tcgen05 attention CTA (bb_flash, bb_sparse_prefill with head_dim 128) first waits for a
 * barrier that nothing completes: the wait runs out after the wait limit, the launch takes its
 * abort path (outputs of aborted tiles are zeros, copies drained, tensor memory freed) and
 * bb_device_fault then reports code 9. Synchronous. No counterpart in the reference. */
BB_API int bb_debug_stall_attention(int on);

/* ------------------------------------------------------------------------------------------
 * RoPE, in place: x[b,h,t,:] <- x*cos[b,t,:] + rotate_half(x)*sin[b,t,:], every op rounded to
 * the element type exactly as the torch expression of modal_rd/attention.py:59 (bit-identical).
 * x: [B, H, T, D] with element strides (sxb, sxh, sxt, 1); cos/sin: [B, T, D] with (scb, sct, 1)
 * (scb may be 0 to broadcast). dtype: BB_F16, BB_BF16 or BB_F32. D must be even.
 */
BB_API int bb_rope_inplace(void* x, int dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                    int64_t sxb, int64_t sxh, int64_t sxt,
                    const void* cos, const void* sin, int64_t scb, int64_t sct,
                    bb_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Routes (RDAttention.routes, modal_rd/attention.py:143-174).
 * For each KV head the routing queries q[h, qpos[i], :] of its `groups` query heads score every
 * key: s = round_to_dtype(q . k) * scaling (the bf16/fp16 matmul output of :164), causal mask
 * key > qpos -> -inf, fp32 softmax over all keys, then the mean (or max) over the r routing
 * queries gives col[h, key]. Columns [0, sink) and the Python slice [n - window:] are set to -1;
 * the `budget` largest columns per query head are returned sorted ascending (int32). Ties at the
 * budget-th score are broken towards lower key positions.
 */
typedef struct {
  const void* q;  int64_t sq_h, sq_t;   /* [H, n, d], innermost stride 1 (post-RoPE queries) */
  const void* k;  int64_t sk_h, sk_t;   /* [Hk, n, d], innermost stride 1 (post-RoPE keys)   */
  const int64_t* qpos;                  /* [r] device positions of the routing queries       */
  int64_t heads, kv_heads, n, d, r;
  int64_t sink, window, budget;
  float scaling;
  int pool;                             /* bb_pool */
  int dtype;                            /* BB_F16 or BB_BF16 */
  int32_t* out_idx; int64_t so_h;       /* [H, budget] int32 */
  float* out_col;                       /* optional [H, n] fp32 copy of the column scores (NULL: none) */
} bb_routes_args;

BB_API int bb_routes_workspace_size(const bb_routes_args* a, size_t* bytes);
BB_API int bb_routes(const bb_routes_args* a, void* workspace, size_t workspace_bytes, bb_stream_t stream);

/* bb_routes for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference. Some host programs reserve the whole GPU for their own memory
 * pool. A serving engine that pre-sizes its KV cache is one example. Some FFI callers have no
 * device allocator at all. Neither can hand this library a fresh workspace. This call computes
 * exactly what bb_routes computes (same kernels, same results). Its scratch lives in one fixed
 * array inside the library, BB_ROUTES_NOALLOC_SCRATCH_BYTES (24 MiB) per GPU. Every GPU that
 * loads the library holds that array until the process exits. It is enough for the 128K-token,
 * 32-query-head layer (about 19 MB). A request needing more is rejected with BB_ERR_WORKSPACE
 * and a message giving both sizes, before anything is launched. The caller still passes q, k,
 * qpos and the outputs.
 * The first call on each device looks up the array's device address, with that device current.
 * Make that first call before any stream capture. All calls share the one array, and it keeps
 * the previous call's contents. That is harmless here: every scratch byte a call reads is
 * written earlier in the same call. Calls that overlap on the GPU race on the array, for
 * example on two streams of one device. Serialize them. The call never runs cudaMalloc,
 * cudaFree or any allocating library routine. */
#define BB_ROUTES_NOALLOC_SCRATCH_BYTES ((size_t)24 << 20)
BB_API int bb_routes_noalloc(const bb_routes_args* a, bb_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Sparse flash attention (bigger_bird_flash, kernels/bigger_bird_flash.py:99-138).
 * One online softmax per query over the union of: sink keys [0, front), the causal window
 * [q - window + 1, q], and routed keys idx[bh, group(q), :] that lie in [front, q - window]
 * (disjoint sets; -1 or out-of-range slots are empty). Query j of T sits at absolute position
 * n - T + j. Query head h reads KV head (h / num_heads) * (num_heads / kv_groups)
 * + (h % num_heads) / kv_groups. token_mask (optional, [B, n] bytes, B = BH / num_heads) drops
 * masked keys and zeroes masked query rows. Fully masked rows give 0.
 * Rows [row_begin, row_end) of T are computed and written; other output rows are untouched.
 * Workspace (bb_flash_workspace_size): split partials of long-key-range calls and, for head_dim
 * 128 with routes, the call's routed K/V rows gathered once ([BH, G, K rounded up to 128, D]
 * each), so that the kernel loads routed tiles like window tiles.
 */
typedef struct {
  const void* q;  int64_t sq_h, sq_t;       /* [BH, T, D] */
  const void* k;  int64_t sk_h, sk_t;       /* [BH/kv_groups, n, D] */
  const void* v;  int64_t sv_h, sv_t;       /* [BH/kv_groups, n, D] */
  const int32_t* idx; int64_t si_h, si_g, si_k; /* [BH, G, K] int32 (K may be 0) */
  const uint8_t* token_mask; int64_t sm_b, sm_t; /* [B, n] or NULL */
  void* out; int64_t so_h, so_t;            /* [BH, T, D] */
  int64_t bh, t, n, d;
  int64_t num_heads, kv_groups;
  int64_t front, window;
  int64_t route_k, route_groups, route_chunk;
  int64_t row_begin, row_end;
  float scale;
  int dtype;                                /* BB_F16 or BB_BF16 */
} bb_flash_args;

BB_API int bb_flash_workspace_size(const bb_flash_args* a, size_t* bytes);
BB_API int bb_flash(const bb_flash_args* a, void* workspace, size_t workspace_bytes, bb_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Whole sparse prefill of one layer (RDAttention.sparse_prefill, modal_rd/attention.py:176-206):
 * [RoPE in place on q and k when cos/sin are given] -> routes -> main sparse pass over rows
 * [0, n - exact_tail) -> exact causal tail over the last exact_tail rows (front=0, window=n).
 * q: [H, n, d]; k, v: [Hk, n, d]; out: [H, n, d]. vertical_scope/scope_chunk as in :187-194.
 * out_idx receives the routes [H, budget] (RDAttention.last_routes).
 */
typedef struct {
  void* q;  int64_t sq_h, sq_t;
  void* k;  int64_t sk_h, sk_t;
  const void* v;  int64_t sv_h, sv_t;
  const void* cos; const void* sin; int64_t sc_t;   /* [n, d] or NULL (no RoPE) */
  const int64_t* qpos;                            /* [r] routing query positions (device) */
  void* out; int64_t so_h, so_t;
  int32_t* out_idx; int64_t si_h;
  int64_t heads, kv_heads, n, d, r;
  int64_t sink, window, budget, exact_tail, vertical_scope, scope_chunk;
  float scaling;
  int pool;
  int dtype;
} bb_prefill_args;

BB_API int bb_sparse_prefill_workspace_size(const bb_prefill_args* a, size_t* bytes);
BB_API int bb_sparse_prefill(const bb_prefill_args* a, void* workspace, size_t workspace_bytes,
                      bb_stream_t stream);

/*
 * KV eviction after a sparse prefill (RDAttention.evict, modal_rd/attention.py:226-259): per KV
 * head, keep the sink keys [0, sink), the `keep` best middle keys and the last `window` keys, and
 * write the kept K/V rows (in position order) and their positions.
 *   score[kv, j]  = max over the KV head's query heads of col[h, j]            (:243, :221)
 *   pooled[kv, j] = max of score[kv, j - pool + 1 .. j + pool_back] (-inf off the ends; pool <= 1
 *                   and pool_back == 0 leave score unchanged)                 (forward_pool :70-75)
 *   prio[kv, j]   = 2 * (j is a route of any of its query heads) + pooled     (:247)
 *   middle keys   = the `keep` largest prio among [sink, n - window), sorted ascending (:248-253;
 *                   equal priorities at the cut are taken in position order)
 * col: [H, n] fp32 column scores (the routing scores of the prefill, or exact-attention scores of
 * the last queries for evict_obs); idx: [H, budget] int32 routes (entries outside [0, n) ignored);
 * k, v: [Hk, n, d]; out_k, out_v: [Hk, sink + keep + window, d]; out_pos: [Hk, sink + keep +
 * window] int64. Requires sink + window <= n and keep <= n - sink - window.
 */
typedef struct {
  const float* col; int64_t sc_h;
  const int32_t* idx; int64_t si_h; int64_t budget;
  const void* k; int64_t sk_h, sk_t;
  const void* v; int64_t sv_h, sv_t;
  void* out_k; int64_t sok_h, sok_t;
  void* out_v; int64_t sov_h, sov_t;
  int64_t* out_pos;                      /* [Hk, sink + keep + window], contiguous */
  int64_t heads, kv_heads, n, d;
  int64_t sink, window, keep, pool, pool_back;
  int dtype;                              /* BB_F16 / BB_BF16 / BB_F32 (element type of k, v) */
} bb_evict_args;

BB_API int bb_kv_evict_workspace_size(const bb_evict_args* a, size_t* bytes);
BB_API int bb_kv_evict(const bb_evict_args* a, void* workspace, size_t workspace_bytes, bb_stream_t stream);

/*
 * Decode (one new query token per head) over a KV cache of capacity `cap`, of which the first n
 * keys are valid: n is the host value `n`, or, when `n_dev` is non-NULL, a device int64 read at
 * run time (so a captured CUDA graph stays valid while the cache grows).
 *
 * bb_decode (bigger_bird_decode, kernels/bigger_bird_decode.py:67-107): each query head attends to
 * the front keys [0, front), the last `window` keys [n - window, n) and its routed keys
 * idx[route row, :] (route rows = Hkv for pooled routes shared by a KV head's query heads, or H for
 * per-head routes; entries outside [0, n) are skipped; routed keys must lie in [front, n - window)
 * and be unique per row). Split-K flash decoding: P is rounded to the cache dtype before P.V.
 * out: [H, d] in the q dtype. route_k = 0: no routed keys (front = 0, window = cap: dense decoding).
 *
 * bb_decode_route (pooled_probs / bigger_bird_route, kernels/bigger_bird_route.py:80-115): per KV
 * head, the probability of every cached key under each query head's softmax over the first n
 * keys, averaged over the KV head's query heads; -1 outside [front, n - window). out_probs (may be
 * NULL): [Hkv, cap] fp32; out_idx (may be NULL): [Hkv, route_k] int32 (int64 with out_idx_i64),
 * the route_k most probable keys, positions ascending.
 */
typedef struct {
  const void* q; int64_t sq_h;              /* [H, d], innermost stride 1 */
  const void* k; int64_t sk_h, sk_t;        /* [Hkv, cap, d] */
  const void* v; int64_t sv_h, sv_t;        /* [Hkv, cap, d] (bb_decode only) */
  const void* idx; int64_t si_r;            /* [route_rows, route_k] int32, or int64 when idx_i64 (bb_decode) */
  int64_t route_rows, route_k;              /* bb_decode_route: route_k = keys to select */
  int64_t n; const int64_t* n_dev;          /* valid keys: n, or *n_dev when n_dev != NULL */
  int64_t cap, heads, kv_heads, d;
  int64_t front, window;
  float scale;
  int64_t splits;                           /* 0: enough chunks for ~4 CTAs per SM */
  void* out; int64_t so_h;                  /* bb_decode: [H, d] */
  float* out_probs;                         /* bb_decode_route: [Hkv, cap] or NULL */
  void* out_idx; int64_t so_i;              /* bb_decode_route: [Hkv, route_k] int32 (int64 when
                                              out_idx_i64) or NULL */
  int dtype;                                /* BB_F16 / BB_BF16 */
  int idx_i64;                              /* bb_decode: 1 when idx holds int64 positions (the
                                              routes' torch dtype, read as is: no conversion pass) */
  int out_idx_i64;                          /* bb_decode_route: 1 to write out_idx as int64 */
} bb_decode_args;

BB_API int bb_decode_workspace_size(const bb_decode_args* a, size_t* bytes);
BB_API int bb_decode(const bb_decode_args* a, void* workspace, size_t workspace_bytes, bb_stream_t stream);
BB_API int bb_decode_route_workspace_size(const bb_decode_args* a, size_t* bytes);
BB_API int bb_decode_route(const bb_decode_args* a, void* workspace, size_t workspace_bytes, bb_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Whole-model prefill memory path (the steps on either side of attention).
 *
 * bb_silu_mul replaces `act_fn(gate_proj(x)) * up_proj(x)` of the Llama MLP that
 * modal_rd/mlp_chunk.py:19-26 runs chunk by chunk: gate <- act(gate) * up in place, rows x cols
 * elements, row strides s_gate / s_up (elements). act(g) = g / (1 + exp(-g)) in fp32 rounded to
 * the dtype, the product in fp32 rounded again: bit-identical to the two HF ops. dtype BB_BF16,
 * BB_F16 or BB_F32.
 *
 * bb_embed_gather replaces CPUEmbedding.forward (modal_rd/cpu_embed.py:21-25): out[i] =
 * table[ids[i]] for n int64 ids on the device, the [vocab, row_bytes] table in page-locked host
 * memory (read by the kernel over the host link, no CPU gather or staging copy) or in device
 * memory. Ids outside [0, vocab) give zero rows and add to *bad (a device int32 the caller zeroes
 * and checks; the reference raises IndexError there). row_bytes a multiple of 16. */
BB_API int bb_silu_mul(void* gate, int64_t s_gate, const void* up, int64_t s_up, int64_t rows, int64_t cols,
                       int dtype, bb_stream_t stream);
BB_API int bb_embed_gather(const void* table, int64_t vocab, int64_t row_bytes, const int64_t* ids, int64_t n,
                           void* out, int32_t* bad, bb_stream_t stream);

/* bb_rmsnorm: y = weight * round(x * rsqrt(mean(x^2) + eps)) per row of `cols` elements, the
 * LlamaRMSNorm arithmetic (HF modeling_llama: fp32 mean of squares, fp32 scale, rounded to the
 * dtype, times the weight) with the fp32 sum in a different order (the normalised value within
 * one ulp of HF's, the output within two). With `residual` non-NULL the row is first updated in
 * place, x <- x + residual (rounded to the dtype, as torch's add_), which fuses the decoder
 * layer's residual add
 * (modal_rd/inplace_residual.py:23-25) with the norm that follows it. Row strides sx/sr/sy in
 * elements; rows and strides 16-byte multiples. B200 extra (opt-in), not a reference entry. */
BB_API int bb_rmsnorm(void* x, int64_t sx, const void* residual, int64_t sr, const void* weight, void* y, int64_t sy,
                      int64_t rows, int64_t cols, float eps, int dtype, bb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* BB_B200_H */
