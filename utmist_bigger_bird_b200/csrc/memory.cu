// Memory path of a whole-model long prefill (the steps on either side of attention):
//
//   silu_mul_kernel      gate <- act(gate) * up for a Llama MLP chunk, in place (SwiGLU). Replaces
//                        `act_fn(gate_proj(x)) * up_proj(x)` inside the per-chunk MLP forward of
//                        modal_rd/mlp_chunk.py:19-26 with one pass (HF: one pass for the
//                        activation, one for the product, each with its own [chunk, I] output).
//                        The roundings are HF's: act(g) = g / (1 + exp(-g)) in fp32 rounded to
//                        the input dtype, then the product in fp32 rounded again, so the output is
//                        bit-identical.
//   embed_gather_kernel  rows of an embedding table held in page-locked host memory gathered
//                        straight into device memory over the host link (modal_rd/cpu_embed.py:
//                        21-25 gathers on the CPU, then copies into pinned staging, then to the
//                        GPU). Ids out of range are counted (the caller raises) and give zero rows.
//
//   rmsnorm_kernel       RMSNorm (optionally fused with the residual add before it) for the B200
//                        model path; HF's arithmetic, the fp32 sum of squares in a different order.
//
// All are bound by bytes moved: silu_mul and rmsnorm by HBM, embed_gather by the host link
// (n * row_bytes).
#include "bb_common.cuh"

namespace bb {
namespace {

template <typename T> __device__ __forceinline__ float silu_round(float x) {
  return Elem<T>::round(x / (1.f + expf(-x)));
}

// One 16-byte vector (8 x 16-bit or 4 x fp32) per thread and step; rows may be strided.
template <typename T>
__global__ void silu_mul_kernel(T* __restrict__ gate, int64_t sg, const T* __restrict__ up, int64_t su, int64_t rows,
                                int64_t cols) {
  constexpr int V = 16 / sizeof(T);
  const int64_t vec_per_row = cols / V;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row, c = (i % vec_per_row) * V;
    uint4 gv = *reinterpret_cast<const uint4*>(gate + r * sg + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(up + r * su + c);
    T* g = reinterpret_cast<T*>(&gv);
    const T* u = reinterpret_cast<const T*>(&uv);
#pragma unroll
    for (int e = 0; e < V; ++e) g[e] = Elem<T>::from_f(silu_round<T>(Elem<T>::to_f(g[e])) * Elem<T>::to_f(u[e]));
    *reinterpret_cast<uint4*>(gate + r * sg + c) = gv;
  }
}

// Scalar tail / unaligned layouts.
template <typename T>
__global__ void silu_mul_scalar_kernel(T* __restrict__ gate, int64_t sg, const T* __restrict__ up, int64_t su,
                                       int64_t rows, int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float g = Elem<T>::to_f(gate[r * sg + c]);
    gate[r * sg + c] = Elem<T>::from_f(silu_round<T>(g) * Elem<T>::to_f(up[r * su + c]));
  }
}

// One warp per row; 16-byte loads from the mapped host table.
__global__ void embed_gather_kernel(const uint4* __restrict__ table, int64_t vocab, int64_t row_vec,
                                    const int64_t* __restrict__ ids, int64_t n, uint4* __restrict__ out,
                                    int32_t* __restrict__ bad) {
  const int lane = threadIdx.x % 32;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += warps) {
    const int64_t id = ids[r];
    uint4* o = out + r * row_vec;
    if (id < 0 || id >= vocab) {
      if (lane == 0) atomicAdd(bad, 1);
      for (int64_t c = lane; c < row_vec; c += 32) o[c] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const uint4* src = table + id * row_vec;
    for (int64_t c = lane; c < row_vec; c += 32) o[c] = src[c];
  }
}

// RMSNorm of one row per warp (optionally after an in-place residual add x <- x + r, rounded to
// the dtype as torch's add_ does): y = w * round(x * rsqrt(mean(x^2) + eps)) with the mean
// accumulated in fp32 (HF LlamaRMSNorm's arithmetic; only the order of the fp32 sum differs).
// The second pass re-reads each lane's own vectors (L1 hits); x is read from HBM once.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(T* __restrict__ x, int64_t sx, const T* __restrict__ r,
                                                      int64_t sr, const T* __restrict__ w, T* __restrict__ y,
                                                      int64_t sy, int64_t rows, int64_t cols, float eps) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x % 32;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  if (row >= rows) return;
  T* xr = x + row * sx;
  const T* rr = r ? r + row * sr : nullptr;
  T* yr = y + row * sy;
  const int64_t nvec = cols / V;
  float acc = 0.f;
  for (int64_t v = lane; v < nvec; v += 32) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + v * V);
    T* xe = reinterpret_cast<T*>(&xv);
    if (rr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rr + v * V);
      const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
      for (int e = 0; e < V; ++e) xe[e] = Elem<T>::from_f(Elem<T>::to_f(xe[e]) + Elem<T>::to_f(re[e]));
      *reinterpret_cast<uint4*>(xr + v * V) = xv;
    }
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float f = Elem<T>::to_f(xe[e]);
      acc = fmaf(f, f, acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  const float inv = rsqrtf(acc / (float)cols + eps);
  for (int64_t v = lane; v < nvec; v += 32) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + v * V);  // this lane's own vector (L1 hit)
    const uint4 wv = *reinterpret_cast<const uint4*>(w + v * V);
    uint4 yv;
    const T* xe = reinterpret_cast<const T*>(&xv);
    const T* we = reinterpret_cast<const T*>(&wv);
    T* ye = reinterpret_cast<T*>(&yv);
#pragma unroll
    for (int e = 0; e < V; ++e)
      ye[e] = Elem<T>::from_f(Elem<T>::to_f(we[e]) * Elem<T>::round(Elem<T>::to_f(xe[e]) * inv));
    *reinterpret_cast<uint4*>(yr + v * V) = yv;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
int launch_silu_mul(void* gate, int64_t sg, const void* up, int64_t su, int64_t rows, int64_t cols, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  T* g = static_cast<T*>(gate);
  const T* u = static_cast<const T*>(up);
  const bool vec = cols % V == 0 && sg % V == 0 && su % V == 0 && al16(gate) && al16(up);
  const int64_t work = vec ? rows * (cols / V) : rows * cols;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)num_sms() * 8));
  if (vec) {
    silu_mul_kernel<T><<<blocks, 256, 0, s>>>(g, sg, u, su, rows, cols);
    BB_CHECK_LAUNCH("silu_mul_kernel");
  } else {
    silu_mul_scalar_kernel<T><<<blocks, 256, 0, s>>>(g, sg, u, su, rows, cols);
    BB_CHECK_LAUNCH("silu_mul_scalar_kernel");
  }
  return BB_OK;
}

}  // namespace

int silu_mul(void* gate, int64_t s_gate, const void* up, int64_t s_up, int64_t rows, int64_t cols, int dtype,
             cudaStream_t stream) {
  if (rows < 0 || cols < 0) return fail(BB_ERR_SHAPE, "silu_mul: negative shape");
  if (rows == 0 || cols == 0) return BB_OK;
  if (!gate || !up) return fail(BB_ERR_ARG, "silu_mul: null pointer");
  if (s_gate < cols || s_up < cols) return fail(BB_ERR_STRIDE, "silu_mul: row stride below the row length");
  switch (dtype) {
    case BB_BF16: return launch_silu_mul<__nv_bfloat16>(gate, s_gate, up, s_up, rows, cols, stream);
    case BB_F16: return launch_silu_mul<__half>(gate, s_gate, up, s_up, rows, cols, stream);
    case BB_F32: return launch_silu_mul<float>(gate, s_gate, up, s_up, rows, cols, stream);
    default: return fail(BB_ERR_DTYPE, "silu_mul: dtype must be bf16, f16 or f32");
  }
}

int rmsnorm(void* x, int64_t sx, const void* r, int64_t sr, const void* w, void* y, int64_t sy, int64_t rows,
            int64_t cols, float eps, int dtype, cudaStream_t stream) {
  if (rows < 0 || cols <= 0) return fail(BB_ERR_SHAPE, "rmsnorm: bad shape");
  if (rows == 0) return BB_OK;
  if (!x || !w || !y) return fail(BB_ERR_ARG, "rmsnorm: null pointer");
  const int es = dtype == BB_F32 ? 4 : 2;
  if (dtype != BB_BF16 && dtype != BB_F16 && dtype != BB_F32) return fail(BB_ERR_DTYPE, "rmsnorm: dtype must be bf16, f16 or f32");
  if ((cols * es) % 16 || (sx * es) % 16 || (sy * es) % 16 || (r && (sr * es) % 16) || !al16(x) || !al16(w) ||
      !al16(y) || (r && !al16(r)))
    return fail(BB_ERR_STRIDE, "rmsnorm: rows must be 16-byte multiples on 16-byte boundaries");
  if (sx < cols || sy < cols || (r && sr < cols)) return fail(BB_ERR_STRIDE, "rmsnorm: row stride below the row length");
  const unsigned blocks = (unsigned)cdiv(rows, 8);
  switch (dtype) {
    case BB_BF16:
      rmsnorm_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
          static_cast<__nv_bfloat16*>(x), sx, static_cast<const __nv_bfloat16*>(r), sr,
          static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), sy, rows, cols, eps);
      break;
    case BB_F16:
      rmsnorm_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<__half*>(x), sx, static_cast<const __half*>(r), sr,
                                                          static_cast<const __half*>(w), static_cast<__half*>(y), sy,
                                                          rows, cols, eps);
      break;
    default:
      rmsnorm_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<float*>(x), sx, static_cast<const float*>(r), sr,
                                                         static_cast<const float*>(w), static_cast<float*>(y), sy,
                                                         rows, cols, eps);
  }
  BB_CHECK_LAUNCH("rmsnorm_kernel");
  return BB_OK;
}

int embed_gather(const void* table, int64_t vocab, int64_t row_bytes, const int64_t* ids, int64_t n, void* out,
                 int32_t* bad, cudaStream_t stream) {
  if (vocab <= 0 || row_bytes <= 0 || n < 0) return fail(BB_ERR_SHAPE, "embed_gather: bad shape");
  if (n == 0) return BB_OK;
  if (!table || !ids || !out || !bad) return fail(BB_ERR_ARG, "embed_gather: null pointer");
  if (row_bytes % 16 || !al16(table) || !al16(out))
    return fail(BB_ERR_UNSUPPORTED, "embed_gather: rows must be a multiple of 16 bytes, table and output 16-byte aligned");
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, table);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(BB_ERR_ARG, "embed_gather: table pointer not known to CUDA: %s", cudaGetErrorString(e));
  }
  const void* dev_table = nullptr;
  if (at.type == cudaMemoryTypeHost) {
    dev_table = at.devicePointer;  // page-locked and mapped: readable by kernels over the host link
  } else if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
    dev_table = table;
  }
  if (!dev_table)
    return fail(BB_ERR_ARG, "embed_gather: the table must be page-locked host memory (pin_memory) or device memory");
  const int64_t row_vec = row_bytes / 16;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 8), (int64_t)num_sms() * 8));
  embed_gather_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(dev_table), vocab, row_vec, ids, n,
                                                   static_cast<uint4*>(out), bad);
  BB_CHECK_LAUNCH("embed_gather_kernel");
  return BB_OK;
}

}  // namespace bb
