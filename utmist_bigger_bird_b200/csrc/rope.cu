// In-place RoPE, bit-identical to rope_inplace (modal_rd/attention.py:51-60), i.e. to the torch
// expression `x * cos + rotate_half(x) * sin` where every op rounds to the tensor's dtype.
// HBM-bound elementwise work: each thread rotates VEC (i, i + D/2) pairs of one row, reading
// and writing x once and cos/sin once.
#include "bb_common.cuh"

namespace bb {
namespace {

template <typename T, int VEC>
__global__ void __launch_bounds__(256) rope_kernel(T* __restrict__ x, const T* __restrict__ cos,
                                                   const T* __restrict__ sin, int64_t B, int64_t H,
                                                   int64_t T_, int64_t D, int64_t sxb, int64_t sxh,
                                                   int64_t sxt, int64_t scb, int64_t sct) {
  using E = Elem<T>;
  const int64_t half = D / 2;
  const int64_t chunks = half / VEC;
  const int64_t total = B * H * T_ * chunks;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total;
       w += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = w % chunks;
    int64_t r = w / chunks;
    const int64_t t = r % T_;
    r /= T_;
    const int64_t h = r % H;
    const int64_t b = r / H;
    T* row = x + b * sxb + h * sxh + t * sxt;
    const T* cr = cos + b * scb + t * sct;
    const T* sr = sin + b * scb + t * sct;
    const int64_t i0 = c * VEC;
    T x1[VEC], x2[VEC], c1[VEC], c2[VEC], s1[VEC], s2[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      x1[j] = row[i0 + j];
      x2[j] = row[i0 + half + j];
      c1[j] = cr[i0 + j];
      c2[j] = cr[i0 + half + j];
      s1[j] = sr[i0 + j];
      s2[j] = sr[i0 + half + j];
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = E::to_f(x1[j]), bq = E::to_f(x2[j]);
      // first half:  x1*cos + (-x2)*sin ; second half: x2*cos + x1*sin
      const float lo = E::round(__fadd_rn(E::round(__fmul_rn(a, E::to_f(c1[j]))),
                                          E::round(__fmul_rn(-bq, E::to_f(s1[j])))));
      const float hi = E::round(__fadd_rn(E::round(__fmul_rn(bq, E::to_f(c2[j]))),
                                          E::round(__fmul_rn(a, E::to_f(s2[j])))));
      row[i0 + j] = E::from_f(lo);
      row[i0 + half + j] = E::from_f(hi);
    }
  }
}

// 16-bit types, rows on 16-byte boundaries, D/2 a multiple of 8: each thread moves one 16-byte
// vector of x from each half of a row (and the matching cos/sin vectors) with single loads and
// stores. Same arithmetic as rope_kernel.
template <typename T>
__global__ void __launch_bounds__(256) rope_vec16_kernel(T* __restrict__ x, const T* __restrict__ cos,
                                                         const T* __restrict__ sin, int64_t B, int64_t H,
                                                         int64_t T_, int64_t D, int64_t sxb, int64_t sxh,
                                                         int64_t sxt, int64_t scb, int64_t sct) {
  using E = Elem<T>;
  const int64_t half = D / 2;
  const int64_t chunks = half / 8;
  const int64_t total = B * H * T_ * chunks;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = w % chunks;
    int64_t r = w / chunks;
    const int64_t t = r % T_;
    r /= T_;
    const int64_t h = r % H;
    const int64_t b = r / H;
    T* row = x + b * sxb + h * sxh + t * sxt + c * 8;
    const T* cr = cos + b * scb + t * sct + c * 8;
    const T* sr = sin + b * scb + t * sct + c * 8;
    uint4 vx1 = *reinterpret_cast<const uint4*>(row);
    uint4 vx2 = *reinterpret_cast<const uint4*>(row + half);
    const uint4 vc1 = __ldg(reinterpret_cast<const uint4*>(cr));
    const uint4 vc2 = __ldg(reinterpret_cast<const uint4*>(cr + half));
    const uint4 vs1 = __ldg(reinterpret_cast<const uint4*>(sr));
    const uint4 vs2 = __ldg(reinterpret_cast<const uint4*>(sr + half));
    T* x1 = reinterpret_cast<T*>(&vx1);
    T* x2 = reinterpret_cast<T*>(&vx2);
    const T* c1 = reinterpret_cast<const T*>(&vc1);
    const T* c2 = reinterpret_cast<const T*>(&vc2);
    const T* s1 = reinterpret_cast<const T*>(&vs1);
    const T* s2 = reinterpret_cast<const T*>(&vs2);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = E::to_f(x1[j]), bq = E::to_f(x2[j]);
      const float lo = E::round(__fadd_rn(E::round(__fmul_rn(a, E::to_f(c1[j]))),
                                          E::round(__fmul_rn(-bq, E::to_f(s1[j])))));
      const float hi = E::round(__fadd_rn(E::round(__fmul_rn(bq, E::to_f(c2[j]))),
                                          E::round(__fmul_rn(a, E::to_f(s2[j])))));
      x1[j] = E::from_f(lo);
      x2[j] = E::from_f(hi);
    }
    *reinterpret_cast<uint4*>(row) = vx1;
    *reinterpret_cast<uint4*>(row + half) = vx2;
  }
}

// Up to two tensors (e.g. a layer's q and k) of D = 128 with one cos/sin table: a thread owns one
// 16-byte chunk pair (i, i + 64) of one position, loads that position's cos/sin vectors once and
// rotates the chunk of every head of both tensors (heads unrolled by 4 so their loads overlap).
// Same arithmetic as rope_vec16_kernel; the cos/sin traffic drops from once per head to once per
// position.
struct RopeTensor {
  void* x;
  int64_t heads, sxh, sxt;
};
template <typename T>
__device__ __forceinline__ void rope_chunk(T* row1, T* row2, const uint4& vc1, const uint4& vc2, const uint4& vs1,
                                           const uint4& vs2) {
  using E = Elem<T>;
  uint4 vx1 = *reinterpret_cast<const uint4*>(row1);
  uint4 vx2 = *reinterpret_cast<const uint4*>(row2);
  T* x1 = reinterpret_cast<T*>(&vx1);
  T* x2 = reinterpret_cast<T*>(&vx2);
  const T* c1 = reinterpret_cast<const T*>(&vc1);
  const T* c2 = reinterpret_cast<const T*>(&vc2);
  const T* s1 = reinterpret_cast<const T*>(&vs1);
  const T* s2 = reinterpret_cast<const T*>(&vs2);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = E::to_f(x1[j]), bq = E::to_f(x2[j]);
    const float lo = E::round(__fadd_rn(E::round(__fmul_rn(a, E::to_f(c1[j]))),
                                        E::round(__fmul_rn(-bq, E::to_f(s1[j])))));
    const float hi = E::round(__fadd_rn(E::round(__fmul_rn(bq, E::to_f(c2[j]))),
                                        E::round(__fmul_rn(a, E::to_f(s2[j])))));
    x1[j] = E::from_f(lo);
    x2[j] = E::from_f(hi);
  }
  *reinterpret_cast<uint4*>(row1) = vx1;
  *reinterpret_cast<uint4*>(row2) = vx2;
}
template <typename T>
__global__ void __launch_bounds__(256) rope_heads_kernel(RopeTensor t0, RopeTensor t1, const T* __restrict__ cos,
                                                         const T* __restrict__ sin, int64_t T_, int64_t sct) {
  const int64_t total = T_ * 8;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = w % 8, t = w / 8;
    const T* cr = cos + t * sct + c * 8;
    const T* sr = sin + t * sct + c * 8;
    const uint4 vc1 = __ldg(reinterpret_cast<const uint4*>(cr));
    const uint4 vc2 = __ldg(reinterpret_cast<const uint4*>(cr + 64));
    const uint4 vs1 = __ldg(reinterpret_cast<const uint4*>(sr));
    const uint4 vs2 = __ldg(reinterpret_cast<const uint4*>(sr + 64));
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const RopeTensor& rt = u ? t1 : t0;
      if (!rt.x) continue;
      T* base = static_cast<T*>(rt.x) + t * rt.sxt + c * 8;
#pragma unroll 4
      for (int64_t h = 0; h < rt.heads; ++h) rope_chunk<T>(base + h * rt.sxh, base + h * rt.sxh + 64, vc1, vc2, vs1, vs2);
    }
  }
}

template <typename T>
int launch_rope(void* x, int64_t B, int64_t H, int64_t T_, int64_t D, int64_t sxb, int64_t sxh,
                int64_t sxt, const void* cos, const void* sin, int64_t scb, int64_t sct,
                cudaStream_t stream) {
  const int64_t half = D / 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if constexpr (sizeof(T) == 2) {
    if (B == 1 && D == 128 && H > 1 && al16(x) && al16(cos) && al16(sin) && (sxh * 2) % 16 == 0 &&
        (sxt * 2) % 16 == 0 && (sct * 2) % 16 == 0) {
      if (T_ == 0) return BB_OK;
      const int64_t grid = std::min<int64_t>(cdiv(T_ * 8, 256), (int64_t)num_sms() * 16);
      rope_heads_kernel<T><<<grid, 256, 0, stream>>>(RopeTensor{x, H, sxh, sxt}, RopeTensor{nullptr, 0, 0, 0},
                                                     static_cast<const T*>(cos), static_cast<const T*>(sin), T_, sct);
      BB_CHECK_LAUNCH("rope_heads_kernel");
      return BB_OK;
    }
    if (half % 8 == 0 && al16(x) && al16(cos) && al16(sin) && (sxb * 2) % 16 == 0 && (sxh * 2) % 16 == 0 &&
        (sxt * 2) % 16 == 0 && (scb * 2) % 16 == 0 && (sct * 2) % 16 == 0) {
      const int64_t total = B * H * T_ * (half / 8);
      if (total == 0) return BB_OK;
      const int64_t grid = std::min<int64_t>(cdiv(total, 256), (int64_t)num_sms() * 16);
      rope_vec16_kernel<T><<<grid, 256, 0, stream>>>(static_cast<T*>(x), static_cast<const T*>(cos),
                                                      static_cast<const T*>(sin), B, H, T_, D, sxb, sxh, sxt,
                                                      scb, sct);
      BB_CHECK_LAUNCH("rope_vec16_kernel");
      return BB_OK;
    }
  }
  const int vec = (half % 8 == 0) ? 8 : ((half % 4 == 0) ? 4 : 1);
  const int64_t total = B * H * T_ * (half / vec);
  if (total == 0) return BB_OK;
  const int64_t grid = std::min<int64_t>(cdiv(total, 256), (int64_t)num_sms() * 16);
  T* xp = static_cast<T*>(x);
  const T* cp = static_cast<const T*>(cos);
  const T* sp = static_cast<const T*>(sin);
  if (vec == 8)
    rope_kernel<T, 8><<<grid, 256, 0, stream>>>(xp, cp, sp, B, H, T_, D, sxb, sxh, sxt, scb, sct);
  else if (vec == 4)
    rope_kernel<T, 4><<<grid, 256, 0, stream>>>(xp, cp, sp, B, H, T_, D, sxb, sxh, sxt, scb, sct);
  else
    rope_kernel<T, 1><<<grid, 256, 0, stream>>>(xp, cp, sp, B, H, T_, D, sxb, sxh, sxt, scb, sct);
  BB_CHECK_LAUNCH("rope_kernel");
  return BB_OK;
}

}  // namespace

// q and k of one layer (batch 1, D = 128, 16-bit, rows on 16-byte boundaries) with one table in one
// launch; returns BB_ERR_UNSUPPORTED when the layout does not qualify (callers then rotate each).
int rope_pair_inplace(void* q, int64_t hq, int64_t sqh, int64_t sqt, void* k, int64_t hk, int64_t skh, int64_t skt,
                      int dtype, int64_t T_, int64_t D, const void* cos, const void* sin, int64_t sct,
                      cudaStream_t stream) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (D != 128 || (dtype != BB_BF16 && dtype != BB_F16) || !al16(q) || !al16(k) || !al16(cos) || !al16(sin) ||
      (sqh * 2) % 16 || (sqt * 2) % 16 || (skh * 2) % 16 || (skt * 2) % 16 || (sct * 2) % 16)
    return BB_ERR_UNSUPPORTED;
  if (T_ == 0) return BB_OK;
  const int64_t grid = std::min<int64_t>(cdiv(T_ * 8, 256), (int64_t)num_sms() * 16);
  const RopeTensor a{q, hq, sqh, sqt}, b{k, hk, skh, skt};
  if (dtype == BB_BF16)
    rope_heads_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(a, b, static_cast<const __nv_bfloat16*>(cos),
                                                               static_cast<const __nv_bfloat16*>(sin), T_, sct);
  else
    rope_heads_kernel<__half><<<grid, 256, 0, stream>>>(a, b, static_cast<const __half*>(cos),
                                                        static_cast<const __half*>(sin), T_, sct);
  BB_CHECK_LAUNCH("rope_heads_kernel");
  return BB_OK;
}

int rope_inplace(void* x, int dtype, int64_t B, int64_t H, int64_t T_, int64_t D, int64_t sxb,
                 int64_t sxh, int64_t sxt, const void* cos, const void* sin, int64_t scb,
                 int64_t sct, cudaStream_t stream) {
  if (!x || !cos || !sin) return fail(BB_ERR_ARG, "rope: null pointer");
  if (B < 0 || H < 0 || T_ < 0 || D <= 0 || (D & 1)) return fail(BB_ERR_SHAPE, "rope: bad shape (D must be even)");
  switch (dtype) {
    case BB_BF16:
      return launch_rope<__nv_bfloat16>(x, B, H, T_, D, sxb, sxh, sxt, cos, sin, scb, sct, stream);
    case BB_F16:
      return launch_rope<__half>(x, B, H, T_, D, sxb, sxh, sxt, cos, sin, scb, sct, stream);
    case BB_F32:
      return launch_rope<float>(x, B, H, T_, D, sxb, sxh, sxt, cos, sin, scb, sct, stream);
    default:
      return fail(BB_ERR_DTYPE, "rope: dtype must be f16, bf16 or f32");
  }
}

}  // namespace bb
