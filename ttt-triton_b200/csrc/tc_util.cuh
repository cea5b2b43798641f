// Helpers shared by the tensor-core kernels: token-major row reductions, 16-bit tile
// unpacking, A-fragment construction from accumulator tiles, and the GELU pieces of the
// MLP on Blackwell's paired fp32 pipe.
#pragma once

#include "mma.cuh"

namespace ttt {

// Sum over the 16 lanes of a half-warp (one token's 64 features, 4 per lane).
__device__ __forceinline__ float red16(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  return v;
}

// Four consecutive 16-bit values -> fp32.
template <typename T>
__device__ __forceinline__ void unpack4(const uint8_t* src, float* v) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  const float2 a = Half2<T>::unpack(u.x), b = Half2<T>::unpack(u.y);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

// A fragment of scale * X^T for a 16 x 16 tile X held as two accumulator tiles
// (columns 0-7 and 8-15).
template <typename T>
__device__ __forceinline__ void transpose_afrag(uint32_t* a, const float (*X)[4], float scale) {
  using H = Half2<T>;
  a[0] = movm_t(H::pack(scale * X[0][0], scale * X[0][1]));
  a[1] = movm_t(H::pack(scale * X[1][0], scale * X[1][1]));
  a[2] = movm_t(H::pack(scale * X[0][2], scale * X[0][3]));
  a[3] = movm_t(H::pack(scale * X[1][2], scale * X[1][3]));
}

// A fragment of scale * X for the same two-tile 16 x 16 X.
template <typename T>
__device__ __forceinline__ void direct_afrag(uint32_t* a, const float (*X)[4], float scale) {
  using H = Half2<T>;
  a[0] = H::pack(scale * X[0][0], scale * X[0][1]);
  a[1] = H::pack(scale * X[0][2], scale * X[0][3]);
  a[2] = H::pack(scale * X[1][0], scale * X[1][1]);
  a[3] = H::pack(scale * X[1][2], scale * X[1][3]);
}

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// gelu (F.gelu approximate="tanh") of a pair, on Blackwell's paired fp32 pipe.
__device__ __forceinline__ float2 gelu2(float2 x) {
  const float2 u = __fmul2_rn(x, x);
  const float2 a = __ffma2_rn(f2(0.044715f), u, f2(1.f));
  const float2 arg = __fmul2_rn(f2(0.7978845608f), __fmul2_rn(x, a));
  const float2 t = make_float2(tanh_fast(arg.x), tanh_fast(arg.y));
  const float2 hx = __fmul2_rn(f2(0.5f), x);
  return __ffma2_rn(hx, t, hx);
}

// gelu and the reference's gelu_bwd (ops/ttt_utils.py:51-54) of a pair, sharing one tanh:
// their tanh arguments differ only in the 10th digit of sqrt(2/pi), far below the
// hardware tanh's error. gelu_bwd is also the exact derivative of the tanh GELU (its
// constant 0.1070322243 is 3 * 0.044715 * sqrt(2/pi)), so it serves autograd's
// gelu'(x) too.
__device__ __forceinline__ void gelu2_and_bwd(float2 x, float2& g, float2& gp) {
  const float2 u = __fmul2_rn(x, x);
  const float2 a = __ffma2_rn(f2(0.044715f), u, f2(1.f));
  const float2 arg = __fmul2_rn(f2(0.7978845608f), __fmul2_rn(x, a));
  const float2 t = make_float2(tanh_fast(arg.x), tanh_fast(arg.y));
  const float2 hx = __fmul2_rn(f2(0.5f), x);
  g = __ffma2_rn(hx, t, hx);
  const float2 poly = __ffma2_rn(f2(0.1070322243f), u, f2(0.79788456f));
  const float2 omt2 = __ffma2_rn(make_float2(-t.x, -t.y), t, f2(1.f));
  const float2 base = __ffma2_rn(f2(0.5f), t, f2(0.5f));
  gp = __ffma2_rn(__fmul2_rn(hx, omt2), poly, base);
}

// Derivative of the reference's gelu_bwd expression (what autograd applies to it):
// with t = tanh(a x (1 + k x^2)), poly = a + c x^2 (c = 3 a k) and om = 1 - t^2,
//   d/dx gelu_bwd(x) = om * (poly + c x^2 - x t poly^2).
__device__ __forceinline__ float2 gelu2_bwd_grad(float2 x) {
  const float2 u = __fmul2_rn(x, x);
  const float2 a = __ffma2_rn(f2(0.044715f), u, f2(1.f));
  const float2 arg = __fmul2_rn(f2(0.79788456f), __fmul2_rn(x, a));
  const float2 t = make_float2(tanh_fast(arg.x), tanh_fast(arg.y));
  const float2 poly = __ffma2_rn(f2(0.1070322243f), u, f2(0.79788456f));
  const float2 om = __ffma2_rn(make_float2(-t.x, -t.y), t, f2(1.f));
  const float2 cx2 = __fmul2_rn(f2(0.1070322243f), u);
  const float2 xtp2 = __fmul2_rn(__fmul2_rn(x, t), __fmul2_rn(poly, poly));
  return __fmul2_rn(om, __fadd2_rn(__fadd2_rn(poly, cx2), make_float2(-xtp2.x, -xtp2.y)));
}

}  // namespace ttt
