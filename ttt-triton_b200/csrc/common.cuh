// Shared device helpers for the TTT dual-form scan kernels (sm_100a).
//
// Layout conventions (all kernels): one (batch, head) pair is a "stream"; stream
// s = b * NH + h. Activations are [B, NH, NC, CS, F] contiguous, eta is
// [B, NH, NC, CS, CS], inner states are fp32 [B, NH, rows, cols].
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ttt {

enum DType : int { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

constexpr float kLnEps = 1e-8f;       // ops/ttt_utils.py:4,21
constexpr float kReadoutEps = 1e-6f;  // kernels/mlp_cached_readout.py:99

// ----------------------------------------------------------------- typed element access
__device__ __forceinline__ float ld_elem(const void* p, long long i, int dt) {
  if (dt == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_elem(void* p, long long i, int dt, float v) {
  if (dt == DT_BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else if (dt == DT_F16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<float*>(p)[i] = v;
  }
}

// Copy n elements of a typed global array (offset base) into fp32 shared memory.
__device__ __forceinline__ void load_tile(float* dst, const void* src, long long base, int n, int dt) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = ld_elem(src, base + i, dt);
}

__device__ __forceinline__ void store_tile(void* dst, long long base, const float* src, int n, int dt) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) st_elem(dst, base + i, dt, src[i]);
}

__device__ __forceinline__ void copy_f32(float* dst, const float* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// ----------------------------------------------------------------- block matmul (fp32 FMA)
// C[m][n] = alpha * sum_k A(m,k) B(k,n) + beta * C[m][n]   (beta == 0 never reads C)
// A(m,k) = TA ? A[k*lda + m] : A[m*lda + k];  B(k,n) = TB ? B[n*ldb + k] : B[k*ldb + n]
// Pointers are generic (shared or global). M and N must be even. The whole block
// participates; callers synchronise before (inputs ready) and after (outputs ready).
// Every output element is owned by one thread, and the owner depends only on (M, N) (and
// the block size), so two calls with the same (M, N) may update the same C without a
// barrier between.
// Shared-memory banks: with a transposed B the lanes of a warp read B[n*ldb + k] at one k
// and n two apart, so for ldb a multiple of 16 floats they all fall in one bank. Each thread
// then runs its k loop from its own offset (lane mod K) and wraps around, spreading the lanes
// over the banks (the order of the sum changes, not its terms). Pairs that sit next to each
// other in memory (A(m, k), A(m+1, k) of a transposed A; B(k, n), B(k, n+1) of a plain B)
// are read as one 8-byte load when their addresses allow it.
template <bool TA, bool TB, bool VA, bool VB>
__device__ __forceinline__ void block_mm_tile(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                              int m, int n, int K, int rot, float alpha, float beta) {
  float c00 = 0.f, c01 = 0.f, c10 = 0.f, c11 = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < K; ++kk) {
    int k = kk + rot;
    if (k >= K) k -= K;
    float a0, a1, b0, b1;
    if (TA) {
      if (VA) {
        const float2 a = *reinterpret_cast<const float2*>(A + (long long)k * lda + m);
        a0 = a.x;
        a1 = a.y;
      } else {
        a0 = A[(long long)k * lda + m];
        a1 = A[(long long)k * lda + m + 1];
      }
    } else {
      a0 = A[(long long)m * lda + k];
      a1 = A[(long long)(m + 1) * lda + k];
    }
    if (TB) {
      b0 = B[(long long)n * ldb + k];
      b1 = B[(long long)(n + 1) * ldb + k];
    } else if (VB) {
      const float2 b = *reinterpret_cast<const float2*>(B + (long long)k * ldb + n);
      b0 = b.x;
      b1 = b.y;
    } else {
      b0 = B[(long long)k * ldb + n];
      b1 = B[(long long)k * ldb + n + 1];
    }
    c00 = fmaf(a0, b0, c00);
    c01 = fmaf(a0, b1, c01);
    c10 = fmaf(a1, b0, c10);
    c11 = fmaf(a1, b1, c11);
  }
  float* c0 = C + (long long)m * ldc + n;
  float* c1 = c0 + ldc;
  if (beta == 0.f) {
    c0[0] = alpha * c00;
    c0[1] = alpha * c01;
    c1[0] = alpha * c10;
    c1[1] = alpha * c11;
  } else {
    c0[0] = fmaf(alpha, c00, beta * c0[0]);
    c0[1] = fmaf(alpha, c01, beta * c0[1]);
    c1[0] = fmaf(alpha, c10, beta * c1[0]);
    c1[1] = fmaf(alpha, c11, beta * c1[1]);
  }
}

// 4 x 4 output tile per thread (two loads per four FMAs instead of one per FMA): used when M
// and N are multiples of 4 and there are at least as many such tiles as threads.
template <bool TA, bool TB>
__device__ __forceinline__ void block_mm_tile4(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                               int m, int n, int K, int rot, float alpha, float beta) {
  float c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.f;
#pragma unroll 2
  for (int kk = 0; kk < K; ++kk) {
    int k = kk + rot;
    if (k >= K) k -= K;
    float a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = TA ? A[(long long)k * lda + m + i] : A[(long long)(m + i) * lda + k];
      b[i] = TB ? B[(long long)(n + i) * ldb + k] : B[(long long)k * ldb + n + i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) c[i][j] = fmaf(a[i], b[j], c[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float* ci = C + (long long)(m + i) * ldc + n;
#pragma unroll
    for (int j = 0; j < 4; ++j) ci[j] = beta == 0.f ? alpha * c[i][j] : fmaf(alpha, c[i][j], beta * ci[j]);
  }
}

template <bool TA, bool TB>
__device__ __forceinline__ void block_mm(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                         int M, int N, int K, float alpha, float beta) {
  const int rot = TB ? (threadIdx.x & 31) % K : 0;
  if ((M & 3) == 0 && (N & 3) == 0 && (M >> 2) * (N >> 2) >= (int)blockDim.x) {
    const int tn = N >> 2;
    const int tiles = (M >> 2) * tn;
    for (int t = threadIdx.x; t < tiles; t += blockDim.x)
      block_mm_tile4<TA, TB>(C, ldc, A, lda, B, ldb, (t / tn) << 2, (t % tn) << 2, K, rot, alpha, beta);
    return;
  }
  const int tn = N >> 1;
  const int tiles = (M >> 1) * tn;
  // 8-byte loads need an even leading dimension and an 8-byte aligned base (m and n are even)
  const bool va = TA && (lda & 1) == 0 && (reinterpret_cast<uintptr_t>(A) & 7) == 0;
  const bool vb = !TB && (ldb & 1) == 0 && (reinterpret_cast<uintptr_t>(B) & 7) == 0;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const int m = (t / tn) << 1;
    const int n = (t % tn) << 1;
    if (va) {
      if (vb)
        block_mm_tile<TA, TB, true, true>(C, ldc, A, lda, B, ldb, m, n, K, rot, alpha, beta);
      else
        block_mm_tile<TA, TB, true, false>(C, ldc, A, lda, B, ldb, m, n, K, rot, alpha, beta);
    } else if (vb) {
      block_mm_tile<TA, TB, false, true>(C, ldc, A, lda, B, ldb, m, n, K, rot, alpha, beta);
    } else {
      block_mm_tile<TA, TB, false, false>(C, ldc, A, lda, B, ldb, m, n, K, rot, alpha, beta);
    }
  }
}

// ----------------------------------------------------------------- block matmul (TF32 tensor cores)
// The same product on mma.sync m16n8k16's TF32 sibling, m16n8k8 (fp32 operands rounded to
// TF32 -- 10 explicit mantissa bits, fp32 range -- and fp32 accumulation): for kernels whose
// activations are 16-bit, where the operands carry no more precision than that anyway (the
// reference's Triton tl.dot also multiplies fp32 operands in TF32). Each warp computes
// 16 x 16 output tiles (two m16n8 accumulators) in turn; M and N multiples of 16, K of 8.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32_16808(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Within each k-step of 8 the MMA's k slots t and t + 4 (t = lane % 4) carry k0 + 2t and
// k0 + 2t + 1 -- the same permutation of k for A and B, so the sum is unchanged -- which makes a
// lane's two A values (row-major A) or B values (B stored transposed) adjacent: one 8-byte
// shared-memory load instead of two scalar ones, at half the bank-conflict replays (tile rows
// here are multiples of 32 floats apart). VA / VB: take that 8-byte load.
template <bool TA, bool TB, bool VA, bool VB>
__device__ __forceinline__ void block_mm_tf32_impl(float* C, int ldc, const float* A, int lda, const float* B,
                                                   int ldb, int M, int N, int K, float alpha, float beta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int tn = N >> 4, tiles = (M >> 4) * tn;
  // strides: per k-step (sa, sb), to row m + 8 of A (ra8) and column n + 8 of B (rb8), to k + 1
  const int sa = TA ? 8 * lda : 8, ra8 = TA ? 8 : 8 * lda, ra1 = TA ? lda : 1;
  const int sb = TB ? 8 : 8 * ldb, rb8 = TB ? 8 * ldb : 8, rb1 = TB ? 1 : ldb;
  auto pair = [](const float* p, int step, bool vec) {
    if (vec) return *reinterpret_cast<const float2*>(p);
    return make_float2(p[0], p[step]);
  };
  for (int tile = warp; tile < tiles; tile += nw) {
    const int m0 = (tile / tn) << 4, n0 = (tile % tn) << 4;
    const float* pa = TA ? A + 2 * t * lda + m0 + g : A + (m0 + g) * lda + 2 * t;
    const float* pb = TB ? B + (n0 + g) * ldb + 2 * t : B + 2 * t * ldb + n0 + g;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 2
    for (int k0 = 0; k0 < K; k0 += 8, pa += sa, pb += sb) {
      const float2 a_lo = pair(pa, ra1, VA), a_hi = pair(pa + ra8, ra1, VA);  // rows m, m + 8
      const uint32_t a[4] = {to_tf32(a_lo.x), to_tf32(a_hi.x), to_tf32(a_lo.y), to_tf32(a_hi.y)};
      const float2 b_lo = pair(pb, rb1, VB), b_hi = pair(pb + rb8, rb1, VB);  // columns n, n + 8
      const uint32_t b0[2] = {to_tf32(b_lo.x), to_tf32(b_lo.y)};
      const uint32_t b1[2] = {to_tf32(b_hi.x), to_tf32(b_hi.y)};
      mma_tf32_16808(acc[0], a, b0);
      mma_tf32_16808(acc[1], a, b1);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float* c = C + (m0 + g + 8 * h) * ldc + n0 + 8 * j + 2 * t;
        const float v0 = acc[j][2 * h], v1 = acc[j][2 * h + 1];
        if (beta == 0.f) {
          c[0] = alpha * v0;
          c[1] = alpha * v1;
        } else {
          c[0] = fmaf(alpha, v0, beta * c[0]);
          c[1] = fmaf(alpha, v1, beta * c[1]);
        }
      }
  }
}

template <bool TA, bool TB>
__device__ __forceinline__ void block_mm_tf32(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                              int M, int N, int K, float alpha, float beta) {
  // 8-byte loads need an even leading dimension and an 8-byte aligned base
  const bool va = !TA && (lda & 1) == 0 && (reinterpret_cast<uintptr_t>(A) & 7) == 0;
  const bool vb = TB && (ldb & 1) == 0 && (reinterpret_cast<uintptr_t>(B) & 7) == 0;
  if (va) {
    if (vb)
      block_mm_tf32_impl<TA, TB, true, true>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
    else
      block_mm_tf32_impl<TA, TB, true, false>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
  } else if (vb) {
    block_mm_tf32_impl<TA, TB, false, true>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
  } else {
    block_mm_tf32_impl<TA, TB, false, false>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
  }
}

// block_mm on the TF32 tensor cores when TC and the shape allows it, else on fp32 FMA.
template <bool TC, bool TA, bool TB>
__device__ __forceinline__ void block_mm_sel(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                             int M, int N, int K, float alpha, float beta) {
  if (TC && (M & 15) == 0 && (N & 15) == 0 && (K & 7) == 0)
    block_mm_tf32<TA, TB>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
  else
    block_mm<TA, TB>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
}

// The same as a real call, for the general backward: it runs some fifty products per
// mini-batch, and inlined they kept its 255 registers busy and spilled; as calls their
// registers are free again between products (128 registers, no spills; the forward, with
// fewer products, is faster inlined).
//
// Inside the call the operand pointers are generic, so their loads would be generic loads
// (tracked like global ones) even for the shared-memory tiles; operands found in shared
// memory are rebased onto the dynamic shared array, which makes them shared-memory loads
// (the general kernels keep every shared tile in that array: they declare no static ones).
__device__ __forceinline__ const float* as_shared(const float* p) {
  extern __shared__ float ttt_dyn_smem[];
  const uint32_t off = (uint32_t)__cvta_generic_to_shared(p) - (uint32_t)__cvta_generic_to_shared(ttt_dyn_smem);
  return ttt_dyn_smem + (off >> 2);
}

template <bool TC, bool TA, bool TB>
__device__ __noinline__ void block_mm_call(float* C, int ldc, const float* A, int lda, const float* B, int ldb,
                                           int M, int N, int K, float alpha, float beta) {
  const bool ash = __isShared(A), bsh = __isShared(B);
  if (ash && bsh)
    block_mm_sel<TC, TA, TB>(C, ldc, as_shared(A), lda, as_shared(B), ldb, M, N, K, alpha, beta);
  else if (ash)
    block_mm_sel<TC, TA, TB>(C, ldc, as_shared(A), lda, B, ldb, M, N, K, alpha, beta);
  else if (bsh)
    block_mm_sel<TC, TA, TB>(C, ldc, A, lda, as_shared(B), ldb, M, N, K, alpha, beta);
  else
    block_mm_sel<TC, TA, TB>(C, ldc, A, lda, B, ldb, M, N, K, alpha, beta);
}

// ----------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ----------------------------------------------------------------- GELU (tanh form)
// Forward and its exact derivative, as F.gelu(approximate="tanh") and its autograd
// (ops/ttt_mlp.py:16,28). tanhf is CUDA's own.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float t = tanhf(k0 * (x + k1 * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

// The reference's gelu_bwd with its truncated constants (ops/ttt_utils.py:51-54) and the
// exact derivative of that expression (what autograd applies to it).
__device__ __forceinline__ float gelu_bwd_ref(float x) {
  const float t = tanhf(0.79788456f * x * (1.f + 0.044715f * x * x));
  return 0.5f * x * ((1.f - t * t) * (0.79788456f + 0.1070322243f * x * x)) + 0.5f * (1.f + t);
}

__device__ __forceinline__ float gelu_bwd_ref_grad(float x) {
  const float a = 0.79788456f, c = 0.1070322243f, k = 0.044715f;
  const float t = tanhf(a * x * (1.f + k * x * x));
  const float dt = (1.f - t * t) * (a + 3.f * a * k * x * x);
  const float poly = a + c * x * x;
  return 0.5f * (1.f - t * t) * poly + 0.5f * x * (-2.f * t * dt * poly + (1.f - t * t) * 2.f * c * x) + 0.5f * dt;
}

// ----------------------------------------------------------------- row-wise LayerNorm pieces
// All row functions: one warp per row (rows strided by warp count), row width F.

// Row statistics: writes mean and 1/std (std = sqrt(var + eps), biased variance).
__device__ __forceinline__ void row_stats(const float* x, int F, float eps, float& mu, float& rstd, float& stdv) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int j = lane; j < F; j += 32) s += x[j];
  mu = warp_sum(s) / F;
  float v = 0.f;
  for (int j = lane; j < F; j += 32) {
    const float d = x[j] - mu;
    v += d * d;
  }
  stdv = sqrtf(warp_sum(v) / F + eps);
  rstd = 1.f / stdv;
}

// G = ln_fused_l2_bwd(Z + b, XV - XK) row by row (ops/ttt_utils.py:21-48). Z holds X W
// on entry and Z + b on exit (bias skipped when bvec is null); G receives the gradient.
// Optionally records each row's mean and std.
__device__ __forceinline__ void ln_fused_rows(float* Z, float* G, const float* bvec, const float* XV, const float* XK,
                                              const float* gam, const float* bet, int C, int F, float* mu_out,
                                              float* std_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < C; r += nw) {
    float* z = Z + r * F;
    if (bvec) {
      for (int j = lane; j < F; j += 32) z[j] += bvec[j];
      __syncwarp();
    }
    float mu, rstd, sd;
    row_stats(z, F, kLnEps, mu, rstd, sd);
    float s1 = 0.f, s2 = 0.f;
    for (int j = lane; j < F; j += 32) {
      const float xh = (z[j] - mu) * rstd;
      const float gh = (gam[j] * xh + bet[j] - (XV[r * F + j] - XK[r * F + j])) * gam[j];
      s1 += gh;
      s2 += gh * xh;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float inv = rstd / F;
    for (int j = lane; j < F; j += 32) {
      const float xh = (z[j] - mu) * rstd;
      const float gh = (gam[j] * xh + bet[j] - (XV[r * F + j] - XK[r * F + j])) * gam[j];
      G[r * F + j] = (F * gh - s1 - xh * s2) * inv;
    }
    if (lane == 0 && mu_out) {
      mu_out[r] = mu;
      std_out[r] = sd;
    }
  }
}

// Backward of G = ln_fused_l2_bwd(Z, T) for every row, given dG (hand derivation of
// autograd through ops/ttt_utils.py:21-48). Z includes its bias; mu/sd are its row
// statistics. Writes dZ, dT (= -d_g_hat * gamma) and keeps d_g_hat in DGH for the
// gamma/beta column sums (ln_fused_bwd_cols); DXH is scratch.
__device__ __forceinline__ void ln_fused_bwd_rows(const float* Z, const float* mu1, const float* sd1, const float* G,
                                                  const float* dG, const float* XV, const float* XK, const float* gam,
                                                  const float* bet, int C, int F, float* DXH, float* DGH, float* dT,
                                                  float* dZ) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < C; r += nw) {
    const float mu = mu1[r], sd = sd1[r], rstd = 1.f / sd;
    float sdG = 0.f, sdGx = 0.f, sgx = 0.f, sdGG = 0.f;
    for (int j = lane; j < F; j += 32) {
      const float xh = (Z[r * F + j] - mu) * rstd;
      const float gh = (gam[j] * xh + bet[j] - (XV[r * F + j] - XK[r * F + j])) * gam[j];
      const float d = dG[r * F + j];
      sdG += d;
      sdGx += d * xh;
      sgx += gh * xh;
      sdGG += d * G[r * F + j];
    }
    sdG = warp_sum(sdG);
    sdGx = warp_sum(sdGx);
    sgx = warp_sum(sgx);
    sdGG = warp_sum(sdGG);
    const float inv = rstd / F;
    const float dstd = -sdGG * rstd;
    float sx = 0.f, sxx = 0.f;
    for (int j = lane; j < F; j += 32) {
      const float xh = (Z[r * F + j] - mu) * rstd;
      const float gh = (gam[j] * xh + bet[j] - (XV[r * F + j] - XK[r * F + j])) * gam[j];
      const float d = dG[r * F + j];
      const float dgh = (F * d - sdG - xh * sdGx) * inv;
      const float dxh = -(d * sgx + gh * sdGx) * inv + dgh * gam[j] * gam[j];
      DXH[r * F + j] = dxh;
      DGH[r * F + j] = dgh;
      dT[r * F + j] = -dgh * gam[j];
      sx += dxh;
      sxx += dxh * xh;
    }
    sx = warp_sum(sx);
    sxx = warp_sum(sxx);
    for (int j = lane; j < F; j += 32) {
      const float xh = (Z[r * F + j] - mu) * rstd;
      dZ[r * F + j] = (F * DXH[r * F + j] - sx - xh * sxx) * inv + dstd * xh / F;
    }
  }
}

// gamma / beta gradient contributions of the fused-LN backward, summed over rows.
__device__ __forceinline__ void ln_fused_bwd_cols(const float* Z, const float* mu1, const float* sd1, const float* DGH,
                                                  const float* XV, const float* XK, const float* gam, const float* bet,
                                                  int C, int F, float* dgam, float* dbet) {
  for (int j = threadIdx.x; j < F; j += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int r = 0; r < C; ++r) {
      const float xh = (Z[r * F + j] - mu1[r]) / sd1[r];
      const float go = gam[j] * xh + bet[j] - (XV[r * F + j] - XK[r * F + j]);
      const float dgh = DGH[r * F + j];
      a += dgh * (go + gam[j] * xh);
      b += dgh * gam[j];
    }
    dgam[j] += a;
    dbet[j] += b;
  }
}

// Readout LayerNorm backward: Zb (bias added in place when bvec is set) becomes x_bar,
// dZb = d LN / d Zb given dO (rows), gamma applied.
__device__ __forceinline__ void readout_ln_bwd_rows(float* Zb, const float* bvec, const float* dO, const float* gam,
                                                    int C, int F, float* dZb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < C; r += nw) {
    float* z = Zb + r * F;
    if (bvec) {
      for (int j = lane; j < F; j += 32) z[j] += bvec[j];
      __syncwarp();
    }
    float mu, rstd, sd;
    row_stats(z, F, kLnEps, mu, rstd, sd);
    float s1 = 0.f, s2 = 0.f;
    for (int j = lane; j < F; j += 32) {
      const float xh = (z[j] - mu) * rstd;
      const float g = dO[r * F + j] * gam[j];
      s1 += g;
      s2 += g * xh;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    __syncwarp();
    for (int j = lane; j < F; j += 32) {
      const float xh = (z[j] - mu) * rstd;
      const float g = dO[r * F + j] * gam[j];
      dZb[r * F + j] = (F * g - s1 - xh * s2) * (rstd / F);
      z[j] = xh;
    }
  }
}

// gamma / beta gradient of the readout LayerNorm: sums over rows of dO * x_bar and dO.
__device__ __forceinline__ void readout_ln_bwd_cols(const float* dO, const float* xbar, int C, int F, float* dgam,
                                                    float* dbet) {
  for (int j = threadIdx.x; j < F; j += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int r = 0; r < C; ++r) {
      a += dO[r * F + j] * xbar[r * F + j];
      b += dO[r * F + j];
    }
    dgam[j] += a;
    dbet[j] += b;
  }
}

// Readout forward: out = XQ + LN(Zb + b) written to global (typed), one warp per row.
__device__ __forceinline__ void readout_ln_store_rows(float* Zb, const float* bvec, const float* XQ, const float* gam,
                                                      const float* bet, int C, int F, float eps, void* out,
                                                      long long base, int dt_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < C; r += nw) {
    float* z = Zb + r * F;
    if (bvec) {
      for (int j = lane; j < F; j += 32) z[j] += bvec[j];
      __syncwarp();
    }
    float mu, rstd, sd;
    row_stats(z, F, eps, mu, rstd, sd);
    for (int j = lane; j < F; j += 32)
      st_elem(out, base + r * F + j, dt_out, XQ[r * F + j] + gam[j] * (z[j] - mu) * rstd + bet[j]);
  }
}

// acc[j] = sum_c w[c] * X[c][j] for j < N (one thread per column).
__device__ __forceinline__ void weighted_colsum(float* acc, const float* w, const float* X, int C, int N) {
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    float a = 0.f;
    for (int c = 0; c < C; ++c) a += w[c] * X[c * N + j];
    acc[j] = a;
  }
}

}  // namespace ttt
