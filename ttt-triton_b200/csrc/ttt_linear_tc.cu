// TTT-Linear forward on the tensor cores (mma.sync bf16/fp16, fp32 accumulate) for the
// benchmark shape: head dim F = 64, mini-batch CS = 16, 16-bit activations.
//
// One CTA (4 warps) per (batch, head) stream. The inner state is held transposed,
// S = W^T (64 x 64 fp32), in mma accumulator fragments for the whole sequence: warp w
// owns output features [16w, 16w + 16). Those fragments are used directly as the A
// operand of Z^T = S [XK; XQ]^T and receive the rank-16 update S -= G^T diag(e) XK as
// an accumulating mma, so the state never leaves the register file between mini-batches.
// Per mini-batch (ops/ttt_linear.py:8-54):
//   Z^T = S XK^T + b, T = XV - XK, G = ln_fused_l2_bwd(Z, T)     (LayerNorm over F:
//     per-warp shuffle reductions + one shared-memory exchange per statistic)
//   A = XQ XK^T, M = eta * (A + 1)     (A's accumulator layout is M^T's B-fragment layout)
//   Zbar^T = S XQ^T + b - G^T M^T,  XQW = XQ + LN(Zbar)
//   S -= G^T diag(eta[CS-1, :]) XK,  b -= eta[CS-1, :] G
// XQ / XK / XV / eta tiles are prefetched three mini-batches ahead with cp.async into
// XOR-swizzled shared memory and read with ldmatrix (plain and transposed).
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mma.cuh"
#include "params.cuh"

namespace ttt {
namespace lin_tc {

constexpr int F = 64, C = 16, NW = 4, NTHREADS = 128, NSTAGE = 3;
constexpr int TILE = C * F * 2;                    // one 16 x 64 16-bit tile
constexpr int ETA = C * C * 2;                     // one 16 x 16 16-bit tile
constexpr int STAGE = 3 * TILE + ETA;              // XQ, XK, XV, eta
constexpr int OFF_XQ = 0, OFF_XK = TILE, OFF_XV = 2 * TILE, OFF_ETA = 3 * TILE;
constexpr int OFF_OUT = NSTAGE * STAGE;            // output staging tile
constexpr int OFF_RED = OFF_OUT + TILE;            // 3 x [NW][C] float2 exchange buffers
constexpr int SMEM = OFF_RED + 3 * NW * C * 8;

template <typename T>
__device__ __forceinline__ void load_stage(uint8_t* st, const LinFwdParams& p, long long s, int n) {
  const int tid = threadIdx.x;
  const long long tb = (s * p.NC + n) * (long long)(C * F) * 2;  // byte offset of the mini-batch tile
  const int row = tid >> 3, ch = tid & 7;
  const uint32_t dst = smem_u32(st) + swz128(row, ch);
  cp_async16(dst + OFF_XQ, (const uint8_t*)p.XQ + tb + row * 128 + ch * 16);
  cp_async16(dst + OFF_XK, (const uint8_t*)p.XK + tb + row * 128 + ch * 16);
  cp_async16(dst + OFF_XV, (const uint8_t*)p.XV + tb + row * 128 + ch * 16);
  if (tid < 32) {
    const long long eb = (s * p.NC + n) * (long long)(C * C) * 2;
    cp_async16(smem_u32(st) + OFF_ETA + tid * 16, (const uint8_t*)p.eta + eb + tid * 16);
  }
}

// Sum over the 8 lanes sharing t = lane % 4 (the 16 feature rows a warp holds per token).
__device__ __forceinline__ float red_g(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// Column (token) statistics of a 64 x 16 fp32 tile spread over 4 warps in accumulator
// layout (tiles x[0], x[1] hold tokens 0-7 / 8-15). Chan's merge of per-warp (mean, M2).
__device__ __forceinline__ void col_stats(const float (*x)[4], float2* red, int warp, int g, int t, float* mu,
                                          float* rstd) {
  float2 part[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int nt = q >> 1, e = q & 1;
    const float m = red_g(x[nt][e] + x[nt][2 + e]) * (1.f / 16.f);
    const float d0 = x[nt][e] - m, d1 = x[nt][2 + e] - m;
    part[q] = make_float2(m, red_g(d0 * d0 + d1 * d1));
  }
  if (g == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) red[warp * C + 8 * (q >> 1) + 2 * t + (q & 1)] = part[q];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int tok = 8 * (q >> 1) + 2 * t + (q & 1);
    float2 v[NW];
    float m = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      v[w] = red[w * C + tok];
      m += v[w].x;
    }
    m *= 1.f / NW;
    float m2 = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) m2 += v[w].y + 16.f * (v[w].x - m) * (v[w].x - m);
    mu[q] = m;
    rstd[q] = 1.f / sqrtf(m2 * (1.f / F) + kLnEps);
  }
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS) linear_fwd_tc_kernel(LinFwdParams p) {
  using H = Half2<T>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  float2* red_a = reinterpret_cast<float2*>(smem + OFF_RED);
  float2* red_b = red_a + NW * C;
  float2* red_c = red_b + NW * C;
  const int f0 = 16 * warp + g, f1 = f0 + 8;  // the two feature rows this thread holds

  // ---- state: S = W^T rows [16w, 16w+16) in accumulator tiles over f_in
  float S[8][4];
  const float* Wi = p.W_init + s * F * F;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int fi = 8 * nt + 2 * t;
    S[nt][0] = Wi[fi * F + f0];
    S[nt][1] = Wi[(fi + 1) * F + f0];
    S[nt][2] = Wi[fi * F + f1];
    S[nt][3] = Wi[(fi + 1) * F + f1];
  }
  float bv0 = p.b_init[s * F + f0], bv1 = p.b_init[s * F + f1];
  const float gm0 = ld_elem(p.ln_w, (long long)h * F + f0, p.dt_ln), gm1 = ld_elem(p.ln_w, (long long)h * F + f1, p.dt_ln);
  const float bt0 = ld_elem(p.ln_b, (long long)h * F + f0, p.dt_ln), bt1 = ld_elem(p.ln_b, (long long)h * F + f1, p.dt_ln);

#pragma unroll
  for (int i = 0; i < NSTAGE - 1; ++i) {
    if (i < p.NC) load_stage<T>(smem + i * STAGE, p, s, i);
    cp_async_commit();
  }

  const int mi = lane >> 3, r8 = lane & 7;
  for (int n = 0; n < p.NC; ++n) {
    cp_async_wait<NSTAGE - 2>();
    __syncthreads();
    {
      const int nn = n + NSTAGE - 1;
      if (nn < p.NC) load_stage<T>(smem + (nn % NSTAGE) * STAGE, p, s, nn);
      cp_async_commit();
    }
    uint8_t* st = smem + (n % NSTAGE) * STAGE;
    const uint32_t sb = smem_u32(st);

    if (n % p.ckpt == 0) {  // state at the start of the group
      const long long k = s * p.K + n / p.ckpt;
      float* Wc = p.W_ckpt + k * F * F;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int fi = 8 * nt + 2 * t;
        Wc[fi * F + f0] = S[nt][0];
        Wc[(fi + 1) * F + f0] = S[nt][1];
        Wc[fi * F + f1] = S[nt][2];
        Wc[(fi + 1) * F + f1] = S[nt][3];
      }
      if (t == 0) {
        p.b_ckpt[k * F + f0] = bv0;
        p.b_ckpt[k * F + f1] = bv1;
      }
    }

    // ---- phase 1: Z^T = S [XK; XQ]^T (tiles 0,1 = XK tokens, 2,3 = XQ tokens), A = XQ XK^T
    float Z[4][4], Aa[2][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) Z[i][0] = Z[i][1] = Z[i][2] = Z[i][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) Aa[i][0] = Aa[i][1] = Aa[i][2] = Aa[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4] = {H::pack(S[2 * kk][0], S[2 * kk][1]), H::pack(S[2 * kk][2], S[2 * kk][3]),
                       H::pack(S[2 * kk + 1][0], S[2 * kk + 1][1]), H::pack(S[2 * kk + 1][2], S[2 * kk + 1][3])};
      uint32_t bk[4], bq[4], aq[4];
      const int tokB = (mi >> 1) * 8 + r8, chB = 2 * kk + (mi & 1);
      ldsm_x4(bk, sb + OFF_XK + swz128(tokB, chB));
      ldsm_x4(bq, sb + OFF_XQ + swz128(tokB, chB));
      ldsm_x4(aq, sb + OFF_XQ + swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1)));
      mma16816<T>(Z[0], a, bk);
      mma16816<T>(Z[1], a, bk + 2);
      mma16816<T>(Z[2], a, bq);
      mma16816<T>(Z[3], a, bq + 2);
      mma16816<T>(Aa[0], aq, bk);
      mma16816<T>(Aa[1], aq, bk + 2);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Z[i][0] += bv0;
      Z[i][1] += bv0;
      Z[i][2] += bv1;
      Z[i][3] += bv1;
    }
    // XV, XK, XQ in the Z^T accumulator layout (rows f, columns tokens)
    float Tg[2][4], Xq[2][4];
    {
      uint32_t v[4], k[4], q[4];
      const uint32_t off = swz128((mi >> 1) * 8 + r8, 2 * warp + (mi & 1));
      ldsm_x4_t(v, sb + OFF_XV + off);
      ldsm_x4_t(k, sb + OFF_XK + off);
      ldsm_x4_t(q, sb + OFF_XQ + off);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fv = H::unpack(v[j]), fk = H::unpack(k[j]), fq = H::unpack(q[j]);
        const int nt = j >> 1, hi = (j & 1) * 2;
        Tg[nt][hi] = fv.x - fk.x;
        Tg[nt][hi + 1] = fv.y - fk.y;
        Xq[nt][hi] = fq.x;
        Xq[nt][hi + 1] = fq.y;
      }
    }

    // ---- G = ln_fused_l2_bwd(Z, T) over the 64 features of each XK token
    float mu[4], rs[4];
    col_stats(Z, red_a, warp, g, t, mu, rs);
    float xh[2][4], gh[2][4];
    float2 part[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int nt = q >> 1, e = q & 1;
      xh[nt][e] = (Z[nt][e] - mu[q]) * rs[q];
      xh[nt][2 + e] = (Z[nt][2 + e] - mu[q]) * rs[q];
      gh[nt][e] = (gm0 * xh[nt][e] + bt0 - Tg[nt][e]) * gm0;
      gh[nt][2 + e] = (gm1 * xh[nt][2 + e] + bt1 - Tg[nt][2 + e]) * gm1;
      part[q] = make_float2(red_g(gh[nt][e] + gh[nt][2 + e]), red_g(gh[nt][e] * xh[nt][e] + gh[nt][2 + e] * xh[nt][2 + e]));
    }
    if (g == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) red_b[warp * C + 8 * (q >> 1) + 2 * t + (q & 1)] = part[q];
    }
    __syncthreads();
    float G[2][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int tok = 8 * (q >> 1) + 2 * t + (q & 1);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float2 v = red_b[w * C + tok];
        s1 += v.x;
        s2 += v.y;
      }
      const int nt = q >> 1, e = q & 1;
      const float inv = rs[q] * (1.f / F);
      G[nt][e] = (F * gh[nt][e] - s1 - xh[nt][e] * s2) * inv;
      G[nt][2 + e] = (F * gh[nt][2 + e] - s1 - xh[nt][2 + e] * s2) * inv;
    }

    // ---- state update S -= G^T diag(e) XK ; b -= e G (old S already consumed above)
    const T* erow = reinterpret_cast<const T*>(st + OFF_ETA) + (C - 1) * C;
    const float e0 = (float)erow[2 * t], e1 = (float)erow[2 * t + 1];
    const float e2 = (float)erow[2 * t + 8], e3 = (float)erow[2 * t + 9];
    {
      uint32_t aU[4] = {H::pack(-e0 * G[0][0], -e1 * G[0][1]), H::pack(-e0 * G[0][2], -e1 * G[0][3]),
                        H::pack(-e2 * G[1][0], -e3 * G[1][1]), H::pack(-e2 * G[1][2], -e3 * G[1][3])};
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm_x4_t(b, sb + OFF_XK + swz128((mi & 1) * 8 + r8, 2 * np + (mi >> 1)));
        mma16816<T>(S[2 * np], aU, b);
        mma16816<T>(S[2 * np + 1], aU, b + 2);
      }
      float d0 = e0 * G[0][0] + e1 * G[0][1] + e2 * G[1][0] + e3 * G[1][1];
      float d1 = e0 * G[0][2] + e1 * G[0][3] + e2 * G[1][2] + e3 * G[1][3];
      d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
      d0 += __shfl_xor_sync(0xffffffffu, d0, 2);
      d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
      d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
      bv0 -= d0;
      bv1 -= d1;
    }

    // ---- read-out: Zbar^T = (S XQ^T + b) - G^T M^T, M = eta * (XQ XK^T + 1)
    {
      uint32_t ev[4];
      ldsm_x4(ev, sb + OFF_ETA + ((mi & 1) * 8 + r8) * 32 + (mi >> 1) * 16);
      float M[2][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 eta2 = H::unpack(ev[j]);
        const int jt = j >> 1, hi = (j & 1) * 2;
        M[jt][hi] = eta2.x * (Aa[jt][hi] + 1.f);
        M[jt][hi + 1] = eta2.y * (Aa[jt][hi + 1] + 1.f);
      }
      uint32_t aG[4] = {H::pack(-G[0][0], -G[0][1]), H::pack(-G[0][2], -G[0][3]), H::pack(-G[1][0], -G[1][1]),
                        H::pack(-G[1][2], -G[1][3])};
      uint32_t bM0[2] = {H::pack(M[0][0], M[0][1]), H::pack(M[1][0], M[1][1])};
      uint32_t bM1[2] = {H::pack(M[0][2], M[0][3]), H::pack(M[1][2], M[1][3])};
      mma16816<T>(Z[2], aG, bM0);
      mma16816<T>(Z[3], aG, bM1);
    }
    float mu2[4], rs2[4];
    col_stats(Z + 2, red_c, warp, g, t, mu2, rs2);
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int nt = q >> 1, e = q & 1;
      const float y0 = Xq[nt][e] + gm0 * (Z[2 + nt][e] - mu2[q]) * rs2[q] + bt0;
      const float y1 = Xq[nt][2 + e] + gm1 * (Z[2 + nt][2 + e] - mu2[q]) * rs2[q] + bt1;
      Z[2 + nt][e] = y0;
      Z[2 + nt][2 + e] = y1;
    }
    o[0] = H::pack(Z[2][0], Z[2][1]);
    o[1] = H::pack(Z[2][2], Z[2][3]);
    o[2] = H::pack(Z[3][0], Z[3][1]);
    o[3] = H::pack(Z[3][2], Z[3][3]);
    // transpose back to [token][feature] in the staging tile (this warp's 16 columns)
    const uint32_t ob = smem_u32(smem + OFF_OUT);
    stsm_x4_t(ob + swz128((mi >> 1) * 8 + r8, 2 * warp + (mi & 1)), o);
    __syncwarp();
    {
      const int row = lane >> 1, ch = 2 * warp + (lane & 1);
      const uint4 v = *reinterpret_cast<const uint4*>(smem + OFF_OUT + swz128(row, ch));
      uint8_t* dst = (uint8_t*)p.out + (s * p.NC + n) * (long long)(C * F) * 2 + row * 128 + ch * 16;
      *reinterpret_cast<uint4*>(dst) = v;
    }
  }
  cp_async_wait<0>();

  float* Wl = p.W_last + s * F * F;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int fi = 8 * nt + 2 * t;
    Wl[fi * F + f0] = S[nt][0];
    Wl[(fi + 1) * F + f0] = S[nt][1];
    Wl[fi * F + f1] = S[nt][2];
    Wl[(fi + 1) * F + f1] = S[nt][3];
  }
  if (t == 0) {
    p.b_last[s * F + f0] = bv0;
    p.b_last[s * F + f1] = bv1;
  }
}

}  // namespace lin_tc

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int linear_fwd_fast(const LinFwdParams& p, cudaStream_t stream) {
  using namespace lin_tc;
  if (p.CS != C || p.F != F) return TTT_NOT_APPLICABLE;
  const int dt = p.dt_xq;
  if (dt != DT_BF16 && dt != DT_F16) return TTT_NOT_APPLICABLE;
  if (p.dt_xk != dt || p.dt_xv != dt || p.dt_eta != dt || p.dt_out != dt) return TTT_NOT_APPLICABLE;
  if (!aligned16(p.XQ) || !aligned16(p.XK) || !aligned16(p.XV) || !aligned16(p.eta) || !aligned16(p.out))
    return TTT_NOT_APPLICABLE;
  int rc;
  if (dt == DT_BF16) {
    rc = prepare_smem(linear_fwd_tc_kernel<__nv_bfloat16>, SMEM, "ttt_linear_fwd");
    if (rc) return rc;
    linear_fwd_tc_kernel<__nv_bfloat16><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(p);
  } else {
    rc = prepare_smem(linear_fwd_tc_kernel<__half>, SMEM, "ttt_linear_fwd");
    if (rc) return rc;
    linear_fwd_tc_kernel<__half><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(p);
  }
  return check_launch("ttt_linear_fwd");
}

}  // namespace ttt
