// TTT-Linear backward on the tensor cores for F = 64, CS = 16, 16-bit activations.
//
// Uses the per-mini-batch pre-activations Z = XK W_n + b_n (fp32) stored by the forward and
// walks the sequence once, last mini-batch first, starting from the final state. The
// state entering mini-batch n is recovered from the state after it by undoing the
// rank-16 update, W_n = W_{n+1} + XK^T (e G_n), b_n = b_{n+1} + e G_n, with G_n rebuilt
// from the stored Z_n. The per-step gradient is the hand derivation of autograd through
// ops/ttt_linear.py:8-54 (full CS x CS d_eta).
//
// One CTA of 8 warps per stream. Warp w owns columns [8w, 8w + 8) of every 64-wide
// product and of the fp32 state / carried gradient (W, b, dW, db in accumulator
// fragments); 16-bit copies of W_n and dW_{n+1} in shared memory serve the products that
// contract over output features. Row phases run token-major (16 lanes per token).
//   R1  G = ln_fused_l2_bwd(Z)                                  (rows)
//   M1  W += XK^T eG, b += 1^T eG; A = XQ XK^T, P = eta*(A+1); Zbar = XQ W + b - P G;
//       XK dW, G dW^T                                           (MMA)
//   R2  dZbar = LN backward of the read-out; dgamma/dbeta      (rows)
//   M2  dXQ, dP -> d_eta, dA; dG = -P^T dZbar - e*(XK dW + db); dW += XQ^T dZbar   (MMA)
//   R3  backward of G = ln_fused_l2_bwd(Z, XV - XK) -> dZ, dXV  (rows)
//   M3  dXK += dZ W^T - dT; dW += XK^T dZ; outputs              (MMA)
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "tc_util.cuh"

namespace ttt {
namespace lin_bwd_tc {

constexpr int F = 64, C = 16, NW = 8, NTHREADS = 32 * NW, NSTAGE = 3;
constexpr int TILE = C * F * 2;
constexpr int ETA = C * C * 2;
constexpr int OFF_XQ = 0, OFF_XK = TILE, OFF_XV = 2 * TILE, OFF_DO = 3 * TILE, OFF_ETA = 4 * TILE;
constexpr int OFF_ZS = OFF_ETA + ETA;                // fp32 [C][F] stored Z of the mini-batch
constexpr int STAGE = OFF_ZS + C * F * 4;            // 12800 bytes
constexpr int LD = F + 8;                            // fp32 row stride of the row-phase tiles
constexpr int OFF_ZB = NSTAGE * STAGE;               // fp32 [C][LD] Zbar
constexpr int OFF_GF = OFF_ZB + C * LD * 4;          // fp32 [C][LD] G
constexpr int OFF_DG = OFF_GF + C * LD * 4;          // fp32 [C][LD] dG
constexpr int OFF_DT = OFF_DG + C * LD * 4;          // fp32 [C][LD] dT
constexpr int OFF_G = OFF_DT + C * LD * 4;           // 16-bit swizzled tiles [C][F]
constexpr int OFF_EG = OFF_G + TILE;
constexpr int OFF_DZB = OFF_EG + TILE;
constexpr int OFF_DZ = OFF_DZB + TILE;
constexpr int OFF_WT = OFF_DZ + TILE;                // 16-bit [F][F] W_n (rows f_in), swizzled
constexpr int OFF_DWT = OFF_WT + F * F * 2;          // 16-bit [F][F] dW_{n+1}
constexpr int OFF_DE = OFF_DWT + F * F * 2;          // fp32 [NW][C] partial d e
constexpr int OFF_DETA = OFF_DE + NW * C * 4;        // fp32 [C][C] d eta
constexpr int OFF_RED = OFF_DETA + C * C * 4;        // fp32 [NW][2][F] final gamma/beta reduction
constexpr int SMEM = OFF_RED + NW * 2 * F * 4;

__device__ __forceinline__ void load_stage(uint8_t* st, const LinBwdParams& p, long long s, int n) {
  const int tid = threadIdx.x;
  const long long tb = (s * p.NC + n) * (long long)(C * F) * 2;
  const int row = (tid & 127) >> 3, ch = tid & 7;
  const uint32_t dst = smem_u32(st) + swz128(row, ch);
  const long long src = tb + row * 128 + ch * 16;
  if (tid < 128) {
    cp_async16(dst + OFF_XQ, (const uint8_t*)p.XQ + src);
    cp_async16(dst + OFF_XK, (const uint8_t*)p.XK + src);
    if (tid < 32) {
      const long long eb = (s * p.NC + n) * (long long)(C * C) * 2;
      cp_async16(smem_u32(st) + OFF_ETA + tid * 16, (const uint8_t*)p.eta + eb + tid * 16);
    }
  } else {
    cp_async16(dst + OFF_XV, (const uint8_t*)p.XV + src);
    cp_async16(dst + OFF_DO, (const uint8_t*)p.dout + src);
  }
  // stored Z: 4 KB = 256 chunks, one per thread
  const float* zsrc = p.Z_saved + (s * p.NC + n) * (long long)(C * F) + tid * 4;
  cp_async16(smem_u32(st) + OFF_ZS + tid * 16, zsrc);
}

// 16-bit copy of a warp's accumulator slice (rows f_in, columns 8w..8w+7) into a
// swizzled [64][64] tile.
template <typename T>
__device__ __forceinline__ void store_slice(uint8_t* tile, const float (*X)[4], int warp, int g, int t) {
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
    *reinterpret_cast<uint32_t*>(tile + swz128(16 * mt + g, warp) + 4 * t) = Half2<T>::pack(X[mt][0], X[mt][1]);
    *reinterpret_cast<uint32_t*>(tile + swz128(16 * mt + g + 8, warp) + 4 * t) = Half2<T>::pack(X[mt][2], X[mt][3]);
  }
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 2) linear_bwd_tc_kernel(LinBwdParams p) {
  using H = Half2<T>;
  extern __shared__ __align__(128) uint8_t smem[];
  // the warp index through redux.sync: provably warp-uniform, so what derives from it stays in
  // uniform registers (fewer spills at the 128-register bound)
  const int tid = threadIdx.x, warp = (int)__reduce_max_sync(0xffffffffu, threadIdx.x >> 5), lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  const int tk = tid >> 4, q = tid & 15;
  const int fc = 8 * warp + 2 * t;
  float* ZB = reinterpret_cast<float*>(smem + OFF_ZB);
  float* GF = reinterpret_cast<float*>(smem + OFF_GF);
  float* DG = reinterpret_cast<float*>(smem + OFF_DG);
  float* DT = reinterpret_cast<float*>(smem + OFF_DT);
  float* DE = reinterpret_cast<float*>(smem + OFF_DE);
  float* DETA = reinterpret_cast<float*>(smem + OFF_DETA);
  const uint32_t sG = smem_u32(smem + OFF_G), sEG = smem_u32(smem + OFF_EG);
  const uint32_t sDZB = smem_u32(smem + OFF_DZB), sDZ = smem_u32(smem + OFF_DZ);
  const uint32_t sWT = smem_u32(smem + OFF_WT), sDWT = smem_u32(smem + OFF_DWT);

  // state after the last mini-batch; carried gradients start at zero
  float W[4][4], Bc[4], dW[4][4], dB[4];
  {
    const float* Wl = p.W_last + s * F * F;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      W[mt][0] = Wl[(16 * mt + g) * F + fc];
      W[mt][1] = Wl[(16 * mt + g) * F + fc + 1];
      W[mt][2] = Wl[(16 * mt + g + 8) * F + fc];
      W[mt][3] = Wl[(16 * mt + g + 8) * F + fc + 1];
      dW[mt][0] = dW[mt][1] = dW[mt][2] = dW[mt][3] = 0.f;
    }
    Bc[0] = Bc[2] = p.b_last[s * F + fc];
    Bc[1] = Bc[3] = p.b_last[s * F + fc + 1];
    dB[0] = dB[1] = dB[2] = dB[3] = 0.f;
  }
  for (int i = tid; i < F * F / 8; i += NTHREADS) reinterpret_cast<uint4*>(smem + OFF_DWT)[i] = make_uint4(0, 0, 0, 0);
  float gm[4], bt[4], dgam[4] = {0.f, 0.f, 0.f, 0.f}, dbet[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    gm[j] = ld_elem(p.ln_w, (long long)h * F + 4 * q + j, p.dt_ln);
    bt[j] = ld_elem(p.ln_b, (long long)h * F + 4 * q + j, p.dt_ln);
  }
  const uint32_t ones = H::pack(1.f, 1.f);
  const uint32_t a_ones[4] = {ones, ones, ones, ones};

  // prefetch the last mini-batches first
#pragma unroll
  for (int i = 0; i < NSTAGE - 1; ++i) {
    const int n = p.NC - 1 - i;
    if (n >= 0) load_stage(smem + i * STAGE, p, s, n);
    cp_async_commit();
  }

  for (int it = 0; it < p.NC; ++it) {
    const int n = p.NC - 1 - it;
    cp_async_wait<NSTAGE - 2>();
    __syncthreads();
    {
      const int ii = it + NSTAGE - 1, nn = p.NC - 1 - ii;
      if (nn >= 0) load_stage(smem + (ii % NSTAGE) * STAGE, p, s, nn);
      cp_async_commit();
    }
    const uint8_t* st = smem + (it % NSTAGE) * STAGE;
    const uint32_t sb = smem_u32(st);
    const T* E = reinterpret_cast<const T*>(st + OFF_ETA);
    const long long xb = (s * p.NC + n) * (long long)(C * F);  // element offset of the mini-batch tile

    // ---------------- R1: G from the stored Z (token tk, features 4q..4q+3)
    float xh[4], gh[4], Gr[4], rstd;
    const uint32_t xo = swz128(tk, q >> 1) + (q & 1) * 8;
    {
      const float4 z4 = *reinterpret_cast<const float4*>(st + OFF_ZS + (tk * F + 4 * q) * 4);
      float z[4] = {z4.x, z4.y, z4.z, z4.w}, xv[4], xk[4];
      unpack4<T>(st + OFF_XV + xo, xv);
      unpack4<T>(st + OFF_XK + xo, xk);
      const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
      float d[4], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      rstd = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xh[j] = d[j] * rstd;
        gh[j] = (gm[j] * xh[j] + bt[j] - (xv[j] - xk[j])) * gm[j];
        s1 += gh[j];
        s2 += gh[j] * xh[j];
      }
      s1 = red16(s1);
      s2 = red16(s2);
      const float inv = rstd * (1.f / F);
#pragma unroll
      for (int j = 0; j < 4; ++j) Gr[j] = (F * gh[j] - s1 - xh[j] * s2) * inv;
      const float e = (float)E[(C - 1) * C + tk];
      *reinterpret_cast<uint2*>(smem + OFF_G + xo) = make_uint2(H::pack(Gr[0], Gr[1]), H::pack(Gr[2], Gr[3]));
      *reinterpret_cast<uint2*>(smem + OFF_EG + xo) =
          make_uint2(H::pack(e * Gr[0], e * Gr[1]), H::pack(e * Gr[2], e * Gr[3]));
      *reinterpret_cast<float4*>(GF + tk * LD + 4 * q) = make_float4(Gr[0], Gr[1], Gr[2], Gr[3]);
    }
    __syncthreads();

    // ---------------- M1
    float A1[2][4], XdW[4], GdWt[4], Zq[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t aNegP[4], aNegPT[4];
    {
      // state reversal (the forward subtracted XK^T (e G) and 1^T (e G))
      uint32_t beg[2];
      ldsm_x2_t(beg, sEG + swz128((lane & 8) + r8, warp));
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t axk[4];
        ldsm_x4_t(axk, sb + OFF_XK + swz128((mi >> 1) * 8 + r8, 2 * mt + (mi & 1)));
        mma16816<T>(W[mt], axk, beg);
      }
      mma16816<T>(Bc, a_ones, beg);
      store_slice<T>(smem + OFF_WT, W, warp, g, t);
      // A1 = XQ XK^T (both j tiles), Zq = XQ W_n, XdW = XK dW_{n+1}
#pragma unroll
      for (int i = 0; i < 2; ++i) A1[i][0] = A1[i][1] = A1[i][2] = A1[i][3] = 0.f;
      XdW[0] = XdW[1] = XdW[2] = XdW[3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t aq[4], ak[4], bk[4];
        const uint32_t aoff = swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
        ldsm_x4(aq, sb + OFF_XQ + aoff);
        ldsm_x4(ak, sb + OFF_XK + aoff);
        ldsm_x4(bk, sb + OFF_XK + swz128((mi >> 1) * 8 + r8, 2 * kk + (mi & 1)));
        mma16816<T>(A1[0], aq, bk);
        mma16816<T>(A1[1], aq, bk + 2);
        const uint32_t bw[2] = {movm_t(H::pack(W[kk][0], W[kk][1])), movm_t(H::pack(W[kk][2], W[kk][3]))};
        mma16816<T>(Zq, aq, bw);
        const uint32_t bd[2] = {movm_t(H::pack(dW[kk][0], dW[kk][1])), movm_t(H::pack(dW[kk][2], dW[kk][3]))};
        mma16816<T>(XdW, ak, bd);
      }
      // P = eta * (A1 + 1) in C layout; -P and -P^T as A fragments
      float P[2][4];
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        const float2 e0 = H::unpack(*reinterpret_cast<const uint32_t*>(E + g * C + 8 * jt + 2 * t));
        const float2 e1 = H::unpack(*reinterpret_cast<const uint32_t*>(E + (g + 8) * C + 8 * jt + 2 * t));
        P[jt][0] = e0.x * (A1[jt][0] + 1.f);
        P[jt][1] = e0.y * (A1[jt][1] + 1.f);
        P[jt][2] = e1.x * (A1[jt][2] + 1.f);
        P[jt][3] = e1.y * (A1[jt][3] + 1.f);
      }
      direct_afrag<T>(aNegP, P, -1.f);
      transpose_afrag<T>(aNegPT, P, -1.f);
      // Zbar = XQ W_n + b_n - P G  -> fp32 tile
      uint32_t bg[2];
      ldsm_x2_t(bg, sG + swz128((lane & 8) + r8, warp));
#pragma unroll
      for (int i = 0; i < 4; ++i) Zq[i] += Bc[i];
      mma16816<T>(Zq, aNegP, bg);
      *reinterpret_cast<float2*>(ZB + g * LD + fc) = make_float2(Zq[0], Zq[1]);
      *reinterpret_cast<float2*>(ZB + (g + 8) * LD + fc) = make_float2(Zq[2], Zq[3]);
      // G dW_{n+1}^T (columns f_in 8w..8w+7)
      GdWt[0] = GdWt[1] = GdWt[2] = GdWt[3] = 0.f;
#pragma unroll
      for (int kf = 0; kf < 4; ++kf) {
        uint32_t ag[4], bdt[2];
        ldsm_x4(ag, sG + swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1)));
        ldsm_x2(bdt, sDWT + swz128(8 * warp + r8, 2 * kf + (mi & 1)));
        mma16816<T>(GdWt, ag, bdt);
      }
    }
    __syncthreads();

    // ---------------- R2: read-out LayerNorm backward -> dZbar
    float dO4[4];
    {
      const float4 z4 = *reinterpret_cast<const float4*>(ZB + tk * LD + 4 * q);
      float z[4] = {z4.x, z4.y, z4.z, z4.w};
      unpack4<T>(st + OFF_DO + xo, dO4);
      const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
      float d[4], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rb = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
      float xb[4], gg[4], s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xb[j] = d[j] * rb;
        gg[j] = dO4[j] * gm[j];
        s1 += gg[j];
        s2 += gg[j] * xb[j];
        dgam[j] += dO4[j] * xb[j];
        dbet[j] += dO4[j];
      }
      s1 = red16(s1);
      s2 = red16(s2);
      float dz[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) dz[j] = (F * gg[j] - s1 - xb[j] * s2) * (rb * (1.f / F));
      *reinterpret_cast<uint2*>(smem + OFF_DZB + xo) = make_uint2(H::pack(dz[0], dz[1]), H::pack(dz[2], dz[3]));
    }
    __syncthreads();

    // ---------------- M2
    float dXQ[4] = {0.f, 0.f, 0.f, 0.f}, dXK[4];
    {
      float dP[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) dP[i][0] = dP[i][1] = dP[i][2] = dP[i][3] = 0.f;
#pragma unroll
      for (int kf = 0; kf < 4; ++kf) {
        uint32_t adz[4], bwt[2], bgt[4];
        ldsm_x4(adz, sDZB + swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1)));
        ldsm_x2(bwt, sWT + swz128(8 * warp + r8, 2 * kf + (mi & 1)));
        ldsm_x4(bgt, sG + swz128((mi >> 1) * 8 + r8, 2 * kf + (mi & 1)));
        mma16816<T>(dXQ, adz, bwt);   // dZbar W^T
        mma16816<T>(dP[0], adz, bgt);  // dZbar G^T (negated below)
        mma16816<T>(dP[1], adz, bgt + 2);
      }
      // dP -> d_eta (dual part), dA = dP * eta
      float dA[2][4];
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        const float2 e0 = H::unpack(*reinterpret_cast<const uint32_t*>(E + g * C + 8 * jt + 2 * t));
        const float2 e1 = H::unpack(*reinterpret_cast<const uint32_t*>(E + (g + 8) * C + 8 * jt + 2 * t));
        const float ev[4] = {e0.x, e0.y, e1.x, e1.y};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float v = -dP[jt][c];
          dA[jt][c] = v * ev[c];
          dP[jt][c] = v * (A1[jt][c] + 1.f);
        }
      }
      if (warp == 0) {
#pragma unroll
        for (int jt = 0; jt < 2; ++jt) {
          *reinterpret_cast<float2*>(DETA + g * C + 8 * jt + 2 * t) = make_float2(dP[jt][0], dP[jt][1]);
          *reinterpret_cast<float2*>(DETA + (g + 8) * C + 8 * jt + 2 * t) = make_float2(dP[jt][2], dP[jt][3]);
        }
      }
      // dG = -P^T dZbar - e (XK dW + db); d e partial (old db)
      const float eg0 = (float)E[(C - 1) * C + g], eg1 = (float)E[(C - 1) * C + g + 8];
      const float2 G0 = *reinterpret_cast<const float2*>(GF + g * LD + fc);
      const float2 G1 = *reinterpret_cast<const float2*>(GF + (g + 8) * LD + fc);
      float de0 = (XdW[0] + dB[0]) * G0.x + (XdW[1] + dB[1]) * G0.y;
      float de1 = (XdW[2] + dB[2]) * G1.x + (XdW[3] + dB[3]) * G1.y;
      de0 += __shfl_xor_sync(0xffffffffu, de0, 1);
      de0 += __shfl_xor_sync(0xffffffffu, de0, 2);
      de1 += __shfl_xor_sync(0xffffffffu, de1, 1);
      de1 += __shfl_xor_sync(0xffffffffu, de1, 2);
      if (t == 0) {
        DE[warp * C + g] = -de0;
        DE[warp * C + g + 8] = -de1;
      }
      float dGc[4] = {-eg0 * (XdW[0] + dB[0]), -eg0 * (XdW[1] + dB[1]), -eg1 * (XdW[2] + dB[2]),
                      -eg1 * (XdW[3] + dB[3])};
      uint32_t bdz[2];
      ldsm_x2_t(bdz, sDZB + swz128((lane & 8) + r8, warp));
      mma16816<T>(dGc, aNegPT, bdz);
      *reinterpret_cast<float2*>(DG + g * LD + fc) = make_float2(dGc[0], dGc[1]);
      *reinterpret_cast<float2*>(DG + (g + 8) * LD + fc) = make_float2(dGc[2], dGc[3]);
      // dXK = -e (G dW^T) + dA^T XQ ; dXQ += dO + dA XK
      dXK[0] = -eg0 * GdWt[0];
      dXK[1] = -eg0 * GdWt[1];
      dXK[2] = -eg1 * GdWt[2];
      dXK[3] = -eg1 * GdWt[3];
      uint32_t aDA[4], aDAT[4], bxq[2], bxk[2];
      direct_afrag<T>(aDA, dA, 1.f);
      transpose_afrag<T>(aDAT, dA, 1.f);
      ldsm_x2_t(bxq, sb + OFF_XQ + swz128((lane & 8) + r8, warp));
      ldsm_x2_t(bxk, sb + OFF_XK + swz128((lane & 8) + r8, warp));
      mma16816<T>(dXK, aDAT, bxq);
      mma16816<T>(dXQ, aDA, bxk);
      const float2 o0 = H::unpack(*reinterpret_cast<const uint32_t*>(st + OFF_DO + swz128(g, warp) + 4 * t));
      const float2 o1 = H::unpack(*reinterpret_cast<const uint32_t*>(st + OFF_DO + swz128(g + 8, warp) + 4 * t));
      dXQ[0] += o0.x;
      dXQ[1] += o0.y;
      dXQ[2] += o1.x;
      dXQ[3] += o1.y;
      // dW += XQ^T dZbar ; db += 1^T dZbar (after the old values were used above)
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t axq[4];
        ldsm_x4_t(axq, sb + OFF_XQ + swz128((mi >> 1) * 8 + r8, 2 * mt + (mi & 1)));
        mma16816<T>(dW[mt], axq, bdz);
      }
      mma16816<T>(dB, a_ones, bdz);
    }
    __syncthreads();

    // ---------------- R3: backward of G = ln_fused_l2_bwd(Z, XV - XK)
    {
      const float4 dg4 = *reinterpret_cast<const float4*>(DG + tk * LD + 4 * q);
      const float dG[4] = {dg4.x, dg4.y, dg4.z, dg4.w};
      float xv[4], xk[4];
      unpack4<T>(st + OFF_XV + xo, xv);
      unpack4<T>(st + OFF_XK + xo, xk);
      float sdG = 0.f, sdGx = 0.f, sgx = 0.f, sdGG = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sdG += dG[j];
        sdGx += dG[j] * xh[j];
        sgx += gh[j] * xh[j];
        sdGG += dG[j] * Gr[j];
      }
      sdG = red16(sdG);
      sdGx = red16(sdGx);
      sgx = red16(sgx);
      sdGG = red16(sdGG);
      const float inv = rstd * (1.f / F);
      const float dstd = -sdGG * rstd;
      float dxh[4], dT[4], sx = 0.f, sxx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float dgh = (F * dG[j] - sdG - xh[j] * sdGx) * inv;
        dxh[j] = -(dG[j] * sgx + gh[j] * sdGx) * inv + dgh * gm[j] * gm[j];
        dT[j] = -dgh * gm[j];
        const float go = gm[j] * xh[j] + bt[j] - (xv[j] - xk[j]);
        dgam[j] += dgh * (go + gm[j] * xh[j]);
        dbet[j] += dgh * gm[j];
        sx += dxh[j];
        sxx += dxh[j] * xh[j];
      }
      sx = red16(sx);
      sxx = red16(sxx);
      float dz[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) dz[j] = (F * dxh[j] - sx - xh[j] * sxx) * inv + dstd * xh[j] * (1.f / F);
      *reinterpret_cast<uint2*>(smem + OFF_DZ + xo) = make_uint2(H::pack(dz[0], dz[1]), H::pack(dz[2], dz[3]));
      *reinterpret_cast<float4*>(DT + tk * LD + 4 * q) = make_float4(dT[0], dT[1], dT[2], dT[3]);
      *reinterpret_cast<uint2*>((uint8_t*)p.dXV + (xb + tk * F + 4 * q) * 2) =
          make_uint2(H::pack(dT[0], dT[1]), H::pack(dT[2], dT[3]));
      if (q == 0) {
        float de = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) de += DE[w * C + tk];
        DETA[(C - 1) * C + tk] += de;
      }
    }
    __syncthreads();

    // ---------------- M3: dXK += dZ W^T - dT ; dW += XK^T dZ ; outputs
    {
#pragma unroll
      for (int kf = 0; kf < 4; ++kf) {
        uint32_t adz[4], bwt[2];
        ldsm_x4(adz, sDZ + swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1)));
        ldsm_x2(bwt, sWT + swz128(8 * warp + r8, 2 * kf + (mi & 1)));
        mma16816<T>(dXK, adz, bwt);
      }
      const float2 t0 = *reinterpret_cast<const float2*>(DT + g * LD + fc);
      const float2 t1 = *reinterpret_cast<const float2*>(DT + (g + 8) * LD + fc);
      dXK[0] -= t0.x;
      dXK[1] -= t0.y;
      dXK[2] -= t1.x;
      dXK[3] -= t1.y;
      uint32_t bdz[2];
      ldsm_x2_t(bdz, sDZ + swz128((lane & 8) + r8, warp));
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t axk[4];
        ldsm_x4_t(axk, sb + OFF_XK + swz128((mi >> 1) * 8 + r8, 2 * mt + (mi & 1)));
        mma16816<T>(dW[mt], axk, bdz);
      }
      mma16816<T>(dB, a_ones, bdz);
      store_slice<T>(smem + OFF_DWT, dW, warp, g, t);
      uint8_t* gq = (uint8_t*)p.dXQ + xb * 2;
      uint8_t* gk = (uint8_t*)p.dXK + xb * 2;
      *reinterpret_cast<uint32_t*>(gq + (g * F + fc) * 2) = H::pack(dXQ[0], dXQ[1]);
      *reinterpret_cast<uint32_t*>(gq + ((g + 8) * F + fc) * 2) = H::pack(dXQ[2], dXQ[3]);
      *reinterpret_cast<uint32_t*>(gk + (g * F + fc) * 2) = H::pack(dXK[0], dXK[1]);
      *reinterpret_cast<uint32_t*>(gk + ((g + 8) * F + fc) * 2) = H::pack(dXK[2], dXK[3]);
      const long long eb = (s * p.NC + n) * (long long)(C * C);
      reinterpret_cast<T*>(p.deta)[eb + tid] = H::from_float(DETA[tid]);
    }
  }
  cp_async_wait<0>();

  // ---- outputs of the whole walk: dW, db (fp32), per-stream gamma / beta partials
  float* dWo = p.dW + s * F * F;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
    dWo[(16 * mt + g) * F + fc] = dW[mt][0];
    dWo[(16 * mt + g) * F + fc + 1] = dW[mt][1];
    dWo[(16 * mt + g + 8) * F + fc] = dW[mt][2];
    dWo[(16 * mt + g + 8) * F + fc + 1] = dW[mt][3];
  }
  if (g == 0) {
    p.db[s * F + fc] = dB[0];
    p.db[s * F + fc + 1] = dB[1];
  }
  // gamma / beta: sum over the 16 tokens (2 per warp, 8 warps)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    dgam[j] += __shfl_xor_sync(0xffffffffu, dgam[j], 16);
    dbet[j] += __shfl_xor_sync(0xffffffffu, dbet[j], 16);
  }
  float* RED = reinterpret_cast<float*>(smem + OFF_RED);
  __syncthreads();
  if ((lane & 16) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      RED[(warp * 2 + 0) * F + 4 * q + j] = dgam[j];
      RED[(warp * 2 + 1) * F + 4 * q + j] = dbet[j];
    }
  }
  __syncthreads();
  if (tid < 2 * F) {
    const int which = tid / F, f = tid % F;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc += RED[(w * 2 + which) * F + f];
    (which == 0 ? p.d_ln_w : p.d_ln_b)[s * F + f] = acc;
  }
}

}  // namespace lin_bwd_tc

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int linear_bwd_fast(const LinBwdParams& p, cudaStream_t stream) {
  using namespace lin_bwd_tc;
  if (!p.Z_saved || !p.W_last || !p.b_last) return TTT_NOT_APPLICABLE;
  if (p.CS != C || p.F != F) return TTT_NOT_APPLICABLE;
  const int dt = p.dt_xq;
  if (dt != DT_BF16 && dt != DT_F16) return TTT_NOT_APPLICABLE;
  if (p.dt_xk != dt || p.dt_xv != dt || p.dt_eta != dt || p.dt_dout != dt || p.dt_grad != dt) return TTT_NOT_APPLICABLE;
  if (!aligned16(p.XQ) || !aligned16(p.XK) || !aligned16(p.XV) || !aligned16(p.eta) || !aligned16(p.dout) ||
      !aligned16(p.Z_saved) || !aligned16(p.dXQ) || !aligned16(p.dXK) || !aligned16(p.dXV))
    return TTT_NOT_APPLICABLE;
  int rc;
  if (dt == DT_BF16) {
    rc = prepare_smem(linear_bwd_tc_kernel<__nv_bfloat16>, SMEM, "ttt_linear_bwd");
    if (rc) return rc;
    linear_bwd_tc_kernel<__nv_bfloat16><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(p);
  } else {
    rc = prepare_smem(linear_bwd_tc_kernel<__half>, SMEM, "ttt_linear_bwd");
    if (rc) return rc;
    linear_bwd_tc_kernel<__half><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(p);
  }
  return check_launch("ttt_linear_bwd");
}

}  // namespace ttt
