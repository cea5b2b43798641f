// TTT-Linear forward on the tensor cores (mma.sync bf16/fp16, fp32 accumulate) for the
// benchmark shape: head dim F = 64, mini-batch CS = 16, 16-bit activations.
//
// One CTA of 8 warps per (batch, head) stream. Warp w owns output features
// [8w, 8w + 8): its slice of the fp32 state W (64 x 8) and bias stay in mma accumulator
// fragments for the whole sequence. Per mini-batch (ops/ttt_linear.py:8-54):
//   A  (MMA)    Z = XK W, Zq = XQ W for the warp's 8 features (W's fragments become B
//               operands through movmatrix); warps 0-1 also form -P = -eta * (XQ XK^T + 1)
//   B           Z + b to shared memory
//   C  (rows)   G = ln_fused_l2_bwd(Z, XV - XK): 16 lanes per token, 4 features per lane,
//               LayerNorm reductions by shuffles inside the half-warp; G and -e*G (e =
//               eta[CS-1, :]) to shared memory as 16-bit tiles
//   D  (MMA)    W += XK^T (-e*G), b += 1^T (-e*G), Zbar = Zq + b_old - P G
//   E  (rows)   XQW = XQ + LN(Zbar), written straight to global memory
// Four CTA barriers per mini-batch. XQ / XK / XV / eta tiles are prefetched three
// mini-batches ahead with cp.async into XOR-swizzled shared memory.
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "tc_util.cuh"

namespace ttt {
namespace lin_tc {

constexpr int F = 64, C = 16, NW = 8, NTHREADS = 32 * NW, NSTAGE = 3;
constexpr int TILE = C * F * 2;                    // one 16 x 64 16-bit tile
constexpr int ETA = C * C * 2;                     // one 16 x 16 16-bit tile
constexpr int STAGE = 3 * TILE + ETA;              // XQ, XK, XV, eta
constexpr int OFF_XQ = 0, OFF_XK = TILE, OFF_XV = 2 * TILE, OFF_ETA = 3 * TILE;
constexpr int ZLD = F + 8;                         // fp32 row stride of the Z tiles (conflict-free float2)
constexpr int OFF_Z = NSTAGE * STAGE;              // fp32 [C][ZLD]: Z + b
constexpr int OFF_ZB = OFF_Z + C * ZLD * 4;        // fp32 [C][ZLD]: Zbar
constexpr int OFF_G = OFF_ZB + C * ZLD * 4;        // 16-bit [C][F] swizzled: G
constexpr int OFF_EG = OFF_G + TILE;               // 16-bit [C][F] swizzled: -e * G
constexpr int OFF_P = OFF_EG + TILE;               // 16-bit [C][C]: -P
constexpr int SMEM = OFF_P + ETA;

__device__ __forceinline__ void load_stage(uint8_t* st, const LinFwdParams& p, long long s, int n) {
  const int tid = threadIdx.x;
  const long long tb = (s * p.NC + n) * (long long)(C * F) * 2;
  if (tid < 128) {
    const int row = tid >> 3, ch = tid & 7;
    const uint32_t dst = smem_u32(st) + swz128(row, ch);
    const uint8_t* src = (const uint8_t*)p.XQ + tb + row * 128 + ch * 16;
    cp_async16(dst + OFF_XQ, src);
    cp_async16(dst + OFF_XK, (const uint8_t*)p.XK + tb + row * 128 + ch * 16);
  } else {
    const int i = tid - 128, row = i >> 3, ch = i & 7;
    cp_async16(smem_u32(st) + OFF_XV + swz128(row, ch), (const uint8_t*)p.XV + tb + row * 128 + ch * 16);
    if (i < 32) {
      const long long eb = (s * p.NC + n) * (long long)(C * C) * 2;
      cp_async16(smem_u32(st) + OFF_ETA + i * 16, (const uint8_t*)p.eta + eb + i * 16);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS) linear_fwd_tc_kernel(LinFwdParams p) {
  using H = Half2<T>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  // row-phase mapping: token tk, features [4q, 4q + 4)
  const int tk = tid >> 4, q = tid & 15;
  const int fc = 8 * warp + 2 * t;  // first of the two output features this lane's C fragments hold
  float* Zs = reinterpret_cast<float*>(smem + OFF_Z);
  float* Zbs = reinterpret_cast<float*>(smem + OFF_ZB);

  // ---- state slice W[:, 8w:8w+8] and bias in accumulator layout (rows f_in / token, cols f_out)
  float W[4][4], Bc[4];
  {
    const float* Wi = p.W_init + s * F * F;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      W[mt][0] = Wi[(16 * mt + g) * F + fc];
      W[mt][1] = Wi[(16 * mt + g) * F + fc + 1];
      W[mt][2] = Wi[(16 * mt + g + 8) * F + fc];
      W[mt][3] = Wi[(16 * mt + g + 8) * F + fc + 1];
    }
    Bc[0] = Bc[2] = p.b_init[s * F + fc];
    Bc[1] = Bc[3] = p.b_init[s * F + fc + 1];
  }
  float gm[4], bt[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    gm[j] = ld_elem(p.ln_w, (long long)h * F + 4 * q + j, p.dt_ln);
    bt[j] = ld_elem(p.ln_b, (long long)h * F + 4 * q + j, p.dt_ln);
  }
  const uint32_t ones = H::pack(1.f, 1.f);
  const uint32_t a_ones[4] = {ones, ones, ones, ones};

#pragma unroll
  for (int i = 0; i < NSTAGE - 1; ++i) {
    if (i < p.NC) load_stage(smem + i * STAGE, p, s, i);
    cp_async_commit();
  }

  for (int n = 0; n < p.NC; ++n) {
    cp_async_wait<NSTAGE - 2>();
    __syncthreads();  // stage n landed; every warp is past mini-batch n-1
    {
      const int nn = n + NSTAGE - 1;
      if (nn < p.NC) load_stage(smem + (nn % NSTAGE) * STAGE, p, s, nn);
      cp_async_commit();
    }
    const uint8_t* st = smem + (n % NSTAGE) * STAGE;
    const uint32_t sb = smem_u32(st);

    if (p.W_ckpt && n % p.ckpt == 0) {  // state at the start of the checkpoint group
      const long long k = s * p.K + n / p.ckpt;
      float* Wc = p.W_ckpt + k * F * F;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        Wc[(16 * mt + g) * F + fc] = W[mt][0];
        Wc[(16 * mt + g) * F + fc + 1] = W[mt][1];
        Wc[(16 * mt + g + 8) * F + fc] = W[mt][2];
        Wc[(16 * mt + g + 8) * F + fc + 1] = W[mt][3];
      }
      if (g == 0) {
        p.b_ckpt[k * F + fc] = Bc[0];
        p.b_ckpt[k * F + fc + 1] = Bc[1];
      }
    }

    // ---- A: Z = XK W, Zq = XQ W (warp's 8 output features); warps 0-1: -P
    float Z[4] = {0.f, 0.f, 0.f, 0.f}, Zq[4] = {0.f, 0.f, 0.f, 0.f}, A1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t bw[2] = {movm_t(H::pack(W[kk][0], W[kk][1])), movm_t(H::pack(W[kk][2], W[kk][3]))};
      uint32_t ak[4], aq[4];
      const uint32_t aoff = swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
      ldsm_x4(ak, sb + OFF_XK + aoff);
      ldsm_x4(aq, sb + OFF_XQ + aoff);
      mma16816<T>(Z, ak, bw);
      mma16816<T>(Zq, aq, bw);
      if (warp < 2) {  // A1[:, 8*warp : 8*warp+8] = XQ XK^T
        uint32_t bk[2];
        ldsm_x2(bk, sb + OFF_XK + swz128(8 * warp + r8, 2 * kk + (mi & 1)));
        mma16816<T>(A1, aq, bk);
      }
    }
    if (warp < 2) {
      const int j0 = 8 * warp + 2 * t;
      const T* E = reinterpret_cast<const T*>(st + OFF_ETA);
      const float2 e_lo = H::unpack(*reinterpret_cast<const uint32_t*>(E + g * C + j0));
      const float2 e_hi = H::unpack(*reinterpret_cast<const uint32_t*>(E + (g + 8) * C + j0));
      *reinterpret_cast<uint32_t*>(smem + OFF_P + (g * C + j0) * 2) =
          H::pack(-e_lo.x * (A1[0] + 1.f), -e_lo.y * (A1[1] + 1.f));
      *reinterpret_cast<uint32_t*>(smem + OFF_P + ((g + 8) * C + j0) * 2) =
          H::pack(-e_hi.x * (A1[2] + 1.f), -e_hi.y * (A1[3] + 1.f));
    }
    // ---- B: Z + b to shared memory; keep Zq + b (old bias) for the read-out
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Z[i] += Bc[i];
      Zq[i] += Bc[i];
    }
    *reinterpret_cast<float2*>(Zs + g * ZLD + fc) = make_float2(Z[0], Z[1]);
    *reinterpret_cast<float2*>(Zs + (g + 8) * ZLD + fc) = make_float2(Z[2], Z[3]);
    __syncthreads();

    // ---- C: G = ln_fused_l2_bwd(Z, XV - XK), token tk, features 4q..4q+3
    {
      const float4 z4 = *reinterpret_cast<const float4*>(Zs + tk * ZLD + 4 * q);
      if (p.Z_out) *reinterpret_cast<float4*>(p.Z_out + (s * p.NC + n) * (long long)(C * F) + tk * F + 4 * q) = z4;
      float z[4] = {z4.x, z4.y, z4.z, z4.w}, xv[4], xk[4];
      const uint32_t xo = swz128(tk, q >> 1) + (q & 1) * 8;
      unpack4<T>(st + OFF_XV + xo, xv);
      unpack4<T>(st + OFF_XK + xo, xk);
      const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
      float d[4], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rstd = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
      float xh[4], gh[4], s1 = 0.f, s2 = 0.f;
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
      float G[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) G[j] = (F * gh[j] - s1 - xh[j] * s2) * inv;
      const float e = (float)reinterpret_cast<const T*>(st + OFF_ETA)[(C - 1) * C + tk];
      *reinterpret_cast<uint2*>(smem + OFF_G + xo) = make_uint2(H::pack(G[0], G[1]), H::pack(G[2], G[3]));
      *reinterpret_cast<uint2*>(smem + OFF_EG + xo) =
          make_uint2(H::pack(-e * G[0], -e * G[1]), H::pack(-e * G[2], -e * G[3]));
    }
    __syncthreads();

    // ---- D: W += XK^T (-e G); b += 1^T (-e G); Zbar = Zq + b_old - P G
    {
      uint32_t beg[2], bg[2], ap[4];
      const uint32_t boff = swz128((lane & 8) + r8, warp);
      ldsm_x2_t(beg, smem_u32(smem + OFF_EG) + boff);
      ldsm_x2_t(bg, smem_u32(smem + OFF_G) + boff);
      ldsm_x4(ap, smem_u32(smem + OFF_P) + ((mi & 1) * 8 + r8) * 32 + (mi >> 1) * 16);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t axk[4];
        ldsm_x4_t(axk, sb + OFF_XK + swz128((mi >> 1) * 8 + r8, 2 * mt + (mi & 1)));
        mma16816<T>(W[mt], axk, beg);
      }
      mma16816<T>(Bc, a_ones, beg);
      mma16816<T>(Zq, ap, bg);
      *reinterpret_cast<float2*>(Zbs + g * ZLD + fc) = make_float2(Zq[0], Zq[1]);
      *reinterpret_cast<float2*>(Zbs + (g + 8) * ZLD + fc) = make_float2(Zq[2], Zq[3]);
    }
    __syncthreads();

    // ---- E: XQW = XQ + LN(Zbar)
    {
      const float4 z4 = *reinterpret_cast<const float4*>(Zbs + tk * ZLD + 4 * q);
      float z[4] = {z4.x, z4.y, z4.z, z4.w}, xq[4];
      unpack4<T>(st + OFF_XQ + swz128(tk, q >> 1) + (q & 1) * 8, xq);
      const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
      float d[4], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rstd = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = xq[j] + gm[j] * d[j] * rstd + bt[j];
      uint8_t* dst = (uint8_t*)p.out + ((s * p.NC + n) * (long long)(C * F) + tk * F + 4 * q) * 2;
      *reinterpret_cast<uint2*>(dst) = make_uint2(H::pack(y[0], y[1]), H::pack(y[2], y[3]));
    }
  }
  cp_async_wait<0>();

  float* Wl = p.W_last + s * F * F;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
    Wl[(16 * mt + g) * F + fc] = W[mt][0];
    Wl[(16 * mt + g) * F + fc + 1] = W[mt][1];
    Wl[(16 * mt + g + 8) * F + fc] = W[mt][2];
    Wl[(16 * mt + g + 8) * F + fc + 1] = W[mt][3];
  }
  if (g == 0) {
    p.b_last[s * F + fc] = Bc[0];
    p.b_last[s * F + fc + 1] = Bc[1];
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
