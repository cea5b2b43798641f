// TTT-Linear forward on the tensor cores (mma.sync bf16/fp16, fp32 accumulate) for the
// benchmark shape: head dim F = 64, mini-batch CS = 16, 16-bit activations.
//
// One CTA of 8 warps per (batch, head) stream. Warp w owns output features
// [8w, 8w + 8): its slice of the fp32 state W (64 x 8) and bias stay in mma accumulator
// fragments for the whole sequence. Per mini-batch (ops/ttt_linear.py:8-54):
//   A  (MMA)    Z = XK W, Zq = XQ W for the warp's 8 features (W's fragments become B
//               operands through movmatrix); one warp turns this mini-batch's XQ XK^T
//               block into -P = -eta * (XQ XK^T + 1)
//   B           Z + b to shared memory
//   C  (rows)   G = ln_fused_l2_bwd(Z, XV - XK): 16 lanes per token, 4 features per lane,
//               LayerNorm reductions by shuffles inside the half-warp; G and -e*G (e =
//               eta[CS-1, :]) to shared memory as 16-bit tiles
//   D  (MMA)    W += XK^T (-e*G), b += 1^T (-e*G), Zbar = Zq + b_old - P G
//   E  (rows)   XQW = XQ + LN(Zbar), written straight to global memory
// Four CTA barriers per mini-batch. XQ / XK / XV / eta tiles of each mini-batch arrive by
// TMA (128-byte swizzled tiles, mbarrier ring three deep), awaited by one copy thread whose
// CTA barrier then publishes them.
//
// The W-independent products XQ XK^T are hoisted out of the chain: for each group of 8
// mini-batches, TMA brings the group's XQ and XK rows as two 128 x 64 tiles and one thread
// issues a 128 x 128 x 64 tcgen05.mma into tensor memory (double-buffered, 2 x 128 fp32
// columns); mini-batch j of the group reads its 16 x 16 diagonal block (lanes and columns
// 16j..16j+15) with tcgen05.ld. The next group's product is issued mid-group, so it is
// ready before it is needed.
#include <type_traits>

#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "tc_util.cuh"
#include "tma.cuh"
#include "tmem.cuh"
#include "umma.cuh"

namespace ttt {
namespace lin_tc {

constexpr int F = 64, C = 16, NW = 8, NTHREADS = 32 * NW, NSTAGE = 3, GRP = 8;
constexpr int TILE = C * F * 2;                    // one 16 x 64 16-bit tile
constexpr int ETA = C * C * 2;                     // one 16 x 16 16-bit tile
// Stage of one mini-batch (TMA): XQ, XK, XV tiles at 1024-byte boundaries, then eta.
constexpr int OFF_XQ = 0, OFF_XK = 2048, OFF_XV = 4096, OFF_ETA = 6144;
constexpr int STAGE = 7168;
constexpr uint32_t STAGE_BYTES = 3 * TILE + ETA;
// Group buffers (two): XQ and XK rows of 8 mini-batches, 128 x 64 each.
constexpr int GTILE = GRP * TILE;                  // 16 KB
constexpr int OFF_GRP = NSTAGE * STAGE;            // 1024-aligned
constexpr int GBUF = 2 * GTILE;
constexpr uint32_t GRP_BYTES = 2 * GTILE;
constexpr int ZLD = F + 8;                         // fp32 row stride of the Z tiles (conflict-free float2)
constexpr int OFF_Z = OFF_GRP + 2 * GBUF;          // fp32 [C][ZLD]: Z + b
constexpr int OFF_ZB = OFF_Z + C * ZLD * 4;        // fp32 [C][ZLD]: Zbar
constexpr int OFF_G = OFF_ZB + C * ZLD * 4;        // 16-bit [C][F] swizzled: G
constexpr int OFF_EG = OFF_G + TILE;               // 16-bit [C][F] swizzled: -e * G
constexpr int OFF_P = OFF_EG + TILE;               // 16-bit [C][C]: -P
constexpr int SMEM = OFF_P + ETA + 1024;           // + slack to align the base to 1024 bytes
constexpr uint32_t TMEM_COLS = 256;                // two 128 x 128 fp32 XQ XK^T accumulators
constexpr int kCopyThread = NTHREADS - 32;         // lane 0 of the last warp: copies and tcgen05.mma
static_assert(OFF_GRP % 1024 == 0 && GBUF % 1024 == 0, "TMA 128-byte swizzle needs 1024-byte aligned tiles");

struct Maps {
  const CUtensorMap* q;   // 16-row tiles
  const CUtensorMap* k;
  const CUtensorMap* v;
  const CUtensorMap* gq;  // 128-row group tiles
  const CUtensorMap* gk;
};

__device__ __forceinline__ void issue_stage(uint32_t st, uint32_t bar, const LinFwdParams& p, const Maps& m,
                                            long long s, int n) {
  const int row = (int)((s * p.NC + n) * C);
  mbar_expect_tx(bar, STAGE_BYTES);
  tma_load_2d(st + OFF_XQ, m.q, 0, row, bar);
  tma_load_2d(st + OFF_XK, m.k, 0, row, bar);
  tma_load_2d(st + OFF_XV, m.v, 0, row, bar);
  bulk_load(st + OFF_ETA, (const uint8_t*)p.eta + (s * p.NC + n) * (long long)ETA, ETA, bar);
}

// XQ and XK rows of mini-batches 8 grp .. 8 grp + 7 (rows past the tensor read as zero).
__device__ __forceinline__ void issue_group(uint32_t gb, uint32_t bar, const LinFwdParams& p, const Maps& m,
                                            long long s, int grp) {
  const int row = (int)((s * p.NC + GRP * grp) * C);
  mbar_expect_tx(bar, GRP_BYTES);
  tma_load_2d(gb, m.gq, 0, row, bar);
  tma_load_2d(gb + GTILE, m.gk, 0, row, bar);
}

// D[128 x 128] = XQ_group XK_group^T (K = 64 in four steps), completion on `bar`.
__device__ __forceinline__ void issue_group_product(uint32_t d_tmem, uint32_t gb, uint32_t bar, uint32_t idesc) {
  tmem_fence_after();
  const uint64_t da = umma_desc_k_sw128(gb), db = umma_desc_k_sw128(gb + GTILE);
#pragma unroll
  for (int k = 0; k < F / 16; ++k) umma_ss(d_tmem, da + 2 * k, db + 2 * k, idesc, k > 0);
  umma_commit(bar);
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS)
    linear_fwd_tc_kernel(LinFwdParams p, const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_gq,
                         const __grid_constant__ CUtensorMap tm_gk) {
  using H = Half2<T>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint32_t tmem_base_sh;
  __shared__ __align__(8) uint64_t full_bar[NSTAGE];  // stage n % NSTAGE landed
  __shared__ __align__(8) uint64_t grp_bar[2];        // group buffer b landed
  __shared__ __align__(8) uint64_t mma_bar[2];        // accumulator b holds its group's XQ XK^T
  __shared__ int abort_sh;                            // a wait gave up: stop waiting
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

  const Maps maps{&tm_q, &tm_k, &tm_v, &tm_gq, &tm_gk};
  const int ngrp = (p.NC + GRP - 1) / GRP;
  const uint32_t idesc = umma_idesc_f32(std::is_same<T, __nv_bfloat16>::value, 128, 128);
  const uint32_t gbuf0 = smem_u32(smem + OFF_GRP);
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == kCopyThread) {
    for (int i = 0; i < NSTAGE; ++i) mbar_init(smem_u32(&full_bar[i]), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&grp_bar[i]), 1);
      mbar_init(smem_u32(&mma_bar[i]), 1);
    }
    abort_sh = 0;
    fence_mbar_init();
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tacc = tmem_base_sh;
  // copy thread: last stage / group / group product issued (for draining after a timeout)
  int last_stage = -1, last_group = -1, last_product = -1;
  if (tid == kCopyThread) {
    for (int i = 0; i < NSTAGE - 1 && i < p.NC; ++i) {
      issue_stage(smem_u32(smem + i * STAGE), smem_u32(&full_bar[i]), p, maps, s, i);
      last_stage = i;
    }
    for (int gi = 0; gi < 2 && gi < ngrp; ++gi) {
      issue_group(gbuf0 + gi * GBUF, smem_u32(&grp_bar[gi]), p, maps, s, gi);
      last_group = gi;
    }
    if (mbar_wait(smem_u32(&grp_bar[0]), 0, p.err)) {
      issue_group_product(tacc, gbuf0, smem_u32(&mma_bar[0]), idesc);
      last_product = 0;
    } else {
      abort_sh = 1;
    }
  }

  for (int n = 0; n < p.NC; ++n) {
    const int grp = n / GRP, j = n % GRP;
    // The copy thread waits for stage n; the CTA barrier publishes it and frees stage n-1.
    if (tid == kCopyThread && !abort_sh &&
        !mbar_wait(smem_u32(&full_bar[n % NSTAGE]), (uint32_t)((n / NSTAGE) & 1), p.err))
      abort_sh = 1;
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    if (tid == kCopyThread && !abort_sh) {
      const int nn = n + NSTAGE - 1;
      if (nn < p.NC) {
        issue_stage(smem_u32(smem + (nn % NSTAGE) * STAGE), smem_u32(&full_bar[nn % NSTAGE]), p, maps, s, nn);
        last_stage = nn;
      }
      // mid-group: the next group's product into the other accumulator (its reads ended a
      // group ago), then the group after it into the buffer that product no longer needs
      if (j == GRP / 2 && grp + 1 < ngrp) {
        const int b = (grp + 1) & 1;
        if (mbar_wait(smem_u32(&grp_bar[b]), (uint32_t)(((grp + 1) >> 1) & 1), p.err)) {
          issue_group_product(tacc + 128 * b, gbuf0 + b * GBUF, smem_u32(&mma_bar[b]), idesc);
          last_product = grp + 1;
        } else {
          abort_sh = 1;
        }
      }
      if (j == 0 && grp >= 1 && grp + 1 < ngrp) {  // group grp+1 into the buffer group grp-1 used
        const int b = (grp + 1) & 1;
        issue_group(gbuf0 + b * GBUF, smem_u32(&grp_bar[b]), p, maps, s, grp + 1);
        last_group = grp + 1;
      }
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

    // ---- A: -P from the hoisted XQ XK^T (warp j/2: its lane quadrant holds rows 16j..16j+15);
    //      Z = XK W, Zq = XQ W (warp's 8 output features)
    if (warp == j / 2) {
      const int b = grp & 1;
      if (lane == 0 && !abort_sh && !mbar_wait(smem_u32(&mma_bar[b]), (uint32_t)((grp >> 1) & 1), p.err))
        abort_sh = 1;
      __syncwarp();
      tmem_fence_after();
      float a[16];
      tmem_ld16(tmem_lane_addr(tacc, warp, 128 * b + 16 * j), a);
      tmem_wait_ld();
      if ((lane >> 4) == (j & 1)) {  // this lane holds row i of the block
        const int i = lane & 15;
        const uint4* er = reinterpret_cast<const uint4*>(st + OFF_ETA + i * 32);
        const uint32_t ew[8] = {er[0].x, er[0].y, er[0].z, er[0].w, er[1].x, er[1].y, er[1].z, er[1].w};
        uint32_t pw[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float2 e = H::unpack(ew[c]);
          pw[c] = H::pack(-e.x * (a[2 * c] + 1.f), -e.y * (a[2 * c + 1] + 1.f));
        }
        uint4* pr = reinterpret_cast<uint4*>(smem + OFF_P + i * 32);
        pr[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        pr[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
      }
    }
    float Z[4] = {0.f, 0.f, 0.f, 0.f}, Zq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t bw[2] = {movm_t(H::pack(W[kk][0], W[kk][1])), movm_t(H::pack(W[kk][2], W[kk][3]))};
      uint32_t ak[4], aq[4];
      const uint32_t aoff = swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
      ldsm_x4(ak, sb + OFF_XK + aoff);
      ldsm_x4(aq, sb + OFF_XQ + aoff);
      mma16816<T>(Z, ak, bw);
      mma16816<T>(Zq, aq, bw);
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
  // after a timeout, copies and products issued but never awaited may still be in flight:
  // drain them (bounded) before shared and tensor memory go away
  if (tid == kCopyThread && abort_sh) {
    for (int m = last_stage - NSTAGE + 1; m <= last_stage; ++m)
      if (m >= 0) mbar_wait(smem_u32(&full_bar[m % NSTAGE]), (uint32_t)((m / NSTAGE) & 1), nullptr);
    for (int m = last_group - 1; m <= last_group; ++m)
      if (m >= 0) mbar_wait(smem_u32(&grp_bar[m & 1]), (uint32_t)((m >> 1) & 1), nullptr);
    for (int m = last_product - 1; m <= last_product; ++m)
      if (m >= 0) mbar_wait(smem_u32(&mma_bar[m & 1]), (uint32_t)((m >> 1) & 1), nullptr);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 0) tmem_dealloc(tacc, TMEM_COLS);

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
  const unsigned long long rows = (unsigned long long)p.B * p.NH * p.NC * C;
  CUtensorMap tq, tk, tv, gq, gk;
  int rc = make_tile_map(&tq, p.XQ, dt, rows, "ttt_linear_fwd");
  if (!rc) rc = make_tile_map(&tk, p.XK, dt, rows, "ttt_linear_fwd");
  if (!rc) rc = make_tile_map(&tv, p.XV, dt, rows, "ttt_linear_fwd");
  if (!rc) rc = make_tile_map(&gq, p.XQ, dt, rows, "ttt_linear_fwd", GRP * C);
  if (!rc) rc = make_tile_map(&gk, p.XK, dt, rows, "ttt_linear_fwd", GRP * C);
  if (rc) return rc;
  LinFwdParams q = p;
  rc = device_error_word(&q.err, "ttt_linear_fwd");
  if (rc) return rc;
  if (dt == DT_BF16) {
    rc = prepare_smem(linear_fwd_tc_kernel<__nv_bfloat16>, SMEM, "ttt_linear_fwd");
    if (rc) return rc;
    linear_fwd_tc_kernel<__nv_bfloat16><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(q, tq, tk, tv, gq, gk);
  } else {
    rc = prepare_smem(linear_fwd_tc_kernel<__half>, SMEM, "ttt_linear_fwd");
    if (rc) return rc;
    linear_fwd_tc_kernel<__half><<<p.B * p.NH, NTHREADS, SMEM, stream>>>(q, tq, tk, tv, gq, gk);
  }
  return check_launch("ttt_linear_fwd");
}

}  // namespace ttt
