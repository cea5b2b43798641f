// TTT-MLP backward on the tensor cores (mma.sync bf16/fp16, fp32 accumulate) for F = 64,
// CS = 16, 16-bit activations and an inner width FF = 32 * NW: the benchmark MLP (FF = 256,
// NW = 8 warps, one CTA per SM) and the layer's F x F inner MLP (FF = 64, NW = 2, two CTAs
// per SM).
//
// Uses the per-mini-batch fp32 pre-activations the forward stored (Z1 = XK W1 + b1,
// Z2 = X2 W2 + b2, Z1bar and Z2bar before their nonlinearities) and walks the sequence
// once, last mini-batch first, from the final weights. The weights entering mini-batch n
// come from those after it by undoing its rank-16 updates:
//   W2_n = W2_{n+1} + X2^T (e G2),   G1 = (G2 W2_n^T) * gelu_bwd(Z1),
//   W1_n = W1_{n+1} + XK^T (e G1)    (e = eta[CS-1, :]).
// The biases never enter a product here (they are inside the stored Z's), so they are not
// reversed. The per-step gradient is autograd through ops/ttt_mlp.py:9-67 (full CS x CS
// d_eta), derived by hand.
//
// One CTA of NW warps per (batch, head) stream; warp w owns hidden units [32w, 32w + 32).
// Its slices of W1, W2 and of the carried gradients dW1, dW2 (fp32, 256 values per thread
// in accumulator-fragment layout) live in tensor memory: 256 columns of the warp's lane
// quadrant (the 8-warp CTA holds all 512 columns). Products that contract over the hidden units ([16 x 64] results, and
// the 16 x 16 A2 / dP1) are per-warp partial sums reduced through shared memory; A2
// enters every formula linearly, so only its partials are formed. Per mini-batch:
//   R1 (rows)  G2 = ln_fused_l2_bwd(Z2, XV - XK); dZ2bar = read-out LayerNorm backward
//   M1 (MMA)   W2 reversal; H = G2 W2^T, G1; W1 reversal; dX2bar, dZ1bar; A1, P1, dP2,
//              A2_w; terms with the carried dW1, dW2; dG1, dH; partial dG2; dW2 updates
//   R2 (rows)  dG2 = sum of partials; backward of ln_fused_l2_bwd -> dZ2, dXV;
//              d_eta and dP1 reductions
//   M2 (MMA)   dX2, dZ1; partial dXQ, dXK; dW1, db1, dW2, db2 updates
//   R3 (rows)  dXQ, dXK = sums of partials (+ dO, - dXV)
// GELU pieces use the hardware tanh (tanh.approx.f32), below the 16-bit operand rounding.
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mlp_tc_common.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "tc_util.cuh"
#include "tmem.cuh"

namespace ttt {
namespace mlp_tc {
namespace bwd {

// Per-phase timeline (built only with -DTTT_PHASE_STAMPS): for the walk's step kBStampIt,
// thread 0 of each CTA records %globaltimer before and after each CTA barrier (11 stamps) and
// its SM id; ttt_bwd_phase_stamps_read copies them out.
#ifdef TTT_PHASE_STAMPS
constexpr int kBStampIt = 64, kBStampCTAs = 4096, kBStamps = 12;
__device__ unsigned long long g_bwd_stamps[kBStampCTAs][kBStamps];
__device__ __forceinline__ unsigned long long bstamp_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define TTT_BSTAMP(k)                                                                              \
  do {                                                                                             \
    if (threadIdx.x == 0 && it == kBStampIt && blockIdx.x < kBStampCTAs) {                         \
      g_bwd_stamps[blockIdx.x][k] = bstamp_ns();                                                   \
      if ((k) == 0) {                                                                              \
        unsigned sm_;                                                                              \
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));                                         \
        g_bwd_stamps[blockIdx.x][11] = sm_;                                                        \
      }                                                                                            \
    }                                                                                              \
  } while (0)
#else
#define TTT_BSTAMP(k) \
  do {                \
  } while (0)
#endif

constexpr int NSTAGE = 2;
constexpr int TILE = C * F * 2;   // one 16 x 64 16-bit tile
constexpr int ETA = C * C * 2;    // one 16 x 16 16-bit tile
constexpr int PLD = F + 8;        // fp32 row stride of the partial tiles
constexpr int OFF_XQ = 0, OFF_XK = TILE, OFF_XV = 2 * TILE, OFF_DO = 3 * TILE, OFF_ETA = 4 * TILE;
constexpr int OFF_Z2 = OFF_ETA + ETA;           // fp32 [C][F]
constexpr int OFF_Z2B = OFF_Z2 + C * F * 4;     // fp32 [C][F]
constexpr int OFF_Z1 = OFF_Z2B + C * F * 4;     // fp32 [C][ZLD]

// Layout of a CTA of NW warps (inner width FFW = 32 * NW).
template <int NW_>
struct Bwd {
  // NW warps own 32 hidden units each (the MMA phases); the row phases (16 threads per token)
  // run on NR >= NW warps: at FF = 64 two more warps join them, which halves the passes over
  // the mini-batch's tokens (registers allow 4 warps per CTA at 2 CTAs per SM)
  static constexpr int NW = NW_, NR = NW_ > 4 ? NW_ : 4, NTHREADS = 32 * NR, FFW = 32 * NW;
  static constexpr int ZLD = FFW + 8;                        // fp32 row stride of the staged Z1 / Z1bar
  static constexpr int OFF_Z1B = OFF_Z1 + C * ZLD * 4;       // fp32 [C][ZLD]
  static constexpr int STAGE = OFF_Z1B + C * ZLD * 4;        // 50688 bytes for FF = 256
  static constexpr int PART = NW * C * PLD * 4;              // one [NW][C][PLD] set of partial tiles
  static constexpr int OFF_PA = NSTAGE * STAGE;              // partial dG2 (M1 -> R2), then partial dXQ (M2 -> R3)
  static constexpr int OFF_PB = OFF_PA + PART;               // partial dXK (M1, M2 -> R3)
  // R1's outputs; with row-only warps (NR > NW) they compute R1 of the next mini-batch while
  // the MMA warps work on this one, so those tiles are double-buffered (mini-batch n in n % 2)
  static constexpr int NRB = NR > NW ? 2 : 1;
  static constexpr int OFF_G = OFF_PB + PART;                // NRB x 16-bit swizzled [C][F]: G2
  static constexpr int OFF_EG = OFF_G + NRB * TILE;          //   e * G2
  static constexpr int OFF_DZB = OFF_EG + NRB * TILE;        //   dZ2bar
  static constexpr int OFF_DZ2 = OFF_DZB + NRB * TILE;       //   dZ2
  static constexpr int OFF_DETAP = OFF_DZ2 + TILE;           // fp32 [NW][C*C] partial d_eta
  static constexpr int OFF_DP1P = OFF_DETAP + NW * C * C * 4;  // fp32 [NW][C*C] partial dP1
  static constexpr int OFF_DP1 = OFF_DP1P + NW * C * C * 4;    // fp32 [C*C] dP1
  static constexpr int OFF_DE = OFF_DP1 + C * C * 4;           // fp32 [NW][C] partial d e
  static constexpr int OFF_DE2 = OFF_DE + NW * C * 4;          // fp32 [C] -G2 . db2
  static constexpr int OFF_DB2 = OFF_DE2 + C * 4;              // fp32 [F] carried db2
  static constexpr int SMEM = OFF_DB2 + F * 4;
  // per warp: W1^T, W2^T, dW1^T, dW2^T slices, 64 columns each, in its lane quadrant
  static constexpr uint32_t TMEM_COLS = NW > 4 ? 512 : 256;
  static constexpr int CTAS_PER_SM = NW > 4 ? 1 : 2;
  static_assert(SMEM * CTAS_PER_SM <= 227 * 1024, "shared memory budget");
  static_assert(PART >= NR * 2 * F * 4, "the gamma / beta reduction reuses one partial set");
  static_assert(OFF_PA % 128 == 0 && OFF_G % 128 == 0 && STAGE % 128 == 0, "tile alignment");
};

// Copies of mini-batch n's stage, issued by the NT threads t0 .. t0 + NT - 1.
template <int NW, int NT>
__device__ __forceinline__ void load_stage(uint8_t* st, const MlpBwdParams& p, long long s, int n, int t0) {
  using L = Bwd<NW>;
  constexpr int FFW = L::FFW, ZLD = L::ZLD;
  const int tid = threadIdx.x - t0;
  const long long mb = s * p.NC + n;  // mini-batch index
  const uint32_t sb = smem_u32(st);
  {
    const long long tb = mb * (long long)(C * F) * 2;
    for (int c = tid; c < 256; c += NT) {  // XQ, XK (chunks 0..127) and XV, dO (128..255)
      const int row = (c & 127) >> 3, ch = c & 7;
      const uint32_t dst = sb + swz128(row, ch);
      const long long src = tb + row * 128 + ch * 16;
      if (c < 128) {
        cp_async16(dst + OFF_XQ, (const uint8_t*)p.XQ + src);
        cp_async16(dst + OFF_XK, (const uint8_t*)p.XK + src);
      } else {
        cp_async16(dst + OFF_XV, (const uint8_t*)p.XV + src);
        cp_async16(dst + OFF_DO, (const uint8_t*)p.dout + src);
      }
    }
    if (tid < 32) cp_async16(sb + OFF_ETA + tid * 16, (const uint8_t*)p.eta + mb * (C * C) * 2 + tid * 16);
  }
  // Z2, Z2bar: 4 KB each, 256 chunks of 16 bytes
  for (int c = tid; c < 256; c += NT) {
    cp_async16(sb + OFF_Z2 + c * 16, p.Z2_saved + mb * (C * F) + c * 4);
    cp_async16(sb + OFF_Z2B + c * 16, p.Z2b_saved + mb * (C * F) + c * 4);
  }
  // Z1, Z1bar: 16 rows of FFW / 4 chunks each, into padded rows
  for (int c = tid; c < C * FFW / 4; c += NT) {
    const int row = c / (FFW / 4), col = c % (FFW / 4);
    const long long src = mb * (C * FFW) + row * FFW + col * 4;
    cp_async16(sb + OFF_Z1 + (row * ZLD + col * 4) * 4, p.Z1_saved + src);
    cp_async16(sb + L::OFF_Z1B + (row * ZLD + col * 4) * 4, p.Z1b_saved + src);
  }
}

// Sum of the NW warps' partial tiles for token tk, features 4q..4q+3.
template <int NW>
__device__ __forceinline__ void sum_part(const float* part, int tk, int q, float* z) {
  float4 acc = *reinterpret_cast<const float4*>(part + tk * PLD + 4 * q);
#pragma unroll
  for (int w = 1; w < NW; ++w) {
    const float4 v = *reinterpret_cast<const float4*>(part + (w * C + tk) * PLD + 4 * q);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  z[0] = acc.x;
  z[1] = acc.y;
  z[2] = acc.z;
  z[3] = acc.w;
}

// A warp's [16 x 64] accumulator tiles -> its partial slot (optionally added to what the
// same threads stored there before).
template <bool kAdd>
__device__ __forceinline__ void put_part(float* pw, const float (*X)[4], int g, int t) {
#pragma unroll
  for (int nf = 0; nf < 8; ++nf) {
    float2* p0 = reinterpret_cast<float2*>(pw + g * PLD + 8 * nf + 2 * t);
    float2* p1 = reinterpret_cast<float2*>(pw + (g + 8) * PLD + 8 * nf + 2 * t);
    if (kAdd) {
      const float2 o0 = *p0, o1 = *p1;
      *p0 = make_float2(o0.x + X[nf][0], o0.y + X[nf][1]);
      *p1 = make_float2(o1.x + X[nf][2], o1.y + X[nf][3]);
    } else {
      *p0 = make_float2(X[nf][0], X[nf][1]);
      *p1 = make_float2(X[nf][2], X[nf][3]);
    }
  }
}

template <typename T, int NW>
__global__ void __launch_bounds__(Bwd<NW>::NTHREADS, Bwd<NW>::CTAS_PER_SM) mlp_bwd_tc_kernel(MlpBwdParams p) {
  using H = Half2<T>;
  using L = Bwd<NW>;
  constexpr int NTHREADS = L::NTHREADS, NR = L::NR, FFW = L::FFW, ZLD = L::ZLD, STAGE = L::STAGE;
  constexpr int OFF_Z1B = L::OFF_Z1B, OFF_PA = L::OFF_PA, OFF_PB = L::OFF_PB, OFF_G = L::OFF_G, OFF_EG = L::OFF_EG;
  constexpr int OFF_DZB = L::OFF_DZB, OFF_DZ2 = L::OFF_DZ2, OFF_DETAP = L::OFF_DETAP, OFF_DP1P = L::OFF_DP1P;
  constexpr int OFF_DP1 = L::OFF_DP1, OFF_DE = L::OFF_DE, OFF_DE2 = L::OFF_DE2, OFF_DB2 = L::OFF_DB2;
  constexpr uint32_t TMEM_COLS = L::TMEM_COLS;
  constexpr int TPP = NTHREADS / 16, NPASS = C / TPP;  // row phases: tokens per pass, passes
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t tmem_base_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  const int tk0 = tid >> 4, q = tid & 15;
  const int fb = 32 * warp;
  float* PA = reinterpret_cast<float*>(smem + OFF_PA);
  float* PB = reinterpret_cast<float*>(smem + OFF_PB);
  float* DETAP = reinterpret_cast<float*>(smem + OFF_DETAP);
  float* DP1P = reinterpret_cast<float*>(smem + OFF_DP1P);
  float* DP1 = reinterpret_cast<float*>(smem + OFF_DP1);
  float* DE = reinterpret_cast<float*>(smem + OFF_DE);
  float* DE2 = reinterpret_cast<float*>(smem + OFF_DE2);
  float* DB2 = reinterpret_cast<float*>(smem + OFF_DB2);
  const uint32_t sDZ2 = smem_u32(smem + OFF_DZ2);

  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tS1 = tmem_lane_addr(tmem_base_sh, warp, 256 * (warp >> 2));
  const uint32_t tS2 = tS1 + 64, tD1 = tS1 + 128, tD2 = tS1 + 192;
  if (warp < NW) {  // the MMA warps' state slices (hidden units fb..fb+31)
    float S1[2][8][4], S2[4][4][4];
    w1_io<2, FFW>(S1, const_cast<float*>(p.W1_last + s * F * FFW), fb, g, t, false);
    w2_io(S2, const_cast<float*>(p.W2_last + s * FFW * F), fb, g, t, false);
    slice_st(tS1, &S1[0][0][0]);
    slice_st(tS2, &S2[0][0][0]);
    float zero[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) zero[i] = 0.f;
    slice_st(tD1, zero);
    slice_st(tD2, zero);
  }
  if (tid < F) DB2[tid] = 0.f;
  float DB1[4][2];  // carried db1 at hidden units fb + 8j + 2t (+1)
#pragma unroll
  for (int j = 0; j < 4; ++j) DB1[j][0] = DB1[j][1] = 0.f;
  float gm[4], bt[4], dgam[4] = {0.f, 0.f, 0.f, 0.f}, dbet[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    gm[j] = ld_elem(p.ln_w, (long long)h * F + 4 * q + j, p.dt_ln);
    bt[j] = ld_elem(p.ln_b, (long long)h * F + 4 * q + j, p.dt_ln);
  }
  const uint32_t ones = H::pack(1.f, 1.f);
  const uint32_t a_ones[4] = {ones, ones, ones, ones};
  const float one_w0 = warp == 0 ? 1.f : 0.f;  // the "+1" of P2 = eta * (A2 + 1) goes to warp 0's partial

  // Row-only warps (NR > NW, FF = 64): while the MMA warps run M1 and M2 of mini-batch n, warps
  // NW.. copy mini-batch n - 1's stage (waiting on their own copies) and compute its R1, whose
  // inputs are the staged tiles only; R1's db2 term moves to R2, where db2 is current.
  constexpr bool kAhead = NR > NW;
  constexpr int NRT = 32 * (NR - NW);  // row-only threads
  auto xo_of = [&](int tk) { return swz128(tk, q >> 1) + (q & 1) * 8; };
  // G2 = ln_fused_l2_bwd(Z2, XV - XK) for token tk of the stage at sx, features 4q.., with its
  // normalised input xh, the scaled residual gh and 1/std
  auto g2_rows_at = [&](const uint8_t* sx, int tk, float* xh, float* gh, float* Gr, float& rstd) {
    const uint32_t xo = xo_of(tk);
    const float4 z4 = *reinterpret_cast<const float4*>(sx + OFF_Z2 + (tk * F + 4 * q) * 4);
    float z[4] = {z4.x, z4.y, z4.z, z4.w}, xv[4], xk[4];
    unpack4<T>(sx + OFF_XV + xo, xv);
    unpack4<T>(sx + OFF_XK + xo, xk);
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
  };
  // R1, part 1: G2 and e * G2 tiles (buffer ob) of the stage at sx, tokens tkb, tkb + tps, ..;
  // with_de2: also -G2 . db2 per token
  auto r1_g = [&](const uint8_t* sx, int ob, int tkb, int tps, bool with_de2) {
    const T* Ex = reinterpret_cast<const T*>(sx + OFF_ETA);
#pragma unroll 4
    for (int tk = tkb; tk < C; tk += tps) {
      const uint32_t xo = xo_of(tk);
      float xh[4], gh[4], Gr[4], rstd;
      g2_rows_at(sx, tk, xh, gh, Gr, rstd);
      const float e = (float)Ex[(C - 1) * C + tk];
      *reinterpret_cast<uint2*>(smem + OFF_G + ob * TILE + xo) = make_uint2(H::pack(Gr[0], Gr[1]), H::pack(Gr[2], Gr[3]));
      *reinterpret_cast<uint2*>(smem + OFF_EG + ob * TILE + xo) =
          make_uint2(H::pack(e * Gr[0], e * Gr[1]), H::pack(e * Gr[2], e * Gr[3]));
      if (with_de2) {
        const float4 db = *reinterpret_cast<const float4*>(DB2 + 4 * q);
        const float dot = red16(Gr[0] * db.x + Gr[1] * db.y + Gr[2] * db.z + Gr[3] * db.w);
        if (q == 0) DE2[tk] = -dot;
      }
    }
  };
  // R1, part 2: read-out LayerNorm backward dZ2bar (buffer ob) from the stored Z2bar and dO,
  // and this thread's share of the TTT LayerNorm gradients
  auto r1_dzb = [&](const uint8_t* sx, int ob, int tkb, int tps) {
#pragma unroll 4
    for (int tk = tkb; tk < C; tk += tps) {
      const uint32_t xo = xo_of(tk);
      const float4 z4 = *reinterpret_cast<const float4*>(sx + OFF_Z2B + (tk * F + 4 * q) * 4);
      float z[4] = {z4.x, z4.y, z4.z, z4.w}, dO4[4];
      unpack4<T>(sx + OFF_DO + xo, dO4);
      const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
      float d[4], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rb = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
      float xbn[4], gg[4], s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xbn[j] = d[j] * rb;
        gg[j] = dO4[j] * gm[j];
        s1 += gg[j];
        s2 += gg[j] * xbn[j];
        dgam[j] += dO4[j] * xbn[j];
        dbet[j] += dO4[j];
      }
      s1 = red16(s1);
      s2 = red16(s2);
      float dz[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) dz[j] = (F * gg[j] - s1 - xbn[j] * s2) * (rb * (1.f / F));
      *reinterpret_cast<uint2*>(smem + OFF_DZB + ob * TILE + xo) = make_uint2(H::pack(dz[0], dz[1]), H::pack(dz[2], dz[3]));
    }
  };
  load_stage<NW, NTHREADS>(smem, p, s, p.NC - 1, 0);
  cp_async_commit();
  if constexpr (kAhead) {  // R1 of the first mini-batch (all threads)
    cp_async_wait<0>();
    __syncthreads();
    r1_g(smem, (p.NC - 1) & 1, tk0, TPP, false);
    r1_dzb(smem, (p.NC - 1) & 1, tk0, TPP);
  }

  for (int it = 0; it < p.NC; ++it) {
    const int n = p.NC - 1 - it;
    TTT_BSTAMP(0);
    cp_async_wait<0>();
    __syncthreads();  // stage of mini-batch n landed; every warp is done with mini-batch n+1
    TTT_BSTAMP(1);
    if (!kAhead && it + 1 < p.NC) load_stage<NW, NTHREADS>(smem + ((it + 1) % NSTAGE) * STAGE, p, s, n - 1, 0);
    cp_async_commit();
    const uint8_t* st = smem + (it % NSTAGE) * STAGE;
    const uint32_t sb = smem_u32(st);
    const T* E = reinterpret_cast<const T*>(st + OFF_ETA);
    const long long xb = (s * p.NC + n) * (long long)(C * F);
    // G2 rows of this mini-batch (formed in R1 and again in R2 rather than kept in registers
    // across M1)
    auto g2_rows = [&](int tk, float* xh, float* gh, float* Gr, float& rstd) { g2_rows_at(st, tk, xh, gh, Gr, rstd); };
    const int ob = kAhead ? (n & 1) : 0;  // R1 output buffer of this mini-batch
    const uint32_t sG = smem_u32(smem + OFF_G + ob * TILE), sEG = smem_u32(smem + OFF_EG + ob * TILE);
    const uint32_t sDZB = smem_u32(smem + OFF_DZB + ob * TILE);

    if constexpr (!kAhead) {
      // ---------------- R1: G2 from the stored Z2; read-out LayerNorm backward from Z2bar
  #pragma unroll
      for (int tk = tk0; tk < C; tk += TPP) {
        const uint32_t xo = xo_of(tk);
        float xh[4], gh[4], Gr[4], rstd;
        g2_rows(tk, xh, gh, Gr, rstd);
        const float e = (float)E[(C - 1) * C + tk];
        *reinterpret_cast<uint2*>(smem + OFF_G + xo) = make_uint2(H::pack(Gr[0], Gr[1]), H::pack(Gr[2], Gr[3]));
        *reinterpret_cast<uint2*>(smem + OFF_EG + xo) =
            make_uint2(H::pack(e * Gr[0], e * Gr[1]), H::pack(e * Gr[2], e * Gr[3]));
        const float4 db = *reinterpret_cast<const float4*>(DB2 + 4 * q);
        const float dot = red16(Gr[0] * db.x + Gr[1] * db.y + Gr[2] * db.z + Gr[3] * db.w);
        if (q == 0) DE2[tk] = -dot;
      }
  #pragma unroll
      for (int tk = tk0; tk < C; tk += TPP) {
        const uint32_t xo = xo_of(tk);
        const float4 z4 = *reinterpret_cast<const float4*>(st + OFF_Z2B + (tk * F + 4 * q) * 4);
        float z[4] = {z4.x, z4.y, z4.z, z4.w}, dO4[4];
        unpack4<T>(st + OFF_DO + xo, dO4);
        const float mu = red16(z[0] + z[1] + z[2] + z[3]) * (1.f / F);
        float d[4], m2 = 0.f;
  #pragma unroll
        for (int j = 0; j < 4; ++j) {
          d[j] = z[j] - mu;
          m2 += d[j] * d[j];
        }
        const float rb = 1.f / sqrtf(red16(m2) * (1.f / F) + kLnEps);
        float xbn[4], gg[4], s1 = 0.f, s2 = 0.f;
  #pragma unroll
        for (int j = 0; j < 4; ++j) {
          xbn[j] = d[j] * rb;
          gg[j] = dO4[j] * gm[j];
          s1 += gg[j];
          s2 += gg[j] * xbn[j];
          dgam[j] += dO4[j] * xbn[j];
          dbet[j] += dO4[j];
        }
        s1 = red16(s1);
        s2 = red16(s2);
        float dz[4];
  #pragma unroll
        for (int j = 0; j < 4; ++j) dz[j] = (F * gg[j] - s1 - xbn[j] * s2) * (rb * (1.f / F));
        *reinterpret_cast<uint2*>(smem + OFF_DZB + xo) = make_uint2(H::pack(dz[0], dz[1]), H::pack(dz[2], dz[3]));
      }
      TTT_BSTAMP(2);
      __syncthreads();
    }
    TTT_BSTAMP(3);

    // ---------------- M1 (the NW MMA warps)
    // carried from M1 into M2 in the MMA warps' registers
    uint32_t X2t[2][4], Zbp[4][2], Zbt[2][4];
    float GP[4][4], dX2[4][4], dZ1[4][4];
    if (warp < NW) {
    tmem_wait_st();  // the previous step's M2 stores of dW1, dW2 (issued without waiting) landed
    const float* Z1s = reinterpret_cast<const float*>(st + OFF_Z1);
    const float* Z1bs = reinterpret_cast<const float*>(st + OFF_Z1B);
    const float eg0 = (float)E[(C - 1) * C + g], eg1 = (float)E[(C - 1) * C + g + 8];
    float ev[2][4];  // eta in accumulator layout
#pragma unroll
    for (int jt = 0; jt < 2; ++jt) {
      const float2 e0 = H::unpack(*reinterpret_cast<const uint32_t*>(E + g * C + 8 * jt + 2 * t));
      const float2 e1 = H::unpack(*reinterpret_cast<const uint32_t*>(E + (g + 8) * C + 8 * jt + 2 * t));
      ev[jt][0] = e0.x;
      ev[jt][1] = e0.y;
      ev[jt][2] = e1.x;
      ev[jt][3] = e1.y;
    }
    // X2 = gelu(Z1), GP = gelu'(Z1) = gelu_bwd(Z1) on the warp's hidden units. GP is
    // rounded to 16 bits as the forward rounded it, so G1 (and with it the W1 reversal)
    // reproduces the forward's values.
    uint32_t X2p[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 z01 = *reinterpret_cast<const float2*>(Z1s + g * ZLD + fb + 8 * j + 2 * t);
      const float2 z23 = *reinterpret_cast<const float2*>(Z1s + (g + 8) * ZLD + fb + 8 * j + 2 * t);
      float2 x01, x23, d01, d23;
      gelu2_and_bwd(z01, x01, d01);
      gelu2_and_bwd(z23, x23, d23);
      X2p[j][0] = H::pack(x01.x, x01.y);
      X2p[j][1] = H::pack(x23.x, x23.y);
      const float2 r01 = H::unpack(H::pack(d01.x, d01.y)), r23 = H::unpack(H::pack(d23.x, d23.y));
      GP[j][0] = r01.x;
      GP[j][1] = r01.y;
      GP[j][2] = r23.x;
      GP[j][3] = r23.y;
      X2t[0][j] = movm_t(X2p[j][0]);
      X2t[1][j] = movm_t(X2p[j][1]);
    }
    // W2^T += (e G2)^T X2 (reversal); H = G2 W2_n^T; dX2bar = dZ2bar W2_n^T
    float Hh[4][4], dX2b[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) Hh[j][c] = dX2b[j][c] = 0.f;
    {
      float S2[4][4][4];
      slice_ld(tS2, &S2[0][0][0]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t a[4];
        ldsm_x4_t(a, sEG + swz128((mi >> 1) * 8 + r8, 2 * m + (mi & 1)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b[2] = {X2t[0][j], X2t[1][j]};
          mma16816<T>(S2[m][j], a, b);
        }
      }
      slice_st_async(tS2, &S2[0][0][0]);
#pragma unroll
      for (int kf = 0; kf < 4; ++kf) {
        uint32_t ag[4], ad[4];
        const uint32_t off = swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1));
        ldsm_x4(ag, sG + off);
        ldsm_x4(ad, sDZB + off);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b[2] = {movm_t(H::pack(S2[kf][j][0], S2[kf][j][1])),
                                 movm_t(H::pack(S2[kf][j][2], S2[kf][j][3]))};
          mma16816<T>(Hh[j], ag, b);
          mma16816<T>(dX2b[j], ad, b);
        }
      }
    }
    float G1[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) G1[j][c] = Hh[j][c] * GP[j][c];
    // W1^T += (e G1)^T XK (reversal)
    {
      uint32_t eb[2][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        eb[0][j] = movm_t(H::pack(eg0 * G1[j][0], eg0 * G1[j][1]));
        eb[1][j] = movm_t(H::pack(eg1 * G1[j][2], eg1 * G1[j][3]));
      }
      float S1[2][8][4];
      slice_ld(tS1, &S1[0][0][0]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bx[4];
        ldsm_x4_t(bx, sb + OFF_XK + swz128((mi & 1) * 8 + r8, 2 * np + (mi >> 1)));
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const uint32_t a[4] = {eb[0][2 * m], eb[0][2 * m + 1], eb[1][2 * m], eb[1][2 * m + 1]};
          mma16816<T>(S1[m][2 * np], a, bx);
          mma16816<T>(S1[m][2 * np + 1], a, bx + 2);
        }
      }
      slice_st_async(tS1, &S1[0][0][0]);
    }
    // dP2 = -dZ2bar G2^T and A1 = XQ XK^T (whole 16 x 16 in every warp)
    float dP2[2][4], A1[2][4];
#pragma unroll
    for (int jt = 0; jt < 2; ++jt)
#pragma unroll
      for (int c = 0; c < 4; ++c) dP2[jt][c] = A1[jt][c] = 0.f;
#pragma unroll
    for (int kf = 0; kf < 4; ++kf) {
      uint32_t adz[4], bgt[4], aq[4], bk[4];
      const uint32_t aoff = swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1));
      const uint32_t boff = swz128((mi >> 1) * 8 + r8, 2 * kf + (mi & 1));
      ldsm_x4(adz, sDZB + aoff);
      ldsm_x4(bgt, sG + boff);
      ldsm_x4(aq, sb + OFF_XQ + aoff);
      ldsm_x4(bk, sb + OFF_XK + boff);
      mma16816<T>(dP2[0], adz, bgt);
      mma16816<T>(dP2[1], adz, bgt + 2);
      mma16816<T>(A1[0], aq, bk);
      mma16816<T>(A1[1], aq, bk + 2);
    }
    float dA2[2][4], P1[2][4];
#pragma unroll
    for (int jt = 0; jt < 2; ++jt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        dP2[jt][c] = -dP2[jt][c];
        dA2[jt][c] = dP2[jt][c] * ev[jt][c];
        P1[jt][c] = ev[jt][c] * (A1[jt][c] + 1.f);
      }
    {  // dX2bar += dA2 X2
      uint32_t a[4];
      direct_afrag<T>(a, dA2, 1.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b[2] = {X2t[0][j], X2t[1][j]};
        mma16816<T>(dX2b[j], a, b);
      }
    }
    // X2bar = gelu(Z1bar); dZ1bar = dX2bar * gelu'(Z1bar); A2_w = X2bar X2^T; dX2 = dA2^T X2bar
    uint32_t XBt[2][4];
    float A2[2][4];
    {
      uint32_t XBp[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 z01 = *reinterpret_cast<const float2*>(Z1bs + g * ZLD + fb + 8 * j + 2 * t);
        const float2 z23 = *reinterpret_cast<const float2*>(Z1bs + (g + 8) * ZLD + fb + 8 * j + 2 * t);
        float2 x01, x23, d01, d23;
        gelu2_and_bwd(z01, x01, d01);
        gelu2_and_bwd(z23, x23, d23);
        XBp[j][0] = H::pack(x01.x, x01.y);
        XBp[j][1] = H::pack(x23.x, x23.y);
        XBt[0][j] = movm_t(XBp[j][0]);
        XBt[1][j] = movm_t(XBp[j][1]);
        Zbp[j][0] = H::pack(dX2b[j][0] * d01.x, dX2b[j][1] * d01.y);
        Zbp[j][1] = H::pack(dX2b[j][2] * d23.x, dX2b[j][3] * d23.y);
        Zbt[0][j] = movm_t(Zbp[j][0]);
        Zbt[1][j] = movm_t(Zbp[j][1]);
      }
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        A2[jt][0] = A2[jt][1] = A2[jt][2] = A2[jt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint32_t a[4] = {XBp[2 * ks][0], XBp[2 * ks][1], XBp[2 * ks + 1][0], XBp[2 * ks + 1][1]};
          const uint32_t b[2] = {X2p[2 * ks][jt], X2p[2 * ks + 1][jt]};
          mma16816<T>(A2[jt], a, b);
        }
      }
      uint32_t aT[4];
      transpose_afrag<T>(aT, dA2, 1.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dX2[j][0] = dX2[j][1] = dX2[j][2] = dX2[j][3] = 0.f;
        const uint32_t b[2] = {XBt[0][j], XBt[1][j]};
        mma16816<T>(dX2[j], aT, b);
      }
    }
    // carried dW2: dX2 -= e (G2 dW2^T), d e -= rowsum(X2 * (G2 dW2^T)); partial dG2 = (-e X2) dW2
    // straight to the warp's partial tile. dW2^T is processed in two halves of feature rows
    // (32 TMEM columns each) to keep registers free.
    float de0 = 0.f, de1 = 0.f;  // d e partials of tokens g, g + 8
    {
      uint32_t aX[4][2];  // -e X2 in accumulator-pair layout
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x01 = H::unpack(X2p[j][0]), x23 = H::unpack(X2p[j][1]);
        aX[j][0] = H::pack(-eg0 * x01.x, -eg0 * x01.y);
        aX[j][1] = H::pack(-eg1 * x23.x, -eg1 * x23.y);
      }
      float GD[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) GD[j][0] = GD[j][1] = GD[j][2] = GD[j][3] = 0.f;
      float* pw = PA + warp * C * PLD;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float D2h[2][4][4];  // feature tiles m = 2 half, 2 half + 1
        tmem_ld32(tD2 + 32 * half, &D2h[0][0][0]);
        tmem_wait_ld();
#pragma unroll
        for (int mm = 0; mm < 2; ++mm) {
          uint32_t ag[4];
          ldsm_x4(ag, sG + swz128((mi & 1) * 8 + r8, 2 * (2 * half + mm) + (mi >> 1)));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t b[2] = {movm_t(H::pack(D2h[mm][j][0], D2h[mm][j][1])),
                                   movm_t(H::pack(D2h[mm][j][2], D2h[mm][j][3]))};
            mma16816<T>(GD[j], ag, b);
          }
        }
#pragma unroll
        for (int nh = 0; nh < 4; ++nh) {  // output feature tiles nf = 4 half + nh
          const int nf = 4 * half + nh, mm = nh >> 1, hh = 2 * (nh & 1);
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint32_t a[4] = {aX[2 * ks][0], aX[2 * ks][1], aX[2 * ks + 1][0], aX[2 * ks + 1][1]};
            const uint32_t b[2] = {H::pack(D2h[mm][2 * ks][hh], D2h[mm][2 * ks][hh + 1]),
                                   H::pack(D2h[mm][2 * ks + 1][hh], D2h[mm][2 * ks + 1][hh + 1])};
            mma16816<T>(acc, a, b);
          }
          *reinterpret_cast<float2*>(pw + g * PLD + 8 * nf + 2 * t) = make_float2(acc[0], acc[1]);
          *reinterpret_cast<float2*>(pw + (g + 8) * PLD + 8 * nf + 2 * t) = make_float2(acc[2], acc[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x01 = H::unpack(X2p[j][0]), x23 = H::unpack(X2p[j][1]);
        dX2[j][0] -= eg0 * GD[j][0];
        dX2[j][1] -= eg0 * GD[j][1];
        dX2[j][2] -= eg1 * GD[j][2];
        dX2[j][3] -= eg1 * GD[j][3];
        de0 -= x01.x * GD[j][0] + x01.y * GD[j][1];
        de1 -= x23.x * GD[j][2] + x23.y * GD[j][3];
      }
    }
    // carried dW1, db1: dG1 = -e (XK dW1 + db1), d e -= rowsum((XK dW1 + db1) * G1);
    // partial dXK = (-e G1) dW1^T. dW1^T in two halves of hidden rows (m-tiles).
    float dG1[4][4];
    {
      float KD[8][4];
#pragma unroll
      for (int nf = 0; nf < 8; ++nf) KD[nf][0] = KD[nf][1] = KD[nf][2] = KD[nf][3] = 0.f;
#pragma unroll
      for (int mh = 0; mh < 2; ++mh) {
        float D1h[8][4];  // hidden rows 16 mh .. of the slice
        tmem_ld32(tD1 + 32 * mh, &D1h[0][0]);
        tmem_wait_ld();
        float XD[2][4];  // hidden tiles j = 2 mh, 2 mh + 1
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) XD[jj][0] = XD[jj][1] = XD[jj][2] = XD[jj][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t ak[4];
          ldsm_x4(ak, sb + OFF_XK + swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1)));
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int hh = 2 * jj;
            const uint32_t b[2] = {H::pack(D1h[2 * kk][hh], D1h[2 * kk][hh + 1]),
                                   H::pack(D1h[2 * kk + 1][hh], D1h[2 * kk + 1][hh + 1])};
            mma16816<T>(XD[jj], ak, b);
          }
        }
        uint32_t aG[2][2];  // -e G1 for j = 2 mh, 2 mh + 1
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * mh + jj;
          const float u0 = XD[jj][0] + DB1[j][0], u1 = XD[jj][1] + DB1[j][1];
          const float u2 = XD[jj][2] + DB1[j][0], u3 = XD[jj][3] + DB1[j][1];
          de0 -= u0 * G1[j][0] + u1 * G1[j][1];
          de1 -= u2 * G1[j][2] + u3 * G1[j][3];
          dG1[j][0] = -eg0 * u0;
          dG1[j][1] = -eg0 * u1;
          dG1[j][2] = -eg1 * u2;
          dG1[j][3] = -eg1 * u3;
          aG[jj][0] = H::pack(-eg0 * G1[j][0], -eg0 * G1[j][1]);
          aG[jj][1] = H::pack(-eg1 * G1[j][2], -eg1 * G1[j][3]);
        }
        const uint32_t a[4] = {aG[0][0], aG[0][1], aG[1][0], aG[1][1]};
#pragma unroll
        for (int nf = 0; nf < 8; ++nf) {
          const uint32_t b[2] = {movm_t(H::pack(D1h[nf][0], D1h[nf][1])), movm_t(H::pack(D1h[nf][2], D1h[nf][3]))};
          mma16816<T>(KD[nf], a, b);
        }
      }
      put_part<false>(PB + warp * C * PLD, KD, g, t);
    }
    // dG1 += -P1^T dZ1bar; dH = dG1 * gelu_bwd(Z1); dZ1 = dG1 * H * gelu_bwd'(Z1)
    uint32_t dHp[4][2];
    {
      uint32_t aPT[4];
      transpose_afrag<T>(aPT, P1, -1.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b[2] = {Zbt[0][j], Zbt[1][j]};
        mma16816<T>(dG1[j], aPT, b);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 z01 = *reinterpret_cast<const float2*>(Z1s + g * ZLD + fb + 8 * j + 2 * t);
        const float2 z23 = *reinterpret_cast<const float2*>(Z1s + (g + 8) * ZLD + fb + 8 * j + 2 * t);
        const float2 q01 = gelu2_bwd_grad(z01), q23 = gelu2_bwd_grad(z23);
        dZ1[j][0] = dG1[j][0] * Hh[j][0] * q01.x;
        dZ1[j][1] = dG1[j][1] * Hh[j][1] * q01.y;
        dZ1[j][2] = dG1[j][2] * Hh[j][2] * q23.x;
        dZ1[j][3] = dG1[j][3] * Hh[j][3] * q23.y;
        dHp[j][0] = H::pack(dG1[j][0] * GP[j][0], dG1[j][1] * GP[j][1]);
        dHp[j][1] = H::pack(dG1[j][2] * GP[j][2], dG1[j][3] * GP[j][3]);
      }
    }
    // partial dG2 += dH W2_n - (eta * (A2_w [+1]))^T dZ2bar (added to the partial tile)
    {
      float PG[8][4];
      uint32_t aYT[4];
      {
        float Y[2][4];
#pragma unroll
        for (int jt = 0; jt < 2; ++jt)
#pragma unroll
          for (int c = 0; c < 4; ++c) Y[jt][c] = ev[jt][c] * (A2[jt][c] + one_w0);
        transpose_afrag<T>(aYT, Y, -1.f);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bz[4];
        ldsm_x4_t(bz, sDZB + swz128((mi & 1) * 8 + r8, 2 * np + (mi >> 1)));
        PG[2 * np][0] = PG[2 * np][1] = PG[2 * np][2] = PG[2 * np][3] = 0.f;
        PG[2 * np + 1][0] = PG[2 * np + 1][1] = PG[2 * np + 1][2] = PG[2 * np + 1][3] = 0.f;
        mma16816<T>(PG[2 * np], aYT, bz);
        mma16816<T>(PG[2 * np + 1], aYT, bz + 2);
      }
      tmem_wait_st();  // the reversed W2 this step stored (without waiting) earlier in M1
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float S2h[2][4][4];
        tmem_ld32(tS2 + 32 * half, &S2h[0][0][0]);
        tmem_wait_ld();
#pragma unroll
        for (int nh = 0; nh < 4; ++nh) {
          const int nf = 4 * half + nh, mm = nh >> 1, hh = 2 * (nh & 1);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint32_t a[4] = {dHp[2 * ks][0], dHp[2 * ks][1], dHp[2 * ks + 1][0], dHp[2 * ks + 1][1]};
            const uint32_t b[2] = {H::pack(S2h[mm][2 * ks][hh], S2h[mm][2 * ks][hh + 1]),
                                   H::pack(S2h[mm][2 * ks + 1][hh], S2h[mm][2 * ks + 1][hh + 1])};
            mma16816<T>(PG[nf], a, b);
          }
        }
      }
      put_part<true>(PA + warp * C * PLD, PG, g, t);
    }
    // dW2^T += dZ2bar^T X2bar + G2^T dH
    {
      uint32_t dHt[2][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dHt[0][j] = movm_t(dHp[j][0]);
        dHt[1][j] = movm_t(dHp[j][1]);
      }
      float D2[4][4][4];
      slice_ld(tD2, &D2[0][0][0]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t a1[4], a2[4];
        const uint32_t off = swz128((mi >> 1) * 8 + r8, 2 * m + (mi & 1));
        ldsm_x4_t(a1, sDZB + off);
        ldsm_x4_t(a2, sG + off);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b1[2] = {XBt[0][j], XBt[1][j]};
          const uint32_t b2[2] = {dHt[0][j], dHt[1][j]};
          mma16816<T>(D2[m][j], a1, b1);
          mma16816<T>(D2[m][j], a2, b2);
        }
      }
      slice_st_async(tD2, &D2[0][0][0]);
    }
    // partial dP1 = -dZ1bar G1^T; partial d_eta = dP2 * (A2_w [+1]) + dP1_w * (A1 + 1); d e
    {
      float dP1[2][4];
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        dP1[jt][0] = dP1[jt][1] = dP1[jt][2] = dP1[jt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint32_t a[4] = {Zbp[2 * ks][0], Zbp[2 * ks][1], Zbp[2 * ks + 1][0], Zbp[2 * ks + 1][1]};
          const uint32_t b[2] = {H::pack(G1[2 * ks][2 * jt], G1[2 * ks][2 * jt + 1]),
                                 H::pack(G1[2 * ks + 1][2 * jt], G1[2 * ks + 1][2 * jt + 1])};
          mma16816<T>(dP1[jt], a, b);
        }
      }
      float* dp = DP1P + warp * C * C;
      float* de = DETAP + warp * C * C;
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        float v[4], w[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[c] = -dP1[jt][c];
          w[c] = dP2[jt][c] * (A2[jt][c] + one_w0) + v[c] * (A1[jt][c] + 1.f);
        }
        const int c0 = 8 * jt + 2 * t;
        *reinterpret_cast<float2*>(dp + g * C + c0) = make_float2(v[0], v[1]);
        *reinterpret_cast<float2*>(dp + (g + 8) * C + c0) = make_float2(v[2], v[3]);
        *reinterpret_cast<float2*>(de + g * C + c0) = make_float2(w[0], w[1]);
        *reinterpret_cast<float2*>(de + (g + 8) * C + c0) = make_float2(w[2], w[3]);
      }
      de0 += __shfl_xor_sync(0xffffffffu, de0, 1);
      de0 += __shfl_xor_sync(0xffffffffu, de0, 2);
      de1 += __shfl_xor_sync(0xffffffffu, de1, 1);
      de1 += __shfl_xor_sync(0xffffffffu, de1, 2);
      if (t == 0) {
        DE[warp * C + g] = de0;
        DE[warp * C + g + 8] = de1;
      }
    }
    }  // M1
    if constexpr (kAhead) {
      if (warp >= NW && it + 1 < p.NC) {  // row-only warps: stage and R1 part 1 of mini-batch n - 1
        uint8_t* nx = smem + ((it + 1) % NSTAGE) * STAGE;
        load_stage<NW, NRT>(nx, p, s, n - 1, 32 * NW);
        cp_async_commit();
        cp_async_wait<0>();
        asm volatile("bar.sync 1, %0;" ::"r"(NRT) : "memory");  // the row-only warps' copies landed
        r1_g(nx, (n - 1) & 1, (tid - 32 * NW) >> 4, NRT / 16, false);
      }
    }
    TTT_BSTAMP(4);
    __syncthreads();
    TTT_BSTAMP(5);

    // ---------------- R2: dG2 -> backward of G2 = ln_fused_l2_bwd(Z2, XV - XK); d_eta, dP1
    float DTr[NPASS][4];
#pragma unroll
    for (int ps = 0; ps < NPASS; ++ps) {
      const int tk = tk0 + ps * TPP;
      const uint32_t xo = xo_of(tk);
      float dG[4], xv[4], xk[4], xh[4], gh[4], Gr[4], rstd;
      g2_rows(tk, xh, gh, Gr, rstd);
      sum_part<NW>(PA, tk, q, dG);
      const float e = (float)E[(C - 1) * C + tk];
      const float4 db = *reinterpret_cast<const float4*>(DB2 + 4 * q);
      if constexpr (kAhead) {  // R1's db2 term, here where db2 is current
        const float dot = red16(Gr[0] * db.x + Gr[1] * db.y + Gr[2] * db.z + Gr[3] * db.w);
        if (q == 0) DE2[tk] = -dot;
      }
      dG[0] -= e * db.x;
      dG[1] -= e * db.y;
      dG[2] -= e * db.z;
      dG[3] -= e * db.w;
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
      float dxh[4], sx = 0.f, sxx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float dgh = (F * dG[j] - sdG - xh[j] * sdGx) * inv;
        dxh[j] = -(dG[j] * sgx + gh[j] * sdGx) * inv + dgh * gm[j] * gm[j];
        DTr[ps][j] = -dgh * gm[j];
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
      *reinterpret_cast<uint2*>(smem + OFF_DZ2 + xo) = make_uint2(H::pack(dz[0], dz[1]), H::pack(dz[2], dz[3]));
      *reinterpret_cast<uint2*>((uint8_t*)p.dXV + (xb + tk * F + 4 * q) * 2) =
          make_uint2(H::pack(DTr[ps][0], DTr[ps][1]), H::pack(DTr[ps][2], DTr[ps][3]));
    }
    if constexpr (kAhead) __syncthreads();  // DE2 of every token written
#pragma unroll
    for (int el = tid; el < C * C; el += NTHREADS) {  // element (el / C, el % C) of d_eta and dP1
      float v = 0.f, u = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        v += DETAP[w * C * C + el];
        u += DP1P[w * C * C + el];
      }
      if ((el >> 4) == C - 1) {
        const int j = el & 15;
        float de = DE2[j];
#pragma unroll
        for (int w = 0; w < NW; ++w) de += DE[w * C + j];
        v += de;
      }
      reinterpret_cast<T*>(p.deta)[(s * p.NC + n) * (long long)(C * C) + el] = H::from_float(v);
      DP1[el] = u;
    }
    TTT_BSTAMP(6);
    __syncthreads();
    TTT_BSTAMP(7);

    // ---------------- M2 (the NW MMA warps)
    if (warp < NW) {
    tmem_wait_st();  // M1's stores of W1, W2, dW2 (issued without waiting) landed
    // dX2 += dZ2 W2_n^T ; dW2^T += dZ2^T X2 ; db2 += 1^T (dZ2bar + dZ2) (warp w: features
    // 8fw..8fw+7 for fw = w, w + NW, ..)
    {
      float S2[4][4][4];
      slice_ld(tS2, &S2[0][0][0]);
#pragma unroll
      for (int kf = 0; kf < 4; ++kf) {
        uint32_t ad[4];
        ldsm_x4(ad, sDZ2 + swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b[2] = {movm_t(H::pack(S2[kf][j][0], S2[kf][j][1])),
                                 movm_t(H::pack(S2[kf][j][2], S2[kf][j][3]))};
          mma16816<T>(dX2[j], ad, b);
        }
      }
    }
    {
      float D2[4][4][4];
      slice_ld(tD2, &D2[0][0][0]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t a[4];
        ldsm_x4_t(a, sDZ2 + swz128((mi >> 1) * 8 + r8, 2 * m + (mi & 1)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b[2] = {X2t[0][j], X2t[1][j]};
          mma16816<T>(D2[m][j], a, b);
        }
      }
      slice_st_async(tD2, &D2[0][0][0]);
    }
#pragma unroll
    for (int fw = warp; fw < F / 8; fw += NW) {
      uint32_t b1[2], b2[2];
      const uint32_t off = swz128((lane & 8) + r8, fw);
      ldsm_x2_t(b1, sDZB + off);
      ldsm_x2_t(b2, sDZ2 + off);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816<T>(acc, a_ones, b1);
      mma16816<T>(acc, a_ones, b2);
      if (g == 0) {
        DB2[8 * fw + 2 * t] += acc[0];
        DB2[8 * fw + 2 * t + 1] += acc[1];
      }
    }
    // dZ1 += dX2 * gelu'(Z1)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) dZ1[j][c] += dX2[j][c] * GP[j][c];
    uint32_t Z1p[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      Z1p[j][0] = H::pack(dZ1[j][0], dZ1[j][1]);
      Z1p[j][1] = H::pack(dZ1[j][2], dZ1[j][3]);
    }
    // dA1 = dP1 * eta as A fragments, plain and transposed
    uint32_t aA1[4], aA1T[4];
    {
      auto da = [&](int r, int c) { return DP1[r * C + c] * (float)E[r * C + c]; };
      aA1[0] = H::pack(da(g, 2 * t), da(g, 2 * t + 1));
      aA1[1] = H::pack(da(g + 8, 2 * t), da(g + 8, 2 * t + 1));
      aA1[2] = H::pack(da(g, 2 * t + 8), da(g, 2 * t + 9));
      aA1[3] = H::pack(da(g + 8, 2 * t + 8), da(g + 8, 2 * t + 9));
      aA1T[0] = H::pack(da(2 * t, g), da(2 * t + 1, g));
      aA1T[1] = H::pack(da(2 * t, g + 8), da(2 * t + 1, g + 8));
      aA1T[2] = H::pack(da(2 * t + 8, g), da(2 * t + 9, g));
      aA1T[3] = H::pack(da(2 * t + 8, g + 8), da(2 * t + 9, g + 8));
    }
    // partial dXQ = dZ1bar W1_n^T (+ dA1 XK), partial dXK += dZ1 W1_n^T (+ dA1^T XQ); the dA1
    // terms go to warp w's columns 8fw..8fw+7 (fw = w, w + NW, ..) only, the reduction adds
    // them once
    {
      float QX[8][4], KX[8][4];
#pragma unroll
      for (int nf = 0; nf < 8; ++nf)
#pragma unroll
        for (int c = 0; c < 4; ++c) QX[nf][c] = KX[nf][c] = 0.f;
      float S1[2][8][4];
      slice_ld(tS1, &S1[0][0][0]);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const uint32_t az[4] = {Zbp[2 * ks][0], Zbp[2 * ks][1], Zbp[2 * ks + 1][0], Zbp[2 * ks + 1][1]};
        const uint32_t a1[4] = {Z1p[2 * ks][0], Z1p[2 * ks][1], Z1p[2 * ks + 1][0], Z1p[2 * ks + 1][1]};
#pragma unroll
        for (int nf = 0; nf < 8; ++nf) {
          const uint32_t b[2] = {movm_t(H::pack(S1[ks][nf][0], S1[ks][nf][1])),
                                 movm_t(H::pack(S1[ks][nf][2], S1[ks][nf][3]))};
          mma16816<T>(QX[nf], az, b);
          mma16816<T>(KX[nf], a1, b);
        }
      }
#pragma unroll
      for (int fw = 0; fw < F / 8; ++fw)
        if (fw % NW == warp) {
          uint32_t bxk[2], bxq[2];
          const uint32_t off = swz128((lane & 8) + r8, fw);
          ldsm_x2_t(bxk, sb + OFF_XK + off);
          ldsm_x2_t(bxq, sb + OFF_XQ + off);
          float cq[4] = {0.f, 0.f, 0.f, 0.f}, ck[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816<T>(cq, aA1, bxk);
          mma16816<T>(ck, aA1T, bxq);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            QX[fw][c] += cq[c];
            KX[fw][c] += ck[c];
          }
        }
      put_part<false>(PA + warp * C * PLD, QX, g, t);
      put_part<true>(PB + warp * C * PLD, KX, g, t);
    }
    // dW1^T += dZ1bar^T XQ + dZ1^T XK ; db1 += 1^T (dZ1bar + dZ1)
    {
      uint32_t Z1t[2][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Z1t[0][j] = movm_t(Z1p[j][0]);
        Z1t[1][j] = movm_t(Z1p[j][1]);
      }
      float D1[2][8][4];
      slice_ld(tD1, &D1[0][0][0]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bq[4], bk[4];
        const uint32_t off = swz128((mi & 1) * 8 + r8, 2 * np + (mi >> 1));
        ldsm_x4_t(bq, sb + OFF_XQ + off);
        ldsm_x4_t(bk, sb + OFF_XK + off);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const uint32_t a1[4] = {Zbt[0][2 * m], Zbt[0][2 * m + 1], Zbt[1][2 * m], Zbt[1][2 * m + 1]};
          const uint32_t a2[4] = {Z1t[0][2 * m], Z1t[0][2 * m + 1], Z1t[1][2 * m], Z1t[1][2 * m + 1]};
          mma16816<T>(D1[m][2 * np], a1, bq);
          mma16816<T>(D1[m][2 * np + 1], a1, bq + 2);
          mma16816<T>(D1[m][2 * np], a2, bk);
          mma16816<T>(D1[m][2 * np + 1], a2, bk + 2);
        }
      }
      slice_st_async(tD1, &D1[0][0][0]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t b1[2] = {Zbt[0][j], Zbt[1][j]};
        const uint32_t b2[2] = {Z1t[0][j], Z1t[1][j]};
        mma16816<T>(acc, a_ones, b1);
        mma16816<T>(acc, a_ones, b2);
        DB1[j][0] += acc[0];
        DB1[j][1] += acc[1];
      }
    }
    }  // M2
    if constexpr (kAhead) {
      if (warp >= NW && it + 1 < p.NC)  // row-only warps: R1 part 2 of mini-batch n - 1
        r1_dzb(smem + ((it + 1) % NSTAGE) * STAGE, (n - 1) & 1, (tid - 32 * NW) >> 4, NRT / 16);
    }
    TTT_BSTAMP(8);
    __syncthreads();
    TTT_BSTAMP(9);

    // ---------------- R3: dXQ = dO + sum of partials, dXK = sum of partials - dXV
#pragma unroll
    for (int ps = 0; ps < NPASS; ++ps) {
      const int tk = tk0 + ps * TPP;
      const uint32_t xo = xo_of(tk);
      float dq[4], dk[4], dO4[4];
      sum_part<NW>(PA, tk, q, dq);
      sum_part<NW>(PB, tk, q, dk);
      unpack4<T>(st + OFF_DO + xo, dO4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dq[j] += dO4[j];
        dk[j] -= DTr[ps][j];
      }
      const long long o = (xb + tk * F + 4 * q) * 2;
      *reinterpret_cast<uint2*>((uint8_t*)p.dXQ + o) = make_uint2(H::pack(dq[0], dq[1]), H::pack(dq[2], dq[3]));
      *reinterpret_cast<uint2*>((uint8_t*)p.dXK + o) = make_uint2(H::pack(dk[0], dk[1]), H::pack(dk[2], dk[3]));
    }
    TTT_BSTAMP(10);
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- outputs of the whole walk: dW1, dW2, db1, db2 (fp32), per-stream gamma / beta partials
  if (warp < NW) {
    float D1[2][8][4];
    tmem_wait_st();
    slice_ld(tD1, &D1[0][0][0]);
    w1_io<2, FFW>(D1, p.dW1 + s * F * FFW, fb, g, t, true);
    float D2[4][4][4];
    slice_ld(tD2, &D2[0][0][0]);
    w2_io(D2, p.dW2 + s * FFW * F, fb, g, t, true);
  }
  if (warp < NW && g == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p.db1[s * FFW + fb + 8 * j + 2 * t] = DB1[j][0];
      p.db1[s * FFW + fb + 8 * j + 2 * t + 1] = DB1[j][1];
    }
  }
  if (tid < F) p.db2[s * F + tid] = DB2[tid];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    dgam[j] += __shfl_xor_sync(0xffffffffu, dgam[j], 16);
    dbet[j] += __shfl_xor_sync(0xffffffffu, dbet[j], 16);
  }
  float* RED = PA;  // [NR][2][F]
  if ((lane & 16) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      RED[(warp * 2 + 0) * F + 4 * q + j] = dgam[j];
      RED[(warp * 2 + 1) * F + 4 * q + j] = dbet[j];
    }
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  for (int e = tid; e < 2 * F; e += NTHREADS) {
    const int which = e / F, f = e % F;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NR; ++w) acc += RED[(w * 2 + which) * F + f];
    (which == 0 ? p.d_ln_w : p.d_ln_b)[s * F + f] = acc;
  }
  // every warp's TMEM accesses are complete (the loads / stores above waited); free the columns
  if (warp == 0) tmem_dealloc(tmem_base_sh, TMEM_COLS);
}

}  // namespace bwd
}  // namespace mlp_tc

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T, int NW>
static int launch_bwd(const MlpBwdParams& p, cudaStream_t stream) {
  using namespace mlp_tc::bwd;
  int rc = prepare_smem(mlp_bwd_tc_kernel<T, NW>, Bwd<NW>::SMEM, "ttt_mlp_bwd");
  if (rc) return rc;
  mlp_bwd_tc_kernel<T, NW><<<p.B * p.NH, Bwd<NW>::NTHREADS, Bwd<NW>::SMEM, stream>>>(p);
  return check_launch("ttt_mlp_bwd");
}

int mlp_bwd_fast(const MlpBwdParams& p, cudaStream_t stream) {
  using namespace mlp_tc;
  using namespace mlp_tc::bwd;
  if (!p.Z1_saved || !p.Z2_saved || !p.Z1b_saved || !p.Z2b_saved || !p.W1_last || !p.W2_last)
    return TTT_NOT_APPLICABLE;
  if (p.CS != C || p.F != F || (p.FF != 256 && p.FF != 64)) return TTT_NOT_APPLICABLE;
  const int dt = p.dt_xq;
  if (dt != DT_BF16 && dt != DT_F16) return TTT_NOT_APPLICABLE;
  if (p.dt_xk != dt || p.dt_xv != dt || p.dt_eta != dt || p.dt_dout != dt || p.dt_grad != dt) return TTT_NOT_APPLICABLE;
  if (!aligned16(p.XQ) || !aligned16(p.XK) || !aligned16(p.XV) || !aligned16(p.eta) || !aligned16(p.dout) ||
      !aligned16(p.Z1_saved) || !aligned16(p.Z2_saved) || !aligned16(p.Z1b_saved) || !aligned16(p.Z2b_saved) ||
      !aligned16(p.dXQ) || !aligned16(p.dXK) || !aligned16(p.dXV))
    return TTT_NOT_APPLICABLE;
  if (p.FF == 256)
    return dt == DT_BF16 ? launch_bwd<__nv_bfloat16, 8>(p, stream) : launch_bwd<__half, 8>(p, stream);
  return dt == DT_BF16 ? launch_bwd<__nv_bfloat16, 2>(p, stream) : launch_bwd<__half, 2>(p, stream);
}

}  // namespace ttt

#ifdef TTT_PHASE_STAMPS
// Copies the backward's timeline: rows x 12 values (11 stamps in ns, SM id).
extern "C" int ttt_bwd_phase_stamps_read(unsigned long long* out, int rows) {
  using namespace ttt::mlp_tc::bwd;
  if (rows < 0 || rows > kBStampCTAs) return TTT_ERR_SHAPE;
  return cudaMemcpyFromSymbol(out, g_bwd_stamps, sizeof(unsigned long long) * kBStamps * rows) == cudaSuccess
             ? TTT_OK
             : TTT_ERR_CUDA;
}
#endif
