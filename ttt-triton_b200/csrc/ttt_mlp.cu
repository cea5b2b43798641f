// TTT-MLP dual-form scan (F -> FF -> F, tanh-GELU): forward, backward and the memo
// read-out, one CTA per (batch, head) stream.
//
// Reference semantics: ops/ttt_mlp.py:9-67 (dual form, full eta, LN eps 1e-8). Launch
// boundaries: mlp_triton.py:130-178 (forward, incl. memo outputs), :274-333 (backward),
// mlp_triton_back.py (same with FF == F) and kernels/mlp_cached_readout.py:112-143.
// The backward is the hand derivation of autograd through the step, with checkpoint-group
// recompute; inside a group the state entering mini-batch n is recovered from the state
// after it: W2_n = W2_{n+1} + X2^T diag(e) G2, then G1 = (G2 W2_n^T) * gelu_bwd(Z1) and
// W1_n = W1_{n+1} + XK^T diag(e) G1, with X2, G2, Z1 rebuilt from the stored Z1, Z2.
//
// This is the general path: fp32 FMA math on shared-memory tiles; the F x FF inner
// weights live in global memory (the W*_last outputs in the forward, the scratch buffer
// in the backward) where they stay L2-resident, per-row activations in shared memory.
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "params.cuh"

namespace ttt {

// Threads of a general-kernel CTA (one stream): up to sixteen warps (the kernels fit 128
// registers per thread). Narrow inner states (F, FF <= 64: the reference's main.py model)
// get sixteen, for latency hiding in their chains of small barrier-separated products
// (forward 0.34 -> 0.24 ms, backward 1.05 -> 0.83 ms there); wider ones keep eight, whose
// products then still fill every thread with 4 x 4 FMA tiles (sixteen warps: 14.6 -> 18.3 ms
// for an fp32 F 64, FF 256 backward).
constexpr int kGenThreads = 512;
static int gen_threads(int F, int FF) { return F <= 64 && FF <= 64 ? 512 : 256; }

__device__ __forceinline__ void copy_state(float* dst, const float* src, long long n) {
  for (long long i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// TC: the products on the TF32 tensor cores (16-bit activations), else on fp32 FMA.
template <bool TC>
__global__ void __launch_bounds__(kGenThreads) mlp_fwd_kernel(MlpFwdParams p) {
  extern __shared__ float sm[];
  const int C = p.CS, F = p.F, FF = p.FF;
  const int CF = C * F, CFF = C * FF, CC = C * C;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);

  float* b1 = sm;
  float* tmp1 = b1 + FF;
  float* b2 = tmp1 + FF;
  float* tmp2 = b2 + F;
  float* gam = tmp2 + F;
  float* bet = gam + F;
  float* XQ = bet + F;
  float* XK = XQ + CF;
  float* XV = XK + CF;
  float* Z2 = XV + CF;
  float* G2 = Z2 + CF;
  float* Z2b = G2 + CF;
  float* XKe = Z2b + CF;
  float* Z1 = XKe + CF;
  float* X2 = Z1 + CFF;
  float* G1 = X2 + CFF;
  float* Z1b = G1 + CFF;  // then X2_bar
  float* X2e = Z1b + CFF;
  float* E = X2e + CFF;
  float* P1 = E + CC;
  float* P2 = P1 + CC;

  float* W1 = p.W1_last + s * F * FF;  // running state, in place
  float* W2 = p.W2_last + s * FF * F;
  copy_state(W1, p.W1_init + s * F * FF, (long long)F * FF);
  copy_state(W2, p.W2_init + s * FF * F, (long long)FF * F);
  copy_f32(b1, p.b1_init + s * FF, FF);
  copy_f32(b2, p.b2_init + s * F, F);
  load_tile(gam, p.ln_w, (long long)h * F, F, p.dt_ln);
  load_tile(bet, p.ln_b, (long long)h * F, F, p.dt_ln);
  __syncthreads();

  for (int n = 0; n < p.NC; ++n) {
    if (p.W1_ckpt && n % p.ckpt == 0) {
      const long long k = s * p.K + n / p.ckpt;
      copy_state(p.W1_ckpt + k * F * FF, W1, (long long)F * FF);
      copy_state(p.W2_ckpt + k * FF * F, W2, (long long)FF * F);
      copy_f32(p.b1_ckpt + k * FF, b1, FF);
      copy_f32(p.b2_ckpt + k * F, b2, F);
    }
    const long long xb = (s * p.NC + n) * CF;
    const long long eb = (s * p.NC + n) * CC;
    load_tile(XQ, p.XQ, xb, CF, p.dt_xq);
    load_tile(XK, p.XK, xb, CF, p.dt_xk);
    load_tile(XV, p.XV, xb, CF, p.dt_xv);
    load_tile(E, p.eta, eb, CC, p.dt_eta);
    __syncthreads();
    const float* e = E + (C - 1) * C;

    block_mm_sel<TC, false, false>(Z1, FF, XK, F, W1, FF, C, FF, F, 1.f, 0.f);   // Z1  = XK W1
    block_mm_sel<TC, false, false>(Z1b, FF, XQ, F, W1, FF, C, FF, F, 1.f, 0.f);  // Z1b = XQ W1
    block_mm_sel<TC, false, true>(P1, C, XQ, F, XK, F, C, C, F, 1.f, 0.f);       // A1 = XQ XK^T
    __syncthreads();
    for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
      const float z = Z1[i] + b1[i % FF];
      Z1[i] = z;
      if (p.Z1_out) p.Z1_out[(s * p.NC + n) * CFF + i] = z;
      const float x2 = gelu_tanh(z);
      X2[i] = x2;
      X2e[i] = e[i / FF] * x2;
      Z1b[i] += b1[i % FF];
    }
    for (int i = threadIdx.x; i < CC; i += blockDim.x) P1[i] = E[i] * (P1[i] + 1.f);
    for (int i = threadIdx.x; i < CF; i += blockDim.x) XKe[i] = e[i / F] * XK[i];
    __syncthreads();
    block_mm_sel<TC, false, false>(Z2, F, X2, FF, W2, F, C, F, FF, 1.f, 0.f);  // Z2 = X2 W2
    __syncthreads();
    ln_fused_rows(Z2, G2, b2, XV, XK, gam, bet, C, F, nullptr, nullptr);
    __syncthreads();
    if (p.Z2_out)
      for (int i = threadIdx.x; i < CF; i += blockDim.x) p.Z2_out[xb + i] = Z2[i];
    block_mm_sel<TC, false, true>(G1, FF, G2, F, W2, F, C, FF, F, 1.f, 0.f);  // H = G2 W2^T
    __syncthreads();
    for (int i = threadIdx.x; i < CFF; i += blockDim.x) G1[i] *= gelu_bwd_ref(Z1[i]);
    __syncthreads();
    block_mm_sel<TC, false, false>(Z1b, FF, P1, C, G1, FF, C, FF, C, -1.f, 1.f);  // Z1b -= P1 G1
    __syncthreads();
    for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
      if (p.Z1b_out) p.Z1b_out[(s * p.NC + n) * CFF + i] = Z1b[i];
      Z1b[i] = gelu_tanh(Z1b[i]);  // X2_bar
    }
    __syncthreads();
    block_mm_sel<TC, false, true>(P2, C, Z1b, FF, X2, FF, C, C, FF, 1.f, 0.f);  // A2 = X2b X2^T
    block_mm_sel<TC, false, false>(Z2b, F, Z1b, FF, W2, F, C, F, FF, 1.f, 0.f);  // Z2b = X2b W2
    __syncthreads();
    for (int i = threadIdx.x; i < CC; i += blockDim.x) P2[i] = E[i] * (P2[i] + 1.f);
    __syncthreads();
    block_mm_sel<TC, false, false>(Z2b, F, P2, C, G2, F, C, F, C, -1.f, 1.f);  // Z2b -= P2 G2
    __syncthreads();
    readout_ln_store_rows(Z2b, b2, XQ, gam, bet, C, F, kLnEps, p.out, xb, p.dt_out);
    if (p.Z2b_out) {
      __syncthreads();
      for (int i = threadIdx.x; i < CF; i += blockDim.x) p.Z2b_out[xb + i] = Z2b[i];
    }
    block_mm_sel<TC, true, false>(W1, FF, XKe, F, G1, FF, F, FF, C, -1.f, 1.f);  // W1 -= (e*XK)^T G1
    block_mm_sel<TC, true, false>(W2, F, X2e, FF, G2, F, FF, F, C, -1.f, 1.f);  // W2 -= (e*X2)^T G2
    weighted_colsum(tmp1, e, G1, C, FF);
    weighted_colsum(tmp2, e, G2, C, F);
    __syncthreads();
    for (int j = threadIdx.x; j < FF; j += blockDim.x) b1[j] -= tmp1[j];
    for (int j = threadIdx.x; j < F; j += blockDim.x) b2[j] -= tmp2[j];
    __syncthreads();
    if (p.W1_memo && n % p.memo == 0) {
      const long long m = s * p.NS + n / p.memo;
      copy_state(p.W1_memo + m * F * FF, W1, (long long)F * FF);
      copy_state(p.W2_memo + m * FF * F, W2, (long long)FF * F);
      copy_f32(p.b1_memo + m * FF, b1, FF);
      copy_f32(p.b2_memo + m * F, b2, F);
    }
  }
  copy_f32(p.b1_last + s * FF, b1, FF);
  copy_f32(p.b2_last + s * F, b2, F);
}

// Shared-memory budget of the general backward's fp32 tiles (bytes; default the opt-in
// maximum per CTA).
#ifndef TTT_BWD_SMEM_CAP
#define TTT_BWD_SMEM_CAP 232448
#endif
constexpr long long kMlpBwdSmemFloats = TTT_BWD_SMEM_CAP / 4;

// The general backward's fp32 tiles, carved in a fixed order: into shared memory while they
// fit in `cap` floats, then (from the first that does not, all the rest) into the stream's
// spill region of the global scratch, which stays L2-resident. Every shape then runs; the
// mini-batch-16 shapes keep every tile on chip. Tiles whose lives within a walk step do not
// overlap share a buffer (noted below); the C x C tiles come last, those read by products
// first, so at large mini-batches (64) the ones that spill are only read element-wise. With
// null bases this only counts: returns the shared-memory floats used and stores the spill
// floats.
struct BwdTiles {
  float *b1, *db1, *tmp1, *b2, *db2, *tmp2, *gam, *bet, *dgam, *dbet, *mu2, *sd2, *de;
  float *XQ, *XK, *XV, *dO, *Z2, *G2, *Z2b, *dZ2b, *dG2, *dXQ, *dXK, *XdW2, *dZ2, *dT, *T1, *T2;
  float *Z1, *X2, *H, *G1, *Z1b, *X2b, *DX2B, *DX2, *DG1;
  float *E, *A1, *P1, *A2, *P2, *dP, *dEta, *dA;
};

struct Carver {
  float* sm;
  float* gl;
  long long cap, off = 0, goff = 0;
  bool out = false;
  __host__ __device__ float* take(long long n) {
    if (!out && off + n <= cap) {
      float* r = sm ? sm + off : nullptr;
      off += n;
      return r;
    }
    out = true;
    float* r = gl ? gl + goff : nullptr;
    goff += n;
    return r;
  }
};

__host__ __device__ inline long long carve_bwd(BwdTiles& t, int C, int F, int FF, long long cap, float* sm,
                                               float* gl, long long* spill) {
  const long long CF = (long long)C * F, CFF = (long long)C * FF, CC = (long long)C * C;
  Carver c{sm, gl, cap};
  t.b1 = c.take(FF); t.db1 = c.take(FF); t.tmp1 = c.take(FF);
  t.b2 = c.take(F); t.db2 = c.take(F); t.tmp2 = c.take(F);
  t.gam = c.take(F); t.bet = c.take(F); t.dgam = c.take(F); t.dbet = c.take(F);
  t.mu2 = c.take(C); t.sd2 = c.take(C); t.de = c.take(C);
  t.XQ = c.take(CF); t.XK = c.take(CF); t.XV = c.take(CF); t.dO = c.take(CF);
  t.Z2 = c.take(CF); t.G2 = c.take(CF); t.Z2b = c.take(CF); t.dZ2b = c.take(CF);
  t.dG2 = c.take(CF); t.dXQ = c.take(CF); t.dXK = c.take(CF); t.XdW2 = c.take(CF); t.T1 = c.take(CF);
  t.dZ2 = t.Z2b;   // Z2bar (then the read-out x_bar) is dead after the gamma / beta columns
  t.T2 = t.XdW2;   // X2 dW2_next is dead after the row loop
  t.dT = t.dZ2b;   // dZ2bar is dead after the dW2 / db2 updates
  t.Z1 = c.take(CFF); t.X2 = c.take(CFF); t.H = c.take(CFF); t.G1 = c.take(CFF); t.Z1b = c.take(CFF);
  t.X2b = c.take(CFF); t.DX2B = c.take(CFF); t.DX2 = c.take(CFF); t.DG1 = c.take(CFF);
  t.A2 = c.take(CC); t.P1 = c.take(CC); t.P2 = c.take(CC);  // read by products
  t.dP = c.take(CC); t.A1 = c.take(CC); t.E = c.take(CC);   // read element-wise only
  t.dA = t.A2;     // A2 is read, element by element, just before dA is written in its place
  t.dEta = t.P2;   // P2 is dead after dG2 = -P2^T dZ2bar
  *spill = c.goff;
  return c.off;
}

template <bool TC>
__global__ void __launch_bounds__(kGenThreads) mlp_bwd_kernel(MlpBwdParams p) {
  extern __shared__ float sm[];
  const int C = p.CS, F = p.F, FF = p.FF;
  const int CF = C * F, CFF = C * FF, CC = C * C;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;

  const long long per_stream = (long long)F * FF * 2 + (long long)p.ckpt * (CFF + CF) + p.spill;
  BwdTiles tl;
  long long spill = 0;
  carve_bwd(tl, C, F, FF, kMlpBwdSmemFloats, sm, p.scratch + s * per_stream + (per_stream - p.spill), &spill);
  float *b1 = tl.b1, *db1 = tl.db1, *tmp1 = tl.tmp1, *b2 = tl.b2, *db2 = tl.db2, *tmp2 = tl.tmp2;
  float *gam = tl.gam, *bet = tl.bet, *dgam = tl.dgam, *dbet = tl.dbet;
  float *XQ = tl.XQ, *XK = tl.XK, *XV = tl.XV, *dO = tl.dO, *Z2 = tl.Z2, *G2 = tl.G2, *Z2b = tl.Z2b;
  float *dZ2b = tl.dZ2b, *dG2 = tl.dG2, *dXQ = tl.dXQ, *dXK = tl.dXK, *XdW2 = tl.XdW2, *dZ2 = tl.dZ2;
  float *dT = tl.dT, *T1 = tl.T1, *T2 = tl.T2;  // T1: e*XK, then d x_hat; T2: d g_hat
  float *Z1 = tl.Z1, *X2 = tl.X2;
  float* H = tl.H;      // G2 W2^T, later dZ1
  float* G1 = tl.G1;
  float* Z1b = tl.Z1b;  // Z1_bar, later XK dW1_next
  float* X2b = tl.X2b;
  float* DX2B = tl.DX2B;  // dX2_bar, then dZ1_bar
  float* DX2 = tl.DX2;    // e*X2, then dX2
  float* DG1 = tl.DG1;    // dG1, then dH
  float *E = tl.E, *A1 = tl.A1, *P1 = tl.P1, *A2 = tl.A2, *P2 = tl.P2, *dP = tl.dP, *dEta = tl.dEta, *dA = tl.dA;
  float *mu2 = tl.mu2, *sd2 = tl.sd2, *de = tl.de;

  float* W1 = p.scratch + s * per_stream;
  float* W2 = W1 + (long long)F * FF;
  float* zs = W2 + (long long)FF * F;
  float* dW1 = p.dW1 + s * F * FF;  // accumulated in place
  float* dW2 = p.dW2 + s * FF * F;

  for (long long i = threadIdx.x; i < (long long)F * FF; i += blockDim.x) {
    dW1[i] = 0.f;
    dW2[i] = 0.f;
  }
  for (int i = threadIdx.x; i < FF; i += blockDim.x) db1[i] = 0.f;
  for (int i = threadIdx.x; i < F; i += blockDim.x) {
    db2[i] = 0.f;
    dgam[i] = 0.f;
    dbet[i] = 0.f;
  }
  load_tile(gam, p.ln_w, (long long)h * F, F, p.dt_ln);
  load_tile(bet, p.ln_b, (long long)h * F, F, p.dt_ln);

  for (int k = p.K - 1; k >= 0; --k) {
    const int n0 = k * p.ckpt;
    const int n1 = min(n0 + p.ckpt, p.NC);
    copy_state(W1, p.W1_ckpt + (s * p.K + k) * F * FF, (long long)F * FF);
    copy_state(W2, p.W2_ckpt + (s * p.K + k) * FF * F, (long long)FF * F);
    copy_f32(b1, p.b1_ckpt + (s * p.K + k) * FF, FF);
    copy_f32(b2, p.b2_ckpt + (s * p.K + k) * F, F);
    __syncthreads();
    // ---- group re-forward: keep Z1, Z2 per mini-batch, advance the state
    for (int n = n0; n < n1; ++n) {
      const long long xb = (s * p.NC + n) * CF;
      const long long eb = (s * p.NC + n) * CC;
      float* z1s = zs + (long long)(n - n0) * (CFF + CF);
      float* z2s = z1s + CFF;
      load_tile(XK, p.XK, xb, CF, p.dt_xk);
      load_tile(XV, p.XV, xb, CF, p.dt_xv);
      load_tile(E + (C - 1) * C, p.eta, eb + (C - 1) * C, C, p.dt_eta);
      __syncthreads();
      const float* e = E + (C - 1) * C;
      block_mm_call<TC, false, false>(Z1, FF, XK, F, W1, FF, C, FF, F, 1.f, 0.f);
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
        const float z = Z1[i] + b1[i % FF];
        Z1[i] = z;
        z1s[i] = z;
        X2[i] = gelu_tanh(z);
        DX2[i] = e[i / FF] * X2[i];
      }
      for (int i = threadIdx.x; i < CF; i += blockDim.x) T1[i] = e[i / F] * XK[i];
      __syncthreads();
      block_mm_call<TC, false, false>(Z2, F, X2, FF, W2, F, C, F, FF, 1.f, 0.f);
      __syncthreads();
      ln_fused_rows(Z2, G2, b2, XV, XK, gam, bet, C, F, nullptr, nullptr);
      __syncthreads();
      for (int i = threadIdx.x; i < CF; i += blockDim.x) z2s[i] = Z2[i];
      block_mm_call<TC, false, true>(H, FF, G2, F, W2, F, C, FF, F, 1.f, 0.f);
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) G1[i] = H[i] * gelu_bwd_ref(Z1[i]);
      __syncthreads();
      block_mm_call<TC, true, false>(W1, FF, T1, F, G1, FF, F, FF, C, -1.f, 1.f);
      block_mm_call<TC, true, false>(W2, F, DX2, FF, G2, F, FF, F, C, -1.f, 1.f);
      weighted_colsum(tmp1, e, G1, C, FF);
      weighted_colsum(tmp2, e, G2, C, F);
      __syncthreads();
      for (int j = threadIdx.x; j < FF; j += blockDim.x) b1[j] -= tmp1[j];
      for (int j = threadIdx.x; j < F; j += blockDim.x) b2[j] -= tmp2[j];
      __syncthreads();
    }
    // ---- reverse walk
    for (int n = n1 - 1; n >= n0; --n) {
      const long long xb = (s * p.NC + n) * CF;
      const long long eb = (s * p.NC + n) * CC;
      const float* z1s = zs + (long long)(n - n0) * (CFF + CF);
      const float* z2s = z1s + CFF;
      load_tile(XQ, p.XQ, xb, CF, p.dt_xq);
      load_tile(XK, p.XK, xb, CF, p.dt_xk);
      load_tile(XV, p.XV, xb, CF, p.dt_xv);
      load_tile(dO, p.dout, xb, CF, p.dt_dout);
      load_tile(E, p.eta, eb, CC, p.dt_eta);
      copy_f32(Z1, z1s, CFF);
      copy_f32(Z2, z2s, CF);
      __syncthreads();
      const float* e = E + (C - 1) * C;
      // rebuild X2, G2; reverse W2 / b2
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
        const float x2 = gelu_tanh(Z1[i]);
        X2[i] = x2;
        DX2[i] = e[i / FF] * x2;
      }
      ln_fused_rows(Z2, G2, nullptr, XV, XK, gam, bet, C, F, mu2, sd2);
      for (int i = threadIdx.x; i < CF; i += blockDim.x) T1[i] = e[i / F] * XK[i];
      block_mm_call<TC, false, true>(A1, C, XQ, F, XK, F, C, C, F, 1.f, 0.f);
      __syncthreads();
      block_mm_call<TC, true, false>(W2, F, DX2, FF, G2, F, FF, F, C, 1.f, 1.f);  // W2 += (e*X2)^T G2
      weighted_colsum(tmp2, e, G2, C, F);
      for (int i = threadIdx.x; i < CC; i += blockDim.x) P1[i] = E[i] * (A1[i] + 1.f);
      __syncthreads();
      for (int j = threadIdx.x; j < F; j += blockDim.x) b2[j] += tmp2[j];
      block_mm_call<TC, false, true>(H, FF, G2, F, W2, F, C, FF, F, 1.f, 0.f);  // H = G2 W2^T
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) G1[i] = H[i] * gelu_bwd_ref(Z1[i]);
      __syncthreads();
      block_mm_call<TC, true, false>(W1, FF, T1, F, G1, FF, F, FF, C, 1.f, 1.f);  // W1 += (e*XK)^T G1
      weighted_colsum(tmp1, e, G1, C, FF);
      __syncthreads();
      for (int j = threadIdx.x; j < FF; j += blockDim.x) b1[j] += tmp1[j];
      // readout recompute
      block_mm_call<TC, false, false>(Z1b, FF, XQ, F, W1, FF, C, FF, F, 1.f, 0.f);
      block_mm_call<TC, false, false>(Z1b, FF, P1, C, G1, FF, C, FF, C, -1.f, 1.f);
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
        const float z = Z1b[i] + b1[i % FF];
        Z1b[i] = z;
        X2b[i] = gelu_tanh(z);
      }
      __syncthreads();
      block_mm_call<TC, false, true>(A2, C, X2b, FF, X2, FF, C, C, FF, 1.f, 0.f);
      block_mm_call<TC, false, false>(Z2b, F, X2b, FF, W2, F, C, F, FF, 1.f, 0.f);
      __syncthreads();
      for (int i = threadIdx.x; i < CC; i += blockDim.x) P2[i] = E[i] * (A2[i] + 1.f);
      __syncthreads();
      block_mm_call<TC, false, false>(Z2b, F, P2, C, G2, F, C, F, C, -1.f, 1.f);
      __syncthreads();
      readout_ln_bwd_rows(Z2b, b2, dO, gam, C, F, dZ2b);  // Z2b -> x_bar
      __syncthreads();
      readout_ln_bwd_cols(dO, Z2b, C, F, dgam, dbet);
      // first-level products of the readout backward (dW*_next = incoming carries)
      block_mm_call<TC, false, true>(DX2B, FF, dZ2b, F, W2, F, C, FF, F, 1.f, 0.f);  // dX2b = dZ2b W2^T
      block_mm_call<TC, false, true>(dP, C, dZ2b, F, G2, F, C, C, F, -1.f, 0.f);     // dP2 = -dZ2b G2^T
      block_mm_call<TC, true, false>(dG2, F, P2, C, dZ2b, F, C, F, C, -1.f, 0.f);    // dG2 = -P2^T dZ2b
      block_mm_call<TC, false, false>(XdW2, F, X2, FF, dW2, F, C, F, FF, 1.f, 0.f);  // X2 dW2_next
      block_mm_call<TC, false, true>(DX2, FF, G2, F, dW2, F, C, FF, F, 1.f, 0.f);    // G2 dW2_next^T
      __syncthreads();
      for (int i = threadIdx.x; i < CC; i += blockDim.x) {
        const float a2 = A2[i];  // dA takes A2's buffer: read it first
        dEta[i] = dP[i] * (a2 + 1.f);
        dA[i] = dP[i] * E[i];
      }
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) DX2[i] *= -e[i / FF];
      __syncthreads();
      block_mm_call<TC, false, false>(DX2B, FF, dA, C, X2, FF, C, FF, C, 1.f, 1.f);  // dX2b += dA2 X2
      block_mm_call<TC, true, false>(DX2, FF, dA, C, X2b, FF, C, FF, C, 1.f, 1.f);   // dX2 += dA2^T X2b
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) DX2B[i] *= gelu_tanh_grad(Z1b[i]);  // dZ1b
      __syncthreads();
      block_mm_call<TC, false, true>(dXQ, F, DX2B, FF, W1, FF, C, F, FF, 1.f, 0.f);   // dXQ = dZ1b W1^T
      block_mm_call<TC, false, true>(dP, C, DX2B, FF, G1, FF, C, C, FF, -1.f, 0.f);   // dP1 = -dZ1b G1^T
      block_mm_call<TC, true, false>(DG1, FF, P1, C, DX2B, FF, C, FF, C, -1.f, 0.f);  // dG1 = -P1^T dZ1b
      block_mm_call<TC, false, false>(Z1b, FF, XK, F, dW1, FF, C, FF, F, 1.f, 0.f);  // XK dW1_next
      block_mm_call<TC, false, true>(dXK, F, G1, FF, dW1, FF, C, F, FF, 1.f, 0.f);    // G1 dW1_next^T
      __syncthreads();
      for (int i = threadIdx.x; i < CC; i += blockDim.x) {
        dEta[i] += dP[i] * (A1[i] + 1.f);
        dA[i] = dP[i] * E[i];
      }
      for (int r = warp; r < C; r += nw) {
        const float er = e[r];
        float acc = 0.f;
        for (int j = lane; j < FF; j += 32) {
          const float g = G1[r * FF + j];
          const float x = Z1b[r * FF + j];
          acc += x * g + g * db1[j];
          DG1[r * FF + j] -= er * (x + db1[j]);
        }
        for (int j = lane; j < F; j += 32) {
          const float g = G2[r * F + j];
          const float x = XdW2[r * F + j];
          acc += x * g + g * db2[j];
          dG2[r * F + j] -= er * (x + db2[j]);
          dXK[r * F + j] *= -er;
          dXQ[r * F + j] += dO[r * F + j];
        }
        acc = warp_sum(acc);
        if (lane == 0) de[r] = -acc;
      }
      __syncthreads();
      for (int c = threadIdx.x; c < C; c += blockDim.x) dEta[(C - 1) * C + c] += de[c];
      block_mm_call<TC, false, false>(dXQ, F, dA, C, XK, F, C, F, C, 1.f, 1.f);         // dXQ += dA1 XK
      block_mm_call<TC, true, false>(dXK, F, dA, C, XQ, F, C, F, C, 1.f, 1.f);          // dXK += dA1^T XQ
      block_mm_call<TC, true, false>(dW2, F, X2b, FF, dZ2b, F, FF, F, C, 1.f, 1.f);     // dW2 += X2b^T dZ2b
      block_mm_call<TC, true, false>(dW1, FF, XQ, F, DX2B, FF, F, FF, C, 1.f, 1.f);     // dW1 += XQ^T dZ1b
      for (int j = threadIdx.x; j < F; j += blockDim.x) {
        float a = 0.f;
        for (int r = 0; r < C; ++r) a += dZ2b[r * F + j];
        db2[j] += a;
      }
      for (int j = threadIdx.x; j < FF; j += blockDim.x) {
        float a = 0.f;
        for (int r = 0; r < C; ++r) a += DX2B[r * FF + j];
        db1[j] += a;
      }
      __syncthreads();
      // G1 = H * gelu_bwd(Z1): dH into DG1, dZ1 into H
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) {
        const float t = DG1[i], z = Z1[i];
        DG1[i] = t * gelu_bwd_ref(z);
        H[i] = t * H[i] * gelu_bwd_ref_grad(z);
      }
      __syncthreads();
      block_mm_call<TC, false, false>(dG2, F, DG1, FF, W2, F, C, F, FF, 1.f, 1.f);  // dG2 += dH W2
      block_mm_call<TC, true, false>(dW2, F, DG1, FF, G2, F, FF, F, C, 1.f, 1.f);   // dW2 += dH^T G2
      __syncthreads();
      ln_fused_bwd_rows(Z2, mu2, sd2, G2, dG2, XV, XK, gam, bet, C, F, T1, T2, dT, dZ2);
      __syncthreads();
      ln_fused_bwd_cols(Z2, mu2, sd2, T2, XV, XK, gam, bet, C, F, dgam, dbet);
      for (int i = threadIdx.x; i < CF; i += blockDim.x) dXK[i] -= dT[i];
      block_mm_call<TC, false, true>(DX2, FF, dZ2, F, W2, F, C, FF, F, 1.f, 1.f);  // dX2 += dZ2 W2^T
      block_mm_call<TC, true, false>(dW2, F, X2, FF, dZ2, F, FF, F, C, 1.f, 1.f);  // dW2 += X2^T dZ2
      for (int j = threadIdx.x; j < F; j += blockDim.x) {
        float a = 0.f;
        for (int r = 0; r < C; ++r) a += dZ2[r * F + j];
        db2[j] += a;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < CFF; i += blockDim.x) H[i] += DX2[i] * gelu_tanh_grad(Z1[i]);  // dZ1
      __syncthreads();
      block_mm_call<TC, false, true>(dXK, F, H, FF, W1, FF, C, F, FF, 1.f, 1.f);  // dXK += dZ1 W1^T
      block_mm_call<TC, true, false>(dW1, FF, XK, F, H, FF, F, FF, C, 1.f, 1.f);  // dW1 += XK^T dZ1
      for (int j = threadIdx.x; j < FF; j += blockDim.x) {
        float a = 0.f;
        for (int r = 0; r < C; ++r) a += H[r * FF + j];
        db1[j] += a;
      }
      __syncthreads();
      store_tile(p.dXQ, xb, dXQ, CF, p.dt_grad);
      store_tile(p.dXK, xb, dXK, CF, p.dt_grad);
      store_tile(p.dXV, xb, dT, CF, p.dt_grad);
      store_tile(p.deta, eb, dEta, CC, p.dt_grad);
      __syncthreads();
    }
  }
  copy_f32(p.db1 + s * FF, db1, FF);
  copy_f32(p.db2 + s * F, db2, F);
  copy_f32(p.d_ln_w + s * F, dgam, F);
  copy_f32(p.d_ln_b + s * F, dbet, F);
}

// Memo read-out: one CTA per (b, h, mini-batch); weights read through L2.
template <bool TC>
__global__ void __launch_bounds__(256) mlp_readout_kernel(ReadoutParams p) {
  extern __shared__ float sm[];
  const int C = p.CS, F = p.F, FF = p.FF;
  const int CF = C * F;
  const long long blk = blockIdx.x;
  const int nc = (int)(blk % p.NCs);
  const long long bh = blk / p.NCs;
  const int h = (int)(bh % p.NH);
  const long long b = bh / p.NH;
  float* gam = sm;
  float* bet = gam + F;
  float* XQ = bet + F;
  float* Z2 = XQ + CF;
  float* Z1 = Z2 + CF;
  const float* W1 = p.W1 + b * p.W1_sb + h * p.W1_sh;
  const float* b1 = p.b1 + b * p.b1_sb + h * p.b1_sh;
  const float* W2 = p.W2 + b * p.W2_sb + h * p.W2_sh;
  const float* b2 = p.b2 + b * p.b2_sb + h * p.b2_sh;
  const long long xb = (bh * p.NCs + nc) * CF;
  load_tile(gam, p.ln_w, (long long)h * F, F, p.dt_ln);
  load_tile(bet, p.ln_b, (long long)h * F, F, p.dt_ln);
  load_tile(XQ, p.XQ, xb, CF, p.dt_xq);
  __syncthreads();
  block_mm_sel<TC, false, false>(Z1, FF, XQ, F, W1, FF, C, FF, F, 1.f, 0.f);
  __syncthreads();
  for (int i = threadIdx.x; i < C * FF; i += blockDim.x) Z1[i] = gelu_tanh(Z1[i] + b1[i % FF]);
  __syncthreads();
  block_mm_sel<TC, false, false>(Z2, F, Z1, FF, W2, F, C, F, FF, 1.f, 0.f);
  __syncthreads();
  // b2 lives in global memory: add it, then LN + residual
  for (int i = threadIdx.x; i < CF; i += blockDim.x) Z2[i] += b2[i % F];
  __syncthreads();
  readout_ln_store_rows(Z2, nullptr, XQ, gam, bet, C, F, kReadoutEps, p.out, xb, DT_F32);
}

static size_t mlp_fwd_smem(int C, int F, int FF) {
  return sizeof(float) * (2 * (size_t)FF + 4 * (size_t)F + 7 * (size_t)C * F + 5 * (size_t)C * FF + 3 * (size_t)C * C);
}

// Shared memory of the general backward and the floats per stream of its tiles that go to
// the global scratch instead (carve_bwd).
static size_t mlp_bwd_smem(int C, int F, int FF, long long* spill) {
  BwdTiles t;
  return sizeof(float) * (size_t)carve_bwd(t, C, F, FF, kMlpBwdSmemFloats, nullptr, nullptr, spill);
}

// The general kernels multiply on the TF32 tensor cores when the activations are 16-bit
// (their operands then carry no more than TF32's precision), on fp32 FMA otherwise.
static bool tc_products(int dt_xq, int dt_xv, int dt_xk) {
  auto half = [](int dt) { return dt == DT_BF16 || dt == DT_F16; };
  return half(dt_xq) && half(dt_xv) && half(dt_xk);
}

static int check_mlp(int B, int NH, int NC, int CS, int F, int FF, int ckpt) {
  TTT_REQUIRE(B > 0 && NH > 0 && NC > 0, TTT_ERR_SHAPE, "B, NH, NC must be positive (got %d, %d, %d)", B, NH, NC);
  TTT_REQUIRE(CS >= 2 && CS <= 64 && CS % 2 == 0, TTT_ERR_SHAPE, "CS must be even and in [2, 64] (got %d)", CS);
  TTT_REQUIRE(F >= 2 && F <= 256 && F % 2 == 0, TTT_ERR_SHAPE, "F must be even and in [2, 256] (got %d)", F);
  TTT_REQUIRE(FF >= 2 && FF <= 4096 && FF % 2 == 0, TTT_ERR_SHAPE, "FF must be even and in [2, 4096] (got %d)", FF);
  TTT_REQUIRE(ckpt > 0, TTT_ERR_SHAPE, "checkpoint_group_size must be positive (got %d)", ckpt);
  return TTT_OK;
}

}  // namespace ttt

using namespace ttt;

extern "C" int ttt_mlp_fwd(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size,
                           int memo_segment_size, const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                           const float* W1_init, const float* b1_init, const float* W2_init, const float* b2_init,
                           const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                           const void* eta, int dt_eta, void* XQW, int dt_out, float* W1_last, float* b1_last,
                           float* W2_last, float* b2_last, float* W1_ckpt, float* b1_ckpt, float* W2_ckpt,
                           float* b2_ckpt, float* W1_memo, float* b1_memo, float* W2_memo, float* b2_memo,
                           float* Z1_out, float* Z2_out, float* Z1b_out, float* Z2b_out, void* stream) {
  int rc = check_mlp(B, NH, NC, CS, F, FF, checkpoint_group_size);
  if (rc) return rc;
  TTT_REQUIRE(memo_segment_size > 0, TTT_ERR_SHAPE, "memo_segment_size must be positive (got %d)", memo_segment_size);
  TTT_REQUIRE(ttt_norm_weight && ttt_norm_bias && W1_init && b1_init && W2_init && b2_init && XQ && XV && XK && eta &&
                  XQW && W1_last && b1_last && W2_last && b2_last,
              TTT_ERR_NULL, "ttt_mlp_fwd: NULL pointer argument");
  const bool any_ck = W1_ckpt || b1_ckpt || W2_ckpt || b2_ckpt;
  const bool all_ck = W1_ckpt && b1_ckpt && W2_ckpt && b2_ckpt;
  TTT_REQUIRE(!any_ck || all_ck, TTT_ERR_NULL, "ttt_mlp_fwd: checkpoint pointers must be all set or all NULL");
  const bool any_memo = W1_memo || b1_memo || W2_memo || b2_memo;
  const bool all_memo = W1_memo && b1_memo && W2_memo && b2_memo;
  TTT_REQUIRE(!any_memo || all_memo, TTT_ERR_NULL, "ttt_mlp_fwd: memo pointers must be all set or all NULL");
  TTT_REQUIRE(valid_dtype(dt_ln) && valid_dtype(dt_xq) && valid_dtype(dt_xv) && valid_dtype(dt_xk) &&
                  valid_dtype(dt_eta) && valid_dtype(dt_out),
              TTT_ERR_DTYPE, "ttt_mlp_fwd: unknown dtype code");
  MlpFwdParams p;
  p.B = B; p.NH = NH; p.NC = NC; p.CS = CS; p.F = F; p.FF = FF;
  p.ckpt = checkpoint_group_size; p.K = (NC + checkpoint_group_size - 1) / checkpoint_group_size;
  p.memo = memo_segment_size; p.NS = (NC + memo_segment_size - 1) / memo_segment_size;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.W1_init = W1_init; p.b1_init = b1_init; p.W2_init = W2_init; p.b2_init = b2_init;
  p.XQ = XQ; p.XV = XV; p.XK = XK; p.eta = eta;
  p.dt_xq = dt_xq; p.dt_xv = dt_xv; p.dt_xk = dt_xk; p.dt_eta = dt_eta;
  p.out = XQW; p.dt_out = dt_out;
  p.W1_last = W1_last; p.b1_last = b1_last; p.W2_last = W2_last; p.b2_last = b2_last;
  p.W1_ckpt = W1_ckpt; p.b1_ckpt = b1_ckpt; p.W2_ckpt = W2_ckpt; p.b2_ckpt = b2_ckpt;
  p.W1_memo = all_memo ? W1_memo : nullptr; p.b1_memo = b1_memo; p.W2_memo = W2_memo; p.b2_memo = b2_memo;
  const bool any_z = Z1_out || Z2_out || Z1b_out || Z2b_out;
  TTT_REQUIRE(!any_z || (Z1_out && Z2_out && Z1b_out && Z2b_out), TTT_ERR_NULL,
              "ttt_mlp_fwd: the four pre-activation outputs must be all set or all NULL");
  p.Z1_out = Z1_out; p.Z2_out = Z2_out; p.Z1b_out = Z1b_out; p.Z2b_out = Z2b_out;
  rc = mlp_fwd_fast(p, (cudaStream_t)stream);
  if (rc != TTT_NOT_APPLICABLE) return rc;
  const size_t smem = mlp_fwd_smem(CS, F, FF);
  auto kern = tc_products(dt_xq, dt_xv, dt_xk) ? mlp_fwd_kernel<true> : mlp_fwd_kernel<false>;
  rc = prepare_smem(kern, smem, "ttt_mlp_fwd");
  if (rc) return rc;
  kern<<<B * NH, gen_threads(F, FF), smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_mlp_fwd");
}

extern "C" size_t ttt_mlp_bwd_scratch_bytes(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size) {
  if (B <= 0 || NH <= 0 || NC <= 0 || CS <= 0 || F <= 0 || FF <= 0 || checkpoint_group_size <= 0) return 0;
  const size_t g = (size_t)(checkpoint_group_size < NC ? checkpoint_group_size : NC);
  long long spill = 0;
  mlp_bwd_smem(CS, F, FF, &spill);
  const size_t per_stream = 2 * (size_t)F * FF + g * (size_t)CS * (FF + F) + (size_t)spill;
  return sizeof(float) * (size_t)B * NH * per_stream;
}

extern "C" int ttt_mlp_bwd(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size,
                           const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln, const float* W1_ckpt,
                           const float* b1_ckpt, const float* W2_ckpt, const float* b2_ckpt, const void* XQ, int dt_xq,
                           const void* XV, int dt_xv, const void* XK, int dt_xk, const void* eta, int dt_eta,
                           const void* dXQW, int dt_dout, const float* Z1_saved, const float* Z2_saved,
                           const float* Z1b_saved, const float* Z2b_saved, const float* W1_last,
                           const float* W2_last, float* d_ln_w, float* d_ln_b, float* dW1, float* db1,
                           float* dW2, float* db2, void* dXQ, void* dXV, void* dXK, void* d_eta, int dt_grad,
                           void* scratch, size_t scratch_bytes, void* stream) {
  int rc = check_mlp(B, NH, NC, CS, F, FF, checkpoint_group_size);
  if (rc) return rc;
  TTT_REQUIRE(ttt_norm_weight && ttt_norm_bias && W1_ckpt && b1_ckpt && W2_ckpt && b2_ckpt && XQ && XV && XK && eta &&
                  dXQW && d_ln_w && d_ln_b && dW1 && db1 && dW2 && db2 && dXQ && dXV && dXK && d_eta,
              TTT_ERR_NULL, "ttt_mlp_bwd: NULL pointer argument");
  TTT_REQUIRE(valid_dtype(dt_ln) && valid_dtype(dt_xq) && valid_dtype(dt_xv) && valid_dtype(dt_xk) &&
                  valid_dtype(dt_eta) && valid_dtype(dt_dout) && valid_dtype(dt_grad),
              TTT_ERR_DTYPE, "ttt_mlp_bwd: unknown dtype code");
  const bool any_saved = Z1_saved || Z2_saved || Z1b_saved || Z2b_saved || W1_last || W2_last;
  TTT_REQUIRE(!any_saved || (Z1_saved && Z2_saved && Z1b_saved && Z2b_saved && W1_last && W2_last), TTT_ERR_NULL,
              "ttt_mlp_bwd: the saved pre-activations and final weights must be all set or all NULL");
  MlpBwdParams p;
  p.B = B; p.NH = NH; p.NC = NC; p.CS = CS; p.F = F; p.FF = FF;
  p.ckpt = checkpoint_group_size < NC ? checkpoint_group_size : NC;
  p.K = (NC + p.ckpt - 1) / p.ckpt;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.W1_ckpt = W1_ckpt; p.b1_ckpt = b1_ckpt; p.W2_ckpt = W2_ckpt; p.b2_ckpt = b2_ckpt;
  p.XQ = XQ; p.XV = XV; p.XK = XK; p.eta = eta;
  p.dt_xq = dt_xq; p.dt_xv = dt_xv; p.dt_xk = dt_xk; p.dt_eta = dt_eta;
  p.dout = dXQW; p.dt_dout = dt_dout;
  p.d_ln_w = d_ln_w; p.d_ln_b = d_ln_b; p.dW1 = dW1; p.db1 = db1; p.dW2 = dW2; p.db2 = db2;
  p.dXQ = dXQ; p.dXV = dXV; p.dXK = dXK; p.deta = d_eta; p.dt_grad = dt_grad;
  p.scratch = (float*)scratch;
  p.Z1_saved = Z1_saved; p.Z2_saved = Z2_saved; p.Z1b_saved = Z1b_saved; p.Z2b_saved = Z2b_saved;
  p.W1_last = W1_last; p.W2_last = W2_last;
  p.spill = 0;
  rc = mlp_bwd_fast(p, (cudaStream_t)stream);
  if (rc != TTT_NOT_APPLICABLE) return rc;
  const size_t need = ttt_mlp_bwd_scratch_bytes(B, NH, NC, CS, F, FF, checkpoint_group_size);
  TTT_REQUIRE(scratch && scratch_bytes >= need, TTT_ERR_SCRATCH, "ttt_mlp_bwd: scratch has %zu bytes, needs %zu",
              scratch ? scratch_bytes : (size_t)0, need);
  const size_t smem = mlp_bwd_smem(CS, F, FF, &p.spill);
  auto kern = tc_products(dt_xq, dt_xv, dt_xk) ? mlp_bwd_kernel<true> : mlp_bwd_kernel<false>;
  rc = prepare_smem(kern, smem, "ttt_mlp_bwd");
  if (rc) return rc;
  kern<<<B * NH, gen_threads(F, FF), smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_mlp_bwd");
}

extern "C" int ttt_mlp_cached_readout(int B, int NH, int NCseg, int CS, int F, int FF, const void* XQ, int dt_xq,
                                      const float* W1, long long W1_sb, long long W1_sh, const float* b1,
                                      long long b1_sb, long long b1_sh, const float* W2, long long W2_sb,
                                      long long W2_sh, const float* b2, long long b2_sb, long long b2_sh,
                                      const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln, float* out,
                                      void* stream) {
  TTT_REQUIRE(B > 0 && NH > 0 && NCseg > 0, TTT_ERR_SHAPE, "B, NH, NCseg must be positive (got %d, %d, %d)", B, NH,
              NCseg);
  TTT_REQUIRE(CS >= 2 && CS <= 64 && CS % 2 == 0, TTT_ERR_SHAPE, "CS must be even and in [2, 64] (got %d)", CS);
  TTT_REQUIRE(F >= 2 && F <= 256 && F % 2 == 0, TTT_ERR_SHAPE, "F must be even and in [2, 256] (got %d)", F);
  TTT_REQUIRE(FF >= 2 && FF <= 4096 && FF % 2 == 0, TTT_ERR_SHAPE, "FF must be even and in [2, 4096] (got %d)", FF);
  TTT_REQUIRE(XQ && W1 && b1 && W2 && b2 && ttt_norm_weight && ttt_norm_bias && out, TTT_ERR_NULL,
              "ttt_mlp_cached_readout: NULL pointer argument");
  TTT_REQUIRE(valid_dtype(dt_xq) && valid_dtype(dt_ln), TTT_ERR_DTYPE, "ttt_mlp_cached_readout: unknown dtype code");
  ReadoutParams p;
  p.B = B; p.NH = NH; p.NCs = NCseg; p.CS = CS; p.F = F; p.FF = FF;
  p.XQ = XQ; p.dt_xq = dt_xq;
  p.W1 = W1; p.W1_sb = W1_sb; p.W1_sh = W1_sh;
  p.b1 = b1; p.b1_sb = b1_sb; p.b1_sh = b1_sh;
  p.W2 = W2; p.W2_sb = W2_sb; p.W2_sh = W2_sh;
  p.b2 = b2; p.b2_sb = b2_sb; p.b2_sh = b2_sh;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.out = out;
  const size_t smem = sizeof(float) * (2 * (size_t)F + 2 * (size_t)CS * F + (size_t)CS * FF);
  auto kern = tc_products(dt_xq, dt_xq, dt_xq) ? mlp_readout_kernel<true> : mlp_readout_kernel<false>;
  const int rc = prepare_smem(kern, smem, "ttt_mlp_cached_readout");
  if (rc) return rc;
  kern<<<(unsigned)((long long)B * NH * NCseg), 256, smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_mlp_cached_readout");
}
