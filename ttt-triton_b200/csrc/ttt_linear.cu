// TTT-Linear dual-form scan: forward and backward, one CTA per (batch, head) stream.
//
// Reference semantics: ops/ttt_linear.py:8-54 (dual form, full eta, LN eps 1e-8); the
// launch boundary is linear_triton.py:96-127 (forward) and :201-246 (backward).
// The backward is the hand derivation of autograd through that step (it emits the full
// CS x CS d_eta), with checkpoint-group recompute: each group is re-run forward from its
// checkpoint keeping only the pre-activation Z per mini-batch, then walked backwards,
// recovering the state entering mini-batch n from the state after it by undoing the
// rank-CS update (W_n = W_{n+1} + XK^T diag(e) G_n).
//
// This is the general path (any CS, F with the shared-memory budget): fp32 FMA math on
// shared-memory tiles. The inner state W (F x F fp32) stays in shared memory for the
// whole sequence.
#include <mutex>

#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "params.cuh"

namespace ttt {

template <bool TC>
__global__ void __launch_bounds__(512) linear_fwd_kernel(LinFwdParams p) {
  extern __shared__ float sm[];
  const int C = p.CS, F = p.F;
  const int CF = C * F, CC = C * C;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);

  float* W = sm;
  float* bvec = W + F * F;
  float* gam = bvec + F;
  float* bet = gam + F;
  float* tmpF = bet + F;
  float* XQ = tmpF + F;
  float* XK = XQ + CF;
  float* XV = XK + CF;
  float* Z = XV + CF;
  float* G = Z + CF;
  float* Zb = G + CF;
  float* XKe = Zb + CF;
  float* E = XKe + CF;
  float* P = E + CC;

  copy_f32(W, p.W_init + s * F * F, F * F);
  copy_f32(bvec, p.b_init + s * F, F);
  load_tile(gam, p.ln_w, (long long)h * F, F, p.dt_ln);
  load_tile(bet, p.ln_b, (long long)h * F, F, p.dt_ln);
  __syncthreads();

  for (int n = 0; n < p.NC; ++n) {
    if (p.W_ckpt && n % p.ckpt == 0) {
      const long long k = s * p.K + n / p.ckpt;
      for (int i = threadIdx.x; i < F * F; i += blockDim.x) p.W_ckpt[k * F * F + i] = W[i];
      for (int i = threadIdx.x; i < F; i += blockDim.x) p.b_ckpt[k * F + i] = bvec[i];
    }
    const long long xb = (s * p.NC + n) * CF;
    const long long eb = (s * p.NC + n) * CC;
    load_tile(XQ, p.XQ, xb, CF, p.dt_xq);
    load_tile(XK, p.XK, xb, CF, p.dt_xk);
    load_tile(XV, p.XV, xb, CF, p.dt_xv);
    load_tile(E, p.eta, eb, CC, p.dt_eta);
    __syncthreads();

    block_mm_sel<TC, false, false>(Z, F, XK, F, W, F, C, F, F, 1.f, 0.f);   // Z  = XK W
    block_mm_sel<TC, false, true>(P, C, XQ, F, XK, F, C, C, F, 1.f, 0.f);   // P  = XQ XK^T
    block_mm_sel<TC, false, false>(Zb, F, XQ, F, W, F, C, F, F, 1.f, 0.f);  // Zb = XQ W
    __syncthreads();

    ln_fused_rows(Z, G, bvec, XV, XK, gam, bet, C, F, nullptr, nullptr);
    for (int i = threadIdx.x; i < CC; i += blockDim.x) P[i] = E[i] * (P[i] + 1.f);
    if (p.Z_out) {
      __syncthreads();
      for (int i = threadIdx.x; i < CF; i += blockDim.x) p.Z_out[xb + i] = Z[i];
    }
    for (int i = threadIdx.x; i < CF; i += blockDim.x) XKe[i] = E[(C - 1) * C + i / F] * XK[i];
    __syncthreads();

    block_mm_sel<TC, false, false>(Zb, F, P, C, G, F, C, F, C, -1.f, 1.f);  // Zb -= (eta*(A+1)) G
    weighted_colsum(tmpF, E + (C - 1) * C, G, C, F);
    __syncthreads();

    // readout: XQW = XQ + LN(Zb + b) with the old b; state update in parallel
    readout_ln_store_rows(Zb, bvec, XQ, gam, bet, C, F, kLnEps, p.out, xb, p.dt_out);
    block_mm_sel<TC, true, false>(W, F, XKe, F, G, F, F, F, C, -1.f, 1.f);  // W -= (e*XK)^T G
    __syncthreads();
    for (int j = threadIdx.x; j < F; j += blockDim.x) bvec[j] -= tmpF[j];
    __syncthreads();
  }
  for (int i = threadIdx.x; i < F * F; i += blockDim.x) p.W_last[s * F * F + i] = W[i];
  for (int i = threadIdx.x; i < F; i += blockDim.x) p.b_last[s * F + i] = bvec[i];
}

template <bool TC>
__global__ void __launch_bounds__(512) linear_bwd_kernel(LinBwdParams p) {
  extern __shared__ float sm[];
  const int C = p.CS, F = p.F;
  const int CF = C * F, CC = C * C;
  const long long s = blockIdx.x;
  const int h = (int)(s % p.NH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;

  float* W = sm;
  float* dW = W + F * F;
  float* bvec = dW + F * F;
  float* db = bvec + F;
  float* gam = db + F;
  float* bet = gam + F;
  float* dgam = bet + F;
  float* dbet = dgam + F;
  float* tmpF = dbet + F;
  float* XQ = tmpF + F;
  float* XK = XQ + CF;
  float* XV = XK + CF;
  float* dO = XV + CF;
  float* Z = dO + CF;     // pre-activation of the fused-LN gradient (bias included)
  float* G = Z + CF;
  float* Zb = G + CF;     // readout pre-activation, then x_bar
  float* dZb = Zb + CF;
  float* dXQ = dZb + CF;
  float* dXK = dXQ + CF;
  float* dG = dXK + CF;
  float* T1 = dG + CF;    // XK e / XK dW^T / d x_hat
  float* T2 = T1 + CF;    // G dW^T / d g_hat
  float* dZ = T2 + CF;
  float* dT = dZ + CF;
  float* E = dT + CF;
  float* A = E + CC;
  float* P = A + CC;
  float* dP = P + CC;
  float* dA = dP + CC;
  float* rowv = dA + CC;  // 4*C: mu, std, mu_bar, std_bar
  float* mu1 = rowv;
  float* sd1 = rowv + C;
  float* de = rowv + 2 * C;

  for (int i = threadIdx.x; i < F * F; i += blockDim.x) dW[i] = 0.f;
  for (int i = threadIdx.x; i < F; i += blockDim.x) {
    db[i] = 0.f;
    dgam[i] = 0.f;
    dbet[i] = 0.f;
  }
  load_tile(gam, p.ln_w, (long long)h * F, F, p.dt_ln);
  load_tile(bet, p.ln_b, (long long)h * F, F, p.dt_ln);
  float* zs = p.scratch + s * (long long)p.ckpt * CF;

  for (int k = p.K - 1; k >= 0; --k) {
    const int n0 = k * p.ckpt;
    const int n1 = min(n0 + p.ckpt, p.NC);
    copy_f32(W, p.W_ckpt + (s * p.K + k) * F * F, F * F);
    copy_f32(bvec, p.b_ckpt + (s * p.K + k) * F, F);
    __syncthreads();
    // ---- group re-forward: keep Z per mini-batch, advance the state
    for (int n = n0; n < n1; ++n) {
      const long long xb = (s * p.NC + n) * CF;
      const long long eb = (s * p.NC + n) * CC;
      load_tile(XK, p.XK, xb, CF, p.dt_xk);
      load_tile(XV, p.XV, xb, CF, p.dt_xv);
      load_tile(E + (C - 1) * C, p.eta, eb + (C - 1) * C, C, p.dt_eta);
      __syncthreads();
      block_mm_sel<TC, false, false>(Z, F, XK, F, W, F, C, F, F, 1.f, 0.f);
      for (int i = threadIdx.x; i < CF; i += blockDim.x) T1[i] = E[(C - 1) * C + i / F] * XK[i];
      __syncthreads();
      ln_fused_rows(Z, G, bvec, XV, XK, gam, bet, C, F, nullptr, nullptr);
      __syncthreads();
      for (int i = threadIdx.x; i < CF; i += blockDim.x) zs[(long long)(n - n0) * CF + i] = Z[i];
      block_mm_sel<TC, true, false>(W, F, T1, F, G, F, F, F, C, -1.f, 1.f);
      weighted_colsum(tmpF, E + (C - 1) * C, G, C, F);
      __syncthreads();
      for (int j = threadIdx.x; j < F; j += blockDim.x) bvec[j] -= tmpF[j];
      __syncthreads();
    }
    // ---- reverse walk
    for (int n = n1 - 1; n >= n0; --n) {
      const long long xb = (s * p.NC + n) * CF;
      const long long eb = (s * p.NC + n) * CC;
      load_tile(XQ, p.XQ, xb, CF, p.dt_xq);
      load_tile(XK, p.XK, xb, CF, p.dt_xk);
      load_tile(XV, p.XV, xb, CF, p.dt_xv);
      load_tile(dO, p.dout, xb, CF, p.dt_dout);
      load_tile(E, p.eta, eb, CC, p.dt_eta);
      for (int i = threadIdx.x; i < CF; i += blockDim.x) Z[i] = zs[(long long)(n - n0) * CF + i];
      __syncthreads();
      // G from the stored Z (its bias is already included)
      block_mm_sel<TC, false, true>(A, C, XQ, F, XK, F, C, C, F, 1.f, 0.f);  // A = XQ XK^T
      for (int i = threadIdx.x; i < CF; i += blockDim.x) T1[i] = E[(C - 1) * C + i / F] * XK[i];
      __syncthreads();
      ln_fused_rows(Z, G, nullptr, XV, XK, gam, bet, C, F, mu1, sd1);
      for (int i = threadIdx.x; i < CC; i += blockDim.x) P[i] = E[i] * (A[i] + 1.f);
      __syncthreads();
      // state reversal: W_n = W_{n+1} + (e*XK)^T G ; b_n = b_{n+1} + e G
      block_mm_sel<TC, true, false>(W, F, T1, F, G, F, F, F, C, 1.f, 1.f);
      weighted_colsum(tmpF, E + (C - 1) * C, G, C, F);
      __syncthreads();
      for (int j = threadIdx.x; j < F; j += blockDim.x) bvec[j] += tmpF[j];
      __syncthreads();
      // readout recompute Zb = XQ W + b - P G
      block_mm_sel<TC, false, false>(Zb, F, XQ, F, W, F, C, F, F, 1.f, 0.f);
      block_mm_sel<TC, false, false>(Zb, F, P, C, G, F, C, F, C, -1.f, 1.f);
      __syncthreads();
      // readout LayerNorm backward: Zb -> x_bar (in place), dZb
      readout_ln_bwd_rows(Zb, bvec, dO, gam, C, F, dZb);
      __syncthreads();
      readout_ln_bwd_cols(dO, Zb, C, F, dgam, dbet);
      block_mm_sel<TC, false, true>(dXQ, F, dZb, F, W, F, C, F, F, 1.f, 0.f);  // dXQ = dZb W^T
      block_mm_sel<TC, false, true>(dP, C, dZb, F, G, F, C, C, F, -1.f, 0.f);  // dP = -dZb G^T
      block_mm_sel<TC, true, false>(dG, F, P, C, dZb, F, C, F, C, -1.f, 0.f);  // dG = -P^T dZb
      block_mm_sel<TC, false, false>(T1, F, XK, F, dW, F, C, F, F, 1.f, 0.f);  // XK dW_next
      block_mm_sel<TC, false, true>(T2, F, G, F, dW, F, C, F, F, 1.f, 0.f);    // G dW_next^T
      __syncthreads();
      for (int i = threadIdx.x; i < CC; i += blockDim.x) {
        dA[i] = dP[i] * E[i];
        dP[i] = dP[i] * (A[i] + 1.f);  // d_eta (dual-form part)
      }
      for (int r = warp; r < C; r += nw) {
        const float e = E[(C - 1) * C + r];
        float acc = 0.f;
        for (int j = lane; j < F; j += 32) {
          const float g = G[r * F + j];
          acc += T1[r * F + j] * g + g * db[j];
          dG[r * F + j] -= e * (T1[r * F + j] + db[j]);
          dXK[r * F + j] = -e * T2[r * F + j];
          dXQ[r * F + j] += dO[r * F + j];
        }
        acc = warp_sum(acc);
        if (lane == 0) de[r] = -acc;
      }
      __syncthreads();
      for (int c = threadIdx.x; c < C; c += blockDim.x) dP[(C - 1) * C + c] += de[c];
      block_mm_sel<TC, false, false>(dXQ, F, dA, C, XK, F, C, F, C, 1.f, 1.f);  // dXQ += dA XK
      block_mm_sel<TC, true, false>(dXK, F, dA, C, XQ, F, C, F, C, 1.f, 1.f);   // dXK += dA^T XQ
      __syncthreads();
      // backward of G = ln_fused_l2_bwd(Z, XV - XK)
      ln_fused_bwd_rows(Z, mu1, sd1, G, dG, XV, XK, gam, bet, C, F, T1, T2, dT, dZ);
      __syncthreads();
      ln_fused_bwd_cols(Z, mu1, sd1, T2, XV, XK, gam, bet, C, F, dgam, dbet);
      for (int i = threadIdx.x; i < CF; i += blockDim.x) dXK[i] -= dT[i];
      __syncthreads();
      block_mm_sel<TC, false, true>(dXK, F, dZ, F, W, F, C, F, F, 1.f, 1.f);   // dXK += dZ W^T
      block_mm_sel<TC, true, false>(dW, F, XQ, F, dZb, F, F, F, C, 1.f, 1.f);  // dW += XQ^T dZb
      block_mm_sel<TC, true, false>(dW, F, XK, F, dZ, F, F, F, C, 1.f, 1.f);   // dW += XK^T dZ
      for (int j = threadIdx.x; j < F; j += blockDim.x) {
        float acc = 0.f;
        for (int r = 0; r < C; ++r) acc += dZb[r * F + j] + dZ[r * F + j];
        db[j] += acc;
      }
      __syncthreads();
      store_tile(p.dXQ, xb, dXQ, CF, p.dt_grad);
      store_tile(p.dXK, xb, dXK, CF, p.dt_grad);
      store_tile(p.dXV, xb, dT, CF, p.dt_grad);
      store_tile(p.deta, eb, dP, CC, p.dt_grad);
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < F * F; i += blockDim.x) p.dW[s * F * F + i] = dW[i];
  for (int i = threadIdx.x; i < F; i += blockDim.x) {
    p.db[s * F + i] = db[i];
    p.d_ln_w[s * F + i] = dgam[i];
    p.d_ln_b[s * F + i] = dbet[i];
  }
}

// The general kernels multiply on the TF32 tensor cores (block_mm_tf32) when the activations
// are 16-bit (their operands then carry no more than TF32's precision), on fp32 FMA otherwise.
static bool lin_tc_products(int dt_xq, int dt_xv, int dt_xk) {
  auto half = [](int dt) { return dt == DT_BF16 || dt == DT_F16; };
  return half(dt_xq) && half(dt_xv) && half(dt_xk);
}

// Threads of a CTA (one stream): sixteen warps for F <= 64, for latency hiding in the chains
// of small barrier-separated products; eight above.
static int lin_threads(int F) { return F <= 64 ? 512 : 256; }

static size_t linear_fwd_smem(int C, int F) {
  return sizeof(float) * ((size_t)F * F + 4 * F + 7 * (size_t)C * F + 2 * (size_t)C * C);
}

static size_t linear_bwd_smem(int C, int F) {
  return sizeof(float) * (2 * (size_t)F * F + 7 * (size_t)F + 15 * (size_t)C * F + 5 * (size_t)C * C + 4 * (size_t)C);
}

static int check_common(int B, int NH, int NC, int CS, int F, int ckpt) {
  TTT_REQUIRE(B > 0 && NH > 0 && NC > 0, TTT_ERR_SHAPE, "B, NH, NC must be positive (got %d, %d, %d)", B, NH, NC);
  TTT_REQUIRE(CS >= 2 && CS <= 64 && CS % 2 == 0, TTT_ERR_SHAPE, "CS must be even and in [2, 64] (got %d)", CS);
  TTT_REQUIRE(F >= 2 && F <= 256 && F % 2 == 0, TTT_ERR_SHAPE, "F must be even and in [2, 256] (got %d)", F);
  TTT_REQUIRE(ckpt > 0, TTT_ERR_SHAPE, "checkpoint_group_size must be positive (got %d)", ckpt);
  return TTT_OK;
}

}  // namespace ttt

using namespace ttt;

extern "C" int ttt_linear_fwd(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                              const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                              const float* W1_init, const float* b1_init, const void* XQ, int dt_xq, const void* XV,
                              int dt_xv, const void* XK, int dt_xk, const void* eta, int dt_eta, void* XQW, int dt_out,
                              float* W1_last, float* b1_last, float* W1_ckpt, float* b1_ckpt, float* Z_out,
                              void* stream) {
  int rc = check_common(B, NH, NC, CS, F, checkpoint_group_size);
  if (rc) return rc;
  TTT_REQUIRE(ttt_norm_weight && ttt_norm_bias && W1_init && b1_init && XQ && XV && XK && eta && XQW && W1_last &&
                  b1_last,
              TTT_ERR_NULL, "ttt_linear_fwd: NULL pointer argument");
  TTT_REQUIRE((W1_ckpt == nullptr) == (b1_ckpt == nullptr), TTT_ERR_NULL,
              "ttt_linear_fwd: checkpoint pointers must be both set or both NULL");
  TTT_REQUIRE(valid_dtype(dt_ln) && valid_dtype(dt_xq) && valid_dtype(dt_xv) && valid_dtype(dt_xk) &&
                  valid_dtype(dt_eta) && valid_dtype(dt_out),
              TTT_ERR_DTYPE, "ttt_linear_fwd: unknown dtype code");
  LinFwdParams p;
  p.B = B; p.NH = NH; p.NC = NC; p.CS = CS; p.F = F; p.ckpt = checkpoint_group_size;
  p.K = (NC + checkpoint_group_size - 1) / checkpoint_group_size;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.W_init = W1_init; p.b_init = b1_init;
  p.XQ = XQ; p.XV = XV; p.XK = XK; p.eta = eta;
  p.dt_xq = dt_xq; p.dt_xv = dt_xv; p.dt_xk = dt_xk; p.dt_eta = dt_eta;
  p.out = XQW; p.dt_out = dt_out;
  p.W_last = W1_last; p.b_last = b1_last; p.W_ckpt = W1_ckpt; p.b_ckpt = b1_ckpt; p.Z_out = Z_out;
  rc = linear_fwd_fast(p, (cudaStream_t)stream);
  if (rc != TTT_NOT_APPLICABLE) return rc;
  const size_t smem = linear_fwd_smem(CS, F);
  auto kern = lin_tc_products(dt_xq, dt_xv, dt_xk) ? linear_fwd_kernel<true> : linear_fwd_kernel<false>;
  rc = prepare_smem(kern, smem, "ttt_linear_fwd");
  if (rc) return rc;
  kern<<<B * NH, lin_threads(F), smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_linear_fwd");
}

extern "C" size_t ttt_linear_bwd_scratch_bytes(int B, int NH, int NC, int CS, int F, int checkpoint_group_size) {
  if (B <= 0 || NH <= 0 || NC <= 0 || CS <= 0 || F <= 0 || checkpoint_group_size <= 0) return 0;
  const size_t g = (size_t)(checkpoint_group_size < NC ? checkpoint_group_size : NC);
  return sizeof(float) * (size_t)B * NH * g * CS * F;
}

extern "C" int ttt_linear_bwd(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                              const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                              const float* W1_ckpt, const float* b1_ckpt, const void* XQ, int dt_xq, const void* XV,
                              int dt_xv, const void* XK, int dt_xk, const void* eta, int dt_eta, const void* dXQW,
                              int dt_dout, const float* Z_saved, const float* W1_last, const float* b1_last,
                              float* d_ln_w, float* d_ln_b, float* dW1, float* db1, void* dXQ, void* dXV, void* dXK,
                              void* d_eta, int dt_grad, void* scratch, size_t scratch_bytes, void* stream) {
  int rc = check_common(B, NH, NC, CS, F, checkpoint_group_size);
  if (rc) return rc;
  TTT_REQUIRE(ttt_norm_weight && ttt_norm_bias && W1_ckpt && b1_ckpt && XQ && XV && XK && eta && dXQW && d_ln_w &&
                  d_ln_b && dW1 && db1 && dXQ && dXV && dXK && d_eta,
              TTT_ERR_NULL, "ttt_linear_bwd: NULL pointer argument");
  TTT_REQUIRE(valid_dtype(dt_ln) && valid_dtype(dt_xq) && valid_dtype(dt_xv) && valid_dtype(dt_xk) &&
                  valid_dtype(dt_eta) && valid_dtype(dt_dout) && valid_dtype(dt_grad),
              TTT_ERR_DTYPE, "ttt_linear_bwd: unknown dtype code");
  LinBwdParams p;
  p.B = B; p.NH = NH; p.NC = NC; p.CS = CS; p.F = F;
  p.ckpt = checkpoint_group_size < NC ? checkpoint_group_size : NC;
  p.K = (NC + p.ckpt - 1) / p.ckpt;
  TTT_REQUIRE(p.K == (NC + checkpoint_group_size - 1) / checkpoint_group_size, TTT_ERR_SHAPE, "internal");
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.W_ckpt = W1_ckpt; p.b_ckpt = b1_ckpt;
  p.XQ = XQ; p.XV = XV; p.XK = XK; p.eta = eta;
  p.dt_xq = dt_xq; p.dt_xv = dt_xv; p.dt_xk = dt_xk; p.dt_eta = dt_eta;
  p.dout = dXQW; p.dt_dout = dt_dout;
  p.d_ln_w = d_ln_w; p.d_ln_b = d_ln_b; p.dW = dW1; p.db = db1;
  p.dXQ = dXQ; p.dXV = dXV; p.dXK = dXK; p.deta = d_eta; p.dt_grad = dt_grad;
  p.scratch = (float*)scratch;
  p.Z_saved = Z_saved; p.W_last = W1_last; p.b_last = b1_last;
  rc = linear_bwd_fast(p, (cudaStream_t)stream);
  if (rc != TTT_NOT_APPLICABLE) return rc;
  const size_t need = ttt_linear_bwd_scratch_bytes(B, NH, NC, CS, F, checkpoint_group_size);
  TTT_REQUIRE(scratch && scratch_bytes >= need, TTT_ERR_SCRATCH, "ttt_linear_bwd: scratch has %zu bytes, needs %zu",
              scratch ? scratch_bytes : (size_t)0, need);
  const size_t smem = linear_bwd_smem(CS, F);
  auto kern = lin_tc_products(dt_xq, dt_xv, dt_xk) ? linear_bwd_kernel<true> : linear_bwd_kernel<false>;
  rc = prepare_smem(kern, smem, "ttt_linear_bwd");
  if (rc) return rc;
  kern<<<B * NH, lin_threads(F), smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_linear_bwd");
}

// ---------------------------------------------------------------------------------------
// Allocation-free backward. Some callers cannot allocate device memory where they enqueue
// work: an inference-engine plugin's enqueue callback that is only handed pre-sized
// buffers, or a service that fixes its whole device-memory budget at start-up. For them,
// the checkpoint-recompute backward can take its scratch from a fixed array compiled into
// this library instead of a caller buffer. Every GPU that loads the library holds this
// array until the process exits.
namespace ttt {
constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_scratch on the current device, looked up once per device.
static int noalloc_scratch(float** out) {
  constexpr int kMaxDevices = 64;
  static float* addr[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "ttt_linear_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(TTT_ERR_UNSUPPORTED, "ttt_linear_bwd_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(TTT_ERR_CUDA, "ttt_linear_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return TTT_OK;
}
}  // namespace ttt

extern "C" int ttt_linear_bwd_noalloc(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                                      const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                                      const float* W1_ckpt, const float* b1_ckpt, const void* XQ, int dt_xq,
                                      const void* XV, int dt_xv, const void* XK, int dt_xk, const void* eta,
                                      int dt_eta, const void* dXQW, int dt_dout, float* d_ln_w, float* d_ln_b,
                                      float* dW1, float* db1, void* dXQ, void* dXV, void* dXK, void* d_eta,
                                      int dt_grad, void* stream) {
  int rc = check_common(B, NH, NC, CS, F, checkpoint_group_size);
  if (rc) return rc;
  TTT_REQUIRE(ttt_norm_weight && ttt_norm_bias && W1_ckpt && b1_ckpt && XQ && XV && XK && eta && dXQW && d_ln_w &&
                  d_ln_b && dW1 && db1 && dXQ && dXV && dXK && d_eta,
              TTT_ERR_NULL, "ttt_linear_bwd_noalloc: NULL pointer argument");
  TTT_REQUIRE(valid_dtype(dt_ln) && valid_dtype(dt_xq) && valid_dtype(dt_xv) && valid_dtype(dt_xk) &&
                  valid_dtype(dt_eta) && valid_dtype(dt_dout) && valid_dtype(dt_grad),
              TTT_ERR_DTYPE, "ttt_linear_bwd_noalloc: unknown dtype code");
  const size_t need = ttt_linear_bwd_scratch_bytes(B, NH, NC, CS, F, checkpoint_group_size);
  TTT_REQUIRE(need <= kNoAllocScratchBytes, TTT_ERR_SCRATCH,
              "ttt_linear_bwd_noalloc: these sizes need %zu bytes of scratch, the library's fixed scratch holds %zu "
              "(use ttt_linear_bwd with a caller buffer)",
              need, kNoAllocScratchBytes);
  float* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  LinBwdParams p;
  p.B = B; p.NH = NH; p.NC = NC; p.CS = CS; p.F = F;
  p.ckpt = checkpoint_group_size < NC ? checkpoint_group_size : NC;
  p.K = (NC + p.ckpt - 1) / p.ckpt;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.W_ckpt = W1_ckpt; p.b_ckpt = b1_ckpt;
  p.XQ = XQ; p.XV = XV; p.XK = XK; p.eta = eta;
  p.dt_xq = dt_xq; p.dt_xv = dt_xv; p.dt_xk = dt_xk; p.dt_eta = dt_eta;
  p.dout = dXQW; p.dt_dout = dt_dout;
  p.d_ln_w = d_ln_w; p.d_ln_b = d_ln_b; p.dW = dW1; p.db = db1;
  p.dXQ = dXQ; p.dXV = dXV; p.dXK = dXK; p.deta = d_eta; p.dt_grad = dt_grad;
  p.scratch = scratch;
  p.Z_saved = nullptr; p.W_last = nullptr; p.b_last = nullptr;
  const size_t smem = linear_bwd_smem(CS, F);
  auto kern = lin_tc_products(dt_xq, dt_xv, dt_xk) ? linear_bwd_kernel<true> : linear_bwd_kernel<false>;
  rc = prepare_smem(kern, smem, "ttt_linear_bwd_noalloc");
  if (rc) return rc;
  kern<<<B * NH, lin_threads(F), smem, (cudaStream_t)stream>>>(p);
  return check_launch("ttt_linear_bwd_noalloc");
}
