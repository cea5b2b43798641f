// Launch parameter blocks shared by the general and the tensor-core kernels.
#pragma once

namespace ttt {

struct LinFwdParams {
  int B, NH, NC, CS, F, ckpt, K;
  const void* ln_w;
  const void* ln_b;
  int dt_ln;
  const float* W_init;
  const float* b_init;
  const void* XQ;
  const void* XV;
  const void* XK;
  const void* eta;
  int dt_xq, dt_xv, dt_xk, dt_eta;
  void* out;
  int dt_out;
  float* W_last;
  float* b_last;
  float* W_ckpt;
  float* b_ckpt;
  float* Z_out;  // optional [B,NH,NC,CS,F] fp32: Z = XK W_n + b_n of every mini-batch
  unsigned int* err;  // device error word (set by the entry point for kernels with bounded waits)
};

struct LinBwdParams {
  int B, NH, NC, CS, F, ckpt, K;
  const void* ln_w;
  const void* ln_b;
  int dt_ln;
  const float* W_ckpt;
  const float* b_ckpt;
  const void* XQ;
  const void* XV;
  const void* XK;
  const void* eta;
  int dt_xq, dt_xv, dt_xk, dt_eta;
  const void* dout;
  int dt_dout;
  float* d_ln_w;
  float* d_ln_b;
  float* dW;
  float* db;
  void* dXQ;
  void* dXV;
  void* dXK;
  void* deta;
  int dt_grad;
  float* scratch;        // [B*NH][ckpt][CS][F] pre-activations Z of one group (checkpoint path)
  const float* Z_saved;  // optional: Z of every mini-batch stored by the forward
  const float* W_last;   // final state (with Z_saved: start of the reverse walk)
  const float* b_last;
};

struct MlpFwdParams {
  int B, NH, NC, CS, F, FF, ckpt, K, memo, NS;
  const void* ln_w;
  const void* ln_b;
  int dt_ln;
  const float* W1_init;
  const float* b1_init;
  const float* W2_init;
  const float* b2_init;
  const void* XQ;
  const void* XV;
  const void* XK;
  const void* eta;
  int dt_xq, dt_xv, dt_xk, dt_eta;
  void* out;
  int dt_out;
  float* W1_last;
  float* b1_last;
  float* W2_last;
  float* b2_last;
  float* W1_ckpt;
  float* b1_ckpt;
  float* W2_ckpt;
  float* b2_ckpt;
  float* W1_memo;
  float* b1_memo;
  float* W2_memo;
  float* b2_memo;
  // optional fp32 pre-activations of every mini-batch, kept for the reverse-walk backward:
  // Z1 = XK W1 + b1, Z1bar (before its GELU) [B,NH,NC,CS,FF]; Z2 = X2 W2 + b2, Z2bar [B,NH,NC,CS,F]
  float* Z1_out;
  float* Z2_out;
  float* Z1b_out;
  float* Z2b_out;
  unsigned int* err;  // device error word (set by the entry point for kernels with bounded waits)
  unsigned long long wait_ns;  // limit of each bounded wait (tensor-core path)
  int hold_stage0;             // wait-expiry test: the first stage's copies are never issued
  // Balanced two-launch schedule of the tensor-core forward (mlp_fwd_fast): 0 = one CTA per
  // stream over the whole sequence; 1 / 2 = its first / second launch, with sched_D SMs running
  // two streams and the paired streams of launch 1 advancing sched_kp mini-batches.
  int sched, sched_D, sched_kp;
};

struct MlpBwdParams {
  int B, NH, NC, CS, F, FF, ckpt, K;
  const void* ln_w;
  const void* ln_b;
  int dt_ln;
  const float* W1_ckpt;
  const float* b1_ckpt;
  const float* W2_ckpt;
  const float* b2_ckpt;
  const void* XQ;
  const void* XV;
  const void* XK;
  const void* eta;
  int dt_xq, dt_xv, dt_xk, dt_eta;
  const void* dout;
  int dt_dout;
  float* d_ln_w;
  float* d_ln_b;
  float* dW1;
  float* db1;
  float* dW2;
  float* db2;
  void* dXQ;
  void* dXV;
  void* dXK;
  void* deta;
  int dt_grad;
  float* scratch;  // per stream: W1 [F*FF], W2 [FF*F], Z1/Z2 of one group [ckpt][CS*(FF+F)]
  // optional: the forward's fp32 pre-activations (ttt_mlp_fwd Z1_out..Z2b_out) and final
  // weights; with them the tensor-core backward walks the sequence once from the end
  const float* Z1_saved;
  const float* Z2_saved;
  const float* Z1b_saved;
  const float* Z2b_saved;
  const float* W1_last;
  const float* W2_last;
  long long spill;  // general kernel: floats per stream of tiles placed in global scratch
};

// Memo-state mixing (ttt_layer.py:503-559); activations [B,NH,NC,16,64] in one 16-bit type.
struct MemoMixParams {
  int B, NH, NC, M, NS, TILES;  // M = memo_segment_size, NS = ceil(NC / M), TILES = 128-token tiles per segment
  int P, NG;  // segments packed per tile (P > 1 when a segment has at most 64 tokens), tile groups per stream
  int dt_ln;
  const void* XQW;
  const void* XQ;
  const void* XK;
  const void* XU;
  const float* W1_memo;  // [B,NH,NS,F,FF]
  const float* b1_memo;  // [B,NH,NS,1,FF]
  const float* W2_memo;  // [B,NH,NS,FF,F]
  const float* b2_memo;  // [B,NH,NS,1,F]
  const void* ln_w;
  const void* ln_b;
  void* out;             // forward
  const void* dOut;      // backward
  void* dXQW;
  void* dXU;
  void* dXK;
  void* W1T;             // scratch: 16-bit [B,NH,NS,FF,F]
  void* W2T;             // scratch: 16-bit [B,NH,NS,F,FF]
  float* summary;        // scratch: [B,NH,NS,F]
  float* dsum;           // scratch: [B,NH,NS,F] (backward)
  unsigned int* err;
};

struct ReadoutParams {
  int B, NH, NCs, CS, F, FF;
  const void* XQ;
  int dt_xq;
  const float* W1;
  long long W1_sb, W1_sh;
  const float* b1;
  long long b1_sb, b1_sh;
  const float* W2;
  long long W2_sb, W2_sh;
  const float* b2;
  long long b2_sb, b2_sh;
  const void* ln_w;
  const void* ln_b;
  int dt_ln;
  float* out;
};

}  // namespace ttt
