/*
 * ttt_b200.h -- C ABI of the B200 (sm_100a) TTT-Linear / TTT-MLP dual-form scan.
 *
 * Drop-in boundary for the Triton launches of Ali-Najar/ttt-triton. Each entry point
 * replaces one `kernel[grid](...)` launch inside the reference's autograd wrappers and
 * takes plain device pointers, sizes, dtype codes and a cudaStream_t (as void*). Nothing
 * here allocates: the caller owns every output and scratch buffer, exactly as the
 * reference wrappers own theirs (torch.empty on the input's device). Work is enqueued
 * asynchronously on `stream`; the functions never synchronise the device.
 *
 * Layout (all contiguous, element strides implied by the shapes):
 *   activations XQ, XK, XV, XQW, dXQW, dXQ, dXK, dXV : [B, NH, NC, CS, F]
 *   eta, d_eta                                       : [B, NH, NC, CS, CS]
 *   ttt_norm_weight / ttt_norm_bias                  : [NH, F]
 *   Linear state W / b                               : [B, NH, F, F] / [B, NH, 1, F]    (fp32)
 *   MLP state W1 / b1 / W2 / b2                      : [B, NH, F, FF] / [B, NH, 1, FF] /
 *                                                      [B, NH, FF, F] / [B, NH, 1, F]   (fp32)
 *   checkpoints (K = ceil(NC / checkpoint_group_size)) : [B, NH, K, ...state...]          (fp32)
 *   memo states (NS = ceil(NC / memo_segment_size))    : [B, NH, NS, ...state...]         (fp32)
 * Per-tensor dtype codes select fp32 / bf16 / fp16 storage; arithmetic is fp32 with fp32
 * inner state (tensor-core operands are rounded to the activation type).
 *
 * Every function returns TTT_OK (0) or a negative TTT_ERR_* code; ttt_last_error()
 * gives the message for the calling thread.
 */
#ifndef TTT_B200_H_
#define TTT_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTT_OK 0
#define TTT_ERR_NULL (-1)        /* a required pointer is NULL */
#define TTT_ERR_SHAPE (-2)       /* a size is out of range or inconsistent */
#define TTT_ERR_DTYPE (-3)       /* unknown dtype code */
#define TTT_ERR_UNSUPPORTED (-4) /* valid request this build cannot run (e.g. shared memory) */
#define TTT_ERR_SCRATCH (-5)     /* scratch buffer smaller than the *_scratch_bytes query */
#define TTT_ERR_CUDA (-6)        /* a CUDA runtime call failed; message has the CUDA error */
#define TTT_ERR_ALIGN (-7)       /* a pointer is not aligned to its element size */

#define TTT_DTYPE_F32 0
#define TTT_DTYPE_BF16 1
#define TTT_DTYPE_F16 2

/* Version of this ABI (major * 10000 + minor * 100 + patch). */
int ttt_abi_version(void);

/* Message of the last failing call on this host thread ("" after a success). */
const char* ttt_last_error(void);

/*
 * TTT-Linear forward scan. Replaces the launch of `ttt_linear_scan_forward` in
 * linear_triton.py:96-127 (TritonLinear._forward_core). Computes, per mini-batch, the
 * dual form of ops/ttt_linear.py:8-54 (LayerNorm eps 1e-8, full eta matrix):
 *   XQW = XQ + LN(XQ W + b - (eta * (XQ XK^T + 1)) G),  G = ln_fused_l2_bwd(XK W + b, XV - XK)
 *   W <- W - XK^T diag(eta[CS-1, :]) G,  b <- b - eta[CS-1, :] G
 * Writes XQW (dtype dt_out), the final state W_last/b_last and the state at the start
 * of every checkpoint group (W_ckpt/b_ckpt, as kernels/linear_forward.py:55-73).
 * W1_ckpt/b1_ckpt may both be NULL when no backward follows (inference).
 * Z_out (optional, NULL to skip) receives the fp32 pre-activation Z = XK W_n + b_n of
 * every mini-batch, [B, NH, NC, CS, F]; ttt_linear_bwd uses it to skip recomputation.
 */
int ttt_linear_fwd(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                   const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                   const float* W1_init, const float* b1_init,
                   const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                   const void* eta, int dt_eta,
                   void* XQW, int dt_out,
                   float* W1_last, float* b1_last, float* W1_ckpt, float* b1_ckpt,
                   float* Z_out, void* stream);

/* Bytes of scratch ttt_linear_bwd needs for these sizes (checkpoint-recompute path). */
size_t ttt_linear_bwd_scratch_bytes(int B, int NH, int NC, int CS, int F, int checkpoint_group_size);

/*
 * TTT-Linear backward. Replaces the launch of `ttt_linear_scan_backward` in
 * linear_triton.py:201-246 (TritonLinear._backward_core), with the full dual-form
 * gradients of ops/ttt_linear.py (d_eta is the whole CS x CS block per mini-batch).
 * Inputs are the forward's inputs plus its checkpoints and dXQW. With Z_saved (the
 * forward's Z_out) and the final state W1_last/b1_last, the backward walks the sequence
 * once from the end, recovering each mini-batch's state by undoing its rank-CS update;
 * otherwise (Z_saved NULL) it re-runs each checkpoint group forward from W1_ckpt/b1_ckpt.
 * Outputs:
 *   d_ln_w, d_ln_b : [B, NH, F] fp32 per-(b,h) partial sums (the caller sums over B,
 *                    as linear_triton.py:251-252 does)
 *   dW1, db1       : [B, NH, F, F], [B, NH, 1, F] fp32
 *   dXQ, dXV, dXK  : [B, NH, NC, CS, F], d_eta : [B, NH, NC, CS, CS], all dtype dt_grad
 * `scratch` must hold ttt_linear_bwd_scratch_bytes(...) bytes (its contents are
 * overwritten; no initialisation needed); it may be NULL when Z_saved is given and the
 * request is inside the tensor-core envelope (CS = 16, F = 64, one 16-bit dtype); the
 * call fails with TTT_ERR_SCRATCH if it is needed and missing.
 */
int ttt_linear_bwd(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                   const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                   const float* W1_ckpt, const float* b1_ckpt,
                   const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                   const void* eta, int dt_eta,
                   const void* dXQW, int dt_dout,
                   const float* Z_saved, const float* W1_last, const float* b1_last,
                   float* d_ln_w, float* d_ln_b, float* dW1, float* db1,
                   void* dXQ, void* dXV, void* dXK, void* d_eta, int dt_grad,
                   void* scratch, size_t scratch_bytes, void* stream);

/*
 * Allocation-free TTT-Linear backward (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory where they enqueue work, for example an
 * inference-engine plugin whose enqueue callback is only handed pre-sized buffers, or a
 * service that fixes its device-memory budget at start-up. Same arguments, algorithm and
 * results as ttt_linear_bwd on its checkpoint-recompute path (no Z_saved), but the
 * scratch comes from a 16 MiB array compiled into the library, which every GPU that
 * loads the library holds until the process exits. Requests needing more than 16 MiB
 * (ttt_linear_bwd_scratch_bytes) fail with TTT_ERR_SCRATCH. The call allocates nothing.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
 * once per device, on the current device); make that first call before any stream
 * capture. All calls on a device share the one array: calls whose work overlaps on the
 * GPU (different streams, no ordering between them) race on it. Each call overwrites
 * the part it uses before reading it, so no clearing is needed between calls.
 */
int ttt_linear_bwd_noalloc(int B, int NH, int NC, int CS, int F, int checkpoint_group_size,
                           const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                           const float* W1_ckpt, const float* b1_ckpt,
                           const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                           const void* eta, int dt_eta,
                           const void* dXQW, int dt_dout,
                           float* d_ln_w, float* d_ln_b, float* dW1, float* db1,
                           void* dXQ, void* dXV, void* dXK, void* d_eta, int dt_grad,
                           void* stream);

/*
 * TTT-MLP forward scan (F -> FF -> F, tanh-GELU). Replaces the launch of
 * `ttt_mlp_scan_forward` in mlp_triton.py:130-178 (TritonMLP._forward_core) and, with
 * FF == F, the F x F launch of mlp_triton_back.py:109-146. Dual form of
 * ops/ttt_mlp.py:9-67. Besides XQW, the final state and the group-start checkpoints, it
 * writes the memo states: the state AFTER mini-batch i for every i with
 * i % memo_segment_size == 0 (kernels/mlp_forward.py:193-226). Memo pointers may all be
 * NULL to skip them, and so may the four checkpoint pointers when no backward follows.
 * Z1_out / Z1b_out ([B, NH, NC, CS, FF]) and Z2_out / Z2b_out ([B, NH, NC, CS, F]),
 * optional (all or none), receive the fp32 pre-activations of every mini-batch:
 * Z1 = XK W1 + b1, Z1bar = XQ W1 + b1 - P1 G1 (before its GELU), Z2 = X2 W2 + b2 and
 * Z2bar = X2bar W2 + b2 - P2 G2; ttt_mlp_bwd uses them to walk the sequence once.
 */
int ttt_mlp_fwd(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size, int memo_segment_size,
                const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                const float* W1_init, const float* b1_init, const float* W2_init, const float* b2_init,
                const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                const void* eta, int dt_eta,
                void* XQW, int dt_out,
                float* W1_last, float* b1_last, float* W2_last, float* b2_last,
                float* W1_ckpt, float* b1_ckpt, float* W2_ckpt, float* b2_ckpt,
                float* W1_memo, float* b1_memo, float* W2_memo, float* b2_memo,
                float* Z1_out, float* Z2_out, float* Z1b_out, float* Z2b_out,
                void* stream);

/*
 * Memo-state mixing of the TTT-MLP layer's output: the segment loop of ttt_layer.py:503-559
 * (per segment i >= 1, softmax over <XU, summary_j> weighting the online output XQW and the
 * cached read-outs of memo states 0..i-1, each one launch of mlp_cached_readout_triton in the
 * reference) as one launch sequence. XQW, XQ, XK, XU, out / dOut, dXQW, dXU, dXK are
 * [B, NH, NC, CS, F] contiguous in one 16-bit type (dt); memo states [B, NH, NS, ...] fp32 as
 * ttt_mlp_fwd writes them, NS = ceil(NC / memo_segment_size). Tensor-core path: CS = 16,
 * F = 64, FF = 256 or 64, NS <= 64. The backward gives dXQW, dXU and the summary part of dXK
 * (the cached read-outs and earlier summaries carry no gradient, as in the reference).
 * Activations, gradients and the memo states must be 16-byte aligned (TTT_ERR_ALIGN).
 * Scratch: ttt_memo_mix_scratch_bytes() bytes, 16-byte aligned; the forward leaves the
 * memo states' 16-bit operand copies and the segment summaries in it, and a backward given
 * that same scratch with scratch_prepped = 1 reuses them instead of preparing them again.
 */
size_t ttt_memo_mix_scratch_bytes(int B, int NH, int NC, int memo_segment_size, int FF);
int ttt_memo_mix_fwd(int B, int NH, int NC, int CS, int F, int FF, int memo_segment_size,
                     const void* XQW, const void* XQ, const void* XK, const void* XU, int dt,
                     const float* W1_memo, const float* b1_memo, const float* W2_memo, const float* b2_memo,
                     const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                     void* out, void* scratch, size_t scratch_bytes, void* stream);
int ttt_memo_mix_bwd(int B, int NH, int NC, int CS, int F, int FF, int memo_segment_size,
                     const void* XQW, const void* XQ, const void* XK, const void* XU, int dt,
                     const float* W1_memo, const float* b1_memo, const float* W2_memo, const float* b2_memo,
                     const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                     const void* dOut, void* dXQW, void* dXU, void* dXK,
                     void* scratch, size_t scratch_bytes, int scratch_prepped, void* stream);

/*
 * Input prologue of the TTT layer, forward: everything TTTBase.process_input
 * (ttt_layer.py:261-330; no text prefix, no multi-scene interleave, no tensor parallelism)
 * does after its projections (get_qkvu_projections :141-148 and the learning-rate gate of
 * get_eta :150-163, which the caller runs as one GEMM). proj is [B * L][ld_proj] (ld_proj a
 * multiple of 8, at least 4 * NH * F + NH) holding, per token, the projections
 * q | k | v | u (NH * F columns each, head-major) and the NH gate logits, biases included.
 * Writes XQ, XK, XU = rope(l2_normalize(.)) (:276-295, utils.py:97-123), the LayerNorm
 * reconstruction target XV (:227-244: unbiased std, eps 1e-8 added to it, ln_w/ln_b
 * [NH][F]) in [B, NH, NC, CS, F] and eta = eta_scale * sigmoid(gate) repeated over the rows
 * of each mini-batch in [B, NH, NC, CS, CS] (:309), eta_scale = ttt_base_lr / (F * CS).
 * rope_cos / rope_sin are [L][F / 2] (real and imaginary parts of freqs_cis rows 0..L-1).
 * F is 16, 32, 64 or 128; L a multiple of CS, CS at most 256. proj, the outputs and eta
 * share dtype dt; every pointer is 16-byte aligned.
 */
int ttt_prologue_fwd(int B, int L, int NH, int F, int CS, const void* proj, int dt, long long ld_proj,
                     const float* ln_w, const float* ln_b, const float* rope_cos, const float* rope_sin,
                     float eta_scale, void* XQ, void* XK, void* XV, void* XU, void* eta, void* stream);

/*
 * Input prologue, backward: from the gradients of XQ, XK, XV, XU, eta (each may be NULL,
 * meaning zero) and the same proj, writes d proj ([B * L][ld_proj], dtype dt; the padding
 * columns past 4 * NH * F + NH are written as zeros) and ADDS the LayerNorm parameter
 * gradients into dln_w / dln_b ([NH][F] fp32) and, when dbias is not NULL, the column sums
 * of d proj (the projection bias gradients) into dbias ([4 * NH * F + NH] fp32). The caller
 * finishes with library GEMMs: d hidden = d proj W_cat, d W_cat = d proj^T hidden.
 * Pointers are 16-byte aligned (d_eta: element aligned); CS is at most 256.
 */
int ttt_prologue_bwd(int B, int L, int NH, int F, int CS, const void* proj, int dt, long long ld_proj,
                     const float* ln_w, const float* ln_b, const float* rope_cos, const float* rope_sin,
                     float eta_scale, const void* dXQ, const void* dXK, const void* dXV, const void* dXU,
                     const void* deta, void* dproj, float* dln_w, float* dln_b, float* dbias, void* stream);

/*
 * Output epilogue, forward: the layer's post_norm (nn.LayerNorm over the width W = NH * F,
 * biased variance, eps inside the square root; ttt_layer.py:77,349) applied to the scan
 * output XQW in its kernel layout [B, NH, NC, CS, F] (L = NC * CS), writing the normalised
 * rows Y [B * L, W] in token order, which is the permute + reshape of TTTMLP.ttt
 * (:563-564) folded into the read. ln_w / ln_b are [W] fp32; XQW and Y share dtype dt;
 * F is a multiple of 16 bytes' worth of elements, W at most 1024 (512 in fp32); pointers
 * 16-byte aligned. The caller applies wo (:350) with a library GEMM.
 */
int ttt_post_norm_fwd(int B, int NH, int L, int F, const void* XQW, int dt, const float* ln_w, const float* ln_b,
                      float eps, void* Y, void* stream);

/*
 * Output epilogue, backward: from dY [B * L, W] (d out @ wo, a library GEMM) writes d XQW
 * in the kernel layout and ADDS the post_norm weight / bias gradients into dln_w / dln_b
 * ([W] fp32). With dOut (the gradient of the wo output, [B * L, W], dtype dt) it also ADDS
 * dOut's column sums, the wo bias gradient, into dbias ([W] fp32); both or neither.
 */
int ttt_post_norm_bwd(int B, int NH, int L, int F, const void* XQW, int dt, const float* ln_w, const float* ln_b,
                      float eps, const void* dY, void* dXQW, float* dln_w, float* dln_b, const void* dOut,
                      float* dbias, void* stream);

/*
 * Reads and clears this library's device error word for the current device, synchronising
 * with it. Non-zero bits mean a kernel gave up waiting for its own asynchronous copies
 * (bit 0: a TMA stage did not land within 2 s) and voided the affected streams' results.
 * No counterpart in the reference (its Triton kernels have no bounded waits).
 */
int ttt_device_status(unsigned int* status);

/*
 * Test switch for the bounded waits (no counterpart in the reference). While enabled
 * (enable != 0), every launch of the tensor-core TTT-MLP forward leaves the copies of each
 * stream's first mini-batch un-issued, so the wait for them can only end by its time limit,
 * which this call sets to wait_limit_ns (0: the library's 2 s; larger values are refused
 * with TTT_ERR_SHAPE). The kernel then sets bit 0 of the device error word
 * (ttt_device_status), waits (bounded) for the copies it did issue, frees its tensor memory
 * and returns; that call's outputs are void. Nothing faults and nothing is left in flight.
 * Disabling restores the 2 s limit. The setting is process-wide and only affects launches
 * enqueued after the call. For tests of failure reporting; off by default.
 */
int ttt_test_hold_first_stage(int enable, unsigned long long wait_limit_ns);

/*
 * Kernels this library has enqueued in this process so far (every successful launch of any
 * entry point). No counterpart in the reference; for benchmarks that count launches.
 */
unsigned long long ttt_kernel_launches(void);

/*
 * Schedule of the tensor-core MLP forward (ttt_mlp_fwd at F = 64, CS = 16, FF = 256, 16-bit
 * activations) when B * NH streams number between the device's SM count M and 4M/3: with
 * `balanced` set (the default) it runs as two launches of one two-stream CTA per SM that
 * swap which streams share an SM halfway, splitting the sequence by `paired_ratio_milli`,
 * the time of a mini-batch on an SM shared by two streams over one alone, x1000 (0: the
 * library's measured 1550; values outside [1000, 4000] are refused with TTT_ERR_SHAPE);
 * with it clear, one CTA per stream runs the whole sequence. Outputs are bit-identical
 * either way; only the time differs. Process-wide; affects launches enqueued after the
 * call. No counterpart in the reference (its grid is one program per stream).
 */
int ttt_set_forward_schedule(int balanced, int paired_ratio_milli);

/*
 * The plan ttt_mlp_fwd's balanced schedule would follow for `streams` = B * NH streams of NC
 * mini-batches on `num_sms` SMs (host only, no GPU needed; paired_ratio_milli 0 = the
 * current setting). *launches = 2 when it applies, 0 when one CTA per stream runs the whole
 * sequence. For 2, rows[6 k .. 6 k + 5] = (launch 1 or 2, CTA, engine 0 or 1, stream, first
 * mini-batch, end mini-batch) for every engine that has work; *n_rows = their count
 * (TTT_ERR_SHAPE if above max_rows). For tests and tuning; no counterpart in the reference.
 */
int ttt_mlp_fwd_schedule_plan(int streams, int NC, int num_sms, int paired_ratio_milli, int* launches, int* rows,
                              int max_rows, int* n_rows);

/* Bytes of scratch ttt_mlp_bwd needs for these sizes. */
size_t ttt_mlp_bwd_scratch_bytes(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size);

/*
 * TTT-MLP backward. Replaces the launch of `ttt_mlp_scan_backward` in
 * mlp_triton.py:274-333 (and the F x F one of mlp_triton_back.py:238-293), with the full
 * dual-form gradients of ops/ttt_mlp.py. Outputs as ttt_linear_bwd plus dW2/db2
 * ([B, NH, FF, F], [B, NH, 1, F] fp32); dW1/db1 are [B, NH, F, FF], [B, NH, 1, FF].
 * Z1_saved .. Z2b_saved (the four ttt_mlp_fwd pre-activation outputs) with W1_last and
 * W2_last, all set or all NULL, let the tensor-core path (F = 64, FF = 256, CS = 16,
 * 16-bit activations) walk the sequence once from the end without re-running the
 * forward; scratch may then be NULL. Otherwise the checkpoints are re-run and scratch
 * must hold ttt_mlp_bwd_scratch_bytes().
 */
int ttt_mlp_bwd(int B, int NH, int NC, int CS, int F, int FF, int checkpoint_group_size,
                const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                const float* W1_ckpt, const float* b1_ckpt, const float* W2_ckpt, const float* b2_ckpt,
                const void* XQ, int dt_xq, const void* XV, int dt_xv, const void* XK, int dt_xk,
                const void* eta, int dt_eta,
                const void* dXQW, int dt_dout,
                const float* Z1_saved, const float* Z2_saved, const float* Z1b_saved, const float* Z2b_saved,
                const float* W1_last, const float* W2_last,
                float* d_ln_w, float* d_ln_b, float* dW1, float* db1, float* dW2, float* db2,
                void* dXQ, void* dXV, void* dXK, void* d_eta, int dt_grad,
                void* scratch, size_t scratch_bytes, void* stream);

/*
 * Read-out of a frozen (memo) MLP state. Replaces `mlp_cached_readout_triton`
 * (kernels/mlp_cached_readout.py:112-143):
 *   out = XQ + LN(gelu(XQ W1 + b1) W2 + b2)   (LayerNorm eps 1e-6, fp32 output)
 * XQ is [B, NH, NCseg, CS, F] contiguous. The state tensors may be strided in their
 * two leading dimensions (the reference passes non-contiguous memo slices
 * W1_memo[:, :, j]); *_sb / *_sh are their batch / head strides in elements, and the
 * trailing matrix of each (b, h) must be contiguous. Unlike the shipped Triton kernel,
 * every (b, h) is read and written at its own offset.
 */
int ttt_mlp_cached_readout(int B, int NH, int NCseg, int CS, int F, int FF,
                           const void* XQ, int dt_xq,
                           const float* W1, long long W1_sb, long long W1_sh,
                           const float* b1, long long b1_sb, long long b1_sh,
                           const float* W2, long long W2_sb, long long W2_sh,
                           const float* b2, long long b2_sb, long long b2_sh,
                           const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln,
                           float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TTT_B200_H_ */
