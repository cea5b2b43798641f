// TTT-MLP forward on the tensor cores (mma.sync bf16/fp16, fp32 accumulate) for F = 64,
// CS = 16, 16-bit activations and an inner width FF = 32 * NW: the benchmark MLP
// (FF = 256, NW = 8 warps) and the layer's F x F inner MLP (FF = 64, NW = 2).
//
// One engine of NW warps per (batch, head) stream: a CTA of its own, or (FF = 256, between
// M and 4M/3 streams on M SMs) one of the two engines of a CTA per SM in the balanced
// two-launch schedule (fwd_segment). Warp w owns hidden units [32w, 32w + 32). Its slices
// of the fp32 state, W1^T (32 x 64) and W2^T (64 x 32), live in tensor memory in mma
// accumulator-fragment order for the whole sequence and are loaded into fragments for each
// product (the accumulator layout of W1^T is the B-operand layout of W1, and of W2^T the B
// layout of W2); the biases live in shared memory. Per mini-batch (ops/ttt_mlp.py:9-67):
//   A (MMA)  Z1 = XK W1 + b1, Z1q = XQ W1 + b1, X2 = gelu(Z1), partial Z2_w = X2_w W2_w;
//            warps 0-1 form -P1 = -eta * (XQ XK^T + 1)
//   C (rows) Z2 = sum_w Z2_w + b2, G2 = ln_fused_l2_bwd(Z2, XV - XK) (16 lanes per token,
//            32 * NW / 16 tokens per pass)
//   D (MMA)  H = G2 W2^T, G1 = H * gelu_bwd(Z1); W1 += XK^T (-e G1), b1 += 1^T (-e G1);
//            Z1bar = Z1q - P1 G1, X2bar = gelu(Z1bar), A2_w = X2bar_w X2_w^T,
//            partial Z2bar_w = X2bar_w W2_w - (eta * A2_w) G2  (- eta G2 once);
//            W2 += X2^T (-e G2), b2 += 1^T (-e G2)
//   E (rows) XQW = XQ + LN(sum_w Z2bar_w + b2_old)
// The dual-form product P2 G2 = (eta * (sum_w A2_w + 1)) G2 is split by linearity over the
// warps' partial A2_w, so no cross-warp reduction of A2 is needed. GELU and its derivative
// use the hardware tanh approximation (tanh.approx.f32, relative error ~2^-11), below the
// 16-bit operand rounding of this path.
#include "capi_common.cuh"
#include "common.cuh"
#include "fast_paths.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "mlp_tc_common.cuh"
#include "tc_util.cuh"
#include "tma.cuh"
#include "tmem.cuh"

namespace ttt {
namespace mlp_tc {

// Per-phase timeline (built only with -DTTT_PHASE_STAMPS, see build.py --phase-stamps): for
// mini-batch kStampN, thread 0 of each CTA records %globaltimer at the phase boundaries
// (before / after each CTA barrier) and its SM id; ttt_phase_stamps_read copies them out.
#ifdef TTT_PHASE_STAMPS
constexpr int kStampN = 64, kStampCTAs = 4096, kStamps = 10;
__device__ unsigned long long g_phase_stamps[kStampCTAs][kStamps];
// Steady-state rate of every engine: %globaltimer at the loop top of mini-batches n0 + 4 and
// n1 - 4, the mini-batches between them and the SM id, per launch of the balanced schedule
// (index 0: one-engine launch or launch 1, 1: launch 2), row blockIdx.x * ENG + eng.
__device__ unsigned long long g_rate_stamps[2][kStampCTAs][4];
#define TTT_RATE_STAMP()                                                                              \
  do {                                                                                                \
    if (tid == 0 && n1 - n0 > 8 && (n == n0 + 4 || n == n1 - 4) && blockIdx.x * ENG + eng < kStampCTAs) { \
      unsigned long long* r_ = g_rate_stamps[p.sched == 2][blockIdx.x * ENG + eng];                  \
      r_[n == n0 + 4 ? 0 : 1] = global_ns();                                                          \
      if (n == n0 + 4) {                                                                              \
        unsigned sm_;                                                                                 \
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));                                            \
        r_[2] = n1 - n0 - 8;                                                                          \
        r_[3] = sm_;                                                                                  \
      }                                                                                               \
    }                                                                                                 \
  } while (0)
#define TTT_STAMP(k)                                                                                  \
  do {                                                                                                \
    if (tid == 0 && eng == 0 && n == kStampN && blockIdx.x < kStampCTAs) g_phase_stamps[blockIdx.x][k] = global_ns(); \
  } while (0)
#define TTT_STAMP_SM()                                                                                \
  do {                                                                                                \
    unsigned sm_;                                                                                     \
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));                                                \
    if (tid == 0 && eng == 0 && n == kStampN && blockIdx.x < kStampCTAs) g_phase_stamps[blockIdx.x][9] = sm_; \
  } while (0)
#else
#define TTT_STAMP(k) \
  do {               \
  } while (0)
#define TTT_RATE_STAMP() \
  do {                   \
  } while (0)
#define TTT_STAMP_SM() \
  do {                 \
  } while (0)
#endif

constexpr int NSTAGE = 3;
constexpr int TILE = C * F * 2;
constexpr int ETA = C * C * 2;
// Stage of one mini-batch, filled by TMA: XQ, XK, XV tiles (1024-byte aligned for the
// 128-byte swizzle) and the eta tile.
constexpr int OFF_XQ = 0, OFF_XK = 1024 * ((TILE + 1023) / 1024), OFF_XV = 2 * OFF_XK, OFF_ETA = 3 * OFF_XK;
constexpr int STAGE = 1024 * ((OFF_ETA + ETA + 1023) / 1024);
constexpr uint32_t STAGE_BYTES = 3 * TILE + ETA;  // bytes the copies of one stage deliver
constexpr int PLD = F + 8;                          // fp32 row stride of the partial tiles
constexpr int OFF_PART = NSTAGE * STAGE;            // fp32 [NW][C][PLD] per-warp partial sums

// Layout of a CTA of NW warps (inner width 32 * NW).
template <int NW_>
struct Fwd {
  static constexpr int NW = NW_, NTHREADS = 32 * NW, FFW = 32 * NW;
  static constexpr int kCopyThread = NTHREADS - 32;      // lane 0 of the last warp issues and awaits the copies
  static constexpr int OFF_G = OFF_PART + NW * C * PLD * 4;  // 16-bit [C][F] swizzled: G2
  static constexpr int OFF_EG = OFF_G + TILE;                // 16-bit [C][F] swizzled: -e * G2
  static constexpr int OFF_P = OFF_EG + TILE;                // 16-bit [C][C]: -P1
  static constexpr int OFF_B1 = OFF_P + ETA;                 // fp32 [FFW]
  static constexpr int OFF_B2 = OFF_B1 + FFW * 4;            // fp32 [2][F] (ping-pong)
  static constexpr int OFF_LN = OFF_B2 + 2 * F * 4;          // fp32 [2][F]: this head's LayerNorm gamma, beta
  static constexpr int SPAN = 1024 * ((OFF_LN + 2 * F * 4 + 1023) / 1024);  // one stream's region
  static constexpr int SMEM = SPAN + 1024;                   // + slack to align the base to 1024 bytes
  // W1^T and W2^T slices: 128 columns per warp in its lane quadrant, two column blocks for 8 warps
  static constexpr uint32_t TMEM_COLS = NW > 4 ? 256 : 128;
  // CTAs per SM: two of 8 warps (registers), four of 2 warps (TMEM: 4 x 128 columns). The
  // launch asks for enough shared memory that no more CTAs become resident than TMEM holds.
  static constexpr int CTAS_PER_SM = NW > 4 ? 2 : 4;
  static constexpr int SMEM_LAUNCH = NW > 4 ? SMEM : (SMEM > 56 * 1024 ? SMEM : 56 * 1024);
};

// The balanced schedule (sched 1, 2) for S streams on M SMs, M < S <= 4M/3: D = S - M SMs must
// hold two streams at any time. A two-stream CTA (two engines of NW warps, one CTA per SM)
// makes that pairing explicit, and two launches swap it:
//   launch 1: CTA c < D runs streams 2c, 2c+1 (set X) for mini-batches [0, kp); CTA c >= D
//             runs stream 2D + c - D (set Y) alone for [0, NC - kp);
//   launch 2: CTA c < D runs the first 2D streams of Y paired, [NC - kp, NC); CTAs D..3D-1
//             finish X alone, [kp, NC); the rest finish Y alone.
// With kp = NC / (1 + r), r the paired / alone time ratio of a mini-batch, both launches take
// kp * r alone-mini-batch times, so no SM holds two streams for the whole sequence. The state
// crosses the launch boundary exactly (fp32 in W*_last / b*_last). Returns false for an idle
// engine.
__host__ __device__ __forceinline__ bool fwd_segment(const MlpFwdParams& p, int c, int eng, long long* s, int* n0,
                                                     int* n1) {
  const int D = p.sched_D, kp = p.sched_kp, ka = p.NC - kp;
  if (c < D) {  // two streams
    *s = p.sched == 1 ? 2 * c + eng : 2 * D + 2 * c + eng;
    *n0 = p.sched == 1 ? 0 : ka;
    *n1 = p.sched == 1 ? kp : p.NC;
    return true;
  }
  if (eng != 0) return false;
  if (p.sched == 1) {
    *s = 2 * D + (c - D);
    *n0 = 0;
    *n1 = ka;
  } else if (c < 3 * D) {
    *s = c - D;
    *n0 = kp;
    *n1 = p.NC;
  } else {
    *s = 4 * D + (c - 3 * D);
    *n0 = ka;
    *n1 = p.NC;
  }
  return true;
}

// One thread: TMA copies of mini-batch n's XQ, XK, XV tiles and eta tile into stage `st`,
// completing on mbarrier `bar`.
__device__ __forceinline__ void issue_stage(uint32_t st, uint32_t bar, const MlpFwdParams& p, const CUtensorMap* tq,
                                            const CUtensorMap* tk, const CUtensorMap* tv, long long s, int n) {
  const int row = (int)((s * p.NC + n) * C);
  mbar_expect_tx(bar, STAGE_BYTES);
  tma_load_2d(st + OFF_XQ, tq, 0, row, bar);
  tma_load_2d(st + OFF_XK, tk, 0, row, bar);
  tma_load_2d(st + OFF_XV, tv, 0, row, bar);
  bulk_load(st + OFF_ETA, (const uint8_t*)p.eta + (s * p.NC + n) * (long long)ETA, ETA, bar);
}

// Row phases: LPT lanes per token, lane rq holding features FPL*rq .. FPL*rq + FPL-1
// (FPL = 64 / LPT). The 8-warp CTA uses 16 lanes per token (one pass over the 16 tokens, short
// per-thread load chains); the 2-warp CTA uses 8 (two passes instead of four).
template <int LPT>
__device__ __forceinline__ float red_lanes(float v) {
#pragma unroll
  for (int o = 1; o < LPT; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of the NW warps' partial tiles for token tk, features FPL*rq.. (FPL = 4 or 8).
template <int NW, int FPL>
__device__ __forceinline__ void sum_partials_rows(const float* part, int tk, int rq, float* z) {
  const float* p0 = part + tk * PLD + FPL * rq;
#pragma unroll
  for (int c = 0; c < FPL / 4; ++c) {
    float4 a = *reinterpret_cast<const float4*>(p0 + 4 * c);
#pragma unroll
    for (int w = 1; w < NW; ++w) {
      const float4 u = *reinterpret_cast<const float4*>(p0 + w * C * PLD + 4 * c);
      a.x += u.x;
      a.y += u.y;
      a.z += u.z;
      a.w += u.w;
    }
    z[4 * c] = a.x;
    z[4 * c + 1] = a.y;
    z[4 * c + 2] = a.z;
    z[4 * c + 3] = a.w;
  }
}

// Adds FPL consecutive fp32 values of a shared / global row (16-byte aligned) to z.
template <int FPL>
__device__ __forceinline__ void add_row(float* z, const float* src) {
#pragma unroll
  for (int c = 0; c < FPL / 4; ++c) {
    const float4 b = *reinterpret_cast<const float4*>(src + 4 * c);
    z[4 * c] += b.x;
    z[4 * c + 1] += b.y;
    z[4 * c + 2] += b.z;
    z[4 * c + 3] += b.w;
  }
}

template <int FPL>
__device__ __forceinline__ void store_row(float* dst, const float* z) {
#pragma unroll
  for (int c = 0; c < FPL / 4; ++c)
    *reinterpret_cast<float4*>(dst + 4 * c) = make_float4(z[4 * c], z[4 * c + 1], z[4 * c + 2], z[4 * c + 3]);
}

// Byte offset of features FPL*rq.. of row tk in a 128-byte-swizzled 16-bit [16][64] tile.
template <int FPL>
__device__ __forceinline__ uint32_t row_off(int tk, int rq) {
  return swz128(tk, (rq * FPL) >> 3) + ((rq * FPL) & 7) * 2;
}

// FPL consecutive 16-bit values -> fp32 (an 8- or 16-byte load).
template <typename T, int FPL>
__device__ __forceinline__ void unpack_row(const uint8_t* src, float* v) {
  if constexpr (FPL == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Half2<T>::unpack(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    unpack4<T>(src, v);
  }
}

// FPL fp32 values -> FPL consecutive 16-bit values (an 8- or 16-byte store).
template <typename T, int FPL>
__device__ __forceinline__ void pack_row(uint8_t* dst, const float* v, float scale) {
  using H = Half2<T>;
  if constexpr (FPL == 8) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(H::pack(scale * v[0], scale * v[1]), H::pack(scale * v[2], scale * v[3]),
                                                H::pack(scale * v[4], scale * v[5]), H::pack(scale * v[6], scale * v[7]));
  } else {
    *reinterpret_cast<uint2*>(dst) = make_uint2(H::pack(scale * v[0], scale * v[1]), H::pack(scale * v[2], scale * v[3]));
  }
}

// CTA barrier of one engine: the whole CTA when it runs one stream, else the engine's own
// named barrier (ids 1, 2) over its 32 * NW threads.
template <int ENG, int NTHREADS>
__device__ __forceinline__ void engine_sync(int eng) {
  if constexpr (ENG == 1)
    __syncthreads();
  else
    named_barrier(1 + eng, NTHREADS);
}

// One engine (NW warps) runs stream s over mini-batches [n0, n1): the state enters from
// W*_init / b*_init (n0 == 0) or from W*_last / b*_last, where it also leaves.
template <typename T, int NW, int ENG>
__device__ __forceinline__ void fwd_stream(const MlpFwdParams& p, const CUtensorMap* tm_q, const CUtensorMap* tm_k,
                                           const CUtensorMap* tm_v, uint8_t* smem, uint64_t* full_bar, int& abort_sh,
                                           uint32_t tmem_base, int eng, int tid, long long s, int n0, int n1) {
  using H = Half2<T>;
  using L = Fwd<NW>;
  constexpr int NTHREADS = L::NTHREADS, FFW = L::FFW, kCopyThread = L::kCopyThread;
  constexpr int OFF_G = L::OFF_G, OFF_EG = L::OFF_EG, OFF_P = L::OFF_P, OFF_B1 = L::OFF_B1, OFF_B2 = L::OFF_B2;
  constexpr int LPT = NW > 4 ? 16 : 8, FPL = F / LPT;  // row phases: lanes per token, features per lane
  constexpr int RTPP = NTHREADS / LPT;                // tokens per pass of the row phases
  if constexpr (ENG == 1) {  // whole sequence: bounds straight from the launch parameters
    s = blockIdx.x;
    n0 = 0;
    n1 = p.NC;
  }
  // (one engine) the warp index as a uniform value as well: without it this kernel spills
  const int warp = ENG == 1 ? (int)__reduce_max_sync(0xffffffffu, (unsigned)tid >> 5) : tid >> 5;
  const int lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const int h = (int)(s % p.NH);
  const int rtk0 = tid / LPT, rq = tid % LPT;  // row phases: token, feature group
  const int fb = 32 * warp;
  float* part = reinterpret_cast<float*>(smem + OFF_PART);
  float* pw = part + warp * C * PLD;
  float* b1s = reinterpret_cast<float*>(smem + OFF_B1);
  float* b2s = reinterpret_cast<float*>(smem + OFF_B2);

  int last_issued = -1;  // (copy thread) last stage index (mini-batch - n0) whose copies were issued
  if (tid == kCopyThread)
    for (int i = 0; i < NSTAGE - 1 && n0 + i < n1; ++i) {
      // (wait-expiry test) stage 0 never issued: nothing is in flight for its barrier
      if (!(p.hold_stage0 && i == 0))
        issue_stage(smem_u32(smem + i * STAGE), smem_u32(&full_bar[i]), p, tm_q, tm_k, tm_v, s, n0 + i);
      last_issued = i;
    }
  // fp32 state slices live in TMEM: warp w uses lanes 32*(w%4).. and columns
  // [128*(w/4), +64) of its engine's 256 for W1^T, [+64, +128) for W2^T.
  const uint32_t tS1 = tmem_lane_addr(tmem_base, warp, L::TMEM_COLS * eng + 128 * (warp >> 2));
  const uint32_t tS2 = tS1 + 64;
  const bool first = n0 == 0;
  {
    float S1[2][8][4], S2[4][4][4];
    w1_io<2, FFW>(S1, const_cast<float*>((first ? p.W1_init : p.W1_last) + s * F * FFW), fb, g, t, false);
    w2_io(S2, const_cast<float*>((first ? p.W2_init : p.W2_last) + s * FFW * F), fb, g, t, false);
    slice_st(tS1, &S1[0][0][0]);
    slice_st(tS2, &S2[0][0][0]);
  }
  {
    const float* b1i = (first ? p.b1_init : p.b1_last) + s * FFW;
    const float* b2i = (first ? p.b2_init : p.b2_last) + s * F;
    for (int i = tid; i < FFW; i += NTHREADS) b1s[i] = b1i[i];
    for (int i = tid; i < F; i += NTHREADS) b2s[i] = b2i[i];
  }
  // the head's LayerNorm parameters, read by the row phases from shared memory (8 per lane)
  float* lns = reinterpret_cast<float*>(smem + L::OFF_LN);
  for (int i = tid; i < F; i += NTHREADS) {
    lns[i] = ld_elem(p.ln_w, (long long)h * F + i, p.dt_ln);
    lns[F + i] = ld_elem(p.ln_b, (long long)h * F + i, p.dt_ln);
  }
  const uint32_t ones = H::pack(1.f, 1.f);
  const uint32_t a_ones[4] = {ones, ones, ones, ones};

  // mini-batches until the next checkpoint / memo state (both taken where n is a multiple)
  int ck_left = n0 ? (p.ckpt - n0 % p.ckpt) % p.ckpt : 0, memo_left = n0 ? (p.memo - n0 % p.memo) % p.memo : 0;
  for (int n = n0; n < n1; ++n) {
    const int i = n - n0;  // stage index: stage i % NSTAGE, its barrier's (i / NSTAGE)-th phase
    // The copy thread waits for stage i; the engine barrier then publishes it to every warp
    // and tells the copy thread that mini-batch n-1 is done, so its stage may be refilled.
    if (tid == kCopyThread && !abort_sh &&
        !mbar_wait(smem_u32(&full_bar[i % NSTAGE]), (uint32_t)((i / NSTAGE) & 1), p.err, p.wait_ns))
      abort_sh = 1;  // results of this stream are void; the error word reports it
    TTT_STAMP(0);
    engine_sync<ENG, NTHREADS>(eng);
    TTT_STAMP(1);
    TTT_RATE_STAMP();
    {
      const int ii = i + NSTAGE - 1;
      if (tid == kCopyThread && n0 + ii < n1 && !abort_sh) {
        issue_stage(smem_u32(smem + (ii % NSTAGE) * STAGE), smem_u32(&full_bar[ii % NSTAGE]), p, tm_q, tm_k, tm_v, s,
                    n0 + ii);
        last_issued = ii;
      }
    }
    const uint8_t* st = smem + (i % NSTAGE) * STAGE;
    const uint32_t sb = smem_u32(st);
    const float* b2_old = b2s + (i & 1) * F;
    float* b2_new = b2s + ((i + 1) & 1) * F;
    tmem_wait_st();  // the previous mini-batch's state stores (issued without waiting) have landed

    if (p.W1_ckpt && ck_left == 0) {  // state at the start of the checkpoint group
      const long long k = s * p.K + n / p.ckpt;
      float S1[2][8][4], S2[4][4][4];
      slice_ld(tS1, &S1[0][0][0]);
      w1_io<2, FFW>(S1, p.W1_ckpt + k * F * FFW, fb, g, t, true);
      slice_ld(tS2, &S2[0][0][0]);
      w2_io(S2, p.W2_ckpt + k * FFW * F, fb, g, t, true);
      for (int i = tid; i < FFW; i += NTHREADS) p.b1_ckpt[k * FFW + i] = b1s[i];
      for (int i = tid; i < F; i += NTHREADS) p.b2_ckpt[k * F + i] = b2_old[i];
      ck_left = p.ckpt;
    }
    --ck_left;

    // ---------------- A: Z1 = XK W1 + b1, Z1q = XQ W1 + b1 (warp's 32 hidden units)
    float Zq[4][4];
    uint32_t X2p[4][2], GPp[4][2];  // gelu(Z1) and gelu_bwd(Z1), 16-bit pairs in C layout
    {
      float S1[2][8][4];
      slice_ld(tS1, &S1[0][0][0]);
      float Z1[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) Z1[j][c] = Zq[j][c] = 0.f;
      float A1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ak[4], aq[4];
        const uint32_t aoff = swz128((mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
        ldsm_x4(ak, sb + OFF_XK + aoff);
        ldsm_x4(aq, sb + OFF_XQ + aoff);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = j >> 1, hh = 2 * (j & 1);
          const uint32_t b[2] = {H::pack(S1[m][2 * kk][hh], S1[m][2 * kk][hh + 1]),
                                 H::pack(S1[m][2 * kk + 1][hh], S1[m][2 * kk + 1][hh + 1])};
          mma16816<T>(Z1[j], ak, b);
          mma16816<T>(Zq[j], aq, b);
        }
        if (warp < 2) {
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
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 bb = *reinterpret_cast<const float2*>(b1s + fb + 8 * j + 2 * t);
        const float2 z01 = __fadd2_rn(make_float2(Z1[j][0], Z1[j][1]), bb);
        const float2 z23 = __fadd2_rn(make_float2(Z1[j][2], Z1[j][3]), bb);
        Zq[j][0] += bb.x;
        Zq[j][1] += bb.y;
        Zq[j][2] += bb.x;
        Zq[j][3] += bb.y;
        if (p.Z1_out) {
          float* zo = p.Z1_out + (s * p.NC + n) * (long long)(C * FFW) + fb + 8 * j + 2 * t;
          *reinterpret_cast<float2*>(zo + g * FFW) = z01;
          *reinterpret_cast<float2*>(zo + (g + 8) * FFW) = z23;
        }
        float2 g01, g23, d01, d23;
        gelu2_and_bwd(z01, g01, d01);
        gelu2_and_bwd(z23, g23, d23);
        X2p[j][0] = H::pack(g01.x, g01.y);
        X2p[j][1] = H::pack(g23.x, g23.y);
        GPp[j][0] = H::pack(d01.x, d01.y);
        GPp[j][1] = H::pack(d23.x, d23.y);
      }
    }
    {
      // partial Z2_w = X2_w W2_w  (B operand of W2 = accumulator layout of W2^T)
      float S2[4][4][4];
      slice_ld(tS2, &S2[0][0][0]);
#pragma unroll
      for (int nf = 0; nf < 8; ++nf) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int m = nf >> 1, hh = 2 * (nf & 1);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint32_t a[4] = {X2p[2 * ks][0], X2p[2 * ks][1], X2p[2 * ks + 1][0], X2p[2 * ks + 1][1]};
          const uint32_t b[2] = {H::pack(S2[m][2 * ks][hh], S2[m][2 * ks][hh + 1]),
                                 H::pack(S2[m][2 * ks + 1][hh], S2[m][2 * ks + 1][hh + 1])};
          mma16816<T>(acc, a, b);
        }
        *reinterpret_cast<float2*>(pw + g * PLD + 8 * nf + 2 * t) = make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(pw + (g + 8) * PLD + 8 * nf + 2 * t) = make_float2(acc[2], acc[3]);
      }
    }
    TTT_STAMP(2);
    engine_sync<ENG, NTHREADS>(eng);
    TTT_STAMP(3);

    // ---------------- C: Z2 = sum + b2, G2 = ln_fused_l2_bwd(Z2, XV - XK)
#pragma unroll
    for (int tk = rtk0; tk < C; tk += RTPP) {  // every lane of a warp takes the same passes
      float z[FPL], xv[FPL], xk[FPL];
      sum_partials_rows<NW, FPL>(part, tk, rq, z);
      add_row<FPL>(z, b2_old + FPL * rq);
      if (p.Z2_out) store_row<FPL>(p.Z2_out + (s * p.NC + n) * (long long)(C * F) + tk * F + FPL * rq, z);
      const uint32_t xo = row_off<FPL>(tk, rq);
      unpack_row<T, FPL>(st + OFF_XV + xo, xv);
      unpack_row<T, FPL>(st + OFF_XK + xo, xk);
      float sz = 0.f;
#pragma unroll
      for (int j = 0; j < FPL; ++j) sz += z[j];
      const float mu = red_lanes<LPT>(sz) * (1.f / F);
      float d[FPL], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < FPL; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rstd = 1.f / sqrtf(red_lanes<LPT>(m2) * (1.f / F) + kLnEps);
      float xh[FPL], gh[FPL], s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int j = 0; j < FPL; ++j) {
        const float gm = lns[FPL * rq + j], bt = lns[F + FPL * rq + j];
        xh[j] = d[j] * rstd;
        gh[j] = (gm * xh[j] + bt - (xv[j] - xk[j])) * gm;
        s1 += gh[j];
        s2 += gh[j] * xh[j];
      }
      s1 = red_lanes<LPT>(s1);
      s2 = red_lanes<LPT>(s2);
      const float inv = rstd * (1.f / F);
      float G[FPL];
#pragma unroll
      for (int j = 0; j < FPL; ++j) G[j] = (F * gh[j] - s1 - xh[j] * s2) * inv;
      const float e = (float)reinterpret_cast<const T*>(st + OFF_ETA)[(C - 1) * C + tk];
      pack_row<T, FPL>(smem + OFF_G + xo, G, 1.f);
      pack_row<T, FPL>(smem + OFF_EG + xo, G, -e);
    }
    TTT_STAMP(4);
    engine_sync<ENG, NTHREADS>(eng);
    TTT_STAMP(5);

    // ---------------- D
    const uint32_t gb = smem_u32(smem + OFF_G), egb = smem_u32(smem + OFF_EG);
    uint32_t ub[2][4], eb[2][4];  // G1 and -e*G1 transposed: [token half][hidden tile]
    {
      // H = G2 W2^T (B operand of W2^T via movmatrix of the W2^T accumulators)
      float Hh[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) Hh[j][0] = Hh[j][1] = Hh[j][2] = Hh[j][3] = 0.f;
      {
        float S2[4][4][4];
        slice_ld(tS2, &S2[0][0][0]);
#pragma unroll
        for (int kf = 0; kf < 4; ++kf) {
          uint32_t ag[4];
          ldsm_x4(ag, gb + swz128((mi & 1) * 8 + r8, 2 * kf + (mi >> 1)));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t b[2] = {movm_t(H::pack(S2[kf][j][0], S2[kf][j][1])),
                                   movm_t(H::pack(S2[kf][j][2], S2[kf][j][3]))};
            mma16816<T>(Hh[j], ag, b);
          }
        }
      }
      const T* E = reinterpret_cast<const T*>(st + OFF_ETA);
      const float eg0 = -(float)E[(C - 1) * C + g], eg1 = -(float)E[(C - 1) * C + g + 8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 gp0 = H::unpack(GPp[j][0]), gp1 = H::unpack(GPp[j][1]);
        const float g0 = Hh[j][0] * gp0.x, g1 = Hh[j][1] * gp0.y, g2 = Hh[j][2] * gp1.x, g3 = Hh[j][3] * gp1.y;
        ub[0][j] = movm_t(H::pack(g0, g1));
        ub[1][j] = movm_t(H::pack(g2, g3));
        eb[0][j] = movm_t(H::pack(eg0 * g0, eg0 * g1));
        eb[1][j] = movm_t(H::pack(eg1 * g2, eg1 * g3));
      }
    }
    // W1^T += (-e G1)^T XK ; b1 += 1^T (-e G1)
    {
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
      slice_st(tS1, &S1[0][0][0]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float db[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t b[2] = {eb[0][j], eb[1][j]};
      mma16816<T>(db, a_ones, b);
      if (g == 0) {
        float2* bp = reinterpret_cast<float2*>(b1s + fb + 8 * j + 2 * t);
        const float2 o = *bp;
        *bp = make_float2(o.x + db[0], o.y + db[1]);
      }
    }
    // Z1bar = Z1q - P1 G1, X2bar = gelu(Z1bar)
    uint32_t XBp[4][2];
    {
      uint32_t ap[4];
      ldsm_x4(ap, smem_u32(smem + OFF_P) + ((mi & 1) * 8 + r8) * 32 + (mi >> 1) * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b[2] = {ub[0][j], ub[1][j]};
        mma16816<T>(Zq[j], ap, b);
        if (p.Z1b_out) {
          float* zo = p.Z1b_out + (s * p.NC + n) * (long long)(C * FFW) + fb + 8 * j + 2 * t;
          *reinterpret_cast<float2*>(zo + g * FFW) = make_float2(Zq[j][0], Zq[j][1]);
          *reinterpret_cast<float2*>(zo + (g + 8) * FFW) = make_float2(Zq[j][2], Zq[j][3]);
        }
        const float2 g01 = gelu2(make_float2(Zq[j][0], Zq[j][1])), g23 = gelu2(make_float2(Zq[j][2], Zq[j][3]));
        XBp[j][0] = H::pack(g01.x, g01.y);
        XBp[j][1] = H::pack(g23.x, g23.y);
      }
    }
    // A2_w = X2bar_w X2_w^T ; a = -(eta * (A2_w [+1 on warp 0]))
    uint32_t aA2[4];
    {
      float A2[2][4];
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
      const T* E = reinterpret_cast<const T*>(st + OFF_ETA);
      const float one = warp == 0 ? 1.f : 0.f;
      float v[2][4];
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        const float2 e0 = H::unpack(*reinterpret_cast<const uint32_t*>(E + g * C + 8 * jt + 2 * t));
        const float2 e1 = H::unpack(*reinterpret_cast<const uint32_t*>(E + (g + 8) * C + 8 * jt + 2 * t));
        v[jt][0] = -e0.x * (A2[jt][0] + one);
        v[jt][1] = -e0.y * (A2[jt][1] + one);
        v[jt][2] = -e1.x * (A2[jt][2] + one);
        v[jt][3] = -e1.y * (A2[jt][3] + one);
      }
      aA2[0] = H::pack(v[0][0], v[0][1]);
      aA2[1] = H::pack(v[0][2], v[0][3]);
      aA2[2] = H::pack(v[1][0], v[1][1]);
      aA2[3] = H::pack(v[1][2], v[1][3]);
    }
    {
      float S2[4][4][4];
      slice_ld(tS2, &S2[0][0][0]);
      // partial Z2bar_w = X2bar_w W2_w + aA2 G2  -> shared memory (old W2)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bg[4];
        ldsm_x4_t(bg, gb + swz128((mi & 1) * 8 + r8, 2 * np + (mi >> 1)));
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int nf = 2 * np + hf, m = nf >> 1, hh = 2 * (nf & 1);
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816<T>(acc, aA2, bg + 2 * hf);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint32_t a[4] = {XBp[2 * ks][0], XBp[2 * ks][1], XBp[2 * ks + 1][0], XBp[2 * ks + 1][1]};
            const uint32_t b[2] = {H::pack(S2[m][2 * ks][hh], S2[m][2 * ks][hh + 1]),
                                   H::pack(S2[m][2 * ks + 1][hh], S2[m][2 * ks + 1][hh + 1])};
            mma16816<T>(acc, a, b);
          }
          *reinterpret_cast<float2*>(pw + g * PLD + 8 * nf + 2 * t) = make_float2(acc[0], acc[1]);
          *reinterpret_cast<float2*>(pw + (g + 8) * PLD + 8 * nf + 2 * t) = make_float2(acc[2], acc[3]);
        }
      }
      // W2^T += (-e G2)^T X2
      uint32_t bx2[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bx2[j][0] = movm_t(X2p[j][0]);
        bx2[j][1] = movm_t(X2p[j][1]);
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t a[4];
        ldsm_x4_t(a, egb + swz128((mi >> 1) * 8 + r8, 2 * m + (mi & 1)));
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816<T>(S2[m][j], a, bx2[j]);
      }
      slice_st_async(tS2, &S2[0][0][0]);
    }
#pragma unroll
    for (int fw = warp; fw < F / 8; fw += NW) {  // b2_new = b2_old + 1^T (-e G2), features 8fw..8fw+7
      uint32_t bg2[2];
      ldsm_x2_t(bg2, egb + swz128((lane & 8) + r8, fw));
      float db[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816<T>(db, a_ones, bg2);
      if (g == 0) {
        const int f = 8 * fw + 2 * t;
        b2_new[f] = b2_old[f] + db[0];
        b2_new[f + 1] = b2_old[f + 1] + db[1];
      }
    }
    TTT_STAMP(6);
    engine_sync<ENG, NTHREADS>(eng);
    TTT_STAMP(7);

    // ---------------- E: XQW = XQ + LN(sum_w Z2bar_w + b2_old)
#pragma unroll
    for (int tk = rtk0; tk < C; tk += RTPP) {
      float z[FPL], xq[FPL];
      sum_partials_rows<NW, FPL>(part, tk, rq, z);
      add_row<FPL>(z, b2_old + FPL * rq);
      if (p.Z2b_out) store_row<FPL>(p.Z2b_out + (s * p.NC + n) * (long long)(C * F) + tk * F + FPL * rq, z);
      unpack_row<T, FPL>(st + OFF_XQ + row_off<FPL>(tk, rq), xq);
      float sz = 0.f;
#pragma unroll
      for (int j = 0; j < FPL; ++j) sz += z[j];
      const float mu = red_lanes<LPT>(sz) * (1.f / F);
      float d[FPL], m2 = 0.f;
#pragma unroll
      for (int j = 0; j < FPL; ++j) {
        d[j] = z[j] - mu;
        m2 += d[j] * d[j];
      }
      const float rstd = 1.f / sqrtf(red_lanes<LPT>(m2) * (1.f / F) + kLnEps);
      float y[FPL];
#pragma unroll
      for (int j = 0; j < FPL; ++j) y[j] = xq[j] + lns[FPL * rq + j] * d[j] * rstd + lns[F + FPL * rq + j];
      pack_row<T, FPL>((uint8_t*)p.out + ((s * p.NC + n) * (long long)(C * F) + tk * F + FPL * rq) * 2, y, 1.f);
    }

    TTT_STAMP(8);
    TTT_STAMP_SM();
    if (p.W1_memo && memo_left == 0) {  // state after this mini-batch
      const long long m = s * p.NS + n / p.memo;
      float S1[2][8][4], S2[4][4][4];
      tmem_wait_st();
      slice_ld(tS1, &S1[0][0][0]);
      w1_io<2, FFW>(S1, p.W1_memo + m * F * FFW, fb, g, t, true);
      slice_ld(tS2, &S2[0][0][0]);
      w2_io(S2, p.W2_memo + m * FFW * F, fb, g, t, true);
      for (int i = tid; i < FFW; i += NTHREADS) p.b1_memo[m * FFW + i] = b1s[i];
      for (int i = tid; i < F; i += NTHREADS) p.b2_memo[m * F + i] = b2_new[i];
      memo_left = p.memo;
    }
    --memo_left;
  }
  engine_sync<ENG, NTHREADS>(eng);
  {
    float S1[2][8][4], S2[4][4][4];
    tmem_wait_st();
    slice_ld(tS1, &S1[0][0][0]);
    w1_io<2, FFW>(S1, p.W1_last + s * F * FFW, fb, g, t, true);
    slice_ld(tS2, &S2[0][0][0]);
    w2_io(S2, p.W2_last + s * FFW * F, fb, g, t, true);
  }
  // after a timeout, copies issued but never awaited may still be in flight: drain them
  // (bounded) before the CTA's shared memory goes away
  if (tid == kCopyThread && abort_sh)
    for (int m = last_issued - NSTAGE + 1; m <= last_issued; ++m)
      if (m >= 0 && !(p.hold_stage0 && m == 0))  // full 2 s limit: these copies were issued
        mbar_wait(smem_u32(&full_bar[m % NSTAGE]), (uint32_t)((m / NSTAGE) & 1), nullptr);
  const float* b2_fin = b2s + ((n1 - n0) & 1) * F;
  for (int i = tid; i < FFW; i += NTHREADS) p.b1_last[s * FFW + i] = b1s[i];
  for (int i = tid; i < F; i += NTHREADS) p.b2_last[s * F + i] = b2_fin[i];
}

// ENG engines of NW warps per CTA: ENG = 1 is one CTA per stream over the whole sequence
// (grid B * NH); ENG = 2 is one two-stream CTA per SM for the balanced schedule (fwd_segment,
// sched 1 or 2).
template <typename T, int NW, int ENG>
__global__ void __launch_bounds__(32 * NW * ENG, ENG == 1 ? Fwd<NW>::CTAS_PER_SM : 1)
    mlp_fwd_tc_kernel(MlpFwdParams p, const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v) {
  using L = Fwd<NW>;
  constexpr uint32_t TMEM_COLS = L::TMEM_COLS * ENG;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ uint32_t tmem_base_sh;
  __shared__ __align__(8) uint64_t full_bar[ENG][NSTAGE];  // engine e: stage i % NSTAGE landed
  __shared__ int abort_sh[ENG];                            // a stage never landed: stop waiting
  // the engine index through redux.sync: provably warp-uniform, so the compiler keeps it and
  // what derives from it (shared-memory base, stream, mini-batch bounds) in uniform registers
  const int eng = ENG == 1 ? 0 : (int)__reduce_max_sync(0xffffffffu, threadIdx.x / L::NTHREADS);
  const int tid = ENG == 1 ? (int)threadIdx.x : (int)(threadIdx.x & (L::NTHREADS - 1));
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) + eng * L::SPAN;
  long long s = blockIdx.x;
  int n0 = 0, n1 = p.NC;
  bool active = true;
  if constexpr (ENG == 2) active = fwd_segment(p, (int)blockIdx.x, eng, &s, &n0, &n1);

  if (threadIdx.x < 32) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < NSTAGE; ++i) mbar_init(smem_u32(&full_bar[eng][i]), 1);
    abort_sh[eng] = 0;
    fence_mbar_init();
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (active)
    fwd_stream<T, NW, ENG>(p, &tm_q, &tm_k, &tm_v, smem, full_bar[eng], abort_sh[eng], tmem_base_sh, eng, tid, s, n0,
                           n1);
  // every warp's TMEM accesses are complete (slice_ld / slice_st wait); free the columns
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem_base_sh, TMEM_COLS);
}

}  // namespace mlp_tc

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T, int NW>
static int launch_fwd(const MlpFwdParams& q, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                      cudaStream_t stream) {
  using namespace mlp_tc;
  int rc = prepare_smem(mlp_fwd_tc_kernel<T, NW, 1>, Fwd<NW>::SMEM_LAUNCH, "ttt_mlp_fwd");
  if (rc) return rc;
  mlp_fwd_tc_kernel<T, NW, 1><<<q.B * q.NH, Fwd<NW>::NTHREADS, Fwd<NW>::SMEM_LAUNCH, stream>>>(q, tq, tk, tv);
  return check_launch("ttt_mlp_fwd");
}

// The balanced schedule's two launches (fwd_segment) on M SMs.
template <typename T>
static int launch_fwd_balanced(const MlpFwdParams& q, const CUtensorMap& tq, const CUtensorMap& tk,
                               const CUtensorMap& tv, int M, int D, int kp, cudaStream_t stream) {
  using namespace mlp_tc;
  using L = Fwd<8>;
  constexpr int kSmem = 2 * L::SPAN + 1024;
  int rc = prepare_smem(mlp_fwd_tc_kernel<T, 8, 2>, kSmem, "ttt_mlp_fwd");
  if (rc) return rc;
  MlpFwdParams a = q;
  a.sched_D = D;
  a.sched_kp = kp;
  for (int phase = 1; phase <= 2; ++phase) {
    a.sched = phase;
    mlp_fwd_tc_kernel<T, 8, 2><<<M, 2 * L::NTHREADS, kSmem, stream>>>(a, tq, tk, tv);
    rc = check_launch("ttt_mlp_fwd");
    if (rc) return rc;
  }
  return TTT_OK;
}

// SMs of the current device (cached per device).
static int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached[dev] = n;
  }
  return cached[dev];
}

// Whether the balanced schedule applies to S streams of NC mini-batches on M SMs (the FF = 256
// forward), and its split: D two-stream SMs, kp mini-batches for the streams paired first.
static bool balanced_split(long long S, int NC, int M, int ratio_milli, int* D, int* kp) {
  if (M <= 0 || S <= M || 3 * (S - M) > M || NC < 4) return false;  // needs M - D >= 2D
  *D = (int)(S - M);
  *kp = (int)((1000LL * NC + (1000 + ratio_milli) / 2) / (1000 + ratio_milli));
  if (*kp < 1) *kp = 1;
  if (*kp > NC - 1) *kp = NC - 1;
  return true;
}

int mlp_fwd_fast(const MlpFwdParams& p, cudaStream_t stream) {
  using namespace mlp_tc;
  if (p.CS != C || p.F != F || (p.FF != 256 && p.FF != 64)) return TTT_NOT_APPLICABLE;
  const int dt = p.dt_xq;
  if (dt != DT_BF16 && dt != DT_F16) return TTT_NOT_APPLICABLE;
  if (p.dt_xk != dt || p.dt_xv != dt || p.dt_eta != dt || p.dt_out != dt) return TTT_NOT_APPLICABLE;
  if (!aligned16(p.XQ) || !aligned16(p.XK) || !aligned16(p.XV) || !aligned16(p.eta) || !aligned16(p.out))
    return TTT_NOT_APPLICABLE;
  const unsigned long long rows = (unsigned long long)p.B * p.NH * p.NC * C;
  CUtensorMap tq, tk, tv;
  int rc = make_tile_map(&tq, p.XQ, dt, rows, "ttt_mlp_fwd");
  if (!rc) rc = make_tile_map(&tk, p.XK, dt, rows, "ttt_mlp_fwd");
  if (!rc) rc = make_tile_map(&tv, p.XV, dt, rows, "ttt_mlp_fwd");
  if (rc) return rc;
  MlpFwdParams q = p;
  rc = device_error_word(&q.err, "ttt_mlp_fwd");
  if (rc) return rc;
  q.wait_ns = test_wait_limit_ns();
  q.hold_stage0 = test_hold_first_stage() ? 1 : 0;
  q.sched = 0;
  if (p.FF == 256) {
    int D = 0, kp = 0;
    const int M = sm_count();
    if (forward_schedule_balanced() &&
        balanced_split((long long)p.B * p.NH, p.NC, M, forward_paired_ratio_milli(), &D, &kp))
      return dt == DT_BF16 ? launch_fwd_balanced<__nv_bfloat16>(q, tq, tk, tv, M, D, kp, stream)
                           : launch_fwd_balanced<__half>(q, tq, tk, tv, M, D, kp, stream);
    return dt == DT_BF16 ? launch_fwd<__nv_bfloat16, 8>(q, tq, tk, tv, stream)
                         : launch_fwd<__half, 8>(q, tq, tk, tv, stream);
  }
  return dt == DT_BF16 ? launch_fwd<__nv_bfloat16, 2>(q, tq, tk, tv, stream)
                       : launch_fwd<__half, 2>(q, tq, tk, tv, stream);
}

}  // namespace ttt

extern "C" int ttt_mlp_fwd_schedule_plan(int streams, int NC, int num_sms, int paired_ratio_milli, int* launches,
                                         int* rows, int max_rows, int* n_rows) {
  using namespace ttt;
  TTT_REQUIRE(launches && n_rows && (rows || max_rows == 0), TTT_ERR_NULL,
              "ttt_mlp_fwd_schedule_plan: NULL pointer argument");
  TTT_REQUIRE(streams > 0 && NC > 0 && num_sms > 0 && max_rows >= 0, TTT_ERR_SHAPE,
              "ttt_mlp_fwd_schedule_plan: sizes must be positive (got %d, %d, %d)", streams, NC, num_sms);
  TTT_REQUIRE(paired_ratio_milli == 0 || (paired_ratio_milli >= 1000 && paired_ratio_milli <= 4000), TTT_ERR_SHAPE,
              "ttt_mlp_fwd_schedule_plan: paired / alone ratio %d (x1000) outside [1000, 4000]", paired_ratio_milli);
  *launches = 0;
  *n_rows = 0;
  MlpFwdParams p{};
  p.NC = NC;
  const int ratio = paired_ratio_milli ? paired_ratio_milli : forward_paired_ratio_milli();
  if (!forward_schedule_balanced() || !balanced_split(streams, NC, num_sms, ratio, &p.sched_D, &p.sched_kp))
    return ok();
  *launches = 2;
  int k = 0;
  for (int l = 1; l <= 2; ++l) {
    p.sched = l;
    for (int c = 0; c < num_sms; ++c)
      for (int e = 0; e < 2; ++e) {
        long long st = 0;
        int n0 = 0, n1 = 0;
        if (!mlp_tc::fwd_segment(p, c, e, &st, &n0, &n1)) continue;
        if (k < max_rows) {
          int* r = rows + 6 * k;
          r[0] = l; r[1] = c; r[2] = e; r[3] = (int)st; r[4] = n0; r[5] = n1;
        }
        ++k;
      }
  }
  *n_rows = k;
  TTT_REQUIRE(k <= max_rows, TTT_ERR_SHAPE, "ttt_mlp_fwd_schedule_plan: %d rows, room for %d", k, max_rows);
  return ok();
}

#ifdef TTT_PHASE_STAMPS
// Copies the engines' steady-state rate stamps: 2 launches x rows x 4 values (start ns, end ns,
// mini-batches between them, SM id).
extern "C" int ttt_rate_stamps_read(unsigned long long* out, int rows) {
  if (rows < 0 || rows > ttt::mlp_tc::kStampCTAs) return TTT_ERR_SHAPE;
  for (int l = 0; l < 2; ++l)
    if (cudaMemcpyFromSymbol(out + (size_t)l * rows * 4, ttt::mlp_tc::g_rate_stamps, sizeof(unsigned long long) * 4 * rows,
                             sizeof(unsigned long long) * 4 * ttt::mlp_tc::kStampCTAs * l) != cudaSuccess)
      return TTT_ERR_CUDA;
  return TTT_OK;
}

// Copies the timeline of the last forward launch: rows x 10 values (9 stamps in ns, SM id).
extern "C" int ttt_phase_stamps_read(unsigned long long* out, int rows) {
  if (rows < 0 || rows > ttt::mlp_tc::kStampCTAs) return TTT_ERR_SHAPE;
  return cudaMemcpyFromSymbol(out, ttt::mlp_tc::g_phase_stamps, sizeof(unsigned long long) * ttt::mlp_tc::kStamps * rows) ==
                 cudaSuccess
             ? TTT_OK
             : TTT_ERR_CUDA;
}
#endif
