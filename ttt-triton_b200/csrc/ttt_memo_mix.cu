// Memo-state mixing of the TTT-MLP layer's output (ttt_layer.py:503-559) in one launch, on
// the 5th-generation tensor cores.
//
// Segment i of a stream covers mini-batches [i M, min((i+1) M, NC)) (M = memo_segment_size).
// For i >= 1 every token t of the segment mixes
//   out_t = g_i(t) XQW_t + sum_{j<i} g_j(t) R_j(XQ_t),   g = softmax_j(<XU_t, summary_j>),
// where summary_j is the mean of segment j's XK and R_j the cached read-out of memo state j:
// R_j(x) = x + LN(gelu(x W1_j + b1_j) W2_j + b2_j) (LayerNorm eps 1e-6,
// kernels/mlp_cached_readout.py:88-101). Segment 0 passes through.
//
// Kernels:
//   memo_prep   one CTA per (stream, memo state j): 16-bit K-major copies of W1_j^T [FF][F]
//               and W2_j^T [F][FF] (the tensor-core B operands) and summary_j.
//   memo_mix    one CTA (8 warps) per (stream, segment, 128-token tile), heavy segments
//               first; segments of at most 64 tokens are packed P = 128 / tokens to a
//               tile (consecutive segments of one stream are consecutive tokens), which
//               reads the union of their earlier states and masks each row to its own
//               segment's. Per earlier state j (inner width FF = 256, or 64 for the layer's
//               F x F inner MLP):
//                 Z1 = XQ W1_j      128 x FF x 64 tcgen05.mma into tensor memory
//                 X2 = gelu(Z1+b1)  all warps (more columns to warps 4-7 when FF = 256):
//                                   32-column TMEM loads, 16-bit K-major swizzled tiles
//                 Z2 = X2 W2_j      128 x 64 x FF tcgen05.mma
//                 R_j              warps 0-3, one token per thread: LayerNorm in registers
//               forward: accumulate g_j R_j; backward: dg_j = <dOut_t, R_j(t)>.
//               W1_j / W2_j arrive by TMA (128-byte swizzle) as soon as the previous
//               product that read their buffer completes; the product for j+1 is issued
//               behind the one for j, so the tensor cores work under the epilogues.
//   memo_dxk    backward only: dXK of segment i's tokens = d summary_i / (tokens in i).
// Backward of the mixing (the read-outs carry no gradient, ttt_layer.py:542): dXQW =
// g_i dOut; ds_j = g_j (dg_j - sum_k g_k dg_k); dXU = sum_j ds_j summary_j; d summary_i =
// sum_t ds_i(t) XU_t (the earlier summaries enter detached).
#include <type_traits>

#include "capi_common.cuh"
#include "common.cuh"
#include "mma.cuh"
#include "params.cuh"
#include "tc_util.cuh"
#include "tma.cuh"
#include "tmem.cuh"
#include "umma.cuh"

namespace ttt {
namespace memo {

constexpr int F = 64, C = 16, ROWS = 128, NS_MAX = 64;
constexpr float kReadoutEps = 1e-6f;  // kernels/mlp_cached_readout.py:99
constexpr int OFF_XQ = 0;             // [128][64] 16-bit, K-major 128-byte swizzle
constexpr int GLD = NS_MAX + 1;       // row stride of the per-token tables (conflict-free)
constexpr uint32_t XQ_BYTES = ROWS * F * 2;

// Shared memory (1024-byte aligned base) and tensor memory of a CTA for inner width FF.
template <int FF>
struct Mix {
  // FF = 64 runs warp-specialised (SPEC): warps 0-3 compute the GELU, warps 4-7 own one token
  // each (mixing weights, read-out LayerNorm, tail) and warp 8 issues the products and the
  // weight copies; the groups meet only through mbarriers. Z1, Z2 and X2 are double-buffered
  // so product 1 runs two states ahead and product 2 of state j under the GELU of j + 1.
  // FF = 256 keeps one schedule for 8 warps with a CTA barrier per state (its tiles do not
  // fit twice): the GELU columns split [0, SPLIT) on warps 0-3, the rest on warps 4-7.
  static constexpr bool SPEC = FF == 64;
  static constexpr int NT = SPEC ? 288 : 256;         // threads
  static constexpr int NX = SPEC ? 2 : 1;             // Z1 / Z2 / X2 buffers (state j in j % NX)
  static constexpr int NB1 = SPEC ? 4 : 1, NB2 = SPEC ? 3 : 1;  // W1 / W2 buffers (fetch lead)
  static constexpr int OFF_W1 = OFF_XQ + ROWS * F * 2;     // NB1 x [FF][64]: W1_j^T
  static constexpr int OFF_W2 = OFF_W1 + NB1 * FF * F * 2; // NB2 x FF/64 x [64][64]: W2_j^T, K chunks of 64
  // NX x FF/64 x [128][64]: gelu(Z1 + b1), K chunks of 64; the backward's d-summary scratch
  // (fp32 [128][RED_LD], padded rows for conflict-free row-per-thread stores) reuses it
  static constexpr int RED_LD = F + 1;
  static constexpr int X2_BUF = ROWS * FF * 2;
  static constexpr int X2_BYTES = NX * X2_BUF > ROWS * RED_LD * 4 ? NX * X2_BUF : ROWS * RED_LD * 4;
  static constexpr int OFF_X2 = OFF_W2 + NB2 * F * FF * 2;
  static constexpr int OFF_G = OFF_X2 + X2_BYTES;        // fp32 [128][GLD]: mixing weights g_j(t)
  static constexpr int OFF_DG = OFF_G + ROWS * GLD * 4;  // fp32 [128][GLD]: dg_j(t) (backward)
  static constexpr int OFF_LN = OFF_DG + ROWS * GLD * 4; // fp32 [2][64]: LayerNorm weight, bias
  // memo-state biases: FF = 64 stages every state's b1, b2 once per CTA (state j in slot j);
  // FF = 256 keeps a 3-slot ring (state j in slot j % 3) refilled two states ahead
  static constexpr int NBIAS = SPEC ? NS_MAX : 3;
  static constexpr int OFF_B1 = OFF_LN + 2 * F * 4;          // fp32 [NBIAS][FF]: b1_j
  static constexpr int OFF_B2 = OFF_B1 + NBIAS * FF * 4;     // fp32 [NBIAS][64]: b2_j
  // fp32 [NS_MAX][64]: the stream's segment summaries, staged once per CTA; for FF = 256 in
  // the upper half of the X2 region (free before the first read-out and, reloaded, in the
  // backward tail), for FF = 64 in a region of its own
  static constexpr bool SUM_IN_X2 = FF == 256;
  static constexpr int OFF_SUM = SUM_IN_X2 ? OFF_X2 + 36864 : OFF_B2 + NBIAS * F * 4;
  static constexpr int SMEM = (SUM_IN_X2 ? OFF_B2 + NBIAS * F * 4 : OFF_SUM + NS_MAX * F * 4) + 1024;  // + alignment slack
  // tensor memory: Z1 buffers at columns [0, NX * FF), Z2 buffers at [Z2_COL, + NX * 64)
  static constexpr int Z2_COL = FF == 256 ? 256 : NX * FF;
  static constexpr uint32_t TMEM_COLS = FF == 256 ? 512 : 256;
  static constexpr uint32_t W1_BYTES = FF * F * 2, W2_BYTES = F * FF * 2;
  static constexpr int CHUNKS = FF / 32, SPLIT = FF == 256 ? 3 : 0;
  static_assert(OFF_W1 % 1024 == 0 && OFF_W2 % 1024 == 0 && OFF_X2 % 1024 == 0,
                "swizzled tiles need 1024-byte alignment");
  static_assert(Z2_COL + NX * F <= (int)TMEM_COLS, "tensor memory budget");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(!SPEC || FF == 64, "the warp-specialised GELU covers 64 columns");
  static_assert(!SUM_IN_X2 || X2_BYTES >= 36864 + NS_MAX * F * 4, "summaries share the X2 region");
  static_assert(ROWS * RED_LD * 4 <= (SUM_IN_X2 ? 36864 : X2_BYTES), "d-summary scratch below the summaries");
  static_assert(OFF_SUM % 16 == 0 && OFF_B1 % 16 == 0 && OFF_B2 % 16 == 0, "16-byte aligned staged rows");
};

struct Maps {
  CUtensorMap xq;  // XQ rows, 128-row boxes
  CUtensorMap w1;  // W1^T copies [B*NH*NS*FF][64], FF-row boxes
  CUtensorMap w2;  // W2^T copies [B*NH*NS*64][FF], 64 x 64 boxes
};

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------------- prep
template <typename T, int FF>
__global__ void __launch_bounds__(256) memo_prep_kernel(MemoMixParams p) {
  using H = Half2<T>;
  const long long sj = blockIdx.x;  // (stream, memo state)
  const long long s = sj / p.NS;
  const int j = (int)(sj - s * p.NS);
  const int tid = threadIdx.x;
  const float* W1 = p.W1_memo + sj * F * FF;  // [F][FF]
  const float* W2 = p.W2_memo + sj * FF * F;  // [FF][F]
  T* W1T = reinterpret_cast<T*>(p.W1T) + sj * FF * F;  // [FF][F]
  T* W2T = reinterpret_cast<T*>(p.W2T) + sj * F * FF;  // [F][FF]
  __shared__ float tile[2][64][65];
  // 64 x 64 blocks of W1 (rows: features, columns: hidden units blk*64..) and of W2 (rows:
  // hidden units blk*64.., columns: features), transposed together through shared memory;
  // 16-byte global loads and stores
  for (int blk = 0; blk < FF / 64; ++blk) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = tid + 256 * k, r = i >> 4, c = 4 * (i & 15);
      const float4 a = *reinterpret_cast<const float4*>(W1 + r * FF + blk * 64 + c);
      const float4 b = *reinterpret_cast<const float4*>(W2 + (blk * 64 + r) * F + c);
      tile[0][r][c] = a.x;
      tile[0][r][c + 1] = a.y;
      tile[0][r][c + 2] = a.z;
      tile[0][r][c + 3] = a.w;
      tile[1][r][c] = b.x;
      tile[1][r][c + 1] = b.y;
      tile[1][r][c + 2] = b.z;
      tile[1][r][c + 3] = b.w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + 256 * k, r = i >> 3, c = 8 * (i & 7);  // output row r, columns c..c+7
      uint32_t u1[4], u2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        u1[e] = H::pack(tile[0][c + 2 * e][r], tile[0][c + 2 * e + 1][r]);
        u2[e] = H::pack(tile[1][c + 2 * e][r], tile[1][c + 2 * e + 1][r]);
      }
      *reinterpret_cast<uint4*>(W1T + (blk * 64 + r) * F + c) = make_uint4(u1[0], u1[1], u1[2], u1[3]);
      *reinterpret_cast<uint4*>(W2T + r * FF + blk * 64 + c) = make_uint4(u2[0], u2[1], u2[2], u2[3]);
    }
    __syncthreads();
  }
  // summary_j = mean of segment j's XK rows: thread (part, chunk) adds rows part, part + 32, ..
  // of 8 features (16-byte loads), then 64 threads add the 32 parts
  const int n0 = j * p.M, n1 = min((j + 1) * p.M, p.NC);
  const long long r0 = (s * p.NC + n0) * C;
  const int nrows = (n1 - n0) * C;
  const T* XK = reinterpret_cast<const T*>(p.XK);
  float* red = &tile[0][0][0];  // [32][64]
  const int part = tid >> 3, ch = tid & 7;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = part; r < nrows; r += 32) {
    const uint4 u = *reinterpret_cast<const uint4*>(XK + (r0 + r) * F + 8 * ch);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 v = H::unpack(w4[e]);
      acc[2 * e] += v.x;
      acc[2 * e + 1] += v.y;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[part * 64 + 8 * ch + e] = acc[e];
  __syncthreads();
  if (tid < 64) {
    float v = 0.f;
#pragma unroll 8
    for (int q = 0; q < 32; ++q) v += red[q * 64 + tid];
    p.summary[sj * F + tid] = v / (float)nrows;
  }
}

// ---------------------------------------------------------------------------------- mix
// blockIdx.x -> (stream, first and last segment of the tile, tile within the segment) with
// the heaviest tiles first. Unpacked (P = 1): one segment, TILES tiles of it. Packed: group
// k holds segments NS-1 - kP - (P-1) .. NS-1 - kP, counted from the last segment, so the one
// group that is not full (it ends at segment 0, which only passes through) is the one that
// reads the fewest memo states.
__device__ __forceinline__ void decode_block(const MemoMixParams& p, long long& s, int& seg_first, int& seg_last,
                                             int& tile) {
  const long long b = blockIdx.x;
  if (p.P == 1) {
    const long long per_seg = (long long)p.B * p.NH * p.TILES;
    seg_first = seg_last = p.NS - 1 - (int)(b / per_seg);
    const long long r = b % per_seg;
    s = r / p.TILES;
    tile = (int)(r % p.TILES);
  } else {
    const long long per_grp = (long long)p.B * p.NH;
    const int k = (int)(b / per_grp);
    s = b % per_grp;
    tile = 0;
    seg_last = p.NS - 1 - k * p.P;
    seg_first = max(0, seg_last - p.P + 1);
  }
}

template <typename T, bool BWD, int FF>
__global__ void __launch_bounds__(Mix<FF>::NT, 1) memo_mix_kernel(MemoMixParams p, const __grid_constant__ Maps maps) {
  using H = Half2<T>;
  using L = Mix<FF>;
  constexpr int OFF_W1 = L::OFF_W1, OFF_W2 = L::OFF_W2, OFF_X2 = L::OFF_X2, OFF_G = L::OFF_G, OFF_DG = L::OFF_DG;
  constexpr int OFF_LN = L::OFF_LN, OFF_B1 = L::OFF_B1, OFF_B2 = L::OFF_B2, OFF_SUM = L::OFF_SUM;
  constexpr uint32_t TMEM_COLS = L::TMEM_COLS, W1_BYTES = L::W1_BYTES, W2_BYTES = L::W2_BYTES;
  constexpr int NB1 = L::NB1, NB2 = L::NB2, NX = L::NX, NT = L::NT;
  constexpr bool kSpecialised = L::SPEC;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint32_t tmem_base_sh;
  // mbarriers: XQ landed; product 1 / product 2 into buffer b complete; W1 / W2 buffer b
  // landed; (warp-specialised) Z2 buffer b read out by the four row warps, X2 buffer b written
  // and Z1 buffer b read by the four GELU warps
  constexpr int BAR_XQ = 0, BAR_P1 = 1, BAR_P2 = BAR_P1 + NX, BAR_W1 = BAR_P2 + NX, BAR_W2 = BAR_W1 + NB1;
  constexpr int BAR_ZF = BAR_W2 + NB2, BAR_GD = BAR_ZF + NX, NBARS = BAR_GD + NX;
  __shared__ __align__(8) uint64_t bars[NBARS];
  __shared__ int last_w1_sh[NB1], last_w2_sh[NB2];  // last state loaded into each buffer (draining)
  __shared__ int commits_sh[2][NX];                 // product 1 / 2 commits per buffer (draining)
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  long long s;
  int seg_first, seg_last, tile;
  decode_block(p, s, seg_first, seg_last, tile);
  const int n0 = seg_first * p.M, n1 = min((seg_last + 1) * p.M, p.NC);
  const int seg_rows = (n1 - n0) * C;  // tokens of the tile's segments
  const int row0 = tile * ROWS;        // first token of the tile within them
  if (row0 >= seg_rows) return;        // empty tail tile (uniform over the CTA)
  const long long tok0 = (s * p.NC + n0) * C + row0;  // global token index of row 0
  const int nrows = min(ROWS, seg_rows - row0);
  const int seg_tok = p.M * C;         // tokens of every segment but a ragged last one
  const int seg = seg_last;            // the tile reads memo states 0 .. seg_last - 1
  const T* XQW = reinterpret_cast<const T*>(p.XQW);
  const T* XU = reinterpret_cast<const T*>(p.XU);

  if (seg_last == 0) {  // segment 0 passes through (forward: out = XQW; backward: dXQW = dOut, dXU = 0)
    const T* src = reinterpret_cast<const T*>(BWD ? p.dOut : p.XQW);
    T* dst = reinterpret_cast<T*>(BWD ? p.dXQW : p.out);
    for (int i = tid; i < nrows * F; i += NT) dst[tok0 * F + i] = src[tok0 * F + i];
    if (BWD)
      for (int i = tid; i < nrows * F; i += NT) reinterpret_cast<T*>(p.dXU)[tok0 * F + i] = H::from_float(0.f);
    return;
  }

  const uint32_t sXQ = smem_u32(smem + OFF_XQ), sW1 = smem_u32(smem + OFF_W1), sW2 = smem_u32(smem + OFF_W2);
  const uint32_t sX2 = smem_u32(smem + OFF_X2);
  float* G = reinterpret_cast<float*>(smem + OFF_G);
  float* DG = reinterpret_cast<float*>(smem + OFF_DG);
  float* LN = reinterpret_cast<float*>(smem + OFF_LN);

  // barrier of state j's buffer (the phase of state j is j / NX, j / NB1, j / NB2)
  const uint32_t b_xq = smem_u32(&bars[BAR_XQ]);
  auto b_p1 = [&](int j) { return smem_u32(&bars[BAR_P1 + j % NX]); };
  auto b_p2 = [&](int j) { return smem_u32(&bars[BAR_P2 + j % NX]); };
  auto b_w1 = [&](int j) { return smem_u32(&bars[BAR_W1 + j % NB1]); };
  auto b_w2 = [&](int j) { return smem_u32(&bars[BAR_W2 + j % NB2]); };
  auto b_zf = [&](int j) { return smem_u32(&bars[BAR_ZF + j % NX]); };
  auto b_gd = [&](int j) { return smem_u32(&bars[BAR_GD + j % NX]); };
  // Thread groups. Row threads own one token each (mixing weights, read-out, tail). In the
  // warp-specialised schedule the GELU group takes warps 0-3, which the warp schedulers favour:
  // the GELU is on the chain of dependent products, the read-out is not. At FF = 256 the bias
  // ring is refilled by the 128 threads from GELU_T0 (warps 4-7).
  constexpr int ROW_T0 = kSpecialised ? 128 : 0, GELU_T0 = 128 - ROW_T0;
  constexpr int kIssuer = kSpecialised ? 256 : 0;  // thread that issues the products
  const bool row_thread = (unsigned)(tid - ROW_T0) < (unsigned)ROWS;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t idesc1 = umma_idesc_f32(kBf16, ROWS, FF), idesc2 = umma_idesc_f32(kBf16, ROWS, F);
  const int h = (int)(s % p.NH);
  const int nstate = seg;  // memo states 0 .. seg-1 are read out

  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < NBARS; ++i) mbar_init(smem_u32(&bars[i]), i >= BAR_ZF ? 4 : 1);  // ZF, GD: one arrival per warp
    for (int b = 0; b < NB1; ++b) last_w1_sh[b] = -1;
    for (int b = 0; b < NB2; ++b) last_w2_sh[b] = -1;
    for (int b = 0; b < NX; ++b) commits_sh[0][b] = commits_sh[1][b] = 0;
    abort_sh = 0;
    fence_mbar_init();
  }
  if (tid < 2 * F) LN[tid] = ld_elem(tid < F ? p.ln_w : p.ln_b, (long long)h * F + (tid % F), p.dt_ln);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tZ1 = tmem_base_sh, tZ2 = tmem_base_sh + L::Z2_COL;

  // state j's weights go to buffers j % NB1 and j % NB2
  auto load_w1 = [&](int j) {
    mbar_expect_tx(b_w1(j), W1_BYTES);
    tma_load_2d(sW1 + (j % NB1) * W1_BYTES, &maps.w1, 0, (int)((s * p.NS + j) * FF), b_w1(j));
    last_w1_sh[j % NB1] = j;
  };
  auto load_w2 = [&](int j) {
    const uint32_t dst = sW2 + (j % NB2) * W2_BYTES;
    mbar_expect_tx(b_w2(j), W2_BYTES);
#pragma unroll
    for (int a = 0; a < FF / 64; ++a)
      tma_load_2d(dst + a * (F * 64 * 2), &maps.w2, 64 * a, (int)((s * p.NS + j) * F), b_w2(j));
    last_w2_sh[j % NB2] = j;
  };
  auto bslot = [&](int j) { return kSpecialised ? j : j % 3; };  // bias slot of state j
  // Biases of state j into slot bslot(j) (plain loads; a barrier publishes them).
  auto load_bias = [&](int j) {  // all threads, blocking (setup)
    float* b1s = reinterpret_cast<float*>(smem + OFF_B1) + bslot(j) * FF;
    float* b2s = reinterpret_cast<float*>(smem + OFF_B2) + bslot(j) * F;
    for (int i = tid; i < FF; i += NT) b1s[i] = __ldg(p.b1_memo + (s * p.NS + j) * FF + i);
    if (tid < F) b2s[tid] = __ldg(p.b2_memo + (s * p.NS + j) * F + tid);
  };
  // Every state's biases of the stream at once (warp-specialised schedule; 16-byte copies)
  auto stage_biases = [&]() {
    const float4* s1 = reinterpret_cast<const float4*>(p.b1_memo + s * p.NS * FF);
    const float4* s2 = reinterpret_cast<const float4*>(p.b2_memo + s * p.NS * F);
    float4* d1 = reinterpret_cast<float4*>(smem + OFF_B1);
    float4* d2 = reinterpret_cast<float4*>(smem + OFF_B2);
    for (int i = tid; i < nstate * (FF / 4); i += NT) d1[i] = s1[i];
    for (int i = tid; i < nstate * (F / 4); i += NT) d2[i] = s2[i];
  };
  // FF = 256 ring: from state 2 on the biases are fetched into registers two states ahead
  // (*_fetch) and written to their slot later (*_put), so the global-load latency stays off
  // the critical path. Slot (j + 2) % 3 is written after the barrier that ends state j, when
  // every reader of its previous occupant (state j - 1) is done; the barrier of state j + 1
  // publishes it. i = this thread's index within warps 4-7.
  float pb[3];  // b1[i], b1[i + 128], b2[i] of the fetched state
  auto b1_fetch = [&](int j, int i) {
    pb[0] = i < FF ? __ldg(p.b1_memo + (s * p.NS + j) * FF + i) : 0.f;
    pb[1] = i + 128 < FF ? __ldg(p.b1_memo + (s * p.NS + j) * FF + i + 128) : 0.f;
  };
  auto b1_put = [&](int j, int i) {
    float* b1s = reinterpret_cast<float*>(smem + OFF_B1) + (j % 3) * FF;
    if (i < FF) b1s[i] = pb[0];
    if (i + 128 < FF) b1s[i + 128] = pb[1];
  };
  auto b2_fetch = [&](int j, int i) { pb[2] = i < F ? __ldg(p.b2_memo + (s * p.NS + j) * F + i) : 0.f; };
  auto b2_put = [&](int j, int i) {
    if (i < F) reinterpret_cast<float*>(smem + OFF_B2)[(j % 3) * F + i] = pb[2];
  };
  float* SUM = reinterpret_cast<float*>(smem + OFF_SUM);
  // the stream's summaries 0..seg_last into shared memory (all threads, 16-byte copies)
  auto stage_summaries = [&]() {
    const float4* src = reinterpret_cast<const float4*>(p.summary + s * p.NS * F);
    float4* dst = reinterpret_cast<float4*>(SUM);
    for (int i = tid; i < (seg_last + 1) * (F / 4); i += NT) dst[i] = src[i];
  };
  // products of state j (issuer thread): into tensor-memory buffer j % NX, committed to that
  // buffer's barrier
  auto product1 = [&](int j) {  // Z1 = XQ W1_j  (K = 64)
    tmem_fence_after();
    const uint32_t d = tZ1 + (j % NX) * FF;
    const uint64_t da = umma_desc_k_sw128(sXQ), db = umma_desc_k_sw128(sW1 + (j % NB1) * W1_BYTES);
#pragma unroll
    for (int k = 0; k < F / 16; ++k) umma_ss(d, da + 2 * k, db + 2 * k, idesc1, k > 0);
    umma_commit(b_p1(j));
    ++commits_sh[0][j % NX];
  };
  auto product2 = [&](int j) {  // Z2 = X2 W2_j  (K = FF in 64-wide chunks)
    tmem_fence_after();
    const uint32_t d = tZ2 + (j % NX) * F, x2b = sX2 + (j % NX) * L::X2_BUF, w2b = sW2 + (j % NB2) * W2_BYTES;
#pragma unroll
    for (int a = 0; a < FF / 64; ++a) {
      const uint64_t da = umma_desc_k_sw128(x2b + a * (ROWS * 64 * 2)), db = umma_desc_k_sw128(w2b + a * (F * 64 * 2));
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_ss(d, da + 2 * k, db + 2 * k, idesc2, (a | k) != 0);
    }
    umma_commit(b_p2(j));
    ++commits_sh[1][j % NX];
  };
  auto wait = [&](uint32_t bar, int phase) {
    if (!abort_sh && !mbar_wait(bar, (uint32_t)(phase & 1), p.err)) abort_sh = 1;
  };

  // copy thread (0): XQ tile and the first weights
  if (tid == 0) {
    mbar_expect_tx(b_xq, XQ_BYTES);
    tma_load_2d(sXQ, &maps.xq, 0, (int)tok0, b_xq);
    for (int j = 0; j < NB1 && j < nstate; ++j) load_w1(j);
    for (int j = 0; j < NB2 && j < nstate; ++j) load_w2(j);
  }
  // 16-bit row c..c+7 of a [.][F] tensor <-> 8 floats (16-byte accesses)
  auto ld_row8 = [&](const T* src, float* x) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = H::unpack(w4[k]);
      x[2 * k] = v.x;
      x[2 * k + 1] = v.y;
    }
  };
  auto st_row8 = [&](T* dst, const float* x) {
    *reinterpret_cast<uint4*>(dst) =
        make_uint4(H::pack(x[0], x[1]), H::pack(x[2], x[3]), H::pack(x[4], x[5]), H::pack(x[6], x[7]));
  };
  const int r = tid - ROW_T0;  // row of a row thread
  const int seg_r = seg_first + (row0 + min(r, nrows - 1)) / seg_tok;
  float xu[F];  // the row's XU, loaded before the summaries are staged so the latencies overlap
  if (row_thread && r < nrows) {
#pragma unroll
    for (int c = 0; c < F; c += 8) ld_row8(XU + (tok0 + r) * F + c, xu + c);
  }
  stage_summaries();
  if constexpr (kSpecialised) {
    stage_biases();
  } else {
    if (nstate > 0) load_bias(0);
    if (nstate > 1) load_bias(1);
  }
  __syncthreads();  // summaries and the first two states' biases in shared memory

  // mixing weights g_j(t), j = 0..seg_r (row threads, one token each; seg_r is the row's own
  // segment)
  if (row_thread && r < nrows) {
    float mx = -INFINITY;
    for (int j = 0; j <= seg_r; ++j) {
      const float4* sm = reinterpret_cast<const float4*>(SUM + j * F);
      float d = 0.f;
#pragma unroll
      for (int c = 0; c < F / 4; ++c) {
        const float4 v = sm[c];  // same address in every thread: a broadcast
        d += xu[4 * c] * v.x + xu[4 * c + 1] * v.y + xu[4 * c + 2] * v.z + xu[4 * c + 3] * v.w;
      }
      G[r * GLD + j] = d;
      mx = fmaxf(mx, d);
    }
    float tot = 0.f;
    for (int j = 0; j <= seg_r; ++j) {
      const float e = __expf(G[r * GLD + j] - mx);
      G[r * GLD + j] = e;
      tot += e;
    }
    const float inv = 1.f / tot;
    for (int j = 0; j <= seg_r; ++j) G[r * GLD + j] *= inv;
  }
  if (tid == kIssuer) {  // product 1 of the first NX states
    wait(b_xq, 0);
    for (int j = 0; j < NX && j < nstate; ++j) {
      wait(b_w1(j), j / NB1);
      if (!abort_sh) product1(j);
    }
  }
  __syncthreads();  // mixing weights written; the XQ tile is in shared memory

  // The read-out of state j is R_j = XQ + ln_w * (y_j - mu_j) rstd_j + ln_b with y_j = Z2_j +
  // b2_j. Its terms that do not change with j are taken out of the loop:
  //   forward  out = sum_j g_j R_j + g_i XQW
  //                = ln_w * sum_j g_j rstd_j (y_j - mu_j) + (XQ + ln_b) sum_j g_j + g_i XQW
  //   backward dg_j = <dOut, R_j> = <dOut, XQ + ln_b> + rstd_j <dOut * ln_w, y_j - mu_j>
  float acc[F];      // forward: sum_j g_j rstd_j (y_j - mu_j);  backward: dOut * ln_w
  float gsum = 0.f;  // forward: sum_j g_j over the states read out
  float k0 = 0.f;    // backward: <dOut, XQ + ln_b>
  // 8 values of the XQ row from the swizzled tile
  auto xq_row8 = [&](int ch, float* x) {
    const uint4 u = *reinterpret_cast<const uint4*>(smem + OFF_XQ + swz128(r, ch));
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = H::unpack(w4[k]);
      x[2 * k] = v.x;
      x[2 * k + 1] = v.y;
    }
  };
  const T* dO = reinterpret_cast<const T*>(p.dOut);
  if (row_thread) {
#pragma unroll
    for (int ch = 0; ch < F / 8; ++ch) {
      if (BWD && r < nrows) {
        float x[8];
        xq_row8(ch, x);
        ld_row8(dO + (tok0 + r) * F + 8 * ch, acc + 8 * ch);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = 8 * ch + e;
          k0 += acc[c] * (x[e] + LN[F + c]);
          acc[c] *= LN[c];
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[8 * ch + e] = 0.f;
      }
    }
  }

  // X2 = gelu(Z1 + b1_j) for 32-column chunks [c_begin, c_end) of the rows of lane quadrant
  // warp % 4, into the K-major swizzled X2 tiles
  auto gelu_chunks = [&](int j, int c_begin, int c_end) {
    const int row = 32 * (warp & 3) + lane;
    const float* b1 = reinterpret_cast<const float*>(smem + OFF_B1) + bslot(j) * FF;
#pragma unroll 1
    for (int c4 = c_begin; c4 < c_end; ++c4) {
      const int col = 32 * c4;
      float z[32];
      tmem_ld32(tmem_lane_addr(tZ1 + (j % NX) * FF, warp, col), z);
      tmem_wait_ld();
      uint32_t pk[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const float2 bb = *reinterpret_cast<const float2*>(b1 + col + 2 * u);
        const float2 g = gelu2(make_float2(z[2 * u] + bb.x, z[2 * u + 1] + bb.y));
        pk[u] = H::pack(g.x, g.y);
      }
      const int atom = col / 64, ch0 = (col % 64) / 8;
      uint8_t* base = smem + OFF_X2 + (j % NX) * L::X2_BUF + atom * (ROWS * 64 * 2);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(base + swz128(row, ch0 + u)) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
    }
  };
  // The same for FF = 64 in one pass: both 32-column loads issued before the wait
  auto gelu64 = [&](int j) {
    const int row = 32 * (warp & 3) + lane;
    const float* b1 = reinterpret_cast<const float*>(smem + OFF_B1) + bslot(j) * FF;
    float z[64];
    tmem_ld32(tmem_lane_addr(tZ1 + (j % NX) * FF, warp, 0), z);
    tmem_ld32(tmem_lane_addr(tZ1 + (j % NX) * FF, warp, 32), z + 32);
    tmem_wait_ld();
    uint8_t* base = smem + OFF_X2 + (j % NX) * L::X2_BUF;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      uint32_t pk[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = 8 * ch + 2 * u;
        const float2 bb = *reinterpret_cast<const float2*>(b1 + c);
        const float2 g = gelu2(__fadd2_rn(make_float2(z[c], z[c + 1]), bb));
        pk[u] = H::pack(g.x, g.y);
      }
      *reinterpret_cast<uint4*>(base + swz128(row, ch)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  };
  // R_j = XQ + LN(Z2 + b2_j) (row threads, one token each): accumulate the forward's sum or
  // record dg_j = <dOut, R_j> (backward). With signal_free each warp arrives on the Z2-free
  // mbarrier as soon as its rows are out of tensor memory.
  auto readout = [&](int j, bool signal_free) {
    if (lane == 0) wait(b_p2(j), j / NX);
    __syncwarp();
    tmem_fence_after();
    float z[F];
    tmem_ld32(tmem_lane_addr(tZ2 + (j % NX) * F, warp, 0), z);
    tmem_ld32(tmem_lane_addr(tZ2 + (j % NX) * F, warp, 32), z + 32);
    tmem_wait_ld();
    if (signal_free) {
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_zf(j));
    }
    // product 2 of j no longer reads its W2 buffer: fetch state j + NB2 into it
    if (tid == ROW_T0 && j + NB2 < nstate && !abort_sh) load_w2(j + NB2);
    const float* b2 = reinterpret_cast<const float*>(smem + OFF_B2) + bslot(j) * F;
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < F; c += 2) {
      const float2 y = __fadd2_rn(make_float2(z[c], z[c + 1]), *reinterpret_cast<const float2*>(b2 + c));
      z[c] = y.x;
      z[c + 1] = y.y;
      s2 = __fadd2_rn(s2, y);
    }
    const float2 nmu = f2(-(s2.x + s2.y) * (1.f / F));
    float2 v2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < F; c += 2) {
      const float2 d = __fadd2_rn(make_float2(z[c], z[c + 1]), nmu);
      z[c] = d.x;
      z[c + 1] = d.y;
      v2 = __ffma2_rn(d, d, v2);
    }
    const float rstd = 1.f / sqrtf((v2.x + v2.y) * (1.f / F) + kReadoutEps);
    if (!BWD) {
      const float gj = r < nrows && j < seg_r ? G[r * GLD + j] : 0.f;  // states of the row's own segment only
      gsum += gj;
      const float2 sj = f2(gj * rstd);
#pragma unroll
      for (int c = 0; c < F; c += 2) {
        const float2 a2 = __ffma2_rn(sj, make_float2(z[c], z[c + 1]), make_float2(acc[c], acc[c + 1]));
        acc[c] = a2.x;
        acc[c + 1] = a2.y;
      }
    } else {
      float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < F; c += 2) d2 = __ffma2_rn(make_float2(acc[c], acc[c + 1]), make_float2(z[c], z[c + 1]), d2);
      if (r < nrows) DG[r * GLD + j] = k0 + rstd * (d2.x + d2.y);
    }
  };

  if constexpr (!kSpecialised) {
    // FF = 256: every warp takes part in the GELU; a CTA barrier per state separates it from
    // the products and the read-out
    for (int j = 0; j < nstate; ++j) {
      if (lane == 0) wait(b_p1(j), j / NX);
      __syncwarp();
      tmem_fence_after();
      // product 1 of j no longer reads its W1 buffer: fetch state j + NB1 into it
      if (tid == 0 && j + NB1 < nstate && !abort_sh) load_w1(j + NB1);
      if (warp >= 4 && j + 2 < nstate) {
        b1_fetch(j + 2, tid - GELU_T0);
        b2_fetch(j + 2, tid - GELU_T0);
      }
      gelu_chunks(j, warp < 4 ? 0 : L::SPLIT, warp < 4 ? L::SPLIT : L::CHUNKS);
      fence_proxy_async();  // X2 stores -> visible to the tensor cores
      tmem_fence_before();
      __syncthreads();
      if (warp >= 4 && j + 2 < nstate) {
        b1_put(j + 2, tid - GELU_T0);
        b2_put(j + 2, tid - GELU_T0);
      }
      if (tid == 0 && !abort_sh) {
        wait(b_w2(j), j / NB2);
        if (!abort_sh) product2(j);
        if (j + 1 < nstate) {
          wait(b_w1(j + 1), (j + 1) / NB1);
          if (!abort_sh) product1(j + 1);  // Z1 of j has been read by every warp
        }
      }
      if (row_thread) readout(j, false);
      tmem_fence_before();
    }
  } else if (warp < 4) {
    // GELU group: X2_j = gelu(Z1_j + b1_j) into buffer j % 2, then one arrival per warp on
    // the GELU-done barrier of that buffer. Product 1 of j was committed after product 2 of
    // j - 2 by the same thread, so its completion also means X2 buffer j % 2 is free.
    for (int j = 0; j < nstate; ++j) {
      if (lane == 0) wait(b_p1(j), j / NX);
      __syncwarp();
      tmem_fence_after();
      gelu64(j);
      fence_proxy_async();  // X2 stores -> visible to the tensor cores
      tmem_fence_before();  // Z1 loads complete before the arrival
      __syncwarp();
      if (lane == 0) mbar_arrive(b_gd(j));
    }
  } else if (warp < 8) {
    // row group: the read-outs, following the product-2 commits
    for (int j = 0; j < nstate; ++j) readout(j, true);
  } else if (tid == kIssuer) {
    // issuer: once the GELU of j is done, product 2 of j (into Z2 buffer j % 2, free once the
    // read-out of j - 2 has taken it out) and product 1 of j + 2 (into the Z1 buffer the GELU
    // of j has just read); W1 buffer j % NB1 is free (product 1 of j has completed)
    for (int j = 0; j < nstate; ++j) {
      wait(b_gd(j), j / NX);
      if (j + NB1 < nstate && !abort_sh) load_w1(j + NB1);
      wait(b_w2(j), j / NB2);
      if (j >= NX) wait(b_zf(j - NX), (j - NX) / NX);
      if (!abort_sh) product2(j);
      if (j + NX < nstate) {
        wait(b_w1(j + NX), (j + NX) / NB1);
        if (!abort_sh) product1(j + NX);
      }
    }
  }
  tmem_fence_before();

  // ---- tail (row threads, one token each)
  if constexpr (BWD && L::SUM_IN_X2) {
    // the read-outs overwrote the summaries' copy in the X2 region; every product is done
    // (the row threads waited for the last one before this barrier): stage them again
    __syncthreads();
    stage_summaries();
    __syncthreads();
  }
  if (row_thread && r < nrows) {
    const long long o = (tok0 + r) * F;
    const float gi = G[r * GLD + seg_r];
    if (!BWD) {
      T* out = reinterpret_cast<T*>(p.out);
#pragma unroll
      for (int ch = 0; ch < F / 8; ++ch) {
        float w[8], x[8], y[8];
        ld_row8(XQW + o + 8 * ch, w);
        xq_row8(ch, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = 8 * ch + e;
          y[e] = LN[c] * acc[c] + (x[e] + LN[F + c]) * gsum + gi * w[e];
        }
        st_row8(out + o + 8 * ch, y);
      }
    } else {
      float dgi = 0.f;
#pragma unroll
      for (int c = 0; c < F; c += 8) {
        float w[8], d8[8];
        ld_row8(XQW + o + c, w);
        ld_row8(dO + o + c, d8);
#pragma unroll
        for (int e = 0; e < 8; ++e) dgi += d8[e] * w[e];
      }
      DG[r * GLD + seg_r] = dgi;
      float sg = 0.f;
      for (int k = 0; k <= seg_r; ++k) sg += G[r * GLD + k] * DG[r * GLD + k];
      float dxu[F];
#pragma unroll
      for (int c = 0; c < F; ++c) dxu[c] = 0.f;
      for (int k = 0; k <= seg_r; ++k) {
        const float ds = G[r * GLD + k] * (DG[r * GLD + k] - sg);
        DG[r * GLD + k] = ds;
        const float4* sm = reinterpret_cast<const float4*>(SUM + k * F);
#pragma unroll
        for (int c = 0; c < F / 4; ++c) {
          const float4 v = sm[c];  // broadcast
          dxu[4 * c] += ds * v.x;
          dxu[4 * c + 1] += ds * v.y;
          dxu[4 * c + 2] += ds * v.z;
          dxu[4 * c + 3] += ds * v.w;
        }
      }
      T* dXU = reinterpret_cast<T*>(p.dXU);
      T* dXQW = reinterpret_cast<T*>(p.dXQW);
#pragma unroll
      for (int c = 0; c < F; c += 8) {
        float q8[8];
        ld_row8(dO + o + c, q8);
#pragma unroll
        for (int e = 0; e < 8; ++e) q8[e] *= gi;
        st_row8(dXU + o + c, dxu + c);
        st_row8(dXQW + o + c, q8);
      }
    }
  }
  if (BWD) {
    // d summary_i += sum over the tile's tokens of segment i of ds_i(t) XU_t  (X2 region as
    // scratch)
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem + OFF_X2);  // [128][RED_LD]
    if (row_thread) {
      const float ds = r < nrows ? DG[r * GLD + seg_r] : 0.f;
#pragma unroll
      for (int c = 0; c < F; c += 2) {
        float2 v = make_float2(0.f, 0.f);
        if (r < nrows) v = H::unpack(*reinterpret_cast<const uint32_t*>(XU + (tok0 + r) * F + c));
        red[r * L::RED_LD + c] = ds * v.x;
        red[r * L::RED_LD + c + 1] = ds * v.y;
      }
    }
    __syncthreads();
    // one (segment, feature) per thread: rows [lo, hi) of the tile belong to segment
    // seg_first + sg
    for (int e = tid; e < (seg_last - seg_first + 1) * F; e += NT) {
      const int sg = e / F, f = e % F;
      const int lo = max(0, sg * seg_tok - row0), hi = min(nrows, (sg + 1) * seg_tok - row0);
      float a = 0.f;
      for (int i = lo; i < hi; ++i) a += red[i * L::RED_LD + f];
      atomicAdd(p.dsum + (s * p.NS + seg_first + sg) * F + f, a);
    }
  }
  // a timed-out wait may leave products in flight: drain (bounded) before freeing memory
  if (tid == 0 && abort_sh) {
    mbar_wait(b_xq, 0, nullptr);
    for (int b = 0; b < NX; ++b) {  // the last commit of each product barrier
      if (commits_sh[0][b] > 0) mbar_wait(smem_u32(&bars[BAR_P1 + b]), (uint32_t)((commits_sh[0][b] - 1) & 1), nullptr);
      if (commits_sh[1][b] > 0) mbar_wait(smem_u32(&bars[BAR_P2 + b]), (uint32_t)((commits_sh[1][b] - 1) & 1), nullptr);
    }
    for (int b = 0; b < NB1; ++b)  // weight loads issued and never awaited
      if (last_w1_sh[b] >= 0) mbar_wait(b_w1(last_w1_sh[b]), (uint32_t)((last_w1_sh[b] / NB1) & 1), nullptr);
    for (int b = 0; b < NB2; ++b)
      if (last_w2_sh[b] >= 0) mbar_wait(b_w2(last_w2_sh[b]), (uint32_t)((last_w2_sh[b] / NB2) & 1), nullptr);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base_sh, TMEM_COLS);
}

// ------------------------------------------------------------- mix, two CTAs per SM (FF = 64)
// The F x F layer with at most NSC memo states per stream (the forecaster's layers) runs two
// 8-warp CTAs per SM, so one CTA's dependency chain (GELU -> product 2 -> read-out) overlaps
// the other's. Warps 0-3 compute the GELU into X2 buffer j % 2 and arrive on a GELU-done
// barrier; warps 4-7 own one token each (mixing weights, read-out, tail) and keep their
// read-out accumulators in tensor memory, which keeps them within the 128 registers that two
// CTAs per SM allow; lane 0 of warp 4 issues the products: product 2 of j once the GELU of j
// is done (Z2 is single-buffered: after the read-out of j - 1 took it out) and product 1 of
// j + 1 (W1 has had a state to land). Product 1 of j + 1 is committed after product 2 of j by
// the same thread, so its completion also frees X2 buffer (j + 1) % 2.
struct Mix2 {
  static constexpr int FF = 64, NT = 256, NSC = 16, GLD2 = NSC + 1;
  static constexpr int OFF_W1 = OFF_XQ + ROWS * F * 2;  // 2 x [64][64]: W1_j^T (state j in j % 2)
  static constexpr int OFF_W2 = OFF_W1 + 2 * FF * F * 2;  // 2 x [64][64]: W2_j^T
  static constexpr int X2_BUF = ROWS * FF * 2;
  // 2 x [128][64] X2; the backward tail's d-summary scratch (fp32 [128][64], columns swizzled
  // by the row) reuses it
  static constexpr int OFF_X2 = OFF_W2 + 2 * F * FF * 2;
  static constexpr int OFF_G = OFF_X2 + 2 * X2_BUF;       // fp32 [128][GLD2]: g_j(t)
  static constexpr int OFF_DG = OFF_G + ROWS * GLD2 * 4;  // fp32 [128][GLD2]: dg_j(t)
  static constexpr int OFF_LN = OFF_DG + ROWS * GLD2 * 4; // fp32 [2][64]
  static constexpr int OFF_B1 = OFF_LN + 2 * F * 4;       // fp32 [NSC][64]: every state's b1
  static constexpr int OFF_B2 = OFF_B1 + NSC * FF * 4;    // fp32 [NSC][64]: every state's b2
  static constexpr int OFF_SUM = OFF_B2 + NSC * F * 4;    // fp32 [NSC][64]: segment summaries
  static constexpr int SMEM = OFF_SUM + NSC * F * 4 + 1024;  // + alignment slack
  // tensor memory: Z1 buffers [0, 128), Z2 [128, 192), the row threads' accumulators [192, 256)
  static constexpr uint32_t TMEM_COLS = 256, W_BYTES = FF * F * 2;
  static_assert(OFF_W1 % 1024 == 0 && OFF_W2 % 1024 == 0 && OFF_X2 % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(OFF_G % 16 == 0 && OFF_B1 % 16 == 0 && OFF_B2 % 16 == 0 && OFF_SUM % 16 == 0, "16-byte aligned rows");
  static_assert(ROWS * F * 4 <= 2 * X2_BUF, "d-summary scratch fits the X2 buffers");
  static_assert(2 * (SMEM + 2048) <= 228 * 1024, "two CTAs per SM");
};

template <typename T, bool BWD>
__global__ void __launch_bounds__(Mix2::NT, 2) memo_mix2_kernel(MemoMixParams p, const __grid_constant__ Maps maps) {
  using H = Half2<T>;
  using L = Mix2;
  constexpr int FF = L::FF, NT = L::NT, GLD2 = L::GLD2;
  constexpr uint32_t W_BYTES = L::W_BYTES;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint32_t tmem_base_sh;
  // mbarriers: XQ landed; product 1 into Z1 buffer b complete; product 2 complete; W1 / W2
  // buffer b landed; Z2 read out by the four row warps; X2 buffer b written (and Z1 buffer b
  // read) by the four GELU warps
  constexpr int BAR_XQ = 0, BAR_P1 = 1, BAR_P2 = 3, BAR_W1 = 4, BAR_W2 = 6, BAR_ZF = 8, BAR_GD = 9, NBARS = 11;
  __shared__ __align__(8) uint64_t bars[NBARS];
  __shared__ int last_w_sh[4];   // last state loaded into W1 buffers 0, 1 and W2 buffers 0, 1 (draining)
  __shared__ int commits_sh[3];  // product-1 commits per Z1 buffer, product-2 commits (draining)
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  long long s;
  int seg_first, seg_last, tile;
  decode_block(p, s, seg_first, seg_last, tile);
  const int n0 = seg_first * p.M, n1 = min((seg_last + 1) * p.M, p.NC);
  const int seg_rows = (n1 - n0) * C;
  const int row0 = tile * ROWS;
  if (row0 >= seg_rows) return;  // empty tail tile (uniform over the CTA)
  const long long tok0 = (s * p.NC + n0) * C + row0;
  const int nrows = min(ROWS, seg_rows - row0);
  const int seg_tok = p.M * C;
  const T* XQW = reinterpret_cast<const T*>(p.XQW);
  const T* XU = reinterpret_cast<const T*>(p.XU);

  if (seg_last == 0) {  // segment 0 passes through (forward: out = XQW; backward: dXQW = dOut, dXU = 0)
    const T* src = reinterpret_cast<const T*>(BWD ? p.dOut : p.XQW);
    T* dst = reinterpret_cast<T*>(BWD ? p.dXQW : p.out);
    for (int i = tid; i < nrows * F; i += NT) dst[tok0 * F + i] = src[tok0 * F + i];
    if (BWD)
      for (int i = tid; i < nrows * F; i += NT) reinterpret_cast<T*>(p.dXU)[tok0 * F + i] = H::from_float(0.f);
    return;
  }

  const uint32_t sXQ = smem_u32(smem + OFF_XQ), sW1 = smem_u32(smem + L::OFF_W1), sW2 = smem_u32(smem + L::OFF_W2);
  const uint32_t sX2 = smem_u32(smem + L::OFF_X2);
  float* G = reinterpret_cast<float*>(smem + L::OFF_G);
  float* DG = reinterpret_cast<float*>(smem + L::OFF_DG);
  float* LN = reinterpret_cast<float*>(smem + L::OFF_LN);
  float* SUM = reinterpret_cast<float*>(smem + L::OFF_SUM);
  // barrier of state j (its phase there: j / 2 for the double buffers, j for P2 and ZF)
  const uint32_t b_xq = smem_u32(&bars[BAR_XQ]), b_p2 = smem_u32(&bars[BAR_P2]), b_zf = smem_u32(&bars[BAR_ZF]);
  auto b_p1 = [&](int j) { return smem_u32(&bars[BAR_P1 + (j & 1)]); };
  auto b_w1 = [&](int j) { return smem_u32(&bars[BAR_W1 + (j & 1)]); };
  auto b_w2 = [&](int j) { return smem_u32(&bars[BAR_W2 + (j & 1)]); };
  auto b_gd = [&](int j) { return smem_u32(&bars[BAR_GD + (j & 1)]); };
  constexpr int ROW_T0 = 128, kIssuer = 128;  // row threads 128..255; lane 0 of warp 4 issues
  const bool row_thread = tid >= ROW_T0;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t idesc1 = umma_idesc_f32(kBf16, ROWS, FF), idesc2 = umma_idesc_f32(kBf16, ROWS, F);
  const int h = (int)(s % p.NH);
  const int nstate = seg_last;  // memo states 0 .. seg_last - 1 are read out

  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, L::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < NBARS; ++i) mbar_init(smem_u32(&bars[i]), i >= BAR_ZF ? 4 : 1);  // ZF, GD: one arrival per warp
    for (int b = 0; b < 4; ++b) last_w_sh[b] = -1;
    for (int b = 0; b < 3; ++b) commits_sh[b] = 0;
    abort_sh = 0;
    fence_mbar_init();
  }
  if (tid < 2 * F) LN[tid] = ld_elem(tid < F ? p.ln_w : p.ln_b, (long long)h * F + (tid % F), p.dt_ln);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tZ1 = tmem_base_sh, tZ2 = tmem_base_sh + 128, tACC = tmem_base_sh + 192;

  auto load_w1 = [&](int j) {
    mbar_expect_tx(b_w1(j), W_BYTES);
    tma_load_2d(sW1 + (j & 1) * W_BYTES, &maps.w1, 0, (int)((s * p.NS + j) * FF), b_w1(j));
    last_w_sh[j & 1] = j;
  };
  auto load_w2 = [&](int j) {
    mbar_expect_tx(b_w2(j), W_BYTES);
    tma_load_2d(sW2 + (j & 1) * W_BYTES, &maps.w2, 0, (int)((s * p.NS + j) * F), b_w2(j));
    last_w_sh[2 + (j & 1)] = j;
  };
  auto product1 = [&](int j) {  // Z1 buffer j % 2 = XQ W1_j  (K = 64)
    tmem_fence_after();
    const uint32_t d = tZ1 + (j & 1) * FF;
    const uint64_t da = umma_desc_k_sw128(sXQ), db = umma_desc_k_sw128(sW1 + (j & 1) * W_BYTES);
#pragma unroll
    for (int k = 0; k < F / 16; ++k) umma_ss(d, da + 2 * k, db + 2 * k, idesc1, k > 0);
    umma_commit(b_p1(j));
    ++commits_sh[j & 1];
  };
  auto product2 = [&](int j) {  // Z2 = X2 (buffer j % 2) W2_j  (K = 64)
    tmem_fence_after();
    const uint64_t da = umma_desc_k_sw128(sX2 + (j & 1) * L::X2_BUF), db = umma_desc_k_sw128(sW2 + (j & 1) * W_BYTES);
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_ss(tZ2, da + 2 * k, db + 2 * k, idesc2, k > 0);
    umma_commit(b_p2);
    ++commits_sh[2];
  };
  auto wait = [&](uint32_t bar, int phase) {
    if (!abort_sh && !mbar_wait(bar, (uint32_t)(phase & 1), p.err)) abort_sh = 1;
  };

  if (tid == 0) {  // XQ tile and the first two states' weights
    mbar_expect_tx(b_xq, XQ_BYTES);
    tma_load_2d(sXQ, &maps.xq, 0, (int)tok0, b_xq);
    for (int j = 0; j < 2 && j < nstate; ++j) {
      load_w1(j);
      load_w2(j);
    }
  }
  auto ld_row8 = [&](const T* src, float* x) {  // 16-bit row c..c+7 -> 8 floats
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = H::unpack(w4[k]);
      x[2 * k] = v.x;
      x[2 * k + 1] = v.y;
    }
  };
  auto st_row8 = [&](T* dst, const float* x) {
    *reinterpret_cast<uint4*>(dst) =
        make_uint4(H::pack(x[0], x[1]), H::pack(x[2], x[3]), H::pack(x[4], x[5]), H::pack(x[6], x[7]));
  };
  const int r = tid - ROW_T0;  // row of a row thread
  const int seg_r = seg_first + (row0 + min(max(r, 0), nrows - 1)) / seg_tok;
  float xu[F];
  if (row_thread && r < nrows) {
#pragma unroll
    for (int c = 0; c < F; c += 8) ld_row8(XU + (tok0 + r) * F + c, xu + c);
  }
  {  // the stream's summaries 0..seg_last and every state's biases (16-byte copies)
    const float4* ss = reinterpret_cast<const float4*>(p.summary + s * p.NS * F);
    const float4* s1 = reinterpret_cast<const float4*>(p.b1_memo + s * p.NS * FF);
    const float4* s2 = reinterpret_cast<const float4*>(p.b2_memo + s * p.NS * F);
    for (int i = tid; i < (seg_last + 1) * (F / 4); i += NT) reinterpret_cast<float4*>(SUM)[i] = ss[i];
    for (int i = tid; i < nstate * (FF / 4); i += NT) reinterpret_cast<float4*>(smem + L::OFF_B1)[i] = s1[i];
    for (int i = tid; i < nstate * (F / 4); i += NT) reinterpret_cast<float4*>(smem + L::OFF_B2)[i] = s2[i];
  }
  __syncthreads();

  // mixing weights g_j(t), j = 0..seg_r (row threads)
  if (row_thread && r < nrows) {
    float mx = -INFINITY;
    for (int j = 0; j <= seg_r; ++j) {
      const float4* sm = reinterpret_cast<const float4*>(SUM + j * F);
      float d = 0.f;
#pragma unroll
      for (int c = 0; c < F / 4; ++c) {
        const float4 v = sm[c];  // broadcast
        d += xu[4 * c] * v.x + xu[4 * c + 1] * v.y + xu[4 * c + 2] * v.z + xu[4 * c + 3] * v.w;
      }
      G[r * GLD2 + j] = d;
      mx = fmaxf(mx, d);
    }
    float tot = 0.f;
    for (int j = 0; j <= seg_r; ++j) {
      const float e = __expf(G[r * GLD2 + j] - mx);
      G[r * GLD2 + j] = e;
      tot += e;
    }
    const float inv = 1.f / tot;
    for (int j = 0; j <= seg_r; ++j) G[r * GLD2 + j] *= inv;
  }
  if (tid == kIssuer) {  // product 1 of state 0
    wait(b_xq, 0);
    wait(b_w1(0), 0);
    if (!abort_sh) product1(0);
  }
  __syncthreads();  // mixing weights written; the XQ tile is in shared memory

  // The read-out of state j is R_j = XQ + ln_w * (y_j - mu_j) rstd_j + ln_b, y_j = Z2_j + b2_j:
  //   forward  out = ln_w * sum_j g_j rstd_j (y_j - mu_j) + (XQ + ln_b) sum_j g_j + g_i XQW
  //   backward dg_j = <dOut, XQ + ln_b> + rstd_j <dOut * ln_w, y_j - mu_j>
  // The per-row vector (forward: the running sum; backward: dOut * ln_w) lives in tensor-memory
  // columns tACC of the row's lane.
  float gsum = 0.f;  // forward: sum_j g_j over the states read out
  float k0 = 0.f;    // backward: <dOut, XQ + ln_b>
  auto xq_row8 = [&](int ch, float* x) {  // 8 values of the XQ row from the swizzled tile
    const uint4 u = *reinterpret_cast<const uint4*>(smem + OFF_XQ + swz128(r, ch));
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = H::unpack(w4[k]);
      x[2 * k] = v.x;
      x[2 * k + 1] = v.y;
    }
  };
  const T* dO = reinterpret_cast<const T*>(p.dOut);
  if (row_thread) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float a[32];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        if (BWD && r < nrows) {
          float x[8];
          xq_row8(4 * hh + ch, x);
          ld_row8(dO + (tok0 + r) * F + 32 * hh + 8 * ch, a + 8 * ch);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = 32 * hh + 8 * ch + e;
            k0 += a[8 * ch + e] * (x[e] + LN[F + c]);
            a[8 * ch + e] *= LN[c];
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) a[8 * ch + e] = 0.f;
        }
      }
      tmem_st32(tmem_lane_addr(tACC, warp, 32 * hh), a);
    }
    tmem_wait_st();
  }

  if (warp < 4) {
    // GELU group: X2_j = gelu(Z1_j + b1_j) into buffer j % 2
    const int row = 32 * warp + lane;
    for (int j = 0; j < nstate; ++j) {
      if (lane == 0) wait(b_p1(j), j >> 1);
      __syncwarp();
      tmem_fence_after();
      const float* b1 = reinterpret_cast<const float*>(smem + L::OFF_B1) + j * FF;
      float z[64];
      tmem_ld32(tmem_lane_addr(tZ1 + (j & 1) * FF, warp, 0), z);
      tmem_ld32(tmem_lane_addr(tZ1 + (j & 1) * FF, warp, 32), z + 32);
      tmem_wait_ld();
      uint8_t* base = smem + L::OFF_X2 + (j & 1) * L::X2_BUF;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t pk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = 8 * ch + 2 * u;
          const float2 bb = *reinterpret_cast<const float2*>(b1 + c);
          const float2 g = gelu2(__fadd2_rn(make_float2(z[c], z[c + 1]), bb));
          pk[u] = H::pack(g.x, g.y);
        }
        *reinterpret_cast<uint4*>(base + swz128(row, ch)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      fence_proxy_async();  // X2 stores -> visible to the tensor cores
      tmem_fence_before();  // Z1 loads complete before the arrival
      __syncwarp();
      if (lane == 0) mbar_arrive(b_gd(j));
    }
  } else {
    // row group: (lane 0 of warp 4) the products of state j, then the read-out of state j
    for (int j = 0; j < nstate; ++j) {
      if (tid == kIssuer) {
        wait(b_gd(j), j >> 1);
        // W1 buffer j % 2 is free (product 1 of j completed before the GELU of j began)
        if (j + 2 < nstate && !abort_sh) load_w1(j + 2);
        wait(b_w2(j), j >> 1);
        if (j >= 1) wait(b_zf, (j - 1) & 1);  // Z2 taken out for state j - 1
        if (!abort_sh) product2(j);
        if (j + 1 < nstate) {
          wait(b_w1(j + 1), (j + 1) >> 1);
          if (!abort_sh) product1(j + 1);
        }
      }
      __syncwarp();
      if (lane == 0) wait(b_p2, j);
      __syncwarp();
      tmem_fence_after();
      float z[F];
      tmem_ld32(tmem_lane_addr(tZ2, warp, 0), z);
      tmem_ld32(tmem_lane_addr(tZ2, warp, 32), z + 32);
      tmem_wait_ld();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_zf);
      // product 2 of j no longer reads W2 buffer j % 2: fetch state j + 2 into it
      if (tid == kIssuer && j + 2 < nstate && !abort_sh) load_w2(j + 2);
      const float* b2 = reinterpret_cast<const float*>(smem + L::OFF_B2) + j * F;
      float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < F; c += 2) {
        const float2 y = __fadd2_rn(make_float2(z[c], z[c + 1]), *reinterpret_cast<const float2*>(b2 + c));
        z[c] = y.x;
        z[c + 1] = y.y;
        s2 = __fadd2_rn(s2, y);
      }
      const float2 nmu = f2(-(s2.x + s2.y) * (1.f / F));
      float2 v2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < F; c += 2) {
        const float2 d = __fadd2_rn(make_float2(z[c], z[c + 1]), nmu);
        z[c] = d.x;
        z[c + 1] = d.y;
        v2 = __ffma2_rn(d, d, v2);
      }
      const float rstd = 1.f / sqrtf((v2.x + v2.y) * (1.f / F) + kReadoutEps);
      if (!BWD) {
        const float gj = r < nrows && j < seg_r ? G[r * GLD2 + j] : 0.f;  // states of the row's own segment only
        gsum += gj;
        const float2 sj = f2(gj * rstd);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float a[32];
          tmem_ld32(tmem_lane_addr(tACC, warp, 32 * hh), a);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float2 a2 = __ffma2_rn(sj, make_float2(z[32 * hh + c], z[32 * hh + c + 1]), make_float2(a[c], a[c + 1]));
            a[c] = a2.x;
            a[c + 1] = a2.y;
          }
          tmem_st32(tmem_lane_addr(tACC, warp, 32 * hh), a);
        }
        tmem_wait_st();
      } else {
        float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float a[32];
          tmem_ld32(tmem_lane_addr(tACC, warp, 32 * hh), a);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c += 2)
            d2 = __ffma2_rn(make_float2(a[c], a[c + 1]), make_float2(z[32 * hh + c], z[32 * hh + c + 1]), d2);
        }
        if (r < nrows) DG[r * GLD2 + j] = k0 + rstd * (d2.x + d2.y);
      }
    }
  }
  tmem_fence_before();

  // ---- tail (row threads, one token each). The tensor-memory loads are warp-collective, so
  // they run for every row thread, before the branch on the tile's ragged row count.
  if (!BWD && row_thread) {
    float a[F];
    tmem_ld32(tmem_lane_addr(tACC, warp, 0), a);
    tmem_ld32(tmem_lane_addr(tACC, warp, 32), a + 32);
    tmem_wait_ld();
    if (r < nrows) {
      const long long o = (tok0 + r) * F;
      const float gi = G[r * GLD2 + seg_r];
      T* out = reinterpret_cast<T*>(p.out);
#pragma unroll
      for (int ch = 0; ch < F / 8; ++ch) {
        float w[8], x[8], y[8];
        ld_row8(XQW + o + 8 * ch, w);
        xq_row8(ch, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = 8 * ch + e;
          y[e] = LN[c] * a[c] + (x[e] + LN[F + c]) * gsum + gi * w[e];
        }
        st_row8(out + o + 8 * ch, y);
      }
    }
  }
  if (BWD && row_thread && r < nrows) {
    const long long o = (tok0 + r) * F;
    const float gi = G[r * GLD2 + seg_r];
    {
      float dgi = 0.f;
#pragma unroll
      for (int c = 0; c < F; c += 8) {
        float w[8], d8[8];
        ld_row8(XQW + o + c, w);
        ld_row8(dO + o + c, d8);
#pragma unroll
        for (int e = 0; e < 8; ++e) dgi += d8[e] * w[e];
      }
      DG[r * GLD2 + seg_r] = dgi;
      float sg = 0.f;
      for (int k = 0; k <= seg_r; ++k) sg += G[r * GLD2 + k] * DG[r * GLD2 + k];
      float dxu[F];
#pragma unroll
      for (int c = 0; c < F; ++c) dxu[c] = 0.f;
      for (int k = 0; k <= seg_r; ++k) {
        const float ds = G[r * GLD2 + k] * (DG[r * GLD2 + k] - sg);
        DG[r * GLD2 + k] = ds;
        const float4* sm = reinterpret_cast<const float4*>(SUM + k * F);
#pragma unroll
        for (int c = 0; c < F / 4; ++c) {
          const float4 v = sm[c];  // broadcast
          dxu[4 * c] += ds * v.x;
          dxu[4 * c + 1] += ds * v.y;
          dxu[4 * c + 2] += ds * v.z;
          dxu[4 * c + 3] += ds * v.w;
        }
      }
      T* dXU = reinterpret_cast<T*>(p.dXU);
      T* dXQW = reinterpret_cast<T*>(p.dXQW);
#pragma unroll
      for (int c = 0; c < F; c += 8) {
        float q8[8];
        ld_row8(dO + o + c, q8);
#pragma unroll
        for (int e = 0; e < 8; ++e) q8[e] *= gi;
        st_row8(dXU + o + c, dxu + c);
        st_row8(dXQW + o + c, q8);
      }
    }
  }
  if (BWD) {
    // d summary_i += sum over the tile's tokens of segment i of ds_i(t) XU_t, through the X2
    // buffers as fp32 [128][64] scratch (column c of row i at c ^ (i % 32): conflict-free row
    // writes and column reads)
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem + L::OFF_X2);
    if (row_thread) {
      const float ds = r < nrows ? DG[r * GLD2 + seg_r] : 0.f;
#pragma unroll
      for (int c = 0; c < F; c += 2) {
        float2 v = make_float2(0.f, 0.f);
        if (r < nrows) v = H::unpack(*reinterpret_cast<const uint32_t*>(XU + (tok0 + r) * F + c));
        red[r * F + (c ^ (r & 31))] = ds * v.x;
        red[r * F + ((c + 1) ^ (r & 31))] = ds * v.y;
      }
    }
    __syncthreads();
    for (int e = tid; e < (seg_last - seg_first + 1) * F; e += NT) {
      const int sg = e / F, f = e % F;
      const int lo = max(0, sg * seg_tok - row0), hi = min(nrows, (sg + 1) * seg_tok - row0);
      float a = 0.f;
      for (int i = lo; i < hi; ++i) a += red[i * F + (f ^ (i & 31))];
      atomicAdd(p.dsum + (s * p.NS + seg_first + sg) * F + f, a);
    }
  }
  // a timed-out wait may leave products in flight: drain (bounded) before freeing memory
  if (tid == 0 && abort_sh) {
    mbar_wait(b_xq, 0, nullptr);
    for (int b = 0; b < 2; ++b)
      if (commits_sh[b] > 0) mbar_wait(smem_u32(&bars[BAR_P1 + b]), (uint32_t)((commits_sh[b] - 1) & 1), nullptr);
    if (commits_sh[2] > 0) mbar_wait(b_p2, (uint32_t)((commits_sh[2] - 1) & 1), nullptr);
    for (int b = 0; b < 2; ++b) {  // weight loads issued and never awaited
      if (last_w_sh[b] >= 0) mbar_wait(b_w1(last_w_sh[b]), (uint32_t)((last_w_sh[b] >> 1) & 1), nullptr);
      if (last_w_sh[2 + b] >= 0) mbar_wait(b_w2(last_w_sh[2 + b]), (uint32_t)((last_w_sh[2 + b] >> 1) & 1), nullptr);
    }
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base_sh, L::TMEM_COLS);
}

// dXK of every token: d summary_i / (tokens of segment i) for i >= 1, zero in segment 0.
// One thread writes 8 features of one token (a 16-byte store); mini-batch rows are indexed
// as (stream, mini-batch) pairs so the only runtime divisions are 32-bit.
template <typename T>
__global__ void memo_dxk_kernel(MemoMixParams p) {
  const int mbs = p.B * p.NH * p.NC;  // (stream, mini-batch) pairs
  const long long total = (long long)mbs * C * (F / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int mb = (int)(i / (C * (F / 8)));         // constant divisor
    const int f0 = 8 * (int)(i % (F / 8));
    const int s = mb / p.NC, n = mb - s * p.NC;
    const int seg = n / p.M;
    float v[8];
    if (seg > 0) {
      const float inv = 1.f / (float)((min((seg + 1) * p.M, p.NC) - seg * p.M) * C);
      const float4 a = *reinterpret_cast<const float4*>(p.dsum + ((long long)s * p.NS + seg) * F + f0);
      const float4 b = *reinterpret_cast<const float4*>(p.dsum + ((long long)s * p.NS + seg) * F + f0 + 4);
      v[0] = a.x * inv, v[1] = a.y * inv, v[2] = a.z * inv, v[3] = a.w * inv;
      v[4] = b.x * inv, v[5] = b.y * inv, v[6] = b.z * inv, v[7] = b.w * inv;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    using H = Half2<T>;
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.dXK) + i * 8) =
        make_uint4(H::pack(v[0], v[1]), H::pack(v[2], v[3]), H::pack(v[4], v[5]), H::pack(v[6], v[7]));
  }
}

}  // namespace memo

using namespace memo;

static bool aligned16(const void* q) { return ((uintptr_t)q & 15) == 0; }

// Scratch layout: W1^T and W2^T 16-bit copies, then summary (and d summary) fp32.
static size_t prep_bytes(long long B, long long NH, long long NS, long long FF) {
  return (size_t)(B * NH * NS) * 2 * F * FF * 2;
}

// prepped: the scratch already holds this call's W1^T / W2^T copies and summaries (the
// forward wrote them), so the prep kernel is skipped.
template <typename T, int FF>
static int run(MemoMixParams p, bool bwd, bool prepped, cudaStream_t stream, const char* who) {
  const long long streams = (long long)p.B * p.NH;
  constexpr int SMEM = Mix<FF>::SMEM;
  int rc = TTT_OK;
  if (!prepped) {
    memo_prep_kernel<T, FF><<<(unsigned)(streams * p.NS), 256, 0, stream>>>(p);
    rc = check_launch(who);
    if (rc) return rc;
  }
  Maps maps;
  const int dt = std::is_same<T, __nv_bfloat16>::value ? DT_BF16 : DT_F16;
  rc = make_tile_map(&maps.xq, p.XQ, dt, (unsigned long long)streams * p.NC * C, who, ROWS);
  if (!rc) rc = make_tile_map(&maps.w1, p.W1T, dt, (unsigned long long)streams * p.NS * FF, who, FF);
  if (!rc) rc = make_map_2d(&maps.w2, p.W2T, dt, FF, (unsigned long long)streams * p.NS * F, FF * 2, 64, 64, true, who);
  if (rc) return rc;
  rc = device_error_word(&p.err, who);
  if (rc) return rc;
  if (bwd) {
    cudaError_t e = cudaMemsetAsync(p.dsum, 0, (size_t)streams * p.NS * F * sizeof(float), stream);
    if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
  }
  const unsigned grid = (unsigned)(p.P == 1 ? streams * p.NS * p.TILES : streams * p.NG);
  if (FF == 64 && p.NS <= Mix2::NSC) {  // two CTAs per SM
    auto kern = bwd ? memo_mix2_kernel<T, true> : memo_mix2_kernel<T, false>;
    rc = prepare_smem(kern, Mix2::SMEM, who);
    if (rc) return rc;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", who, cudaGetErrorString(e));
    kern<<<grid, Mix2::NT, Mix2::SMEM, stream>>>(p, maps);
    if (!bwd) return check_launch(who);
    rc = check_launch(who);
    if (rc) return rc;
    memo_dxk_kernel<T><<<148 * 8, 256, 0, stream>>>(p);
    return check_launch(who);
  }
  if (!bwd) {
    rc = prepare_smem(memo_mix_kernel<T, false, FF>, SMEM, who);
    if (rc) return rc;
    memo_mix_kernel<T, false, FF><<<grid, Mix<FF>::NT, SMEM, stream>>>(p, maps);
  } else {
    rc = prepare_smem(memo_mix_kernel<T, true, FF>, SMEM, who);
    if (rc) return rc;
    memo_mix_kernel<T, true, FF><<<grid, Mix<FF>::NT, SMEM, stream>>>(p, maps);
    rc = check_launch(who);
    if (rc) return rc;
    memo_dxk_kernel<T><<<148 * 8, 256, 0, stream>>>(p);
  }
  return check_launch(who);
}

static int check_mix(int B, int NH, int NC, int CS, int F_, int FF_, int M, int dt, int dt_ln, const char* who) {
  TTT_REQUIRE(B > 0 && NH > 0 && NC > 0 && M > 0, TTT_ERR_SHAPE, "%s: B, NH, NC, memo_segment_size must be positive",
              who);
  TTT_REQUIRE(CS == C && F_ == F && (FF_ == 256 || FF_ == 64), TTT_ERR_UNSUPPORTED,
              "%s: implemented for CS = 16, F = 64, FF = 256 or 64 (got %d, %d, %d)", who, CS, F_, FF_);
  TTT_REQUIRE((NC + M - 1) / M <= NS_MAX, TTT_ERR_UNSUPPORTED, "%s: at most %d memo segments (got %d)", who, NS_MAX,
              (NC + M - 1) / M);
  TTT_REQUIRE(dt == DT_BF16 || dt == DT_F16, TTT_ERR_DTYPE, "%s: activations must be bf16 or f16", who);
  TTT_REQUIRE(valid_dtype(dt_ln), TTT_ERR_DTYPE, "%s: unknown LayerNorm dtype code", who);
  return TTT_OK;
}

static void fill_common(MemoMixParams& p, int B, int NH, int NC, int M) {
  p.B = B;
  p.NH = NH;
  p.NC = NC;
  p.M = M;
  p.NS = (NC + M - 1) / M;
  p.TILES = (M * C + ROWS - 1) / ROWS;
  // segments of at most 64 tokens share 128-row tiles, P consecutive segments each
  p.P = M * C <= ROWS / 2 ? ROWS / (M * C) : 1;
  p.NG = p.P == 1 ? p.NS : (p.NS + p.P - 1) / p.P;
}

}  // namespace ttt

using namespace ttt;

extern "C" size_t ttt_memo_mix_scratch_bytes(int B, int NH, int NC, int memo_segment_size, int FF) {
  if (B <= 0 || NH <= 0 || NC <= 0 || memo_segment_size <= 0 || FF <= 0) return 0;
  const long long NS = (NC + memo_segment_size - 1) / memo_segment_size;
  return prep_bytes(B, NH, NS, FF) + (size_t)B * NH * NS * memo::F * sizeof(float) * 2;
}

extern "C" int ttt_memo_mix_fwd(int B, int NH, int NC, int CS, int F, int FF, int memo_segment_size, const void* XQW,
                                const void* XQ, const void* XK, const void* XU, int dt, const float* W1_memo,
                                const float* b1_memo, const float* W2_memo, const float* b2_memo,
                                const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln, void* out,
                                void* scratch, size_t scratch_bytes, void* stream) {
  const char* who = "ttt_memo_mix_fwd";
  int rc = check_mix(B, NH, NC, CS, F, FF, memo_segment_size, dt, dt_ln, who);
  if (rc) return rc;
  TTT_REQUIRE(XQW && XQ && XK && XU && W1_memo && b1_memo && W2_memo && b2_memo && ttt_norm_weight && ttt_norm_bias &&
                  out && scratch,
              TTT_ERR_NULL, "%s: NULL pointer argument", who);
  TTT_REQUIRE(aligned16(XQW) && aligned16(XQ) && aligned16(XK) && aligned16(XU) && aligned16(scratch), TTT_ERR_ALIGN,
              "%s: activations and scratch must be 16-byte aligned", who);
  TTT_REQUIRE(aligned16(W1_memo) && aligned16(W2_memo) && aligned16(b1_memo) && aligned16(b2_memo), TTT_ERR_ALIGN,
              "%s: memo states must be 16-byte aligned", who);
  const size_t need = ttt_memo_mix_scratch_bytes(B, NH, NC, memo_segment_size, FF);
  TTT_REQUIRE(scratch_bytes >= need, TTT_ERR_SCRATCH, "%s: scratch has %zu bytes, needs %zu", who, scratch_bytes, need);
  TTT_REQUIRE(aligned16(out), TTT_ERR_ALIGN, "%s: out must be 16-byte aligned", who);
  MemoMixParams p = {};
  fill_common(p, B, NH, NC, memo_segment_size);
  p.XQW = XQW; p.XQ = XQ; p.XK = XK; p.XU = XU;
  p.W1_memo = W1_memo; p.b1_memo = b1_memo; p.W2_memo = W2_memo; p.b2_memo = b2_memo;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  p.out = out;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  const size_t half = prep_bytes(B, NH, p.NS, FF) / 2;
  p.W1T = sc;
  p.W2T = sc + half;
  p.summary = reinterpret_cast<float*>(sc + 2 * half);
  p.dsum = p.summary + (size_t)B * NH * p.NS * memo::F;
  if (FF == 64)
    return dt == DT_BF16 ? run<__nv_bfloat16, 64>(p, false, false, (cudaStream_t)stream, who)
                         : run<__half, 64>(p, false, false, (cudaStream_t)stream, who);
  return dt == DT_BF16 ? run<__nv_bfloat16, 256>(p, false, false, (cudaStream_t)stream, who)
                       : run<__half, 256>(p, false, false, (cudaStream_t)stream, who);
}

extern "C" int ttt_memo_mix_bwd(int B, int NH, int NC, int CS, int F, int FF, int memo_segment_size, const void* XQW,
                                const void* XQ, const void* XK, const void* XU, int dt, const float* W1_memo,
                                const float* b1_memo, const float* W2_memo, const float* b2_memo,
                                const void* ttt_norm_weight, const void* ttt_norm_bias, int dt_ln, const void* dOut,
                                void* dXQW, void* dXU, void* dXK, void* scratch, size_t scratch_bytes,
                                int scratch_prepped, void* stream) {
  const char* who = "ttt_memo_mix_bwd";
  int rc = check_mix(B, NH, NC, CS, F, FF, memo_segment_size, dt, dt_ln, who);
  if (rc) return rc;
  TTT_REQUIRE(XQW && XQ && XK && XU && W1_memo && b1_memo && W2_memo && b2_memo && ttt_norm_weight && ttt_norm_bias &&
                  dOut && dXQW && dXU && dXK && scratch,
              TTT_ERR_NULL, "%s: NULL pointer argument", who);
  TTT_REQUIRE(aligned16(XQW) && aligned16(XQ) && aligned16(XK) && aligned16(XU) && aligned16(scratch), TTT_ERR_ALIGN,
              "%s: activations and scratch must be 16-byte aligned", who);
  TTT_REQUIRE(aligned16(W1_memo) && aligned16(W2_memo) && aligned16(b1_memo) && aligned16(b2_memo), TTT_ERR_ALIGN,
              "%s: memo states must be 16-byte aligned", who);
  const size_t need = ttt_memo_mix_scratch_bytes(B, NH, NC, memo_segment_size, FF);
  TTT_REQUIRE(scratch_bytes >= need, TTT_ERR_SCRATCH, "%s: scratch has %zu bytes, needs %zu", who, scratch_bytes, need);
  MemoMixParams p = {};
  fill_common(p, B, NH, NC, memo_segment_size);
  p.XQW = XQW; p.XQ = XQ; p.XK = XK; p.XU = XU;
  p.W1_memo = W1_memo; p.b1_memo = b1_memo; p.W2_memo = W2_memo; p.b2_memo = b2_memo;
  p.ln_w = ttt_norm_weight; p.ln_b = ttt_norm_bias; p.dt_ln = dt_ln;
  TTT_REQUIRE(aligned16(dOut) && aligned16(dXQW) && aligned16(dXU) && aligned16(dXK), TTT_ERR_ALIGN,
              "%s: gradients must be 16-byte aligned", who);
  p.dOut = dOut; p.dXQW = dXQW; p.dXU = dXU; p.dXK = dXK;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  const size_t half = prep_bytes(B, NH, p.NS, FF) / 2;
  p.W1T = sc;
  p.W2T = sc + half;
  p.summary = reinterpret_cast<float*>(sc + 2 * half);
  p.dsum = p.summary + (size_t)B * NH * p.NS * memo::F;
  const bool prepped = scratch_prepped != 0;
  if (FF == 64)
    return dt == DT_BF16 ? run<__nv_bfloat16, 64>(p, true, prepped, (cudaStream_t)stream, who)
                         : run<__half, 64>(p, true, prepped, (cudaStream_t)stream, who);
  return dt == DT_BF16 ? run<__nv_bfloat16, 256>(p, true, prepped, (cudaStream_t)stream, who)
                       : run<__half, 256>(p, true, prepped, (cudaStream_t)stream, who);
}
