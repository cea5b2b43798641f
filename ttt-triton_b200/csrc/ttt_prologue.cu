// Input prologue of the TTT layer (TTTBase.process_input, ttt_layer.py:261-330, with no
// text prefix, no multi-scene interleave and no tensor parallelism), everything after the
// projections:
//   XQ, XK, XU = rope(l2_normalize(P_q)), rope(l2_normalize(P_k)), rope(l2_normalize(P_u))
//   XV         = gamma_h * (Y - mean Y) / (std Y + 1e-8) + beta_h + XK,  Y = P_v - XK
//   eta[b, h, n, i, j] = eta_scale * sigmoid(P_gate[b, n * CS + j, h])   for every row i
// with P = hidden @ [wq | wk | wv | wu | lr_w]^T + bias (one library GEMM the caller runs),
// std the unbiased standard deviation over the head dimension and eta_scale =
// ttt_base_lr / (head_dim * mini_batch_size). The outputs are written in the scan's
// [B, NH, NC, CS, F] / [B, NH, NC, CS, CS] layout, so the projection rows are read once
// and each output is written once.
//
// A warp owns one mini-batch of one head at a time and works on 4 of its tokens at once: 8
// lanes per token, each holding F / 8 contiguous head elements (whole rotary pairs, one
// 16-byte access for F = 64 in 16 bits), so the L2 norms and LayerNorm moments are 3-step
// shuffle reductions. Owning the mini-batch lets the warp write its [CS][CS] eta block (and
// read the d_eta block) as contiguous vectors. The grid is [mini-batch chunks, heads]: a
// CTA works on one head, so the backward sums the LayerNorm parameter and projection bias
// gradients in registers and shared memory before one atomic per element per CTA.
#include <type_traits>

#include "capi_common.cuh"
#include "common.cuh"

namespace ttt {
namespace prologue {

constexpr int kWarps = 8;
constexpr int kMaxCS = 128;  // per-warp gate buffer in shared memory

// Lanes per token (G), head elements per lane (V) and tokens per warp pass (32 / G): 8
// elements (16 bytes in 16 bits) per lane from F = 64 up, 8 lanes per token below.
template <int F>
struct Shape {
  static constexpr int G = F >= 64 ? F / 8 : 8;
  static constexpr int V = F / G;
  static constexpr int TPP = 32 / G;
};
constexpr float kNormEps = 1e-12f;        // torch.nn.functional.normalize default (ttt_layer.py:276-278)

struct Params {
  int B, L, NH, CS;
  long long ld;        // row stride of P / dP in elements
  const void* P;       // [B * L][ld]
  const float* ln_w;   // [NH][F]
  const float* ln_b;
  const float* cosv;   // [L][F / 2]
  const float* sinv;
  float eta_scale;
  void *XQ, *XK, *XV, *XU, *eta;             // forward outputs
  const void *dXQ, *dXK, *dXV, *dXU, *deta;  // backward inputs (NULL = zero)
  void* dP;                                  // [B * L][ld]
  float *dln_w, *dln_b;                      // [NH][F], accumulated
  float* dbias;                              // [ld] column sums of dP, accumulated (optional)
};

template <typename T>
__device__ __forceinline__ float to_f(T x) {
  if constexpr (std::is_same<T, float>::value) return x;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(x);
  else return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x) {
  if constexpr (std::is_same<T, float>::value) return x;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
  else return __float2half_rn(x);
}

// V contiguous elements of T moved in chunks of at most 16 bytes (one vector access each).
template <typename T, int V>
struct VecIO {
  static constexpr int kBytes = (int)sizeof(T) * V;
  static constexpr int kChunk = kBytes < 16 ? kBytes : 16;
  static constexpr int kEpc = kChunk / (int)sizeof(T);
  struct alignas(kChunk) Chunk {
    T v[kEpc];
  };
  __device__ __forceinline__ static void load(const T* p, float (&x)[V]) {
#pragma unroll
    for (int c = 0; c < V / kEpc; ++c) {
      const Chunk ch = reinterpret_cast<const Chunk*>(p)[c];
#pragma unroll
      for (int e = 0; e < kEpc; ++e) x[c * kEpc + e] = to_f(ch.v[e]);
    }
  }
  __device__ __forceinline__ static void store(T* p, const float (&x)[V]) {
#pragma unroll
    for (int c = 0; c < V / kEpc; ++c) {
      Chunk ch;
#pragma unroll
      for (int e = 0; e < kEpc; ++e) ch.v[e] = from_f<T>(x[c * kEpc + e]);
      reinterpret_cast<Chunk*>(p)[c] = ch;
    }
  }
};

template <typename T, int V>
__device__ __forceinline__ void load_or_zero(const void* base, long long off, bool on, float (&x)[V]) {
  if (base && on) {
    VecIO<T, V>::load(static_cast<const T*>(base) + off, x);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) x[i] = 0.f;
  }
}

// Sum over the G lanes of a token group.
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int V>
__device__ __forceinline__ float dot(const float (&x)[V], const float (&y)[V]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) s = fmaf(x[i], y[i], s);
  return s;
}

// Rotation of the pairs (x[2i], x[2i+1]) by the angle with cosine c[i], sine s[i]
// (utils.py:97-123: the pair is a complex number multiplied by freqs_cis); sign -1
// applies the inverse rotation (the transposed Jacobian in the backward).
template <int V>
__device__ __forceinline__ void rotate(float (&x)[V], const float (&c)[V / 2], const float (&s)[V / 2], float sign) {
#pragma unroll
  for (int i = 0; i < V / 2; ++i) {
    const float a = x[2 * i], b = x[2 * i + 1], sn = sign * s[i];
    x[2 * i] = a * c[i] - b * sn;
    x[2 * i + 1] = a * sn + b * c[i];
  }
}

template <int F, int V>
__device__ __forceinline__ void load_rope(const Params& p, int l, int r, bool on, float (&c)[V / 2],
                                          float (&s)[V / 2]) {
  if (on) {
    VecIO<float, V / 2>::load(p.cosv + (long long)l * (F / 2) + r * (V / 2), c);
    VecIO<float, V / 2>::load(p.sinv + (long long)l * (F / 2) + r * (V / 2), s);
  } else {
#pragma unroll
    for (int i = 0; i < V / 2; ++i) c[i] = 1.f, s[i] = 0.f;
  }
}

// Grid: x over mini-batches (b, n), y = head. Warp w of CTA x takes mini-batches
// x * kWarps + w, + gridDim.x * kWarps, ...; within one, token group g takes tokens
// g, g + 32 / G, ... of the mini-batch.
template <int F, typename T>
__global__ void __launch_bounds__(kWarps * 32, 3) prologue_fwd_kernel(Params p) {
  constexpr int G = Shape<F>::G, V = Shape<F>::V, TPP = Shape<F>::TPP;
  using IO = VecIO<T, V>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane / G, r = lane % G;
  const int h = blockIdx.y, W = p.NH * F, NC = p.L / p.CS, CS = p.CS;
  const int n_mb = p.B * NC;
  const T* P = static_cast<const T*>(p.P);
  __shared__ float gate_sh[kWarps][kMaxCS];

  float gam[V], bet[V];  // this lane's LayerNorm weight and bias columns
  VecIO<float, V>::load(p.ln_w + h * F + r * V, gam);
  VecIO<float, V>::load(p.ln_b + h * F + r * V, bet);

  for (int m = blockIdx.x * kWarps + warp; m < n_mb; m += gridDim.x * kWarps) {
    const int b = m / NC, n = m - b * NC;
    for (int t0 = 0; t0 < CS; t0 += TPP) {
      const int t = t0 + grp;
      const bool on = t < CS;
      const int l = n * CS + t;
      const long long row = (long long)b * p.L + l;
      const long long pin = row * p.ld + h * F + r * V;
      float q[V], k[V], v[V], w[V], c[V / 2], s[V / 2];
      load_or_zero<T, V>(P, pin, on, q);
      load_or_zero<T, V>(P, pin + W, on, k);
      load_or_zero<T, V>(P, pin + 2 * W, on, v);
      load_or_zero<T, V>(P, pin + 3 * W, on, w);
      load_rope<F, V>(p, l, r, on, c, s);
      const float gate = on && r == 0 ? to_f(P[row * p.ld + 4 * W + h]) : 0.f;

      const float iq = 1.f / fmaxf(sqrtf(group_sum<G>(dot(q, q))), kNormEps);
      const float ik = 1.f / fmaxf(sqrtf(group_sum<G>(dot(k, k))), kNormEps);
      const float iu = 1.f / fmaxf(sqrtf(group_sum<G>(dot(w, w))), kNormEps);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        q[i] *= iq;
        k[i] *= ik;
        w[i] *= iu;
      }
      rotate<V>(q, c, s, 1.f);
      rotate<V>(k, c, s, 1.f);
      rotate<V>(w, c, s, 1.f);
      // LayerNorm reconstruction target on Y = XV - XK (ttt_layer.py:227-244).
      float ysum = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[i] -= k[i];
        ysum += v[i];
      }
      const float mu = group_sum<G>(ysum) * (1.f / F);
      float nsq = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[i] -= mu;
        nsq = fmaf(v[i], v[i], nsq);
      }
      const float rs = 1.f / (sqrtf(group_sum<G>(nsq) * (1.f / (F - 1))) + kLnEps);
#pragma unroll
      for (int i = 0; i < V; ++i) v[i] = fmaf(gam[i], v[i] * rs, bet[i]) + k[i];

      if (on) {
        const long long o = (((long long)b * p.NH + h) * p.L + l) * F + r * V;
        IO::store(static_cast<T*>(p.XQ) + o, q);
        IO::store(static_cast<T*>(p.XK) + o, k);
        IO::store(static_cast<T*>(p.XV) + o, v);
        IO::store(static_cast<T*>(p.XU) + o, w);
        if (r == 0) gate_sh[warp][t] = p.eta_scale / (1.f + __expf(-gate));
      }
    }
    __syncwarp();
    // eta block [CS][CS] of (b, h, n): every row i holds the mini-batch's gates.
    T* eta = static_cast<T*>(p.eta) + (((long long)b * p.NH + h) * NC + n) * CS * CS;
    constexpr int EV = 16 / (int)sizeof(T);
    if (CS % EV == 0) {
      using EIO = VecIO<T, EV>;
      for (int e = lane * EV; e < CS * CS; e += 32 * EV) {
        const int j0 = e % CS;
        float x[EV];
#pragma unroll
        for (int u = 0; u < EV; ++u) x[u] = gate_sh[warp][j0 + u];
        EIO::store(eta + e, x);
      }
    } else {
      for (int e = lane; e < CS * CS; e += 32) eta[e] = from_f<T>(gate_sh[warp][e % CS]);
    }
    __syncwarp();
  }
}

template <int F, typename T>
__global__ void __launch_bounds__(kWarps * 32, 2) prologue_bwd_kernel(Params p) {
  constexpr int G = Shape<F>::G, V = Shape<F>::V, TPP = Shape<F>::TPP;
  constexpr int C = V < 4 ? V : 4;  // floats per shared-memory access of the bias partials
  using IO = VecIO<T, V>;
  using SIO = VecIO<float, C>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane / G, r = lane % G;
  const int h = blockIdx.y, W = p.NH * F, NC = p.L / p.CS, CS = p.CS;
  const int ncols = 4 * W + p.NH;
  const int n_mb = p.B * NC;
  const T* P = static_cast<const T*>(p.P);
  T* dP = static_cast<T*>(p.dP);
  __shared__ float de_sh[kWarps][kMaxCS];

  // Per-lane partial sums over this warp's tokens: LayerNorm weight / bias gradients in
  // registers, the column sums of dP (projection bias gradients) of q, k, v, u in
  // lane-private shared-memory slots ([warp][projection][chunk][lane], conflict-free).
  __shared__ __align__(16) float bacc[kWarps][4][V / C][32][C];
  float a_g[V], a_b[V];
  float a_gate = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) a_g[i] = a_b[i] = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int ch = 0; ch < V / C; ++ch)
#pragma unroll
      for (int e = 0; e < C; ++e) bacc[warp][c][ch][lane][e] = 0.f;
  auto add_bias = [&](int c, const float (&x)[V]) {
#pragma unroll
    for (int ch = 0; ch < V / C; ++ch) {
      float cur[C];
      SIO::load(&bacc[warp][c][ch][lane][0], cur);
#pragma unroll
      for (int e = 0; e < C; ++e) cur[e] += x[ch * C + e];
      SIO::store(&bacc[warp][c][ch][lane][0], cur);
    }
  };
  float gam[V];  // this lane's LayerNorm weight columns
  VecIO<float, V>::load(p.ln_w + h * F + r * V, gam);

  for (int m = blockIdx.x * kWarps + warp; m < n_mb; m += gridDim.x * kWarps) {
    const int b = m / NC, n = m - b * NC;
    // Column sums of this mini-batch's d_eta block: eta column j is one gate in every row.
    if (p.deta) {
      const T* deta = static_cast<const T*>(p.deta) + (((long long)b * p.NH + h) * NC + n) * CS * CS;
      for (int j = lane; j < CS; j += 32) {
        float acc = 0.f;
        for (int i = 0; i < CS; ++i) acc += to_f(deta[i * CS + j]);
        de_sh[warp][j] = acc;
      }
    }
    __syncwarp();
    for (int t0 = 0; t0 < CS; t0 += TPP) {
      const int t = t0 + grp;
      const bool on = t < CS;
      const int l = n * CS + t;
      const long long row = (long long)b * p.L + l;
      const long long pin = row * p.ld + h * F + r * V;
      const long long o = (((long long)b * p.NH + h) * p.L + l) * F + r * V;
      float q[V], k[V], v[V], w[V], c[V / 2], s[V / 2];
      float dv[V], dk[V], dq[V], du[V];
      load_or_zero<T, V>(P, pin, on, q);
      load_or_zero<T, V>(P, pin + W, on, k);
      load_or_zero<T, V>(P, pin + 2 * W, on, v);
      load_or_zero<T, V>(P, pin + 3 * W, on, w);
      load_or_zero<T, V>(p.dXV, o, on, dv);
      load_or_zero<T, V>(p.dXK, o, on, dk);
      load_or_zero<T, V>(p.dXQ, o, on, dq);
      load_or_zero<T, V>(p.dXU, o, on, du);
      load_rope<F, V>(p, l, r, on, c, s);
      const float gate = on && r == 0 ? to_f(P[row * p.ld + 4 * W + h]) : 0.f;

      const float nq = sqrtf(group_sum<G>(dot(q, q))), nk = sqrtf(group_sum<G>(dot(k, k))),
                  nu = sqrtf(group_sum<G>(dot(w, w)));
      const float iq = 1.f / fmaxf(nq, kNormEps), ik = 1.f / fmaxf(nk, kNormEps), iu = 1.f / fmaxf(nu, kNormEps);
      float kr[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        q[i] *= iq;  // unit vectors (before rotation)
        k[i] *= ik;
        w[i] *= iu;
        kr[i] = k[i];
      }
      rotate<V>(kr, c, s, 1.f);
      float ysum = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[i] -= kr[i];
        ysum += v[i];
      }
      const float mu = group_sum<G>(ysum) * (1.f / F);
      float nsq = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[i] -= mu;  // n = Y - mean
        nsq = fmaf(v[i], v[i], nsq);
      }
      const float sigma = sqrtf(group_sum<G>(nsq) * (1.f / (F - 1)));
      const float rs = 1.f / (sigma + kLnEps);

      // XV = gamma * n * rs + beta + XK_rot: dXV reaches n through the LayerNorm and XK_rot
      // directly; the LayerNorm input Y = P_v - XK_rot sends -dY back to XK_rot.
      float dyh_sum = 0.f, dyh_n = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        a_g[i] = fmaf(dv[i], v[i] * rs, a_g[i]);
        a_b[i] += dv[i];
        const float dyh = gam[i] * dv[i];
        dyh_sum += dyh;
        dyh_n = fmaf(dyh, v[i], dyh_n);
      }
      dyh_sum = group_sum<G>(dyh_sum);
      dyh_n = group_sum<G>(dyh_n);
      // dY = (dyh - mean dyh) * rs - n * <dyh, n> * rs^2 / ((F - 1) sigma)
      const float cn = sigma > 0.f ? dyh_n * rs * rs / ((F - 1) * sigma) : 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float dy = (gam[i] * dv[i] - dyh_sum * (1.f / F)) * rs - v[i] * cn;
        dk[i] += dv[i] - dy;
        dv[i] = dy;  // d P_v
      }
      rotate<V>(dq, c, s, -1.f);
      rotate<V>(dk, c, s, -1.f);
      rotate<V>(du, c, s, -1.f);
      // l2-normalise backward: (d - xhat <xhat, d>) / |x|, or d / eps below the clamp. The
      // shuffles run on every lane (the clamp differs between token groups of one warp).
      const float sq = group_sum<G>(dot(q, dq)), sk = group_sum<G>(dot(k, dk)), su = group_sum<G>(dot(w, du));
      const float pq = nq > kNormEps ? sq : 0.f;
      const float pk = nk > kNormEps ? sk : 0.f;
      const float pu = nu > kNormEps ? su : 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        dq[i] = (dq[i] - q[i] * pq) * iq;
        dk[i] = (dk[i] - k[i] * pk) * ik;
        du[i] = (du[i] - w[i] * pu) * iu;
      }
      add_bias(0, dq);
      add_bias(1, dk);
      add_bias(2, dv);
      add_bias(3, du);
      if (on) {
        const long long dout = row * p.ld + h * F + r * V;
        IO::store(dP + dout, dq);
        IO::store(dP + dout + W, dk);
        IO::store(dP + dout + 2 * W, dv);
        IO::store(dP + dout + 3 * W, du);
        if (r == 0) {
          // Gate: eta column t is eta_scale * sigmoid(gate) in every row of the block.
          const float sg = 1.f / (1.f + __expf(-gate));
          const float dgate = p.deta ? p.eta_scale * sg * (1.f - sg) * de_sh[warp][t] : 0.f;
          dP[row * p.ld + 4 * W + h] = from_f<T>(dgate);
          a_gate += dgate;
        }
        // The padding columns past the gates are zeroed (head 0's CTAs), so the caller's
        // GEMMs may run over the full aligned row.
        if (h == 0 && ncols + r < p.ld) dP[row * p.ld + ncols + r] = from_f<T>(0.f);
      }
    }
    __syncwarp();
  }

  // Reduce the partial sums: token groups (shuffles) -> warps (shared memory) -> one
  // atomic per element per CTA.
  __shared__ float red[kWarps][2][F];
  __shared__ float red_gate[kWarps];
  auto fold = [&](const float (&acc)[V], int a) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float x = acc[i];
#pragma unroll
      for (int o = G; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (grp == 0) red[warp][a][r * V + i] = x;
    }
  };
  fold(a_g, 0);
  fold(a_b, 1);
#pragma unroll
  for (int o = G; o < 32; o <<= 1) a_gate += __shfl_xor_sync(0xffffffffu, a_gate, o);
  if (lane == 0) red_gate[warp] = a_gate;
  __syncthreads();
  for (int e = threadIdx.x; e < 2 * F; e += blockDim.x) {
    const int a = e / F, col = e % F;
    float t = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < kWarps; ++w2) t += red[w2][a][col];
    atomicAdd((a ? p.dln_b : p.dln_w) + h * F + col, t);
  }
  if (p.dbias) {
    // Column col = r * V + ch * C + e of projection c sums the slots of lanes (g, r).
    for (int e = threadIdx.x; e < 4 * F; e += blockDim.x) {
      const int c = e / F, col = e % F, rr = col / V, ch = (col % V) / C, el = col % C;
      float t = 0.f;
      for (int w2 = 0; w2 < kWarps; ++w2)
#pragma unroll
        for (int g2 = 0; g2 < TPP; ++g2) t += bacc[w2][c][ch][g2 * G + rr][el];
      atomicAdd(p.dbias + c * W + h * F + col, t);
    }
  }
  if (threadIdx.x == 0 && p.dbias) {
    float t = 0.f;
    for (int w2 = 0; w2 < kWarps; ++w2) t += red_gate[w2];
    atomicAdd(p.dbias + 4 * W + h, t);
  }
}

// ------------------------------------------------------------------------------ host
// CTAs along x per head: one wave of resident CTAs over all heads (occupancy API), at most
// one mini-batch per warp.
template <typename K>
static int grid_x(K kernel, long long n_mb, int NH) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWarps * 32, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  long long want = ((long long)sms * per_sm + NH - 1) / NH;
  long long most = (n_mb + kWarps - 1) / kWarps;
  long long x = want < most ? want : most;
  if (x < 1) x = 1;
  if (x > 0x7fffffffLL) x = 0x7fffffffLL;
  return (int)x;
}

template <bool BWD, int F, typename T>
static void launch_t(const Params& p, cudaStream_t st) {
  const long long n_mb = (long long)p.B * (p.L / p.CS);
  if (BWD)
    prologue_bwd_kernel<F, T><<<dim3(grid_x(prologue_bwd_kernel<F, T>, n_mb, p.NH), p.NH), kWarps * 32, 0, st>>>(p);
  else
    prologue_fwd_kernel<F, T><<<dim3(grid_x(prologue_fwd_kernel<F, T>, n_mb, p.NH), p.NH), kWarps * 32, 0, st>>>(p);
}

template <bool BWD, int F>
static void launch_f(const Params& p, int dt, cudaStream_t st) {
  if (dt == DT_BF16)
    launch_t<BWD, F, __nv_bfloat16>(p, st);
  else if (dt == DT_F16)
    launch_t<BWD, F, __half>(p, st);
  else
    launch_t<BWD, F, float>(p, st);
}

template <bool BWD>
static void launch(const Params& p, int F, int dt, cudaStream_t st) {
  switch (F) {
    case 16: launch_f<BWD, 16>(p, dt, st); break;
    case 32: launch_f<BWD, 32>(p, dt, st); break;
    case 64: launch_f<BWD, 64>(p, dt, st); break;
    default: launch_f<BWD, 128>(p, dt, st); break;
  }
}

static bool aligned(const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

static int check_common(const char* who, int B, int L, int NH, int F, int CS, const void* P, int dt,
                        long long ld, const float* ln_w, const float* ln_b, const float* cosv, const float* sinv) {
  TTT_REQUIRE(P && ln_w && ln_b && cosv && sinv, TTT_ERR_NULL, "%s: NULL pointer argument", who);
  TTT_REQUIRE(B >= 1 && L >= 1 && NH >= 1 && NH <= 65535, TTT_ERR_SHAPE, "%s: bad sizes B=%d L=%d NH=%d", who, B, L,
              NH);
  TTT_REQUIRE((long long)B * L < (1LL << 31), TTT_ERR_SHAPE, "%s: B * L = %lld tokens is too many", who,
              (long long)B * L);
  TTT_REQUIRE(F == 16 || F == 32 || F == 64 || F == 128, TTT_ERR_SHAPE,
              "%s: head_dim F=%d not supported (16, 32, 64 or 128)", who, F);
  TTT_REQUIRE(CS >= 1 && L % CS == 0, TTT_ERR_SHAPE, "%s: seq len %d is not a multiple of mini_batch_size %d", who, L,
              CS);
  TTT_REQUIRE(CS <= kMaxCS, TTT_ERR_SHAPE, "%s: mini_batch_size %d above %d", who, CS, kMaxCS);
  TTT_REQUIRE(valid_dtype(dt), TTT_ERR_DTYPE, "%s: bad dtype code %d", who, dt);
  const long long W = (long long)NH * F;
  TTT_REQUIRE(ld >= 4 * W + NH && ld % 8 == 0, TTT_ERR_SHAPE,
              "%s: projection row stride %lld must be a multiple of 8 and at least 4 * NH * F + NH = %lld", who, ld,
              4 * W + NH);
  TTT_REQUIRE(aligned(P, 16), TTT_ERR_ALIGN, "%s: projection rows must be 16-byte aligned", who);
  TTT_REQUIRE(aligned(ln_w, 16) && aligned(ln_b, 16), TTT_ERR_ALIGN,
              "%s: LayerNorm parameters must be 16-byte aligned", who);
  return TTT_OK;
}

}  // namespace prologue
}  // namespace ttt

using namespace ttt;

extern "C" int ttt_prologue_fwd(int B, int L, int NH, int F, int CS, const void* proj, int dt, long long ld_proj,
                                const float* ln_w, const float* ln_b, const float* rope_cos, const float* rope_sin,
                                float eta_scale, void* XQ, void* XK, void* XV, void* XU, void* eta, void* stream) {
  const char* who = "ttt_prologue_fwd";
  int rc = prologue::check_common(who, B, L, NH, F, CS, proj, dt, ld_proj, ln_w, ln_b, rope_cos, rope_sin);
  if (rc) return rc;
  TTT_REQUIRE(XQ && XK && XV && XU && eta, TTT_ERR_NULL, "%s: NULL output pointer", who);
  const void* outs[] = {XQ, XK, XV, XU};
  for (const void* o : outs)
    TTT_REQUIRE(prologue::aligned(o, 16), TTT_ERR_ALIGN, "%s: outputs must be 16-byte aligned", who);
  TTT_REQUIRE(prologue::aligned(eta, 16), TTT_ERR_ALIGN, "%s: eta must be 16-byte aligned", who);
  TTT_REQUIRE(prologue::aligned(rope_cos, 16) && prologue::aligned(rope_sin, 16), TTT_ERR_ALIGN,
              "%s: rotary tables must be 16-byte aligned", who);
  prologue::Params p{};
  p.B = B, p.L = L, p.NH = NH, p.CS = CS, p.ld = ld_proj, p.P = proj;
  p.ln_w = ln_w, p.ln_b = ln_b, p.cosv = rope_cos, p.sinv = rope_sin, p.eta_scale = eta_scale;
  p.XQ = XQ, p.XK = XK, p.XV = XV, p.XU = XU, p.eta = eta;
  prologue::launch<false>(p, F, dt, static_cast<cudaStream_t>(stream));
  return check_launch(who);
}

extern "C" int ttt_prologue_bwd(int B, int L, int NH, int F, int CS, const void* proj, int dt, long long ld_proj,
                                const float* ln_w, const float* ln_b, const float* rope_cos, const float* rope_sin,
                                float eta_scale, const void* dXQ, const void* dXK, const void* dXV, const void* dXU,
                                const void* deta, void* dproj, float* dln_w, float* dln_b, float* dbias,
                                void* stream) {
  const char* who = "ttt_prologue_bwd";
  int rc = prologue::check_common(who, B, L, NH, F, CS, proj, dt, ld_proj, ln_w, ln_b, rope_cos, rope_sin);
  if (rc) return rc;
  TTT_REQUIRE(dproj && dln_w && dln_b, TTT_ERR_NULL, "%s: NULL output pointer", who);
  const void* ins[] = {dXQ, dXK, dXV, dXU, dproj};
  for (const void* o : ins)
    TTT_REQUIRE(!o || prologue::aligned(o, 16), TTT_ERR_ALIGN, "%s: gradients must be 16-byte aligned", who);
  TTT_REQUIRE(!deta || prologue::aligned(deta, dt == DT_F32 ? 4 : 2), TTT_ERR_ALIGN, "%s: d_eta misaligned", who);
  TTT_REQUIRE(prologue::aligned(rope_cos, 16) && prologue::aligned(rope_sin, 16), TTT_ERR_ALIGN,
              "%s: rotary tables must be 16-byte aligned", who);
  prologue::Params p{};
  p.B = B, p.L = L, p.NH = NH, p.CS = CS, p.ld = ld_proj, p.P = proj;
  p.ln_w = ln_w, p.ln_b = ln_b, p.cosv = rope_cos, p.sinv = rope_sin, p.eta_scale = eta_scale;
  p.dXQ = dXQ, p.dXK = dXK, p.dXV = dXV, p.dXU = dXU, p.deta = deta;
  p.dP = dproj, p.dln_w = dln_w, p.dln_b = dln_b, p.dbias = dbias;
  prologue::launch<true>(p, F, dt, static_cast<cudaStream_t>(stream));
  return check_launch(who);
}
