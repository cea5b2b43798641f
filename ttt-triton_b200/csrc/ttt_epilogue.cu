// Output epilogue of the TTT layer (TTTBase.forward, ttt_layer.py:345-350): the scan output
// XQW_batch is permuted from the kernel layout [B, NH, NC, CS, F] to [B, L, NH * F]
// (TTTMLP.ttt :563-564, TTTLinear.ttt :405,420), layer-normalised over the width by
// post_norm (nn.LayerNorm(width, eps=1e-6), :77) and projected by wo. The reference
// materialises the permuted copy and the normalised copy; here ONE kernel reads the scan
// output in its own layout and writes the normalised rows the wo GEMM (a library call)
// consumes, so the permute costs nothing and one full round trip of the activations is
// saved. The backward kernel reads the gradient of the normalised rows (d out @ wo, library
// GEMM) and writes d XQW straight back into the scan layout, summing the LayerNorm
// parameter gradients on the way.
//
// A warp works on TPW tokens at once (all their loads issued before any arithmetic, so
// enough bytes are in flight to cover DRAM latency): the W = NH * F values of token (b, l)
// are NH head segments of F contiguous elements in the scan layout; lane i holds 16-byte
// chunks i, i + 32, ... of each (a chunk never straddles two heads because F is a multiple
// of the chunk), so the mean and variance are warp-shuffle reductions and every access is a
// 16-byte vector. The backward also sums d out over tokens: the wo bias gradient.
#include <type_traits>

#include "capi_common.cuh"
#include "common.cuh"

namespace ttt {
namespace epilogue {

constexpr int kWarps = 8;
constexpr int kMaxW = 1024;  // widest row (16-bit; 512 in fp32): four chunks per lane

struct Params {
  int B, NH, L, F;
  const void* X;       // [B, NH, L, F]
  const float* ln_w;   // [W]
  const float* ln_b;
  float eps;
  void* Y;             // [B * L, W]
  const void* dY;      // [B * L, W]
  void* dX;            // [B, NH, L, F]
  float *dln_w, *dln_b;  // [W], accumulated
  const void* dOut;    // [B * L, W] gradient of the wo output (optional)
  float* dbias;        // [W] column sums of dOut, accumulated (with dOut)
};

// Tokens per warp iteration: about 2 KB of loads per warp in flight.
template <int NCL>
struct Tpw {
  static constexpr int value = NCL >= 4 ? 1 : 4 / NCL;
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

template <typename T>
struct Chunk {
  static constexpr int V = 16 / (int)sizeof(T);
  struct alignas(16) Raw {
    T v[V];
  };
  __device__ __forceinline__ static void load(const T* p, float (&x)[V]) {
    const Raw r = *reinterpret_cast<const Raw*>(p);
#pragma unroll
    for (int e = 0; e < V; ++e) x[e] = to_f(r.v[e]);
  }
  __device__ __forceinline__ static void store(T* p, const float (&x)[V]) {
    Raw r;
#pragma unroll
    for (int e = 0; e < V; ++e) r.v[e] = from_f<T>(x[e]);
    *reinterpret_cast<Raw*>(p) = r;
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Columns cV .. cV + V - 1 of an fp32 [W] vector (16-byte loads), or zeros when !on.
template <int V>
__device__ __forceinline__ void load_cols(const float* v, int c, bool on, float (&x)[V]) {
#pragma unroll
  for (int q = 0; q < V / 4; ++q) {
    const float4 t = on ? __ldg(reinterpret_cast<const float4*>(v + c * V) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    x[4 * q] = t.x, x[4 * q + 1] = t.y, x[4 * q + 2] = t.z, x[4 * q + 3] = t.w;
  }
}

// Scan-layout offset of chunk c (V elements) relative to the token's row in head 0:
// head h = cV / F sits h * L * F elements further. Computed once per lane.
__device__ __forceinline__ long long chunk_off(const Params& p, int c, int V) {
  const int e = c * V, h = e / p.F;
  return (long long)h * p.L * p.F + (e - h * p.F);
}
// Scan-layout offset of token tok = b * L + l in head 0 (one 32-bit division).
__device__ __forceinline__ long long token_base(const Params& p, int tok) {
  const int b = tok / p.L, l = tok - b * p.L;
  return ((long long)b * p.NH * p.L + l) * p.F;
}

template <typename T, int NCL>
__global__ void __launch_bounds__(kWarps * 32) post_norm_fwd_kernel(Params p) {
  constexpr int V = Chunk<T>::V, TPW = Tpw<NCL>::value;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = p.NH * p.F, nch = W / V;
  const int tokens = p.B * p.L;
  const float inv_w = 1.f / W;
  long long coff[NCL];
  float gam[NCL][V], bet[NCL][V];  // this lane's LayerNorm columns, loaded once
#pragma unroll
  for (int i = 0; i < NCL; ++i) {
    const int c = lane + 32 * i;
    coff[i] = chunk_off(p, c, V);
    load_cols(p.ln_w, c, c < nch, gam[i]);
    load_cols(p.ln_b, c, c < nch, bet[i]);
  }
  const int stride = gridDim.x * kWarps * TPW;
  for (int tok0 = (blockIdx.x * kWarps + warp) * TPW; tok0 < tokens; tok0 += stride) {
    float x[TPW][NCL][V];
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tok = tok0 + u;
      const long long base = token_base(p, tok);
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const int c = lane + 32 * i;
        if (c < nch && tok < tokens) {
          Chunk<T>::load(static_cast<const T*>(p.X) + base + coff[i], x[u][i]);
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) x[u][i][e] = 0.f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tok = tok0 + u;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NCL; ++i)
#pragma unroll
        for (int e = 0; e < V; ++e) s += x[u][i][e];
      const float mu = warp_sum(s) * inv_w;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const bool on = lane + 32 * i < nch;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          x[u][i][e] = on ? x[u][i][e] - mu : 0.f;
          q = fmaf(x[u][i][e], x[u][i][e], q);
        }
      }
      const float rstd = rsqrtf(warp_sum(q) * inv_w + p.eps);  // biased variance (nn.LayerNorm)
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const int c = lane + 32 * i;
        if (c < nch && tok < tokens) {
          float y[V];
#pragma unroll
          for (int e = 0; e < V; ++e)
            y[e] = fmaf(x[u][i][e] * rstd, gam[i][e], bet[i][e]);
          Chunk<T>::store(static_cast<T*>(p.Y) + (long long)tok * W + c * V, y);
        }
      }
    }
  }
}

template <typename T, int NCL>
__global__ void __launch_bounds__(kWarps * 32, NCL == 1 ? 2 : 1) post_norm_bwd_kernel(Params p) {
  constexpr int V = Chunk<T>::V, TPW = Tpw<NCL>::value;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = p.NH * p.F, nch = W / V;
  const int tokens = p.B * p.L;
  const float inv_w = 1.f / W;
  long long coff[NCL];
  float gam[NCL][V];  // this lane's LayerNorm weight columns (zero past the row), loaded once
#pragma unroll
  for (int i = 0; i < NCL; ++i) {
    const int c = lane + 32 * i;
    coff[i] = chunk_off(p, c, V);
    load_cols(p.ln_w, c, c < nch, gam[i]);
  }
  // this lane's columns: sums of dy * xhat, of dy, and of d out
  float ag[NCL][V], ab[NCL][V], ao[NCL][V];
#pragma unroll
  for (int i = 0; i < NCL; ++i)
#pragma unroll
    for (int e = 0; e < V; ++e) ag[i][e] = ab[i][e] = ao[i][e] = 0.f;

  const int stride = gridDim.x * kWarps * TPW;
  for (int tok0 = (blockIdx.x * kWarps + warp) * TPW; tok0 < tokens; tok0 += stride) {
    float x[TPW][NCL][V], dy[TPW][NCL][V];
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tok = tok0 + u;
      const long long base = token_base(p, tok);
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const int c = lane + 32 * i;
        if (c < nch && tok < tokens) {
          Chunk<T>::load(static_cast<const T*>(p.X) + base + coff[i], x[u][i]);
          Chunk<T>::load(static_cast<const T*>(p.dY) + (long long)tok * W + c * V, dy[u][i]);
          if (p.dOut) {
            float o[V];
            Chunk<T>::load(static_cast<const T*>(p.dOut) + (long long)tok * W + c * V, o);
#pragma unroll
            for (int e = 0; e < V; ++e) ao[i][e] += o[e];
          }
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) x[u][i][e] = dy[u][i][e] = 0.f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tok = tok0 + u;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NCL; ++i)
#pragma unroll
        for (int e = 0; e < V; ++e) s += x[u][i][e];
      const float mu = warp_sum(s) * inv_w;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const bool on = lane + 32 * i < nch;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          x[u][i][e] = on ? x[u][i][e] - mu : 0.f;
          q = fmaf(x[u][i][e], x[u][i][e], q);
        }
      }
      const float rstd = rsqrtf(warp_sum(q) * inv_w + p.eps);
      // dx = rstd * (dxh - mean(dxh) - xhat * mean(dxh * xhat)),  dxh = dy * gamma
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const float xh = x[u][i][e] * rstd;
          x[u][i][e] = xh;
          const float dxh = dy[u][i][e] * gam[i][e];
          ag[i][e] = fmaf(dy[u][i][e], xh, ag[i][e]);
          ab[i][e] += dy[u][i][e];
          dy[u][i][e] = dxh;
          s1 += dxh;
          s2 = fmaf(dxh, xh, s2);
        }
      }
      s1 = warp_sum(s1) * inv_w;
      s2 = warp_sum(s2) * inv_w;
#pragma unroll
      for (int i = 0; i < NCL; ++i) {
        const int c = lane + 32 * i;
        if (c < nch && tok < tokens) {
          float dx[V];
#pragma unroll
          for (int e = 0; e < V; ++e) dx[e] = rstd * (dy[u][i][e] - s1 - x[u][i][e] * s2);
          Chunk<T>::store(static_cast<T*>(p.dX) + token_base(p, tok) + coff[i], dx);
        }
      }
    }
  }

  // LayerNorm parameter gradients: warps -> shared memory -> one atomic per column per CTA,
  // weight then bias through the same buffer.
  __shared__ float red[kWarps][kMaxW];
  const int passes = p.dOut ? 3 : 2;
  for (int pass = 0; pass < passes; ++pass) {
#pragma unroll
    for (int i = 0; i < NCL; ++i) {
      const int c = lane + 32 * i;
      if (c < nch)
#pragma unroll
        for (int e = 0; e < V; ++e) red[warp][c * V + e] = pass == 0 ? ag[i][e] : pass == 1 ? ab[i][e] : ao[i][e];
    }
    __syncthreads();
    float* dst = pass == 0 ? p.dln_w : pass == 1 ? p.dln_b : p.dbias;
    for (int col = threadIdx.x; col < W; col += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kWarps; ++w2) t += red[w2][col];
      atomicAdd(dst + col, t);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------ host
// One wave: as many CTAs as fit on the device at once (from the occupancy API), at most one
// token group per warp.
template <typename K>
static int n_ctas(K kernel, long long tokens, int tpw) {  // tokens < 2^31
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWarps * 32, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  long long want = (long long)sms * per_sm, most = (tokens + kWarps * tpw - 1) / (kWarps * tpw);
  return (int)(want < most ? want : most);
}

template <bool BWD, typename T, int NCL>
static void launch_t(const Params& p, cudaStream_t st) {
  const long long tokens = (long long)p.B * p.L;
  const int grid = BWD ? n_ctas(post_norm_bwd_kernel<T, NCL>, tokens, Tpw<NCL>::value)
                       : n_ctas(post_norm_fwd_kernel<T, NCL>, tokens, Tpw<NCL>::value);
  if (BWD)
    post_norm_bwd_kernel<T, NCL><<<grid, kWarps * 32, 0, st>>>(p);
  else
    post_norm_fwd_kernel<T, NCL><<<grid, kWarps * 32, 0, st>>>(p);
}

template <bool BWD, typename T>
static void launch_ncl(const Params& p, cudaStream_t st) {
  const int nch = p.NH * p.F / Chunk<T>::V;
  if (nch <= 32)
    launch_t<BWD, T, 1>(p, st);
  else if (nch <= 64)
    launch_t<BWD, T, 2>(p, st);
  else
    launch_t<BWD, T, 4>(p, st);
}

template <bool BWD>
static void launch(const Params& p, int dt, cudaStream_t st) {
  if (dt == DT_BF16)
    launch_ncl<BWD, __nv_bfloat16>(p, st);
  else if (dt == DT_F16)
    launch_ncl<BWD, __half>(p, st);
  else
    launch_ncl<BWD, float>(p, st);
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

static int check(const char* who, int B, int NH, int L, int F, const void* X, int dt, const float* ln_w,
                 const float* ln_b, float eps) {
  TTT_REQUIRE(X && ln_w && ln_b, TTT_ERR_NULL, "%s: NULL pointer argument", who);
  TTT_REQUIRE(B >= 1 && NH >= 1 && L >= 1 && F >= 1, TTT_ERR_SHAPE, "%s: bad sizes B=%d NH=%d L=%d F=%d", who, B, NH,
              L, F);
  TTT_REQUIRE((long long)B * L < (1LL << 31) - (1LL << 20), TTT_ERR_SHAPE, "%s: B * L = %lld tokens is too many", who,
              (long long)B * L);
  TTT_REQUIRE(valid_dtype(dt), TTT_ERR_DTYPE, "%s: bad dtype code %d", who, dt);
  const int V = dt == DT_F32 ? 4 : 8;
  TTT_REQUIRE(F % V == 0, TTT_ERR_SHAPE, "%s: head_dim %d must be a multiple of %d", who, F, V);
  TTT_REQUIRE((long long)NH * F <= (dt == DT_F32 ? kMaxW / 2 : kMaxW), TTT_ERR_SHAPE,
              "%s: width %d above %d", who, NH * F, dt == DT_F32 ? kMaxW / 2 : kMaxW);
  TTT_REQUIRE(eps >= 0.f, TTT_ERR_SHAPE, "%s: negative eps", who);
  TTT_REQUIRE(aligned16(X) && aligned16(ln_w) && aligned16(ln_b), TTT_ERR_ALIGN,
              "%s: XQW and the LayerNorm parameters must be 16-byte aligned", who);
  return TTT_OK;
}

}  // namespace epilogue
}  // namespace ttt

using namespace ttt;

extern "C" int ttt_post_norm_fwd(int B, int NH, int L, int F, const void* XQW, int dt, const float* ln_w,
                                 const float* ln_b, float eps, void* Y, void* stream) {
  const char* who = "ttt_post_norm_fwd";
  int rc = epilogue::check(who, B, NH, L, F, XQW, dt, ln_w, ln_b, eps);
  if (rc) return rc;
  TTT_REQUIRE(Y, TTT_ERR_NULL, "%s: NULL output pointer", who);
  TTT_REQUIRE(epilogue::aligned16(Y), TTT_ERR_ALIGN, "%s: output must be 16-byte aligned", who);
  epilogue::Params p{};
  p.B = B, p.NH = NH, p.L = L, p.F = F, p.X = XQW, p.ln_w = ln_w, p.ln_b = ln_b, p.eps = eps, p.Y = Y;
  epilogue::launch<false>(p, dt, static_cast<cudaStream_t>(stream));
  return check_launch(who);
}

extern "C" int ttt_post_norm_bwd(int B, int NH, int L, int F, const void* XQW, int dt, const float* ln_w,
                                 const float* ln_b, float eps, const void* dY, void* dXQW, float* dln_w, float* dln_b,
                                 const void* dOut, float* dbias, void* stream) {
  const char* who = "ttt_post_norm_bwd";
  int rc = epilogue::check(who, B, NH, L, F, XQW, dt, ln_w, ln_b, eps);
  if (rc) return rc;
  TTT_REQUIRE(dY && dXQW && dln_w && dln_b, TTT_ERR_NULL, "%s: NULL pointer argument", who);
  TTT_REQUIRE(epilogue::aligned16(dY) && epilogue::aligned16(dXQW), TTT_ERR_ALIGN,
              "%s: gradients must be 16-byte aligned", who);
  TTT_REQUIRE(!dOut == !dbias, TTT_ERR_NULL, "%s: dOut and dbias are given together", who);
  TTT_REQUIRE(!dOut || epilogue::aligned16(dOut), TTT_ERR_ALIGN, "%s: dOut must be 16-byte aligned", who);
  epilogue::Params p{};
  p.B = B, p.NH = NH, p.L = L, p.F = F, p.X = XQW, p.ln_w = ln_w, p.ln_b = ln_b, p.eps = eps;
  p.dY = dY, p.dX = dXQW, p.dln_w = dln_w, p.dln_b = dln_b, p.dOut = dOut, p.dbias = dbias;
  epilogue::launch<true>(p, dt, static_cast<cudaStream_t>(stream));
  return check_launch(who);
}
