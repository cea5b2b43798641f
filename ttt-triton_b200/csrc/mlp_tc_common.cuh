// Pieces shared by the tensor-core TTT-MLP kernels (F = 64, CS = 16, inner width FF = 256
// or the F x F layer's 64): the
// accumulator-fragment layout of a warp's state slices and their TMEM / global copies.
//
// A warp owns 16 M consecutive hidden units (M = 2: 32 units, M = 1: 16). Its slice of W1
// is held as W1^T (16M x 64, fragments [M][8][4]: hidden rows 16m + g (+8), feature columns
// 8nf + 2t (+1)), its slice of W2 as W2^T (64 x 16M, fragments [4][2M][4]: feature rows
// 16m + g (+8), hidden columns 8j + 2t (+1)). These accumulator layouts are directly the
// mma B-operand layouts of W1 and W2 (k = feature resp. hidden); movmatrix turns them into
// those of W1^T, W2^T.
#pragma once

#include "tmem.cuh"

namespace ttt {
namespace mlp_tc {

constexpr int F = 64, FF = 256, C = 16;

// State slices <-> global [F][FFS] (W1) and [FFS][F] (W2) layouts (FFS: the inner width,
// 256 by default, 64 for the F x F inner MLP). A warp owning 16 * M hidden units from fb
// holds W1^T as M x 8 accumulator tiles and W2^T as 4 x 2M tiles.
template <int M = 2, int FFS = FF>
__device__ __forceinline__ void w1_io(float (*S1)[8][4], float* W1, int fb, int g, int t, bool store) {
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int nf = 0; nf < 8; ++nf) {
      const int f = 8 * nf + 2 * t, ff = fb + 16 * m + g;
      float* p0 = W1 + f * FFS + ff;
      if (store) {
        p0[0] = S1[m][nf][0];
        p0[FFS] = S1[m][nf][1];
        p0[8] = S1[m][nf][2];
        p0[FFS + 8] = S1[m][nf][3];
      } else {
        S1[m][nf][0] = p0[0];
        S1[m][nf][1] = p0[FFS];
        S1[m][nf][2] = p0[8];
        S1[m][nf][3] = p0[FFS + 8];
      }
    }
}
template <int M = 2>
__device__ __forceinline__ void w2_io(float (*S2)[2 * M][4], float* W2, int fb, int g, int t, bool store) {
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int j = 0; j < 2 * M; ++j) {
      const int f = 16 * m + g, ff = fb + 8 * j + 2 * t;
      float* p0 = W2 + ff * F + f;
      if (store) {
        p0[0] = S2[m][j][0];
        p0[F] = S2[m][j][1];
        p0[8] = S2[m][j][2];
        p0[F + 8] = S2[m][j][3];
      } else {
        S2[m][j][0] = p0[0];
        S2[m][j][1] = p0[F];
        S2[m][j][2] = p0[8];
        S2[m][j][3] = p0[F + 8];
      }
    }
}

// A warp's state slice of NV values (32 or 64) <-> its NV TMEM columns.
template <int NV = 64>
__device__ __forceinline__ void slice_ld(uint32_t a, float* v) {
  tmem_ld32(a, v);
  if (NV == 64) tmem_ld32(a + 32, v + 32);
  tmem_wait_ld();
}
template <int NV = 64>
__device__ __forceinline__ void slice_st(uint32_t a, const float* v) {
  tmem_st32(a, v);
  if (NV == 64) tmem_st32(a + 32, v + 32);
  tmem_wait_st();
}
// The same store without waiting for it to land: the caller issues tmem_wait_st() before its
// next tcgen05.ld of these columns (and before the CTA's final barrier), at a point by which
// the store has long completed, so the store latency leaves the dependency chain.
template <int NV = 64>
__device__ __forceinline__ void slice_st_async(uint32_t a, const float* v) {
  tmem_st32(a, v);
  if (NV == 64) tmem_st32(a + 32, v + 32);
}

}  // namespace mlp_tc
}  // namespace ttt
