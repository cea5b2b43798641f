// Tensor-core specialisations. Each returns TTT_NOT_APPLICABLE (without touching the GPU)
// when the request is outside its shape / dtype / alignment envelope, so the caller runs
// the general kernel instead; any other value is the entry point's status.
#pragma once

#include <cuda_runtime.h>

#include "params.cuh"

#define TTT_NOT_APPLICABLE 1

namespace ttt {

int linear_fwd_fast(const LinFwdParams& p, cudaStream_t stream);
int mlp_fwd_fast(const MlpFwdParams& p, cudaStream_t stream);
int linear_bwd_fast(const LinBwdParams& p, cudaStream_t stream);
int mlp_bwd_fast(const MlpBwdParams& p, cudaStream_t stream);

}  // namespace ttt
