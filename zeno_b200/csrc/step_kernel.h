// Launcher for the fused step kernel (step_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "zeno_types.h"

namespace zb {

// Shared memory one environment needs for the whole step.
uint32_t env_smem_bytes(uint32_t B, uint32_t J, uint32_t M);

// Run args.substeps substeps for all args.num_envs environments on `stream`.
// lanes: threads per environment (4, 8, 16 or 32); envs_per_block * lanes threads per block.
cudaError_t launch_step(const StepArgs& args, int lanes, int envs_per_block, cudaStream_t stream);

}  // namespace zb

namespace zb {
// Masked restore of the initial template (mask == nullptr: every env).
cudaError_t launch_reset(float* pos, float* quat, float* vel, float* ang, float* jpos, float* jvel, const float* init,
                         uint32_t E, uint32_t B, uint32_t J, const uint8_t* mask, cudaStream_t stream);
// dst[e, b, :] = src[e, b, :] for masked envs (float4 per body).
cudaError_t launch_masked_copy(float* dst, const float* src, uint32_t E, uint32_t B, const uint8_t* mask,
                               cudaStream_t stream);
}  // namespace zb
