// Launchers for the two step kernels.
//   fast_step.cu    environment-per-lane kernel, model in the constant bank (default)
//   step_kernel.cu  general kernel, L lanes per environment, model in device tables
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "fast_model.h"
#include "zeno_types.h"

namespace zb {

// Shared memory one environment needs for the whole step (general kernel).  grid_geoms
// and grid_buckets are 0 unless the grid broad phase runs; lanes: threads per environment.
uint32_t env_smem_bytes(uint32_t B, uint32_t J, uint32_t M, uint32_t grid_geoms = 0, uint32_t grid_buckets = 0,
                        uint32_t lanes = 8);

// General kernel: run args.substeps substeps on `stream`, for all args.num_envs
// environments, or (args.env_list set) for the *args.env_count listed ones.
// lanes: threads per environment (4, 8, 16 or 32); envs_per_block * lanes threads per block.
cudaError_t launch_step(const StepArgs& args, int lanes, int envs_per_block, cudaStream_t stream);

// Shared memory one environment needs in the compressed-state kernel with L lanes per env.
uint32_t fast_env_smem_bytes(uint32_t B, uint32_t J, uint32_t M, uint32_t H, uint32_t L);

// Compressed-state kernel: `lanes` (1 or 2) lanes per environment, envs_per_block
// (1..32) environments per block.  Environments it cannot
// represent are appended to args.odd_list / odd_count untouched, for a following
// list-mode launch_step.
bool fast_lanes_supported(int lanes);
cudaError_t launch_fast_step(const StepArgs& args, const FModel& model, int lanes, int envs_per_block,
                             cudaStream_t stream);

// Resident blocks per SM for a given shape (0 when it does not fit).
int fast_max_active_blocks(const StepArgs& args, const FModel& model, int lanes, int envs_per_block);

// Masked restore of the initial template (mask == nullptr: every env).
cudaError_t launch_reset(float* pos, float* quat, float* vel, float* ang, float* jpos, float* jvel, const float* init,
                         uint32_t E, uint32_t B, uint32_t J, const uint8_t* mask, cudaStream_t stream);
// dst[e, b, :] = src[e, b, :] for masked envs (float4 per body).
cudaError_t launch_masked_copy(float* dst, const float* src, uint32_t E, uint32_t B, const uint8_t* mask,
                               cudaStream_t stream);

}  // namespace zb
