// World runtime: owns the device model tables and the batched state of one world on
// one GPU (the CUDA device current when the world is created), and drives the fused
// step kernel.  Mirrors src/world/world.zig (World.init/step/stepSubset/reset/setters).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "fast_model.h"
#include "model.h"
#include "zeno_types.h"

namespace zb {

struct WorldConfig {  // ZenoConfig fields the world uses (src/main.zig:75-86)
  uint32_t num_envs = 1;
  float timestep = 0.0f;  // 0: MJCF timestep
  uint32_t contact_iterations = 4;
  uint32_t max_contacts_per_env = 64;
  uint64_t seed = 42;
  uint32_t substeps = 1;
  bool enable_profiling = false;
};

struct Profiling {  // ZenoProfilingData (src/main.zig:105-113)
  float integrate_ns = 0, collision_broad_ns = 0, collision_narrow_ns = 0, constraint_solve_ns = 0,
        total_step_ns = 0;
  uint32_t num_contacts = 0, num_active_constraints = 0;
};

class World {
 public:
  // Returns nullptr and sets *err on failure.
  static World* create(const Scene& sc, const WorldConfig& cfg, std::string* err);
  ~World();

  // World.step: actions may be host or device memory (E*A floats).  Synchronous unless
  // async is set, in which case the caller synchronizes the world stream.
  cudaError_t step(const float* actions, uint32_t substeps, bool async = false);
  cudaError_t step_subset(const float* actions, const uint8_t* mask, uint32_t substeps);
  void reset(const uint8_t* mask);
  int reset_to_state(const float* pos, const float* quat, const float* vel, const float* angvel,
                     const uint8_t* mask);
  // reset_to_state staged through caller-provided device memory of at least
  // num_envs * num_bodies float4 (no allocation; used by the no-allocation entry point).
  int reset_to_state_staged(const float* pos, const float* quat, const float* vel, const float* angvel,
                            const uint8_t* mask, float* staging);
  int set_positions(const float* pos, const uint8_t* mask);
  int set_velocities(const float* vel, const uint8_t* mask);
  void set_gravity(float gx, float gy, float gz);
  int set_timestep(float ts);
  int set_task(const DTask& t);
  // 0: the reference's GPU narrow phase (default); 1: its CPU detectCollision routines.
  int set_narrow_phase(uint32_t mode);
  uint32_t narrow_phase() const { return narrow_mode_; }
  // Broad phase: 0 auto (the grid above 512 geoms, as the reference switches to its
  // spatial hash), 1 all candidate pairs, 2 grid.  Both give the same slots.
  int set_broad_phase(uint32_t mode);
  uint32_t broad_phase() const { return broad_mode_; }
  bool grid_on() const { return broad_mode_ == 2 || (broad_mode_ == 0 && model_.G > 512); }
  // lanes 1, 2: compressed-state kernel with that many lanes per environment and
  // envs_per_block (1..32) environments per block; lanes 8, 16, 32: general kernel only.
  // -6 when the shape is invalid or unsupported.
  // Shared memory of one environment in the general kernel with `lanes` lanes.
  uint32_t general_env_bytes(int lanes) const;
  int set_launch(int lanes, int envs_per_block);
  cudaError_t synchronize();
  void set_stream(cudaStream_t s) { stream_ = s ? s : own_stream_; }
  cudaStream_t stream() const { return stream_; }

  const HostModel& model() const { return model_; }
  const WorldConfig& config() const { return cfg_; }
  float timestep() const { return timestep_; }
  uint64_t memory_usage() const { return bytes_; }
  int device() const { return device_; }
  Profiling profiling() const { return prof_; }
  void reset_profiling() {
    prof_ = Profiling{};
    stage_valid_ = false;
  }
  // Stage profile of the last synchronous step of a profiling world on the
  // environment-per-lane kernel: per-stage clock cycles averaged over the blocks
  // (kStageCount values, Stage order), then the average block span in cycles, the
  // nanoseconds per cycle, the largest block span in cycles and the per-stage maxima over
  // the blocks (kStageCount values).  Returns the values written, 0 when no profile exists.
  uint32_t stage_cycles(double* out, uint32_t n) const;
  // The contacts buffer pointer for the caller (zeno_world_get_contacts).  From then on
  // every step reads the contact records themselves, so that the caller's writes count.
  Contact* expose_contacts() {
    contacts_exposed_ = true;
    return contacts;
  }
  int lanes() const { return use_fast_ ? fast_lanes_ : lanes_; }
  int envs_per_block() const { return use_fast_ ? fast_epb_ : envs_per_block_; }
  bool fast_available() const { return fast_ok_; }

  // Host copies of the step outputs (pinned memory), returned by the ABI getters.  The
  // synchronous step copies them right behind its kernel; after an asynchronous step the
  // first read brings all stale outputs over in one round of DMA copies on the stream
  // the step ran on.  (A host read of managed memory would instead migrate
  // the pages one fault at a time: 1.5 ms for Ant's 16384 x 29 observations, four
  // times the step.)  Host writes to a copy last until the next step that produces it.
  float* host_obs();
  float* host_rewards();
  uint8_t* host_dones();

  // ABI-visible state (managed memory: host and device addressable)
  float* pos = nullptr;
  float* quat = nullptr;
  float* vel = nullptr;
  float* angvel = nullptr;
  float* acc = nullptr;
  float* jpos = nullptr;
  float* jvel = nullptr;
  float* jtorque = nullptr;
  // step outputs, device memory (written by the step kernels, never read by them)
  float* obs = nullptr;
  float* rewards = nullptr;
  uint8_t* dones = nullptr;
  Contact* contacts = nullptr;
  uint32_t* counts = nullptr;

 private:
  World() = default;
  StepArgs args(uint32_t substeps, const float* actions, const uint8_t* mask) const;
  void choose_fast_shape();
  // General kernel with 8 lanes: environments per block for the current narrow phase
  // (more when GJK + EPA runs, see world.cpp).  A caller's set_launch shape is kept.
  void choose_general_blocking();
  cudaError_t launch(uint32_t substeps, const float* actions, const uint8_t* mask);
  template <class T>
  cudaError_t managed(T** p, size_t n);
  template <class T>
  cudaError_t device_buf(T** p, size_t n);
  template <class T>
  cudaError_t pinned(T** p, size_t n);
  cudaError_t queue_output_copies();  // stale outputs -> host copies, on the last step's stream
  cudaError_t refresh_outputs();

  Scene scene_;
  HostModel model_;
  WorldConfig cfg_;
  float timestep_ = 0.0f;
  float gravity_[3] = {0, 0, -9.81f};
  int device_ = 0;
  int lanes_ = 8;            // general kernel shape (also the hand-over launch)
  int envs_per_block_ = 4;
  bool fast_ok_ = false;     // the model packs into FModel
  bool use_fast_ = false;
  bool prefer_general_ = false;  // the caller selected the general kernel
  int fast_lanes_ = 2;
  int fast_epb_ = 32;
  FModel fmodel_{};
  std::vector<uint8_t> hot_image_;
  uint8_t* d_hot_ = nullptr;
  size_t hot_capacity_ = 0;
  uint32_t narrow_mode_ = 0;
  uint32_t broad_mode_ = 0;
  float4* pose_scratch_ = nullptr;
  // slot cache of the environment-per-lane kernel (StepArgs.slot_cache_*): used until the
  // contacts buffer is handed to the caller; its flags are cleared when a launch did not
  // maintain it (general kernel, model re-pack)
  uint32_t* d_cache_w_ = nullptr;
  float* d_cache_imp_ = nullptr;
  uint8_t* d_cache_ok_ = nullptr;
  bool contacts_exposed_ = false;
  bool cache_dirty_ = true;
  unsigned long long* d_stage_ = nullptr;  // profiling: the kernel's stage sums (kStageSlots)
  unsigned long long* h_stage_ = nullptr;  // pinned copy
  bool stage_valid_ = false;
  uint64_t bytes_ = 0;
  cudaStream_t own_stream_ = nullptr;
  cudaStream_t stream_ = nullptr;
  Profiling prof_;
  DTask task_{};
  // device model
  DBody* d_bodies_ = nullptr;
  uint32_t* d_jf_ = nullptr;
  DJoint* d_joints_ = nullptr;
  DGeom* d_geoms_ = nullptr;
  DPair* d_pairs_ = nullptr;
  uint32_t* d_pair_bodies_ = nullptr;
  float4* d_pair_la_ = nullptr;
  float4* d_pair_lb_ = nullptr;
  DActuator* d_act_ = nullptr;
  DSensor* d_sensors_ = nullptr;
  DConstraint* d_cons_ = nullptr;
  uint32_t* d_colors_ = nullptr;
  uint32_t* d_jgroups_ = nullptr;       // hinge groups by level (HostModel::jgroup_words)
  uint32_t* d_jgroup_levels_ = nullptr;
  uint32_t* d_subtree_ = nullptr;
  float* d_init_ = nullptr;
  float* d_bound_ = nullptr;
  uint32_t* d_planes_ = nullptr;
  // internal state
  uint32_t* prev_counts_ = nullptr;
  Contact* prev_contacts_ = nullptr;
  uint8_t* prev_sep_ = nullptr;
  uint32_t* episode_ = nullptr;
  float* d_actions_ = nullptr;
  uint8_t* d_mask_ = nullptr;
  uint32_t* d_odd_ = nullptr;  // [0] hand-over count, [1] blocks done, [2..] env indices
  std::vector<void*> allocations_;
  std::vector<void*> host_allocations_;
  float* h_obs_ = nullptr;
  float* h_rewards_ = nullptr;
  uint8_t* h_dones_ = nullptr;
  bool obs_stale_ = false;   // a step wrote obs since the host copy was taken
  bool task_stale_ = false;  // ... rewards and dones (written only with the task on)
  cudaStream_t out_stream_ = nullptr;  // the stream of the last step
};

}  // namespace zb
