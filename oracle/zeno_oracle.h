// TEST INFRASTRUCTURE ONLY -- C entry points of the CPU oracle, loaded with ctypes by
// tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py.  The product
// (zeno_b200/, include/) never includes or links this header or its library.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Same byte layout as ZenoConfig (reference src/main.zig:75-86).
typedef struct {
  uint32_t num_envs;
  float timestep;
  uint32_t contact_iterations;
  uint32_t max_contacts_per_env;
  uint64_t seed;
  uint32_t substeps;
  bool enable_profiling;
  uint32_t max_bodies_per_env;
  uint32_t max_joints_per_env;
  uint32_t max_geoms_per_env;
} ZoConfig;

typedef struct {
  uint32_t enabled, body, auto_reset, _pad;
  float z_min, z_max, noise, forward_weight, alive_bonus, ctrl_cost;
  uint64_t seed, env_offset;
} ZoTask;

void* zo_create(const char* mjcf_xml, const ZoConfig* cfg);
/* semantics 0: the reference; 1: corrected (MJCF compiler rules, geom frames, B->A normals) */
void* zo_create_ex(const char* mjcf_xml, const ZoConfig* cfg, uint32_t semantics);
void zo_destroy(void* h);
int zo_step(void* h, const float* actions, uint32_t substeps);
int zo_step_subset(void* h, const float* actions, const uint8_t* mask, uint32_t substeps);
int zo_reset(void* h, const uint8_t* mask);
int zo_reset_to_state(void* h, const float* pos, const float* quat, const float* vel, const float* angvel,
                      const uint8_t* mask);
int zo_set_gravity(void* h, float gx, float gy, float gz);
int zo_set_timestep(void* h, float ts);
int zo_set_task(void* h, const ZoTask* t);
// dims: [E, B, J, A, G, S, M, K, obs, num_colors]
void zo_dims(void* h, uint32_t out[10]);
// Named state buffers ("positions", "quaternions", "velocities", "angular_velocities",
// "accelerations", "joint_positions", "joint_velocities", "joint_torques", "observations",
// "rewards", "dones", "contacts", "contact_counts", "prev_contacts", "prev_contact_counts",
// "actions") and model tables ("bodies", "joints", "geoms", "actuators", "sensors",
// "constraints", "constraint_template", "color_ranges", "inv_mass_inertia").
void* zo_buffer(void* h, const char* name, size_t* nbytes);
// Run n steps with per-step actions drawn by the caller (actions: n*E*A floats).
int zo_run(void* h, const float* actions, uint32_t nsteps, uint32_t substeps);
// Same, with environments split across `threads` host threads (identical results).
int zo_run_threads(void* h, const float* actions, uint32_t nsteps, uint32_t substeps, uint32_t threads);

#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
extern "C" {
#endif
float zo_atan2(float y, float x);
int zo_set_narrow_mode(void* h, uint32_t mode);
/* 0: canonical arithmetic (default); 1: literal IEEE arithmetic of the reference kernels;
   2: the literal source compiled with FMA contraction */
int zo_set_arithmetic(void* h, uint32_t mode);
int zo_eval_math(uint32_t fn, const float* x, const float* y, float* out, uint64_t n);
int zo_gjk_epa(const float* geom_a, const float* body_a, const float* geom_b, const float* body_b, float* out);
int zo_narrow_cpu(const float* geom_a, const float* body_a, const float* geom_b, const float* body_b, float* out,
                  uint32_t mode);
float zo_asin(float x);
float zo_effective_mass(float ima, float imb, const float* Ia, const float* Ib, const float* ra, const float* rb,
                        const float* n);
#ifdef __cplusplus
}
#endif
