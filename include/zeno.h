/*
 * zeno.h -- C ABI of libzeno.so, the B200 (sm_100a) implementation of Zeno's batched
 * rigid-body step.
 *
 * Every function below the "reference ABI" line has the exact name, argument list,
 * struct layout and error behaviour of the reference export it replaces; the citation
 * after each declaration is the reference definition (src/main.zig in Lulzx/zeno) and
 * the cffi declaration that binds it (python/zeno/_ffi.py).  Functions below the
 * "extensions" line are new.
 *
 * Threading and devices: a world binds to the CUDA device that is current on the calling
 * thread when it is created (cudaSetDevice before zeno_world_create).  A world is not
 * re-entrant; use one world per thread or process.
 *
 * Memory: pointers returned by zeno_world_get_* are CUDA managed memory.  They are valid
 * until zeno_world_destroy, readable and writable from the host between calls (as the
 * reference's zero-copy numpy views require), and addressable from the GPU.
 */
#ifndef ZENO_H
#define ZENO_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- reference ABI */

typedef void* ZenoWorldHandle;
typedef void* ZenoSwarmHandle;

/* main.zig:75-86, _ffi.py:45-56 */
typedef struct {
  uint32_t num_envs;
  float timestep; /* 0: use the MJCF <option timestep> */
  uint32_t contact_iterations;
  uint32_t max_contacts_per_env;
  uint64_t seed;
  uint32_t substeps;
  bool enable_profiling;
  uint32_t max_bodies_per_env;
  uint32_t max_joints_per_env;
  uint32_t max_geoms_per_env;
} ZenoConfig;

/* main.zig:89-102, _ffi.py:58-71; metal_available reports a usable CUDA device */
typedef struct {
  uint32_t num_envs;
  uint32_t num_bodies;
  uint32_t num_joints;
  uint32_t num_actuators;
  uint32_t num_sensors;
  uint32_t num_geoms;
  uint32_t obs_dim;
  uint32_t action_dim;
  float timestep;
  uint64_t memory_usage;
  uint64_t gpu_memory_usage;
  bool metal_available;
} ZenoInfo;

/* main.zig:105-113, _ffi.py:73-81 */
typedef struct {
  float integrate_ns;
  float collision_broad_ns;
  float collision_narrow_ns;
  float constraint_solve_ns;
  float total_step_ns;
  uint32_t num_contacts;
  uint32_t num_active_constraints;
} ZenoProfilingData;

/* main.zig:116-125, _ffi.py:83-92 */
typedef enum {
  ZENO_SUCCESS = 0,
  ZENO_INVALID_HANDLE = -1,
  ZENO_FILE_NOT_FOUND = -2,
  ZENO_PARSE_ERROR = -3,
  ZENO_METAL_ERROR = -4, /* any CUDA runtime error */
  ZENO_OUT_OF_MEMORY = -5,
  ZENO_INVALID_ARGUMENT = -6,
  ZENO_NOT_IMPLEMENTED = -7,
} ZenoError;

/* Contact slot, 64 bytes (contact.zig:210-247, read by _ffi.py:926-931) */
typedef struct {
  float position_pen[4];    /* point xyz, penetration (< 0: slot invalid) */
  float normal_friction[4]; /* normal xyz, combined friction */
  uint32_t indices[4];      /* body_a, body_b, geom_a, geom_b */
  float impulses[4];        /* normal, tangent1, tangent2, restitution */
} ZenoContact;

ZenoWorldHandle zeno_world_create(const char* mjcf_path, const ZenoConfig* config);          /* main.zig:139-178 */
ZenoWorldHandle zeno_world_create_from_string(const char* mjcf_string, const ZenoConfig* config); /* main.zig:181-216 */
void zeno_world_destroy(ZenoWorldHandle world);                                                /* main.zig:218-225 */
int zeno_world_step(ZenoWorldHandle world, const float* actions, uint32_t substeps);          /* main.zig:228-244 */
int zeno_world_step_subset(ZenoWorldHandle world, const float* actions, const uint8_t* env_mask,
                           uint32_t substeps);                                                 /* main.zig:247-268 */
int zeno_world_reset(ZenoWorldHandle world, const uint8_t* env_mask);                         /* main.zig:271-287 */
int zeno_world_reset_to_state(ZenoWorldHandle world, const float* positions, const float* quaternions,
                              const float* velocities, const float* angular_velocities,
                              const uint8_t* env_mask);                                        /* main.zig:290-385 */
float* zeno_world_get_observations(ZenoWorldHandle world);            /* main.zig:388-393 */
float* zeno_world_get_rewards(ZenoWorldHandle world);                 /* main.zig:396-401 */
uint8_t* zeno_world_get_dones(ZenoWorldHandle world);                 /* main.zig:404-409 */
uint32_t zeno_world_num_envs(ZenoWorldHandle world);                  /* main.zig:412-417 */
uint32_t zeno_world_num_bodies(ZenoWorldHandle world);                /* main.zig:420-425 */
uint32_t zeno_world_num_joints(ZenoWorldHandle world);                /* main.zig:428-433 */
uint32_t zeno_world_num_sensors(ZenoWorldHandle world);               /* main.zig:436-441 */
uint32_t zeno_world_obs_dim(ZenoWorldHandle world);                   /* main.zig:444-449 */
uint32_t zeno_world_action_dim(ZenoWorldHandle world);                /* main.zig:452-457 */
int zeno_world_get_info(ZenoWorldHandle world, ZenoInfo* info);       /* main.zig:460-483 */
float* zeno_world_get_body_positions(ZenoWorldHandle world);          /* main.zig:485-494 */
float* zeno_world_get_body_quaternions(ZenoWorldHandle world);        /* main.zig:496-505 */
float* zeno_world_get_body_velocities(ZenoWorldHandle world);         /* main.zig:507-513 */
float* zeno_world_get_body_angular_velocities(ZenoWorldHandle world); /* main.zig:515-521 */
float* zeno_world_get_body_accelerations(ZenoWorldHandle world);      /* main.zig:523-529 */
float* zeno_world_get_joint_positions(ZenoWorldHandle world);         /* main.zig:531-537 */
float* zeno_world_get_joint_velocities(ZenoWorldHandle world);        /* main.zig:539-545 */
float* zeno_world_get_joint_forces(ZenoWorldHandle world);            /* main.zig:547-555 */
uint32_t* zeno_world_get_contact_counts(ZenoWorldHandle world);       /* main.zig:557-563 */
float* zeno_world_get_sensor_data(ZenoWorldHandle world);             /* main.zig:565-571 */
void* zeno_world_get_contacts(ZenoWorldHandle world);                 /* main.zig:573-579 */
int zeno_world_set_body_positions(ZenoWorldHandle world, const float* positions,
                                  const uint8_t* env_mask);           /* main.zig:581-606 */
int zeno_world_set_body_velocities(ZenoWorldHandle world, const float* velocities,
                                   const uint8_t* env_mask);          /* main.zig:608-630 */
int zeno_world_set_gravity(ZenoWorldHandle world, float gx, float gy, float gz); /* main.zig:633-647 */
int zeno_world_set_timestep(ZenoWorldHandle world, float timestep);   /* main.zig:650-663 */
int zeno_world_get_profiling(ZenoWorldHandle world, ZenoProfilingData* data); /* main.zig:666-683 */
void zeno_world_reset_profiling(ZenoWorldHandle world);               /* main.zig:686-690 */
uint64_t zeno_world_memory_usage(ZenoWorldHandle world);              /* main.zig:693-698 */
void zeno_world_compact_memory(ZenoWorldHandle world);                /* main.zig:701-703 (no-op) */
const char* zeno_error_string(int error_code);                        /* main.zig:706-718 */
const char* zeno_version(void);                                       /* main.zig:721-723 ("0.1.0") */
uint32_t zeno_world_max_contacts_per_env(ZenoWorldHandle world);      /* main.zig:726-730 */
bool zeno_metal_available(void);                                      /* main.zig:733-736: true if a CUDA device is usable */

/* Swarm platform (main.zig:756-910, _ffi.py:218-300).  The swarm platform is outside
 * the physics step and is not implemented: creation returns NULL, calls taking a swarm
 * return ZENO_INVALID_HANDLE for NULL and ZENO_NOT_IMPLEMENTED otherwise, and pointer
 * getters return NULL.  The symbols exist so the reference's cffi binding loads. */
typedef struct ZenoSwarmConfig ZenoSwarmConfig;
typedef struct ZenoSwarmMetrics ZenoSwarmMetrics;
typedef struct ZenoAgentState ZenoAgentState;
typedef struct ZenoTaskResult ZenoTaskResult;
typedef struct ZenoAttackConfig ZenoAttackConfig;
typedef struct ZenoReplayStats ZenoReplayStats;
ZenoSwarmHandle zeno_swarm_create(ZenoWorldHandle world, const ZenoSwarmConfig* config); /* main.zig:756-770 */
void zeno_swarm_destroy(ZenoSwarmHandle swarm);                                          /* main.zig:773-779 */
int zeno_swarm_step(ZenoSwarmHandle swarm, ZenoWorldHandle world, float* actions);       /* main.zig:783-808 */
int zeno_swarm_get_metrics(ZenoSwarmHandle swarm, ZenoSwarmMetrics* metrics);            /* main.zig:810-816 */
ZenoAgentState* zeno_swarm_get_agent_states(ZenoSwarmHandle swarm);                      /* main.zig:818-824 */
int zeno_swarm_get_neighbor_counts(ZenoSwarmHandle swarm, uint32_t* out, uint32_t count); /* main.zig:826-832 */
void zeno_swarm_set_body_offset(ZenoSwarmHandle swarm, uint32_t offset);                 /* main.zig:834-839 */
int zeno_swarm_evaluate_task(ZenoSwarmHandle swarm, void* world, uint32_t task_type, const float params[8],
                             ZenoTaskResult* result);                                    /* main.zig:841-859 */
int zeno_swarm_apply_attack(ZenoSwarmHandle swarm, const ZenoAttackConfig* config);     /* main.zig:862-870 */
uint32_t* zeno_swarm_get_neighbor_index_ptr(ZenoSwarmHandle swarm);                      /* main.zig:873-878 */
uint32_t* zeno_swarm_get_neighbor_row_ptr(ZenoSwarmHandle swarm);                        /* main.zig:881-886 */
int zeno_swarm_start_recording(ZenoSwarmHandle swarm);                                   /* main.zig:889-894 */
int zeno_swarm_stop_recording(ZenoSwarmHandle swarm);                                    /* main.zig:897-902 */
int zeno_swarm_get_replay_stats(ZenoSwarmHandle swarm, ZenoReplayStats* stats);          /* main.zig:905-910 */

/* ---------------------------------------------------------------- extensions */

/* zeno_world_step without the final stream synchronization: the step is queued on the
 * world's stream.  `actions` may be host or device memory; host memory is copied before
 * the call returns.  Call zeno_world_synchronize before reading state. */
int zeno_world_step_async(ZenoWorldHandle world, const float* actions, uint32_t substeps);
int zeno_world_synchronize(ZenoWorldHandle world);

/* The CUDA stream (cudaStream_t) the world launches on; set_stream(NULL) restores the
 * world's own non-blocking stream.  The stream must belong to the world's device. */
void* zeno_world_get_stream(ZenoWorldHandle world);
int zeno_world_set_stream(ZenoWorldHandle world, void* cuda_stream);
int zeno_world_device(ZenoWorldHandle world);

/* The step outputs in device memory, for consumers on the GPU.  The reference getters
 * zeno_world_get_observations / _rewards / _dones / _sensor_data return pinned host
 * copies of these buffers instead.  zeno_world_step copies the outputs right behind its
 * kernel, before it returns; after zeno_world_step_async the first of these getters waits
 * for the step and copies the stale outputs over in one round of DMA copies, and later
 * calls return at once.  (The reference's buffers are CPU/GPU shared memory; here a host read of
 * device-resident managed memory would migrate it page by page.) */
float* zeno_world_get_observations_device(ZenoWorldHandle world);
float* zeno_world_get_rewards_device(ZenoWorldHandle world);
uint8_t* zeno_world_get_dones_device(ZenoWorldHandle world);

/* Episode task: rewards, dones and device-side auto reset.  The reference never writes
 * rewards or dones (state.zig:93-94 allocates them; no kernel fills them), so this is
 * off by default and the default behaviour matches the reference.  When enabled, after
 * every step:
 *   done    = !(z_min <= pos[body].z <= z_max)
 *   reward  = forward_weight * vel[body].x + alive_bonus - ctrl_cost * sum(actions^2)
 *   if done and auto_reset: the env is restored to its initial state, the root body
 *   position and every hinge angle get uniform noise in [-noise, noise) from a
 *   counter-based generator keyed by (seed, env_offset + env, episode), and the env's
 *   contact count is zeroed. */
typedef struct {
  uint32_t enabled;
  uint32_t body;
  uint32_t auto_reset;
  uint32_t _pad;
  float z_min, z_max, noise, forward_weight, alive_bonus, ctrl_cost;
  uint64_t seed;
  uint64_t env_offset; /* global index of this world's env 0 (multi-GPU sharding) */
} ZenoTaskConfig;
int zeno_world_set_task(ZenoWorldHandle world, const ZenoTaskConfig* task);

/* Narrow phase (no counterpart export in the reference).  0 (default): the reference's
 * GPU narrow phase (src/shaders/all_shaders.metal:751-894: sphere-sphere, sphere-plane,
 * capsule-plane, geoms placed by unrotated offsets).  1: the reference's CPU collision
 * routines (src/collision/narrow_phase.zig:28-512, detectCollision): also sphere-capsule,
 * sphere-box, capsule-capsule, box-plane and box-box (SAT), geoms placed by their body's
 * pose.  2: as 1, plus box-capsule through the reference's GJK + EPA
 * (src/collision/gjk.zig:152-574, which the reference runs only for meshes).  Returns 0,
 * or -6 for another mode. */
int zeno_world_set_narrow_phase(ZenoWorldHandle world, uint32_t mode);
uint32_t zeno_world_get_narrow_phase(ZenoWorldHandle world);

/* Broad phase of the general kernel (replaces the reference's choice at world.zig:534 and
 * its racy spatial hash, all_shaders.metal:557-703).  0 (default): a hashed grid above 512
 * geoms, else all candidate pairs; 1: all candidate pairs; 2: the grid.  The grid emits
 * exactly the all-pairs sweep's slots, in its order (an environment whose geom centres are
 * not finite, or more than 500 cells from the origin, is swept for that substep).  Returns
 * 0, or -6 for another mode or when the grid's shared memory does not fit. */
int zeno_world_set_broad_phase(ZenoWorldHandle world, uint32_t mode);
uint32_t zeno_world_get_broad_phase(ZenoWorldHandle world);

/* Launch shape of the step.  lanes 1 or 2: the compressed-state kernel with that many
 * lanes per environment and envs_per_block (1..32) environments per block; lanes 8, 16
 * or 32: the general kernel (lanes * envs_per_block <= 256, shared memory permitting).
 * Returns -6 when the shape does not fit the model. */
int zeno_world_set_launch(ZenoWorldHandle world, int lanes, int envs_per_block);
int zeno_world_get_launch(ZenoWorldHandle world, int* lanes, int* envs_per_block);

/* Model tables in the reference's GPU record layouts, for parity checks:
 * "bodies" (BodyDataGPU, 80 B), "joints" (JointDataGPU, 80 B), "geoms" (GeomGPU, 64 B),
 * "actuators" (ActuatorDataGPU, 32 B), "sensors" (SensorGPU, 32 B), "constraints"
 * (XPBDConstraint template of env 0, colour-sorted, 96 B), "color_ranges" (u32 pairs).
 * Returns NULL for an unknown name. */
const void* zeno_world_model_table(ZenoWorldHandle world, const char* name, uint64_t* nbytes);

/* Stage profile (extends zeno_world_get_profiling, main.zig:666-683).  A world created
 * with ZenoConfig.enable_profiling runs an instrumented instantiation of its step kernel
 * (compressed-state or general) whose blocks time each stage of the step with the SM clock
 * (the general kernel: the block's first environment).
 * After each synchronous zeno_world_step, zeno_world_get_profiling's integrate / broad /
 * narrow / constraint fields hold those stages' device times (summed over the substeps,
 * averaged over the blocks, which run side by side), and this call writes up to n values:
 * the average cycles per block of the 14 stages -- 0 prologue (block loads), 1 actions and
 * kinematic bodies, 2 wrenches and integration, 3 broad phase, 4 sort, 5 narrow phase and
 * warm start, 6 contact schedule, 7 joint constraints, 8 contact solve, 9 velocity
 * update, 10 joint states and sensors, 11 contact write-back, 12 caches and task,
 * 13 block epilogue -- then the average block span in cycles, nanoseconds per cycle, the
 * slowest block's span in cycles (the kernel's duration is the slowest block's), and the
 * 14 stages' largest per-block cycles.  Returns the number of values written (31 at most),
 * 0 when no profile exists (profiling off or no synchronous step yet), -1 for NULL. */
int zeno_world_get_stage_cycles(ZenoWorldHandle world, double* out, uint32_t n);

/* Message of the last failed zeno_world_create* on this thread ("" if none). */
const char* zeno_last_error(void);

/* No counterpart in the reference.  zeno_world_reset_to_state without any device
 * allocation, for callers that cannot allocate device memory at that point (their HBM is
 * already reserved by another allocator, or they cannot risk an allocation blocking or
 * failing mid-episode).  The host arrays are staged through a fixed 16 MiB array in the
 * library's static device memory, so num_envs * num_bodies must be <= 1,048,576; larger
 * worlds get ZENO_INVALID_ARGUMENT and a message in zeno_last_error().  The array is
 * shared by all calls and worlds on a device (overlapping calls on the GPU race; serialize
 * them) and is held by every GPU that loads the library until exit.  The first call on a
 * device resolves the array's address; make it before any stream capture.  Results are
 * identical to zeno_world_reset_to_state. */
int zeno_world_reset_to_state_noalloc(ZenoWorldHandle world, const float* positions, const float* quaternions,
                                      const float* velocities, const float* angular_velocities,
                                      const uint8_t* env_mask);

/* Model semantics (no counterpart in the reference).  ZENO_SEMANTICS_REFERENCE: the
 * reference's loader and step, quirks included (what zeno_world_create builds).
 * ZENO_SEMANTICS_CORRECTED: the MJCF compiler rules the reference loader skips (compiler
 * angle units and euler sequence; parent-rotation composition of body frames; child-frame
 * joint anchors and normalised axes; geom orientation, including fromto capsules; rotated
 * geom inertia, diagonal kept; frame/site sensors resolved to their body), and in the
 * step: geom offsets rotated with their body in the broad phase with whole-geom bounding
 * radii, the contact list rebuilt every substep (the reference's counter never resets,
 * so its list freezes with duplicate slots), each geom placed by its own world frame in
 * the narrow phase, and every contact normal pointing from B to A as the contact solver
 * expects.  Corrected worlds use narrow
 * phase 2 (mode 0 is refused) and run on the general kernel. */
#define ZENO_SEMANTICS_REFERENCE 0u
#define ZENO_SEMANTICS_CORRECTED 1u
ZenoWorldHandle zeno_world_create_ex(const char* mjcf_path, const ZenoConfig* config, uint32_t semantics);
ZenoWorldHandle zeno_world_create_from_string_ex(const char* mjcf_string, const ZenoConfig* config,
                                                 uint32_t semantics);

/* Diagnostic (no counterpart in the reference): evaluates one of the step kernels'
 * canonical scalar functions on the current GPU for n host values, results into out.
 * fn 0: rsq_(x), 1: rcp_(x), 2: atan2r(x, y), 3: asinr(x), 4: len((x, y, x/2)).  y is
 * needed for fn 2 and 4.  Returns 0, -6 for a bad argument, -4 for a CUDA error. */
int zeno_eval_math(uint32_t fn, const float* x, const float* y, float* out, uint64_t n);

/* Host-only model build (no GPU needed): parse MJCF text and build the model tables;
 * zeno_model_table takes the same names as zeno_world_model_table. */
void* zeno_model_create_from_string(const char* mjcf_string);
void* zeno_model_create_from_string_ex(const char* mjcf_string, uint32_t semantics);
void zeno_model_destroy(void* model);
const void* zeno_model_table(void* model, const char* name, uint64_t* nbytes);

#ifdef __cplusplus
}
#endif

#endif /* ZENO_H */
