// extern "C" exports of libzeno.so (declared in include/zeno.h; reference: src/main.zig).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/zeno.h"
#include "scene.h"
#include "world.h"

using zb::World;

namespace {
thread_local std::string g_last_error;

World* W(ZenoWorldHandle h) { return static_cast<World*>(h); }

ZenoWorldHandle create_world(const zb::Scene& sc, const ZenoConfig* c) {
  zb::WorldConfig wc;
  wc.num_envs = c->num_envs;
  wc.timestep = c->timestep;
  wc.contact_iterations = c->contact_iterations;
  wc.max_contacts_per_env = c->max_contacts_per_env;
  wc.seed = c->seed;
  wc.substeps = c->substeps;
  wc.enable_profiling = c->enable_profiling;
  std::string err;
  World* w = World::create(sc, wc, &err);
  if (!w) {
    g_last_error = err;
    std::fprintf(stderr, "zeno: failed to create world: %s\n", err.c_str());
  }
  return w;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? ZENO_SUCCESS : ZENO_METAL_ERROR; }
}  // namespace

namespace zb {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace zb

extern "C" {

ZenoWorldHandle zeno_world_create_ex(const char* mjcf_path, const ZenoConfig* config, uint32_t semantics) {
  if (!mjcf_path || !config) return nullptr;
  if (semantics > ZENO_SEMANTICS_CORRECTED) {
    g_last_error = "unknown semantics";
    return nullptr;
  }
  zb::Scene sc;
  std::string err;
  if (!zb::load_mjcf_file(mjcf_path, &sc, &err, semantics == ZENO_SEMANTICS_CORRECTED)) {
    g_last_error = err;
    std::fprintf(stderr, "zeno: failed to parse MJCF: %s\n", err.c_str());
    return nullptr;
  }
  return create_world(sc, config);
}

ZenoWorldHandle zeno_world_create_from_string_ex(const char* mjcf_string, const ZenoConfig* config,
                                                 uint32_t semantics) {
  if (!mjcf_string || !config) return nullptr;
  if (semantics > ZENO_SEMANTICS_CORRECTED) {
    g_last_error = "unknown semantics";
    return nullptr;
  }
  zb::Scene sc;
  std::string err;
  if (!zb::load_mjcf(mjcf_string, ".", &sc, &err, semantics == ZENO_SEMANTICS_CORRECTED)) {
    g_last_error = err;
    return nullptr;
  }
  return create_world(sc, config);
}

ZenoWorldHandle zeno_world_create(const char* mjcf_path, const ZenoConfig* config) {
  return zeno_world_create_ex(mjcf_path, config, ZENO_SEMANTICS_REFERENCE);
}

ZenoWorldHandle zeno_world_create_from_string(const char* mjcf_string, const ZenoConfig* config) {
  return zeno_world_create_from_string_ex(mjcf_string, config, ZENO_SEMANTICS_REFERENCE);
}

void zeno_world_destroy(ZenoWorldHandle world) { delete W(world); }

int zeno_world_step(ZenoWorldHandle world, const float* actions, uint32_t substeps) {
  if (!world) return ZENO_INVALID_HANDLE;
  return cuda_status(W(world)->step(actions, substeps));
}

int zeno_world_step_subset(ZenoWorldHandle world, const float* actions, const uint8_t* env_mask, uint32_t substeps) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!env_mask) return ZENO_INVALID_ARGUMENT;
  return cuda_status(W(world)->step_subset(actions, env_mask, substeps));
}

int zeno_world_reset(ZenoWorldHandle world, const uint8_t* env_mask) {
  if (!world) return ZENO_INVALID_HANDLE;
  W(world)->reset(env_mask);
  return ZENO_SUCCESS;
}

int zeno_world_reset_to_state(ZenoWorldHandle world, const float* positions, const float* quaternions,
                              const float* velocities, const float* angular_velocities, const uint8_t* env_mask) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!positions || !quaternions) return ZENO_INVALID_ARGUMENT;
  return W(world)->reset_to_state(positions, quaternions, velocities, angular_velocities, env_mask);
}

// host copies, refreshed by the first read after a step (World::host_obs)
float* zeno_world_get_observations(ZenoWorldHandle world) { return world ? W(world)->host_obs() : nullptr; }
float* zeno_world_get_rewards(ZenoWorldHandle world) { return world ? W(world)->host_rewards() : nullptr; }
uint8_t* zeno_world_get_dones(ZenoWorldHandle world) { return world ? W(world)->host_dones() : nullptr; }
float* zeno_world_get_observations_device(ZenoWorldHandle world) { return world ? W(world)->obs : nullptr; }
float* zeno_world_get_rewards_device(ZenoWorldHandle world) { return world ? W(world)->rewards : nullptr; }
uint8_t* zeno_world_get_dones_device(ZenoWorldHandle world) { return world ? W(world)->dones : nullptr; }
uint32_t zeno_world_num_envs(ZenoWorldHandle world) { return world ? W(world)->config().num_envs : 0; }
uint32_t zeno_world_num_bodies(ZenoWorldHandle world) { return world ? W(world)->model().B : 0; }
uint32_t zeno_world_num_joints(ZenoWorldHandle world) { return world ? W(world)->model().J : 0; }
uint32_t zeno_world_num_sensors(ZenoWorldHandle world) { return world ? W(world)->model().S : 0; }
uint32_t zeno_world_obs_dim(ZenoWorldHandle world) { return world ? W(world)->model().obs_dim : 0; }
uint32_t zeno_world_action_dim(ZenoWorldHandle world) { return world ? W(world)->model().A : 0; }

int zeno_world_get_info(ZenoWorldHandle world, ZenoInfo* info) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!info) return ZENO_INVALID_ARGUMENT;
  const World* w = W(world);
  const zb::HostModel& m = w->model();
  ZenoInfo r;
  std::memset(&r, 0, sizeof(r));
  r.num_envs = w->config().num_envs;
  r.num_bodies = m.B;
  r.num_joints = m.J;
  r.num_actuators = m.A;
  r.num_sensors = m.S;
  r.num_geoms = m.G;
  r.obs_dim = m.obs_dim;
  r.action_dim = m.A;
  r.timestep = w->timestep();
  r.memory_usage = w->memory_usage();
  r.gpu_memory_usage = w->memory_usage();
  r.metal_available = true;
  *info = r;
  return ZENO_SUCCESS;
}

float* zeno_world_get_body_positions(ZenoWorldHandle world) { return world ? W(world)->pos : nullptr; }
float* zeno_world_get_body_quaternions(ZenoWorldHandle world) { return world ? W(world)->quat : nullptr; }
float* zeno_world_get_body_velocities(ZenoWorldHandle world) { return world ? W(world)->vel : nullptr; }
float* zeno_world_get_body_angular_velocities(ZenoWorldHandle world) {
  return world ? W(world)->angvel : nullptr;
}
float* zeno_world_get_body_accelerations(ZenoWorldHandle world) { return world ? W(world)->acc : nullptr; }
float* zeno_world_get_joint_positions(ZenoWorldHandle world) { return world ? W(world)->jpos : nullptr; }
float* zeno_world_get_joint_velocities(ZenoWorldHandle world) { return world ? W(world)->jvel : nullptr; }
float* zeno_world_get_joint_forces(ZenoWorldHandle world) { return world ? W(world)->jtorque : nullptr; }
uint32_t* zeno_world_get_contact_counts(ZenoWorldHandle world) { return world ? W(world)->counts : nullptr; }
float* zeno_world_get_sensor_data(ZenoWorldHandle world) { return zeno_world_get_observations(world); }
void* zeno_world_get_contacts(ZenoWorldHandle world) { return world ? W(world)->expose_contacts() : nullptr; }

int zeno_world_set_body_positions(ZenoWorldHandle world, const float* positions, const uint8_t* env_mask) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!positions) return ZENO_INVALID_ARGUMENT;
  return W(world)->set_positions(positions, env_mask);
}

int zeno_world_set_body_velocities(ZenoWorldHandle world, const float* velocities, const uint8_t* env_mask) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!velocities) return ZENO_INVALID_ARGUMENT;
  return W(world)->set_velocities(velocities, env_mask);
}

int zeno_world_set_gravity(ZenoWorldHandle world, float gx, float gy, float gz) {
  if (!world) return ZENO_INVALID_HANDLE;
  W(world)->set_gravity(gx, gy, gz);
  return ZENO_SUCCESS;
}

int zeno_world_set_timestep(ZenoWorldHandle world, float timestep) {
  if (!world) return ZENO_INVALID_HANDLE;
  return W(world)->set_timestep(timestep);
}

int zeno_world_get_profiling(ZenoWorldHandle world, ZenoProfilingData* data) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!data) return ZENO_INVALID_ARGUMENT;
  const zb::Profiling p = W(world)->profiling();
  data->integrate_ns = p.integrate_ns;
  data->collision_broad_ns = p.collision_broad_ns;
  data->collision_narrow_ns = p.collision_narrow_ns;
  data->constraint_solve_ns = p.constraint_solve_ns;
  data->total_step_ns = p.total_step_ns;
  data->num_contacts = p.num_contacts;
  data->num_active_constraints = p.num_active_constraints;
  return ZENO_SUCCESS;
}

int zeno_world_get_stage_cycles(ZenoWorldHandle world, double* out, uint32_t n) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!out && n) return ZENO_INVALID_ARGUMENT;
  return int(W(world)->stage_cycles(out, n));
}

void zeno_world_reset_profiling(ZenoWorldHandle world) {
  if (world) W(world)->reset_profiling();
}

uint64_t zeno_world_memory_usage(ZenoWorldHandle world) { return world ? W(world)->memory_usage() : 0; }
void zeno_world_compact_memory(ZenoWorldHandle) {}

const char* zeno_error_string(int error_code) {
  switch (error_code) {
    case 0: return "success";
    case -1: return "invalid handle";
    case -2: return "file not found";
    case -3: return "parse error";
    case -4: return "metal error";
    case -5: return "out of memory";
    case -6: return "invalid argument";
    case -7: return "not implemented";
    default: return "unknown error";
  }
}

const char* zeno_version(void) { return "0.1.0"; }

uint32_t zeno_world_max_contacts_per_env(ZenoWorldHandle world) {
  return world ? W(world)->config().max_contacts_per_env : 0;
}

bool zeno_metal_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return n > 0;
}

// ---- swarm platform: not implemented (outside the physics step) ----
ZenoSwarmHandle zeno_swarm_create(ZenoWorldHandle, const ZenoSwarmConfig*) { return nullptr; }
void zeno_swarm_destroy(ZenoSwarmHandle) {}
int zeno_swarm_step(ZenoSwarmHandle s, ZenoWorldHandle w, float*) {
  return (!s || !w) ? ZENO_INVALID_HANDLE : ZENO_NOT_IMPLEMENTED;
}
int zeno_swarm_get_metrics(ZenoSwarmHandle s, ZenoSwarmMetrics*) { return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE; }
ZenoAgentState* zeno_swarm_get_agent_states(ZenoSwarmHandle) { return nullptr; }
int zeno_swarm_get_neighbor_counts(ZenoSwarmHandle s, uint32_t*, uint32_t) {
  return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE;
}
void zeno_swarm_set_body_offset(ZenoSwarmHandle, uint32_t) {}
int zeno_swarm_evaluate_task(ZenoSwarmHandle s, void* w, uint32_t, const float*, ZenoTaskResult*) {
  return (!s || !w) ? ZENO_INVALID_HANDLE : ZENO_NOT_IMPLEMENTED;
}
int zeno_swarm_apply_attack(ZenoSwarmHandle s, const ZenoAttackConfig*) { return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE; }
uint32_t* zeno_swarm_get_neighbor_index_ptr(ZenoSwarmHandle) { return nullptr; }
uint32_t* zeno_swarm_get_neighbor_row_ptr(ZenoSwarmHandle) { return nullptr; }
int zeno_swarm_start_recording(ZenoSwarmHandle s) { return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE; }
int zeno_swarm_stop_recording(ZenoSwarmHandle s) { return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE; }
int zeno_swarm_get_replay_stats(ZenoSwarmHandle s, ZenoReplayStats*) { return s ? ZENO_NOT_IMPLEMENTED : ZENO_INVALID_HANDLE; }

// ---- extensions ----
int zeno_world_step_async(ZenoWorldHandle world, const float* actions, uint32_t substeps) {
  if (!world) return ZENO_INVALID_HANDLE;
  return cuda_status(W(world)->step(actions, substeps, true));
}

int zeno_world_synchronize(ZenoWorldHandle world) {
  if (!world) return ZENO_INVALID_HANDLE;
  return cuda_status(W(world)->synchronize());
}

void* zeno_world_get_stream(ZenoWorldHandle world) { return world ? static_cast<void*>(W(world)->stream()) : nullptr; }

int zeno_world_set_stream(ZenoWorldHandle world, void* cuda_stream) {
  if (!world) return ZENO_INVALID_HANDLE;
  W(world)->set_stream(static_cast<cudaStream_t>(cuda_stream));
  return ZENO_SUCCESS;
}

int zeno_world_device(ZenoWorldHandle world) { return world ? W(world)->device() : -1; }

int zeno_world_set_narrow_phase(ZenoWorldHandle world, uint32_t mode) {
  if (!world) return ZENO_INVALID_HANDLE;
  return W(world)->set_narrow_phase(mode);
}

uint32_t zeno_world_get_narrow_phase(ZenoWorldHandle world) { return world ? W(world)->narrow_phase() : 0u; }

int zeno_world_set_broad_phase(ZenoWorldHandle world, uint32_t mode) {
  if (!world) return ZENO_INVALID_HANDLE;
  return W(world)->set_broad_phase(mode);
}

uint32_t zeno_world_get_broad_phase(ZenoWorldHandle world) { return world ? W(world)->broad_phase() : 0u; }

int zeno_world_set_task(ZenoWorldHandle world, const ZenoTaskConfig* t) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!t) return ZENO_INVALID_ARGUMENT;
  zb::DTask d;
  std::memset(&d, 0, sizeof(d));
  d.enabled = t->enabled;
  d.body = t->body;
  d.auto_reset = t->auto_reset;
  d.z_min = t->z_min, d.z_max = t->z_max, d.noise = t->noise;
  d.forward_weight = t->forward_weight, d.alive_bonus = t->alive_bonus, d.ctrl_cost = t->ctrl_cost;
  d.seed = t->seed, d.env_offset = t->env_offset;
  return W(world)->set_task(d);
}

int zeno_world_set_launch(ZenoWorldHandle world, int lanes, int envs_per_block) {
  if (!world) return ZENO_INVALID_HANDLE;
  return W(world)->set_launch(lanes, envs_per_block);
}

int zeno_world_get_launch(ZenoWorldHandle world, int* lanes, int* envs_per_block) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (lanes) *lanes = W(world)->lanes();
  if (envs_per_block) *envs_per_block = W(world)->envs_per_block();
  return ZENO_SUCCESS;
}

const void* zeno_model_table(void* model, const char* name, uint64_t* nbytes);

const void* zeno_world_model_table(ZenoWorldHandle world, const char* name, uint64_t* nbytes) {
  if (!world) return nullptr;
  return zeno_model_table(const_cast<zb::HostModel*>(&W(world)->model()), name, nbytes);
}

const char* zeno_last_error(void) { return g_last_error.c_str(); }

void* zeno_model_create_from_string_ex(const char* mjcf_string, uint32_t semantics) {
  if (!mjcf_string || semantics > ZENO_SEMANTICS_CORRECTED) return nullptr;
  zb::Scene sc;
  std::string err;
  auto* m = new zb::HostModel();
  if (!zb::load_mjcf(mjcf_string, ".", &sc, &err, semantics == ZENO_SEMANTICS_CORRECTED) ||
      !zb::build_model(sc, m, &err)) {
    g_last_error = err;
    delete m;
    return nullptr;
  }
  return m;
}

void* zeno_model_create_from_string(const char* mjcf_string) {
  return zeno_model_create_from_string_ex(mjcf_string, ZENO_SEMANTICS_REFERENCE);
}

void zeno_model_destroy(void* model) { delete static_cast<zb::HostModel*>(model); }

const void* zeno_model_table(void* model, const char* name, uint64_t* nbytes) {
  if (!model || !name) return nullptr;
  const zb::HostModel& m = *static_cast<zb::HostModel*>(model);
  std::string n(name);
  const std::vector<uint8_t>* v = nullptr;
  if (n == "bodies") v = &m.ref_bodies;
  else if (n == "joints") v = &m.ref_joints;
  else if (n == "geoms") v = &m.ref_geoms;
  else if (n == "actuators") v = &m.ref_actuators;
  else if (n == "sensors") v = &m.ref_sensors;
  else if (n == "constraints") v = &m.ref_constraints;
  if (v) {
    if (nbytes) *nbytes = v->size();
    return v->data();
  }
  if (n == "color_ranges") {
    if (nbytes) *nbytes = m.color_ranges.size() * 4;
    return m.color_ranges.data();
  }
  if (n == "pairs") {  // broad-phase candidates (ga, gb, min_dist_sq, plane) in emission order
    if (nbytes) *nbytes = m.pairs.size() * sizeof(zb::DPair);
    return m.pairs.data();
  }
  return nullptr;
}

}  // extern "C"
