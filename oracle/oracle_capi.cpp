// TEST INFRASTRUCTURE ONLY -- C entry points of the CPU oracle (see zeno_oracle.h).
// reset_to_state / set_gravity / set_timestep follow src/main.zig:290-385, 633-663.
#include <cstring>
#include <string>

#include "oracle_model.h"
#include "zeno_oracle.h"

using namespace zo;

extern "C" {

void* zo_create_ex(const char* xml, const ZoConfig* c, uint32_t semantics) {
  if (!xml || !c || semantics > 1) return nullptr;
  Scene sc;
  if (!parse_mjcf(std::string(xml), &sc, semantics == 1)) return nullptr;
  Config cfg;
  cfg.num_envs = c->num_envs;
  cfg.timestep = c->timestep;
  cfg.contact_iterations = c->contact_iterations;
  cfg.max_contacts_per_env = c->max_contacts_per_env;
  cfg.seed = c->seed;
  cfg.substeps = c->substeps;
  cfg.enable_profiling = c->enable_profiling;
  World* w = new World();
  if (!world_init(w, sc, cfg)) {
    delete w;
    return nullptr;
  }
  return w;
}

void* zo_create(const char* xml, const ZoConfig* c) { return zo_create_ex(xml, c, 0); }

void zo_destroy(void* h) { delete static_cast<World*>(h); }

int zo_step(void* h, const float* actions, uint32_t substeps) {
  if (!h) return -1;
  world_step(static_cast<World*>(h), actions, substeps);
  return 0;
}

int zo_run(void* h, const float* actions, uint32_t nsteps, uint32_t substeps) {
  return zo_run_threads(h, actions, nsteps, substeps, 1);
}

int zo_run_threads(void* h, const float* actions, uint32_t nsteps, uint32_t substeps, uint32_t threads) {
  if (!h) return -1;
  World* w = static_cast<World*>(h);
  for (uint32_t s = 0; s < nsteps; s++) world_step(w, actions + size_t(s) * w->E * w->A, substeps, threads);
  return 0;
}

int zo_step_subset(void* h, const float* actions, const uint8_t* mask, uint32_t substeps) {
  if (!h) return -1;
  return world_step_subset(static_cast<World*>(h), actions, mask, substeps);
}

int zo_reset(void* h, const uint8_t* mask) {
  if (!h) return -1;
  world_reset(static_cast<World*>(h), mask);
  return 0;
}

int zo_reset_to_state(void* h, const float* pos, const float* quat, const float* vel, const float* angvel,
                      const uint8_t* mask) {
  if (!h) return -1;
  World* w = static_cast<World*>(h);
  const size_t per = size_t(w->B) * 4;
  auto copy_in = [&](std::vector<float>& dst, const float* src) {
    for (uint32_t e = 0; e < w->E; e++) {
      if (mask && !mask[e]) continue;
      std::memcpy(&dst[e * per], &src[e * per], per * sizeof(float));
    }
  };
  copy_in(w->pos, pos);
  copy_in(w->quat, quat);
  if (vel) copy_in(w->vel, vel);
  if (angvel) copy_in(w->angvel, angvel);
  std::fill(w->counts.begin(), w->counts.end(), 0u);
  return 0;
}

int zo_set_gravity(void* h, float gx, float gy, float gz) {
  if (!h) return -1;
  World* w = static_cast<World*>(h);
  w->params.gravity[0] = gx;
  w->params.gravity[1] = gy;
  w->params.gravity[2] = gz;
  return 0;
}

int zo_set_timestep(void* h, float ts) {
  if (!h) return -1;
  if (ts <= 0) return -6;
  World* w = static_cast<World*>(h);
  w->timestep = ts;
  uint32_t s = w->cfg.substeps > 1 ? w->cfg.substeps : 1;
  w->params.dt = ts / float(s);
  return 0;
}

int zo_set_task(void* h, const ZoTask* t) {
  if (!h || !t) return -1;
  World* w = static_cast<World*>(h);
  if (t->enabled && t->body >= w->B) return -6;
  w->task.enabled = t->enabled != 0;
  w->task.body = t->body;
  w->task.auto_reset = t->auto_reset != 0;
  w->task.z_min = t->z_min;
  w->task.z_max = t->z_max;
  w->task.noise = t->noise;
  w->task.forward_weight = t->forward_weight;
  w->task.alive_bonus = t->alive_bonus;
  w->task.ctrl_cost = t->ctrl_cost;
  w->task.seed = t->seed;
  w->task_env_offset = t->env_offset;
  return 0;
}

void zo_dims(void* h, uint32_t out[10]) {
  World* w = static_cast<World*>(h);
  uint32_t d[10] = {w->E, w->B, w->J, w->A, w->G, w->S, w->M, w->K, w->obs, w->num_colors};
  std::memcpy(out, d, sizeof(d));
}

void* zo_buffer(void* h, const char* name, size_t* nbytes) {
  World* w = static_cast<World*>(h);
  std::string n(name);
  auto ret = [&](auto& v) -> void* {
    *nbytes = v.size() * sizeof(v[0]);
    return v.empty() ? nullptr : (void*)v.data();
  };
  if (n == "positions") return ret(w->pos);
  if (n == "quaternions") return ret(w->quat);
  if (n == "velocities") return ret(w->vel);
  if (n == "angular_velocities") return ret(w->angvel);
  if (n == "accelerations") return ret(w->acc);
  if (n == "joint_positions") return ret(w->jpos);
  if (n == "joint_velocities") return ret(w->jvel);
  if (n == "joint_torques") return ret(w->jtorque);
  if (n == "observations") return ret(w->obs_buf);
  if (n == "rewards") return ret(w->rewards);
  if (n == "dones") return ret(w->dones);
  if (n == "contacts") return ret(w->contacts);
  if (n == "contact_counts") return ret(w->counts);
  if (n == "prev_contacts") return ret(w->prev_contacts);
  if (n == "prev_contact_counts") return ret(w->prev_counts);
  if (n == "actions") return ret(w->actions);
  if (n == "bodies") return ret(w->bodies);
  if (n == "joints") return ret(w->joints);
  if (n == "geoms") return ret(w->geoms);
  if (n == "actuators") return ret(w->actuators);
  if (n == "sensors") return ret(w->sensors);
  if (n == "constraints") return ret(w->constraints);
  if (n == "constraint_template") return ret(w->templ);
  if (n == "color_ranges") return ret(w->color_ranges);
  if (n == "inv_mass_inertia") return ret(w->inv_mi);
  *nbytes = 0;
  return nullptr;
}

}  // extern "C"

// ---- helpers for the known-answer tests ----
#include "oracle_math.h"
extern "C" {
float zo_atan2(float y, float x) { return zo::atan2_r(y, x); }

// Arithmetic of the step: 0 canonical (default), 1 literal, 2 literal with FMA contraction
// (oracle_literal.cpp; the reference semantics only, so a corrected-semantics world
// refuses 1 and 2).
int zo_set_arithmetic(void* h, uint32_t mode) {
  if (!h || mode > 2 || (static_cast<World*>(h)->scene.corrected && mode != 0)) return -6;
  static_cast<World*>(h)->arithmetic = mode;
  return 0;
}

int zo_set_narrow_mode(void* h, uint32_t mode) {
  if (!h || mode > 2 || (static_cast<World*>(h)->scene.corrected && mode == 0)) return -6;
  static_cast<World*>(h)->narrow_mode = mode;
  return 0;
}

// One detectCollision call on two free-standing geoms (known-answer tests).  geom_*:
// type, local pos xyz, size xyz; body_*: pos xyz, quat xyzw.  out: point xyz, normal
// xyz, penetration.  mode 2 adds GJK + EPA for box-capsule pairs.  Returns 1 on contact.
int zo_narrow_cpu(const float* geom_a, const float* body_a, const float* geom_b, const float* body_b, float* out,
                  uint32_t mode) {
  GeomRec ga{}, gb{};
  ga.type_body[0] = uint32_t(geom_a[0]), gb.type_body[0] = uint32_t(geom_b[0]);
  for (int k = 0; k < 3; ++k) ga.pos_size0[k] = geom_a[1 + k], gb.pos_size0[k] = geom_b[1 + k];
  ga.pos_size0[3] = geom_a[4], ga.params[0] = geom_a[5], ga.params[1] = geom_a[6];
  gb.pos_size0[3] = geom_b[4], gb.params[0] = geom_b[5], gb.params[1] = geom_b[6];
  return narrow_cpu(ga, body_a, body_a + 3, gb, body_b, body_b + 3, out, out + 3, out + 6, mode == 2) ? 1 : 0;
}
// gjk + epa on two free-standing shapes (same argument layout as zo_narrow_cpu).
int zo_gjk_epa(const float* geom_a, const float* body_a, const float* geom_b, const float* body_b, float* out) {
  GeomRec ga{}, gb{};
  ga.type_body[0] = uint32_t(geom_a[0]), gb.type_body[0] = uint32_t(geom_b[0]);
  for (int k = 0; k < 3; ++k) ga.pos_size0[k] = geom_a[1 + k], gb.pos_size0[k] = geom_b[1 + k];
  ga.pos_size0[3] = geom_a[4], ga.params[0] = geom_a[5], ga.params[1] = geom_a[6];
  gb.pos_size0[3] = geom_b[4], gb.params[0] = geom_b[5], gb.params[1] = geom_b[6];
  return gjk_epa_query(ga, body_a, body_a + 3, gb, body_b, body_b + 3, out);
}
float zo_asin(float x) { return zo::asin_r(x); }
// The oracle's canonical scalar functions over an array (same numbering as the product's
// zeno_eval_math): 0 rsq_r, 1 rcp_r, 2 atan2_r(x, y), 3 asin_r, 4 length((x, y, x/2)).
int zo_eval_math(uint32_t fn, const float* x, const float* y, float* out, uint64_t n) {
  using namespace zo;
  if (fn > 4 || !x || !out || ((fn == 2 || fn == 4) && !y)) return -6;
  for (uint64_t i = 0; i < n; ++i) {
    const float a = x[i];
    switch (fn) {
      case 0: out[i] = rsq_r(a); break;
      case 1: out[i] = rcp_r(a); break;
      case 2: out[i] = atan2_r(a, y[i]); break;
      case 3: out[i] = asin_r(a); break;
      default: out[i] = length(F3{a, y[i], 0.5f * a}); break;
    }
  }
  return 0;
}
// Generalised inverse mass of a contact or positional constraint, the expression the
// solvers use (all_shaders.metal:1683-1687; xpbd.zig:495-529 computeEffectiveMass):
// w = 1/m_a + (r_a x n)^T I_a^-1 (r_a x n) + 1/m_b + (r_b x n)^T I_b^-1 (r_b x n)
float zo_effective_mass(float ima, float imb, const float* Ia, const float* Ib, const float* ra, const float* rb,
                        const float* n) {
  using namespace zo;
  F3 N{n[0], n[1], n[2]}, RA{ra[0], ra[1], ra[2]}, RB{rb[0], rb[1], rb[2]};
  F3 IA{Ia[0], Ia[1], Ia[2]}, IB{Ib[0], Ib[1], Ib[2]};
  F3 rna = cross(RA, N), rnb = cross(RB, N);
  return (ima + dot(mulv(rna, IA), rna)) + (imb + dot(mulv(rnb, IB), rnb));
}
}
