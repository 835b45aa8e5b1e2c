// World runtime (src/world/world.zig equivalents on CUDA).
//
// Memory: ABI-visible state is CUDA managed memory with the device as preferred
// location, so a pointer handed out by a zeno_world_get_* call is valid on the host (the
// reference's numpy views read and write it, src/python/zeno/_ffi.py:600-620) and on
// the GPU (torch / DLPack consumers), and host writes between steps are seen by the
// next step.  Model tables and internal caches are plain device memory.
#include "world.h"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <vector>

#include "step_kernel.h"

namespace zb {

namespace {
int opt_in_smem(int dev) {
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return v;
}
}  // namespace

template <class T>
cudaError_t World::managed(T** p, size_t n) {
  n = n ? n : 1;
  void* q = nullptr;
  cudaError_t e = cudaMallocManaged(&q, n * sizeof(T));
  if (e != cudaSuccess) return e;
  allocations_.push_back(q);
  cudaMemset(q, 0, n * sizeof(T));
  cudaMemAdvise(q, n * sizeof(T), cudaMemAdviseSetPreferredLocation, device_);
  bytes_ += n * sizeof(T);
  *p = static_cast<T*>(q);
  return cudaSuccess;
}

template <class T>
cudaError_t World::pinned(T** p, size_t n) {
  n = n ? n : 1;
  void* q = nullptr;
  cudaError_t e = cudaHostAlloc(&q, n * sizeof(T), cudaHostAllocDefault);
  if (e != cudaSuccess) return e;
  host_allocations_.push_back(q);
  std::memset(q, 0, n * sizeof(T));
  *p = static_cast<T*>(q);
  return cudaSuccess;
}

template <class T>
cudaError_t World::device_buf(T** p, size_t n) {
  n = n ? n : 1;
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, n * sizeof(T));
  if (e != cudaSuccess) return e;
  allocations_.push_back(q);
  cudaMemset(q, 0, n * sizeof(T));
  bytes_ += n * sizeof(T);
  *p = static_cast<T*>(q);
  return cudaSuccess;
}

World* World::create(const Scene& sc, const WorldConfig& cfg, std::string* err) {
  auto fail = [&](const std::string& m, World* w) -> World* {
    if (err) *err = m;
    delete w;
    return nullptr;
  };
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail("no CUDA device", nullptr);
  if (cfg.num_envs == 0) return fail("num_envs must be at least 1", nullptr);  // state.zig buffers of size 0 fail
  World* w = new World();
  cudaGetDevice(&w->device_);
  w->scene_ = sc;
  w->cfg_ = cfg;
  w->timestep_ = cfg.timestep > 0 ? cfg.timestep : sc.timestep;
  std::memcpy(w->gravity_, sc.gravity, 12);
  std::string merr;
  if (!build_model(sc, &w->model_, &merr)) return fail(merr, w);
  const HostModel& m = w->model_;
  const uint32_t E = cfg.num_envs, B = m.B, J1 = m.J ? m.J : 1, M = cfg.max_contacts_per_env;
  if (M > 65535) return fail("max_contacts_per_env above 65535", w);

  // General-kernel shape: 8 lanes per env, 4 envs per block (small blocks pack the SM's
  // shared memory tightly and balance the tail wave better).  An environment too large
  // for two per block, or so large that fewer than two such blocks fit in one SM (large
  // contact lists, many bodies), gets a whole warp instead, 32 lanes x 1, which keeps
  // more of the SM busy (collision stress, 256 slots: 2.3 against 7.7 ms per step).
  const int smem_cap = opt_in_smem(w->device_);
  const uint32_t env_bytes = w->general_env_bytes(8);
  int sm_smem = 0;
  cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, w->device_);
  if (2 * uint64_t(env_bytes) > uint64_t(smem_cap) ||
      (2 * 4 * uint64_t(env_bytes) > uint64_t(sm_smem) && w->general_env_bytes(32) <= uint32_t(smem_cap))) {
    if (w->general_env_bytes(32) > uint32_t(smem_cap))
      return fail("model does not fit in shared memory (reduce max_contacts_per_env)", w);
    w->lanes_ = 32;
    w->envs_per_block_ = 1;
  } else {
    w->lanes_ = 8;
    w->envs_per_block_ = int(std::min<uint32_t>(4u, uint32_t(smem_cap) / env_bytes));
  }
  // environment-per-lane kernel when the model packs into its fixed-capacity tables
  std::string why;
  if (m.corrected) w->narrow_mode_ = 2;  // corrected semantics use the CPU routines + GJK
  w->choose_general_blocking();
  w->fast_ok_ = pack_fast_model(m, M, w->narrow_mode_, &w->fmodel_, &w->hot_image_, &why);

  if (cudaStreamCreateWithFlags(&w->own_stream_, cudaStreamNonBlocking) != cudaSuccess) return fail("stream", w);
  w->stream_ = w->own_stream_;

  cudaError_t e = cudaSuccess;
  const size_t nb4 = size_t(E) * B * 4;
  e = e ? e : w->managed(&w->pos, nb4);
  e = e ? e : w->managed(&w->quat, nb4);
  e = e ? e : w->managed(&w->vel, nb4);
  e = e ? e : w->managed(&w->angvel, nb4);
  e = e ? e : w->managed(&w->acc, nb4);
  e = e ? e : w->managed(&w->jpos, size_t(E) * J1);
  e = e ? e : w->managed(&w->jvel, size_t(E) * J1);
  e = e ? e : w->managed(&w->jtorque, size_t(E) * J1);
  e = e ? e : w->device_buf(&w->obs, size_t(E) * (m.obs_dim ? m.obs_dim : 1));
  e = e ? e : w->device_buf(&w->rewards, E);
  e = e ? e : w->device_buf(&w->dones, E);
  e = e ? e : w->pinned(&w->h_obs_, size_t(E) * (m.obs_dim ? m.obs_dim : 1));
  e = e ? e : w->pinned(&w->h_rewards_, E);
  e = e ? e : w->pinned(&w->h_dones_, E);
  e = e ? e : w->managed(&w->contacts, size_t(E) * M);
  e = e ? e : w->managed(&w->counts, E);
  e = e ? e : w->device_buf(&w->prev_counts_, E);
  e = e ? e : w->device_buf(&w->prev_sep_, E);
  e = e ? e : w->device_buf(&w->episode_, E);
  e = e ? e : w->device_buf(&w->d_actions_, size_t(E) * (m.A ? m.A : 1));
  e = e ? e : w->device_buf(&w->d_mask_, E);
  e = e ? e : w->device_buf(&w->d_odd_, size_t(E) + 2);
  auto upload = [&](auto** dst, const auto& v) {
    if (e != cudaSuccess) return;
    e = w->device_buf(dst, v.size());
    if (e == cudaSuccess && !v.empty()) e = cudaMemcpy(*dst, v.data(), v.size() * sizeof(v[0]), cudaMemcpyHostToDevice);
  };
  upload(&w->d_bodies_, m.bodies);
  upload(&w->d_jf_, m.jf_list);
  upload(&w->d_joints_, m.joints);
  upload(&w->d_geoms_, m.geoms);
  upload(&w->d_pairs_, m.pairs);
  {
    std::vector<uint32_t> pb;
    std::vector<float4> la, lb;
    for (const DPair& p : m.pairs) {
      const DGeom &ga = m.geoms[p.ga], &gb = m.geoms[p.gb];
      pb.push_back(ga.body | (gb.body << 16));
      la.push_back(make_float4(ga.pos_size0[0], ga.pos_size0[1], ga.pos_size0[2], ga.pos_size0[3]));
      lb.push_back(make_float4(gb.pos_size0[0], gb.pos_size0[1], gb.pos_size0[2], gb.pos_size0[3]));
    }
    upload(&w->d_pair_bodies_, pb);
    upload(&w->d_pair_la_, la);
    upload(&w->d_pair_lb_, lb);
  }
  upload(&w->d_act_, m.actuators);
  upload(&w->d_sensors_, m.sensors);
  upload(&w->d_cons_, m.constraints);
  upload(&w->d_colors_, m.kcolor_ranges);
  upload(&w->d_jgroups_, m.jgroup_words);
  upload(&w->d_jgroup_levels_, m.jgroup_levels);
  upload(&w->d_subtree_, m.subtree);
  upload(&w->d_init_, m.init_state);
  upload(&w->d_bound_, m.geom_bound);
  upload(&w->d_planes_, m.plane_geoms);
  if (w->fast_ok_) {
    upload(&w->d_hot_, w->hot_image_);
    w->hot_capacity_ = w->hot_image_.size();
    w->fmodel_.hot = reinterpret_cast<const uint4*>(w->d_hot_);
    e = e ? e : w->device_buf(&w->pose_scratch_, size_t(2) * B * E);
    e = e ? e : w->device_buf(&w->d_cache_w_, size_t(M) * E);
    e = e ? e : w->device_buf(&w->d_cache_imp_, size_t(M) * E);
    e = e ? e : w->device_buf(&w->d_cache_ok_, size_t(E));
  }
  if (cfg.enable_profiling) {
    e = e ? e : w->device_buf(&w->d_stage_, size_t(kStageSlots));
    e = e ? e : w->pinned(&w->h_stage_, size_t(kStageSlots));
  }
  if (e != cudaSuccess) return fail(std::string("CUDA allocation failed: ") + cudaGetErrorString(e), w);

  // initializeState (world.zig:663-691): every env starts from the body definitions
  e = launch_reset(w->pos, w->quat, w->vel, w->angvel, w->jpos, w->jvel, w->d_init_, E, B, m.J, nullptr, w->stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(w->stream_);
  if (e != cudaSuccess) return fail(std::string("CUDA init failed: ") + cudaGetErrorString(e), w);
  if (w->fast_ok_) w->choose_fast_shape();
  return w;
}

// Shape of the compressed-state kernel.  Lanes per environment: 2 when splitting the
// model's colours over two lanes cuts the sequential constraint steps per sweep by at
// least 1.75x (a second lane per environment also doubles the warps that share an SM
// scheduler, which slows each step; measured on B200: Humanoid, colours of 6,6,6,4,4,4,
// 2,2,2,1,1,1 -> 1.66x faster with 2 lanes; Ant, 4,4,4,2,2,2,1 x 6 -> 3 % slower), else 1.
// Environments per block: the largest count that still lets every environment be
// resident at once; when none does, the shape with the most resident environments per SM.
void World::choose_fast_shape() {
  uint32_t steps1 = 0, steps2 = 0;
  for (uint32_t col = 0; col < model_.num_colors; ++col) {
    const uint32_t c = model_.kcolor_ranges[2 * col + 1];
    steps1 += c;
    steps2 += (c + 1) / 2;
  }
  const int kDefaultLanes = (steps2 > 0 && 4 * steps1 >= 7 * steps2) ? 2 : 1;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_);
  const StepArgs a = args(cfg_.substeps, nullptr, nullptr);
  int best = 0, best_res = 0;
  for (int epb = 32; epb >= 1; --epb) {
    const int bps = fast_max_active_blocks(a, fmodel_, kDefaultLanes, epb);
    if (bps <= 0) continue;
    const uint64_t resident = uint64_t(bps) * epb;
    if (resident * uint64_t(sms) >= cfg_.num_envs) {
      best = epb;
      break;
    }
    if (int(resident) > best_res) best_res = int(resident), best = epb;
  }
  if (best == 0) {
    fast_ok_ = false;
    return;
  }
  fast_lanes_ = kDefaultLanes;
  fast_epb_ = best;
  use_fast_ = true;
}

World::~World() {
  if (own_stream_) cudaStreamSynchronize(own_stream_);
  if (stream_ && stream_ != own_stream_) cudaStreamSynchronize(stream_);
  for (void* p : allocations_) cudaFree(p);
  for (void* p : host_allocations_) cudaFreeHost(p);
  if (own_stream_) cudaStreamDestroy(own_stream_);
}

cudaError_t World::queue_output_copies() {
  const size_t E = cfg_.num_envs;
  cudaError_t e = cudaSuccess;
  if (obs_stale_) e = cudaMemcpyAsync(h_obs_, obs, E * model_.obs_dim * sizeof(float), cudaMemcpyDeviceToHost, out_stream_);
  if (e == cudaSuccess && task_stale_) {
    e = cudaMemcpyAsync(h_rewards_, rewards, E * sizeof(float), cudaMemcpyDeviceToHost, out_stream_);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_dones_, dones, E, cudaMemcpyDeviceToHost, out_stream_);
  }
  return e;
}

cudaError_t World::refresh_outputs() {
  if (!obs_stale_ && !task_stale_) return cudaSuccess;
  cudaError_t e = queue_output_copies();
  if (e == cudaSuccess) e = cudaStreamSynchronize(out_stream_);
  if (e == cudaSuccess) obs_stale_ = task_stale_ = false;
  return e;
}

float* World::host_obs() {
  refresh_outputs();
  return h_obs_;
}

float* World::host_rewards() {
  refresh_outputs();
  return h_rewards_;
}

uint8_t* World::host_dones() {
  refresh_outputs();
  return h_dones_;
}

StepArgs World::args(uint32_t substeps, const float* actions, const uint8_t* mask) const {
  const HostModel& m = model_;
  StepArgs a;
  std::memset(&a, 0, sizeof(a));
  a.num_envs = cfg_.num_envs;
  a.B = m.B, a.J = m.J, a.A = m.A, a.G = m.G, a.S = m.S, a.M = cfg_.max_contacts_per_env, a.K = m.K;
  a.obs_dim = m.obs_dim, a.num_colors = m.num_colors, a.num_pairs = uint32_t(m.pairs.size());
  a.iterations = cfg_.contact_iterations;
  a.substeps = substeps;
  a.actuators_unique = m.actuators_unique ? 1u : 0u;
  a.narrow_mode = narrow_mode_;
  a.corrected = model_.corrected ? 1u : 0u;
  a.broad_grid = grid_on() ? 1u : 0u;
  a.grid_buckets = m.grid_buckets, a.grid_inv_cell = m.grid_inv_cell;
  a.num_planes = uint32_t(m.plane_geoms.size()), a.plane_geoms = d_planes_, a.geom_bound = d_bound_;
  a.dt = timestep_ / float(substeps > 1 ? substeps : 1u);  // world.zig:699-702
  a.inv_dt = 1.0f / a.dt;
  a.inv_step = timestep_ > 0 ? 1.0f / timestep_ : 0.0f;  // world.zig:736
  std::memcpy(a.gravity, gravity_, 12);
  a.baumgarte = scene_.baumgarte, a.slop = scene_.slop, a.restitution = scene_.restitution;
  a.bodies = d_bodies_, a.jf_list = d_jf_, a.joints = d_joints_, a.geoms = d_geoms_, a.pairs = d_pairs_;
  a.pair_bodies = d_pair_bodies_, a.pair_la = d_pair_la_, a.pair_lb = d_pair_lb_;
  a.actuators = d_act_, a.sensors = d_sensors_, a.constraints = d_cons_, a.color_ranges = d_colors_;
  a.jgroups = reinterpret_cast<const uint2*>(d_jgroups_);
  a.jgroup_levels = d_jgroup_levels_;
  a.num_jlevels = m.jgroup_levels.empty() ? 0u : uint32_t(m.jgroup_levels.size() - 1);
  a.subtree = d_subtree_, a.init_state = d_init_;
  a.pos = pos, a.quat = quat, a.vel = vel, a.angvel = angvel, a.acc = acc;
  a.jpos = jpos, a.jvel = jvel, a.jtorque = jtorque, a.obs = obs, a.rewards = rewards, a.dones = dones;
  a.contacts = contacts, a.counts = counts, a.prev_counts = prev_counts_, a.prev_contacts = prev_contacts_;
  a.prev_sep = prev_sep_, a.episode = episode_, a.actions = actions, a.step_mask = mask;
  a.task = task_;
  a.odd_count = d_odd_;
  a.odd_list = d_odd_ + 2;
  a.pose_scratch = pose_scratch_;
  return a;
}

uint32_t World::stage_cycles(double* out, uint32_t n) const {
  if (!stage_valid_ || !h_stage_ || h_stage_[kStageCount + 2] == 0) return 0;
  const double blocks = double(h_stage_[kStageCount + 2]);
  const double span = double(h_stage_[kStageCount]);
  const uint32_t total = 2 * kStageCount + 3;
  uint32_t k = 0;
  for (; k < n && k < kStageCount; ++k) out[k] = double(h_stage_[k]) / blocks;
  if (k < n) out[k++] = span / blocks;
  if (k < n) out[k++] = span > 0 ? double(h_stage_[kStageCount + 1]) / span : 0.0;
  if (k < n) out[k++] = double(h_stage_[kStageCount + 3]);
  for (uint32_t i = 0; k < n && i < kStageCount; ++i) out[k++] = double(h_stage_[kStageMax + i]);
  return k < total ? k : total;
}

cudaError_t World::launch(uint32_t substeps, const float* actions, const uint8_t* mask) {
  StepArgs a = args(substeps, actions, mask);
  // host copies of what this step writes go stale (read_sensors writes every obs entry;
  // rewards and dones only with the task on, as the reference never writes them)
  obs_stale_ = obs_stale_ || model_.obs_dim > 0;
  task_stale_ = task_stale_ || task_.enabled != 0;
  out_stream_ = stream_;
  if (!use_fast_) {
    cache_dirty_ = true;  // the general kernel does not maintain the slot cache
    if (!d_stage_) return launch_step(a, lanes_, envs_per_block_, stream_);
    // profiling world: the general kernel's stage-profiling instantiation
    a.stage_clk = d_stage_;
    cudaError_t e = cudaMemsetAsync(d_stage_, 0, kStageSlots * sizeof(unsigned long long), stream_);
    if (e == cudaSuccess) e = launch_step(a, lanes_, envs_per_block_, stream_);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(h_stage_, d_stage_, kStageSlots * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                          stream_);
    return e;
  }
  if (d_cache_w_ && !contacts_exposed_) {  // the slot cache (see World::expose_contacts)
    if (cache_dirty_) {
      cudaError_t e = cudaMemsetAsync(d_cache_ok_, 0, cfg_.num_envs, stream_);
      if (e != cudaSuccess) return e;
      cache_dirty_ = false;
    }
    a.slot_cache_w = d_cache_w_, a.slot_cache_imp = d_cache_imp_, a.slot_cache_ok = d_cache_ok_;
  }
  if (d_stage_) {  // profiling world: the stage-profiling instantiation, its sums copied back
    a.stage_clk = d_stage_;
    cudaError_t e = cudaMemsetAsync(d_stage_, 0, kStageSlots * sizeof(unsigned long long), stream_);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = launch_fast_step(a, fmodel_, fast_lanes_, fast_epb_, stream_);
  if (e != cudaSuccess) return e;
  if (d_stage_) {
    e = cudaMemcpyAsync(h_stage_, d_stage_, kStageSlots * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                        stream_);
    if (e != cudaSuccess) return e;
    a.stage_clk = nullptr;
  }
  a.slot_cache_w = nullptr, a.slot_cache_imp = nullptr, a.slot_cache_ok = nullptr;
  // environments the fast kernel handed over (normally none): general kernel, list mode
  a.env_list = d_odd_ + 2;
  a.env_count = d_odd_;
  a.env_done = d_odd_ + 1;
  return launch_step(a, lanes_, envs_per_block_, stream_);
}

cudaError_t World::step(const float* actions, uint32_t substeps, bool async) {
  const auto t0 = std::chrono::steady_clock::now();
  // substeps == 0 selects the adaptive count, which stays at the configured value
  // (its violation probe reads a constraint field no kernel writes, world.zig:767-791)
  const uint32_t ns = substeps == 0 ? cfg_.substeps : substeps;
  const size_t na = size_t(cfg_.num_envs) * model_.A;
  const float* dev_actions = d_actions_;
  if (na > 0 && actions) {
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, actions) == cudaSuccess &&
        (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged)) {
      dev_actions = actions;  // already device-addressable: no copy
    } else {
      cudaGetLastError();
      cudaError_t e = cudaMemcpyAsync(d_actions_, actions, na * sizeof(float), cudaMemcpyHostToDevice, stream_);
      if (e != cudaSuccess) return e;
    }
  }
  cudaError_t e = launch(ns, dev_actions, nullptr);
  if (e != cudaSuccess) return e;
  if (async) return cudaSuccess;
  // the synchronous step (the reference's) is followed by reads of its outputs: their
  // host copies ride behind the kernel and share its synchronization
  e = queue_output_copies();
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) return e;
  obs_stale_ = task_stale_ = false;
  if (cfg_.enable_profiling) {
    prof_.total_step_ns =
        float(std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    uint64_t total = 0;
    std::vector<uint32_t> c(cfg_.num_envs);
    cudaMemcpy(c.data(), counts, c.size() * 4, cudaMemcpyDefault);
    for (uint32_t v : c) total += v;
    prof_.num_contacts = uint32_t(total > 0xFFFFFFFFull ? 0xFFFFFFFFull : total);
    prof_.num_active_constraints = model_.K * cfg_.num_envs;
    // stage times (either kernel): the blocks run side by side, so a stage's time is its
    // average over the blocks, in cycles converted with the measured ns/cycle
    double st[kStageCount + 2];
    stage_valid_ = d_stage_ != nullptr;
    if (stage_valid_ && stage_cycles(st, kStageCount + 2) == kStageCount + 2) {
      const double ns = st[kStageCount + 1];
      prof_.integrate_ns = float((st[kStActions] + st[kStIntegrate] + st[kStVelocities]) * ns);
      prof_.collision_broad_ns = float((st[kStBroad] + st[kStSort]) * ns);
      prof_.collision_narrow_ns = float((st[kStNarrow] + st[kStSchedule]) * ns);
      prof_.constraint_solve_ns = float((st[kStJoints] + st[kStContacts]) * ns);
    }
  } else {
    prof_ = Profiling{};
  }
  return cudaSuccess;
}

cudaError_t World::step_subset(const float* actions, const uint8_t* mask, uint32_t substeps) {
  const uint32_t E = cfg_.num_envs;
  uint32_t active = 0;
  for (uint32_t i = 0; i < E; ++i) active += mask[i] != 0;
  if (active == 0) return cudaSuccess;
  if (active == E) return step(actions, substeps);
  cudaError_t e = cudaSuccess;
  if (!prev_contacts_) {
    e = device_buf(&prev_contacts_, size_t(E) * cfg_.max_contacts_per_env);
    if (e != cudaSuccess) return e;
  }
  const uint32_t ns = substeps == 0 ? cfg_.substeps : substeps;
  const size_t na = size_t(E) * model_.A;
  if (na > 0) {
    e = cudaMemcpyAsync(d_actions_, actions, na * sizeof(float), cudaMemcpyDefault, stream_);
    if (e != cudaSuccess) return e;
  }
  e = cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_);
  if (e != cudaSuccess) return e;
  e = launch(ns, d_actions_, d_mask_);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(stream_);
}

void World::reset(const uint8_t* mask) {
  const uint32_t E = cfg_.num_envs;
  const uint8_t* dm = nullptr;
  if (mask) {
    cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_);
    dm = d_mask_;
  }
  launch_reset(pos, quat, vel, angvel, jpos, jvel, d_init_, E, model_.B, model_.J, dm, stream_);
  cudaMemsetAsync(counts, 0, size_t(E) * 4, stream_);  // all envs, world.zig:1313
  cudaStreamSynchronize(stream_);
}

int World::set_positions(const float* p, const uint8_t* mask) {
  const uint32_t E = cfg_.num_envs;
  const uint8_t* dm = nullptr;
  if (mask) {
    cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_);
    dm = d_mask_;
  }
  float* staging = nullptr;
  const size_t n = size_t(E) * model_.B * 4;
  if (cudaMallocAsync(reinterpret_cast<void**>(&staging), n * 4, stream_) != cudaSuccess) return -5;
  cudaMemcpyAsync(staging, p, n * 4, cudaMemcpyDefault, stream_);
  launch_masked_copy(pos, staging, E, model_.B, dm, stream_);
  cudaFreeAsync(staging, stream_);
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

int World::set_velocities(const float* v, const uint8_t* mask) {
  const uint32_t E = cfg_.num_envs;
  const uint8_t* dm = nullptr;
  if (mask) {
    cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_);
    dm = d_mask_;
  }
  float* staging = nullptr;
  const size_t n = size_t(E) * model_.B * 4;
  if (cudaMallocAsync(reinterpret_cast<void**>(&staging), n * 4, stream_) != cudaSuccess) return -5;
  cudaMemcpyAsync(staging, v, n * 4, cudaMemcpyDefault, stream_);
  launch_masked_copy(vel, staging, E, model_.B, dm, stream_);
  cudaFreeAsync(staging, stream_);
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

int World::reset_to_state(const float* p, const float* q, const float* v, const float* w, const uint8_t* mask) {
  const uint32_t E = cfg_.num_envs;
  const uint8_t* dm = nullptr;
  if (mask) {
    cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_);
    dm = d_mask_;
  }
  const size_t n = size_t(E) * model_.B * 4;
  float* staging = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&staging), n * 4, stream_) != cudaSuccess) return -5;
  const float* srcs[4] = {p, q, v, w};
  float* dsts[4] = {pos, quat, vel, angvel};
  for (int k = 0; k < 4; ++k) {
    if (!srcs[k]) continue;
    cudaMemcpyAsync(staging, srcs[k], n * 4, cudaMemcpyDefault, stream_);
    launch_masked_copy(dsts[k], staging, E, model_.B, dm, stream_);
  }
  cudaFreeAsync(staging, stream_);
  cudaMemsetAsync(counts, 0, size_t(E) * 4, stream_);  // main.zig:383
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

int World::reset_to_state_staged(const float* p, const float* q, const float* v, const float* w, const uint8_t* mask,
                                 float* staging) {
  const uint32_t E = cfg_.num_envs;
  const uint8_t* dm = nullptr;
  if (mask) {
    if (cudaMemcpyAsync(d_mask_, mask, E, cudaMemcpyDefault, stream_) != cudaSuccess) return -4;
    dm = d_mask_;
  }
  const size_t n = size_t(E) * model_.B * 4;
  const float* srcs[4] = {p, q, v, w};
  float* dsts[4] = {pos, quat, vel, angvel};
  for (int k = 0; k < 4; ++k) {
    if (!srcs[k]) continue;
    if (cudaMemcpyAsync(staging, srcs[k], n * 4, cudaMemcpyDefault, stream_) != cudaSuccess) return -4;
    if (launch_masked_copy(dsts[k], staging, E, model_.B, dm, stream_) != cudaSuccess) return -4;
  }
  if (cudaMemsetAsync(counts, 0, size_t(E) * 4, stream_) != cudaSuccess) return -4;  // main.zig:383
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

void World::set_gravity(float gx, float gy, float gz) {
  gravity_[0] = gx, gravity_[1] = gy, gravity_[2] = gz;
}

int World::set_timestep(float ts) {
  if (!(ts > 0)) return -6;
  timestep_ = ts;
  return 0;
}

int World::set_task(const DTask& t) {
  if (t.enabled && t.body >= model_.B) return -6;
  task_ = t;
  return 0;
}

int World::set_launch(int lanes, int envs_per_block) {
  if (fast_lanes_supported(lanes)) {
    if (!fast_ok_ || envs_per_block < 1 || envs_per_block > 32) return -6;
    if (fast_max_active_blocks(args(cfg_.substeps, nullptr, nullptr), fmodel_, lanes, envs_per_block) <= 0)
      return -6;
    fast_lanes_ = lanes;
    fast_epb_ = envs_per_block;
    use_fast_ = true;
    prefer_general_ = false;
    return 0;
  }
  if (lanes != 8 && lanes != 16 && lanes != 32) return -6;
  const uint32_t env_bytes = general_env_bytes(lanes);
  if (envs_per_block < 1 || lanes * envs_per_block > 256 ||
      uint64_t(env_bytes) * envs_per_block > uint64_t(opt_in_smem(device_)))
    return -6;
  lanes_ = lanes;
  envs_per_block_ = envs_per_block;
  use_fast_ = false;
  prefer_general_ = true;
  return 0;
}

// With GJK + EPA on box-capsule pairs, each lane running EPA keeps a polytope of about
// 7 KB in local memory, and with 4 environments per block six blocks share an SM, so most
// of those loads miss L1.  Blocks of 16 environments (larger blocks, fewer per SM) measured
// faster there (Humanoid narrow phase 2: 7.60 -> 6.59 ms per step; corrected semantics
// 12.3 -> 11.2) and slower without EPA (narrow phase 1: 1.65 -> 1.84; Ant corrected
// semantics 1.44 -> 1.68), so the larger block is used only when EPA can run.
void World::choose_general_blocking() {
  if (prefer_general_ || lanes_ != 8) return;
  bool epa = false;
  if (narrow_mode_ == 2)
    for (const DPair& p : model_.pairs) {
      const uint32_t ta = model_.geoms[p.ga].type, tb = model_.geoms[p.gb].type;
      epa = epa || (ta == 1 && tb == 2) || (ta == 2 && tb == 1);
    }
  const uint32_t fit = uint32_t(opt_in_smem(device_)) / std::max(general_env_bytes(8), 1u);
  envs_per_block_ = int(std::max(1u, std::min(epa ? 16u : 4u, fit)));
}

uint32_t World::general_env_bytes(int lanes) const {
  const bool g = grid_on();
  return env_smem_bytes(model_.B, model_.J, cfg_.max_contacts_per_env, g ? model_.G : 0u,
                        g ? model_.grid_buckets : 0u, uint32_t(lanes));
}

// Selects the broad phase of the general kernel.  The grid adds per-environment shared
// memory; when the current shape no longer fits, one environment per warp is tried.
int World::set_broad_phase(uint32_t mode) {
  if (mode > 2) return -6;
  if (cudaStreamSynchronize(stream_) != cudaSuccess) return -4;
  const uint32_t old = broad_mode_;
  broad_mode_ = mode;
  const uint64_t cap = uint64_t(opt_in_smem(device_));
  if (uint64_t(general_env_bytes(lanes_)) * uint64_t(envs_per_block_) <= cap) return 0;
  if (general_env_bytes(32) <= cap) {
    lanes_ = 32;
    envs_per_block_ = 1;
    return 0;
  }
  broad_mode_ = old;
  return -6;
}

// Selects the narrow phase and re-packs the compressed-state model (its hittable pairs
// depend on it); a model that no longer fits runs on the general kernel.
int World::set_narrow_phase(uint32_t mode) {
  if (mode > 2 || (model_.corrected && mode == 0)) return -6;
  if (mode == narrow_mode_) return 0;
  if (cudaStreamSynchronize(stream_) != cudaSuccess) return -4;
  narrow_mode_ = mode;
  choose_general_blocking();
  cache_dirty_ = true;  // hittable indices in the cached slot words depend on the narrow phase
  std::string why;
  std::vector<uint8_t> img;
  FModel fm{};
  const bool ok = pack_fast_model(model_, cfg_.max_contacts_per_env, mode, &fm, &img, &why);
  if (ok && img.size() > hot_capacity_) {
    uint8_t* p = nullptr;
    if (device_buf(&p, img.size()) != cudaSuccess) return -5;
    d_hot_ = p;
    hot_capacity_ = img.size();
  }
  if (ok && !pose_scratch_ &&
      device_buf(&pose_scratch_, size_t(2) * model_.B * cfg_.num_envs) != cudaSuccess)
    return -5;
  if (ok && cudaMemcpy(d_hot_, img.data(), img.size(), cudaMemcpyHostToDevice) != cudaSuccess) return -4;
  const bool was_fast = use_fast_;
  fast_ok_ = ok;
  fmodel_ = fm;
  hot_image_ = std::move(img);
  fmodel_.hot = reinterpret_cast<const uint4*>(d_hot_);
  use_fast_ = false;
  if (fast_ok_ && !prefer_general_) {  // keep a caller's shape when it still fits
    const int lanes = fast_lanes_, epb = fast_epb_;
    choose_fast_shape();
    if (was_fast && set_launch(lanes, epb) != 0) choose_fast_shape();
  }
  return 0;
}

cudaError_t World::synchronize() { return cudaStreamSynchronize(stream_); }

}  // namespace zb
