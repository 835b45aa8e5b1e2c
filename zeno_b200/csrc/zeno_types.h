// Plain-old-data types shared by the host runtime (C++) and the sm_100a step kernel.
//
// Layout notes
//  * ABI-visible per-env state keeps the reference's SoA layout exactly
//    (src/physics/state.zig:56-117): float4 per body for positions, quaternions,
//    velocities, angular velocities and accelerations; one f32 per joint for joint
//    positions / velocities / torques; E*obs_dim f32 observations; E f32 rewards;
//    E u8 dones; E*max_contacts 64-byte ContactGPU records; E u32 contact counts.
//  * Model data shared by every environment (bodies, joints, geoms, actuators, sensors,
//    colour-sorted constraints) is stored once, compacted for the kernel.  The reference
//    replicates constraints per environment (src/world/world.zig:492-501) but only the
//    Lagrange multipliers are per-env, and those never influence the state: compliance
//    is 0 for every constraint (world.zig:323), so alpha~ = 0 and the XPBD update
//    dlambda = (-C - alpha~*lambda)/(w + alpha~) does not read lambda.
#pragma once
#include <stdint.h>
#include <vector_types.h>

#ifdef __CUDACC__
#define ZB_HD __host__ __device__
#else
#define ZB_HD
#endif

namespace zb {

// Contact record, byte-identical to ContactGPU (src/physics/contact.zig:210-247).
struct Contact {
  float position_pen[4];     // point xyz, penetration (w < 0: invalid)
  float normal_friction[4];  // normal xyz, combined friction
  uint32_t indices[4];       // body_a, body_b, geom_a, geom_b
  float impulses[4];         // normal, tangent1, tangent2, restitution
};
static_assert(sizeof(Contact) == 64, "ContactGPU is 64 bytes");

// Body table (template; identical for every env).
struct DBody {
  float inv_mass_inertia[4];  // 1/m, 1/Ixx, 1/Iyy, 1/Izz  (body.zig:53-75)
  float com[4];               // centre-of-mass offset, body frame
  uint32_t type;              // 0 static, 1 kinematic, 2 dynamic
  uint32_t jf_begin, jf_end;  // range in jf_list: joints acting on this body, joint order
  uint32_t _pad;
};

// Joint table (JointDataGPU fields the step reads, world.zig:1598-1619).
struct DJoint {
  float anchor_parent[4];
  float anchor_child[4];
  float axis[4];
  uint32_t type, parent, child, _pad;
};

// Geom table (GeomGPU, primitives.zig:424-441).
struct DGeom {
  float pos_size0[4];  // local position (unrotated by the body), size[0]
  float quat[4];       // local quaternion xyzw
  float size12_fr_rest[4];  // size[1], size[2], friction, restitution
  uint32_t type, body, contype, conaffinity;
};

// A broad-phase candidate: a geom pair that passes the static filters of the reference
// broad phase (different bodies, contype/conaffinity, all_shaders.metal:494-507), kept in
// the reference's emission order (geom a ascending, then b ascending).
struct DPair {
  uint32_t ga, gb;
  float min_dist_sq;  // ((r_a + r_b) + 0.1)^2, evaluated on the host in float (r: size[0], or
                      // the bounding radius under corrected semantics)
  uint32_t plane;     // 1: plane pair, always emitted
};

struct DActuator {
  uint32_t joint, _pad[3];
  float ctrl_min, ctrl_max, gear, _pad2;
  float force_min, force_max, _pad3[2];
};

struct DSensor {
  uint32_t type, object, offset, dim;
};

// Constraint record for the solver: the XPBDConstraint fields that stay constant
// (xpbd.zig:50-76), type in the low byte of `type`.
struct DConstraint {
  uint32_t body_a, body_b, type, _pad;
  float anchor_a[4];
  float anchor_b[4];
  float axis_target[4];
  float limits[4];
};

// Episode task extension (no reference counterpart).
struct DTask {
  uint32_t enabled, body, auto_reset, _pad;
  float z_min, z_max, noise, forward_weight, alive_bonus, ctrl_cost;
  uint64_t seed, env_offset;
};

// Everything the step kernel needs, by value.
struct StepArgs {
  // dimensions
  uint32_t num_envs, B, J, A, G, S, M, K, obs_dim, num_colors, num_pairs, iterations;
  uint32_t substeps;
  uint32_t actuators_unique;  // 1: no two actuators drive the same joint
  uint32_t narrow_mode;       // 0: reference GPU narrow phase; 1: its CPU detectCollision;
                              // 2: as 1 plus GJK + EPA for box-capsule pairs
  uint32_t corrected;         // 1: corrected semantics (geom frames, bounds, B->A normals)
  // grid broad phase (same pairs, in the same order, as the all-pairs sweep)
  uint32_t broad_grid;        // 1: hashed grid; 0: all candidate pairs
  uint32_t grid_buckets;      // power of two
  float grid_inv_cell;        // 1 / cell edge (cell edge >= largest pair distance bound)
  uint32_t num_planes;
  const uint32_t* plane_geoms;  // plane geoms, ascending
  const float* geom_bound;      // per geom: the radius of the broad-phase distance test
  float dt, inv_dt, inv_step;  // dt = timestep/substeps, inv_dt = 1/dt, inv_step = 1/timestep
  float gravity[3];
  float baumgarte, slop, restitution;
  // model (device pointers)
  const DBody* bodies;
  const uint32_t* jf_list;  // joint index | (1u<<31 if the body is the joint's parent)
  const DJoint* joints;
  const DGeom* geoms;
  const DPair* pairs;
  // per candidate pair, so that the sweep's loads do not wait on the geom table:
  // body a | body b << 16, and the two geoms' local offsets (xyz, size[0])
  const uint32_t* pair_bodies;
  const float4* pair_la;
  const float4* pair_lb;
  const DActuator* actuators;
  const DSensor* sensors;
  const DConstraint* constraints;
  const uint32_t* color_ranges;  // 2*num_colors (start, count)
  // hinge groups by dependency level (general kernel; num_jlevels 0: solve by colour):
  // per group (k0 | k1 << 16, k2 | kind << 16), jgroup_levels[lv]..[lv + 1] per level
  const uint2* jgroups;
  const uint32_t* jgroup_levels;
  uint32_t num_jlevels;
  const uint32_t* subtree;       // per-body subtree size (task reset noise)
  const float* init_state;       // template: B*4 pos, B*4 quat, B*4 vel, B*4 angvel, J jpos, J jvel
  // state (device-accessible)
  float* pos;
  float* quat;
  float* vel;
  float* angvel;
  float* acc;
  float* jpos;
  float* jvel;
  float* jtorque;
  float* obs;
  float* rewards;
  uint8_t* dones;
  Contact* contacts;
  uint32_t* counts;
  uint32_t* prev_counts;
  Contact* prev_contacts;    // used only for envs whose flag is set (see prev_sep)
  uint8_t* prev_sep;         // 1: prev contacts live in prev_contacts, not in contacts
  uint32_t* episode;         // task extension: per-env reset counter
  const float* actions;      // E*A
  const uint8_t* step_mask;  // null, or per-env: 0 = compute but publish only the caches
  DTask task;
  // hand-over from the environment-per-lane kernel to the general kernel
  uint32_t* odd_list;        // environments the fast kernel left untouched
  uint32_t* odd_count;
  const uint32_t* env_list;  // general kernel: step only these (null: all envs)
  uint32_t* env_count;
  uint32_t* env_done;        // blocks finished (the last one clears env_count)
  float4* pose_scratch;      // environment-per-lane kernel: 2 * B * num_envs poses before integration
  // stage profile (environment-per-lane kernel, when profiling is enabled; null otherwise):
  // kStageCount per-stage clock64 sums over the blocks' first threads, then the sums of the
  // blocks' clock64 and %globaltimer (ns) spans, the number of blocks, the largest block
  // span in cycles and in ns, then kStageCount per-stage maxima over the blocks
  unsigned long long* stage_clk;
  // slot cache (environment-per-lane kernel; null when the contacts buffer has been handed
  // to the caller, whose writes the next step must then read): per environment the contact
  // list as the kernel left it, [slot][env]: slot words (candidate | slot << 8 | hittable
  // << 16 | key rank << 24) and impulses[0] of every slot, and a per-env flag set when the
  // environment's entries are current
  uint32_t* slot_cache_w;
  float* slot_cache_imp;
  uint8_t* slot_cache_ok;
};

// Stages of the stage profile, in step order.
enum Stage : uint32_t {
  kStPrologue = 0,     // block loads: model image, state, contact lists, hand-over checks
  kStActions,          // actions -> joint torques, kinematic bodies
  kStIntegrate,        // gravity and joint wrenches, semi-implicit Euler
  kStBroad,            // broad phase
  kStSort,             // contact list sort / merge
  kStNarrow,           // narrow phase and warm-start match
  kStSchedule,         // contact schedule and slot impulses
  kStJoints,           // XPBD joint constraints
  kStContacts,         // contact solve
  kStVelocities,       // velocities from the pose change
  kStJointState,       // joint states and sensors (last substep)
  kStWriteBack,        // contact records back to memory
  kStTask,             // caches, counters, task extension
  kStEpilogue,         // deferred record writes, coalesced state stores
  kStageCount
};
// sums, then clock span, ns span, blocks, largest clock span, largest ns span, then maxima
constexpr uint32_t kStageMax = kStageCount + 5;
constexpr uint32_t kStageSlots = kStageMax + kStageCount;

}  // namespace zb
