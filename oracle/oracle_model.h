// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle for the batched physics step.
// Nothing in the product (zeno_b200/, include/) may include or link this file.
//
// Scene and per-world data of the oracle.  The GPU-side record layouts follow the
// reference's extern structs byte for byte so that the product's model tables can be
// compared with the oracle's: BodyDataGPU / JointDataGPU / ActuatorDataGPU
// (src/world/world.zig:1573-1637), GeomGPU (src/collision/primitives.zig:434-441),
// SensorGPU (src/world/sensors.zig:155-160), XPBDConstraint (src/physics/xpbd.zig:50-76),
// ContactGPU (src/physics/contact.zig:210-247).
#pragma once
#include <cstdint>
#include <limits>
#include <map>
#include <string>
#include <vector>

namespace zo {

// ----- scene (host description), src/physics/body.zig, joint.zig, primitives.zig -----
enum BodyType : uint8_t { kStatic = 0, kKinematic = 1, kDynamic = 2 };
enum JointType : uint8_t { kFixed = 0, kRevolute = 1, kPrismatic = 2, kBall = 3, kFree = 4, kUniversal = 5 };
enum GeomType : uint8_t { kSphere = 0, kCapsule = 1, kBox = 2, kPlane = 3, kCylinder = 4, kMesh = 5, kHeightfield = 6 };
enum SensorType : uint8_t {
  kJointPos = 0, kJointVel = 1, kAccelerometer = 2, kGyro = 3, kTouch = 4, kForce = 5, kTorque = 6,
  kFramePos = 7, kFrameQuat = 8, kFrameLinVel = 9, kFrameAngVel = 10, kSubtreeCom = 11, kUser = 12
};

struct BodyDef {
  std::string name;
  BodyType type = kDynamic;
  float pos[3] = {0, 0, 0};
  float quat[4] = {0, 0, 0, 1};
  float mass = 1.0f;
  float inertia[3] = {0, 0, 0};
  int32_t parent = -1;
  float com[3] = {0, 0, 0};
  float inv_mass() const;         // body.zig:53-58
  void inv_inertia(float o[3]) const;  // body.zig:62-75
};

struct JointDef {
  std::string name;
  JointType type = kRevolute;
  uint32_t parent = 0, child = 0;
  float anchor_parent[3] = {0, 0, 0};
  float anchor_child[3] = {0, 0, 0};
  float axis[3] = {0, 0, 1};
  float axis2[3] = {0, 1, 0};
  float lower = -std::numeric_limits<float>::infinity();
  float upper = std::numeric_limits<float>::infinity();
  float damping = 0, stiffness = 0, armature = 0, ref = 0;
  bool limited = false;
  bool has_limits() const { return limited && lower < upper; }  // joint.zig:75-77
};

struct GeomDef {
  GeomType type = kSphere;
  uint32_t body = 0;
  float pos[3] = {0, 0, 0};
  float quat[4] = {0, 0, 0, 1};
  float size[3] = {1, 1, 1};
  float friction = 1.0f;
  float restitution = 0.0f;
  uint32_t contype = 0;      // "group" in the reference
  uint32_t conaffinity = 0xFFFFFFFFu;  // "mask" in the reference
};

struct ActuatorDef {
  uint32_t joint = 0;
  float ctrl_min = -1.0f, ctrl_max = 1.0f;
  float force_min = -std::numeric_limits<float>::infinity();
  float force_max = std::numeric_limits<float>::infinity();
  float gear = 1.0f, kp = 0.0f, kv = 0.0f;
};

struct SensorDef {
  SensorType type = kJointPos;
  uint32_t object = 0;
  uint32_t dim = 1;
  float noise = 0, cutoff = 0;
};

struct Scene {
  std::vector<BodyDef> bodies;
  std::vector<JointDef> joints;
  std::vector<GeomDef> geoms;
  std::vector<ActuatorDef> actuators;
  std::vector<SensorDef> sensors;
  std::map<std::string, uint32_t> body_names, joint_names;
  float timestep = 0.002f;
  float gravity[3] = {0, 0, -9.81f};
  float friction = 1.0f, restitution = 0.0f, baumgarte = 0.2f, slop = 0.005f;  // constants.zig
  bool corrected = false;  // loaded with corrected semantics
  uint32_t obs_dim() const {
    uint32_t d = 0;
    for (auto& s : sensors) d += s.dim;
    return d;
  }
};

// Parse MJCF text (parser.zig semantics).  Returns false on failure (file errors only;
// the reference parser accepts almost any text).
// corrected = true applies the MJCF compiler rules the reference skips (oracle_mjcf.cpp).
bool parse_mjcf(const std::string& xml, Scene* out, bool corrected = false);

// ----- GPU-layout records -----
struct BodyRec { float position[4], quaternion[4], inv_mass_inertia[4], params[4], com_offset[4]; };
struct JointRec { float anchor_parent[4], anchor_child[4], axis[4], params[4], params2[4]; };
struct GeomRec { uint32_t type_body[4]; float pos_size0[4], quat[4], params[4]; };
struct ActuatorRec { float params[4], params2[4]; };
struct SensorRec { uint32_t type_object[4]; float params[4]; };
struct ConstraintRec { uint32_t indices[4]; float anchor_a[4], anchor_b[4], axis_target[4], limits[4], state[4]; };
struct ContactRec { float position_pen[4], normal_friction[4]; uint32_t indices[4]; float impulses[4]; };
static_assert(sizeof(BodyRec) == 80, "BodyDataGPU");
static_assert(sizeof(JointRec) == 80, "JointDataGPU");
static_assert(sizeof(GeomRec) == 64, "GeomGPU");
static_assert(sizeof(ActuatorRec) == 32, "ActuatorDataGPU");
static_assert(sizeof(SensorRec) == 32, "SensorGPU");
static_assert(sizeof(ConstraintRec) == 96, "XPBDConstraint");
static_assert(sizeof(ContactRec) == 64, "ContactGPU");

struct Config {  // ZenoConfig, src/main.zig:75-86
  uint32_t num_envs = 1;
  float timestep = 0;
  uint32_t contact_iterations = 4;
  uint32_t max_contacts_per_env = 64;
  uint64_t seed = 42;
  uint32_t substeps = 1;
  bool enable_profiling = false;
  uint32_t max_bodies_per_env = 0, max_joints_per_env = 0, max_geoms_per_env = 0;
};

struct Params {  // SimParams, world.zig:35-56
  uint32_t num_envs, num_bodies, num_joints, num_actuators, num_geoms, num_sensors, max_contacts,
      contact_iterations;
  float dt, gravity[3], friction, restitution, baumgarte, slop;
  uint32_t obs_dim;
};

// Episode termination / reward extension (not in the reference, whose step never writes
// rewards or dones).  Off by default.
struct Task {
  bool enabled = false;
  uint32_t body = 1;
  float z_min = -std::numeric_limits<float>::infinity();
  float z_max = std::numeric_limits<float>::infinity();
  bool auto_reset = false;
  float noise = 0.0f;
  uint64_t seed = 0;
  float forward_weight = 1.0f, alive_bonus = 1.0f, ctrl_cost = 0.01f;
};

struct World {
  Scene scene;
  Config cfg;
  Params params;
  float timestep = 0;
  uint32_t E = 0, B = 0, J = 0, A = 0, G = 0, S = 0, M = 0, K = 0, obs = 0;
  // model tables
  std::vector<BodyRec> bodies;
  std::vector<JointRec> joints;
  std::vector<GeomRec> geoms;
  std::vector<ActuatorRec> actuators;
  std::vector<SensorRec> sensors;
  std::vector<ConstraintRec> constraints;  // E*K, sorted by colour within each env
  std::vector<ConstraintRec> templ;        // K (colour-sorted template)
  uint32_t num_colors = 0;
  std::vector<uint32_t> color_ranges;      // 2*num_colors: (start, count)
  // state (state.zig:56-117)
  std::vector<float> pos, vel, acc, angvel, quat, force, torque, inv_mi;  // E*B*4
  std::vector<float> jpos, jvel, jtorque;                                 // E*max(J,1)
  std::vector<float> actions;                                             // E*max(A,1)
  std::vector<float> obs_buf;                                             // E*max(obs,1)
  std::vector<float> rewards;                                             // E
  std::vector<uint8_t> dones;                                             // E
  std::vector<ContactRec> contacts, prev_contacts;                        // E*M
  std::vector<uint32_t> counts, prev_counts;                              // E
  std::vector<float> prev_pos, prev_quat, prev_vel;                       // E*B*4
  // initial state template (state.zig:358-411, env 0)
  std::vector<float> init_pos, init_quat, init_vel, init_angvel, init_jpos, init_jvel;
  uint32_t adaptive_substeps = 1;
  Task task;
  uint64_t task_env_offset = 0;     // global index of env 0 (multi-GPU sharding)
  uint32_t narrow_mode = 0;         // 0: reference GPU narrow phase; 1: CPU detectCollision;
                                    // 2: as 1, plus GJK + EPA for box-capsule pairs
  uint32_t arithmetic = 0;          // 0: canonical (the product's arithmetic, bit for bit);
                                    // 1: literal (the reference kernels' own IEEE arithmetic);
                                    // 2: literal compiled with FMA contraction
  std::vector<uint32_t> episode;    // per-env reset counter (task extension RNG stream)
  std::vector<uint32_t> subtree;    // per-body subtree size (depth-first body order)
};

bool world_init(World* w, const Scene& scene, const Config& cfg);
void world_step(World* w, const float* actions, uint32_t substeps, uint32_t threads = 1);
int world_step_subset(World* w, const float* actions, const uint8_t* mask, uint32_t substeps);
void world_reset(World* w, const uint8_t* mask);
void world_apply_task(World* w, const uint8_t* mask);
void world_reset_env_noise(World* w, uint32_t e);
// One substep of one environment in the literal arithmetic (oracle_literal.cpp).
void substep_env_literal(World* w, uint32_t e);
void substep_env_literal_contracted(World* w, uint32_t e);
// detectCollision of the reference CPU collision code for one geom pair placed by its
// bodies' poses (oracle_narrow.cpp).
bool narrow_cpu(const GeomRec& ga, const float* body_pos_a, const float* body_quat_a, const GeomRec& gb,
                const float* body_pos_b, const float* body_quat_b, float point[3], float normal[3], float* pen,
                bool gjk_pairs);
// Corrected semantics helpers (oracle_narrow.cpp).
void geom_world_pose(const GeomRec& g, const float* body_pos, const float* body_quat, float wp[3], float wq[4]);
bool normal_a_to_b(uint32_t ta, uint32_t tb);
// GJK + EPA of the reference (src/collision/gjk.zig) on two free-standing shapes.
int gjk_epa_query(const GeomRec& ga, const float* body_pos_a, const float* body_quat_a, const GeomRec& gb,
                  const float* body_pos_b, const float* body_quat_b, float out[10]);

}  // namespace zo
