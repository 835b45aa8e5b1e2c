// Host-side scene description and model building (cold path, run once per world).
//
// The loader reproduces the reference MJCF loader's semantics (src/mjcf/parser.zig,
// src/mjcf/schema.zig) including its quirks, because the model tables -- masses,
// inertias, constraint templates, graph colouring -- must match the reference exactly:
//  * body positions accumulate parent offsets without parent rotation (parser.zig:910-913)
//  * joint ranges are used verbatim as radians (parser.zig:990-994)
//  * capsule fromto sets the midpoint and half length but keeps an identity local quat
//  * bodies without joints receive an implicit fixed joint (weld) to their parent
//  * frame sensors observe body 0 (object id is resolved only for joint sensors)
// A world created with corrected semantics (ZENO_SEMANTICS_CORRECTED) instead follows the
// MJCF compiler rules for these items; see load_mjcf.
#pragma once
#include <cstdint>
#include <limits>
#include <string>
#include <unordered_map>
#include <vector>

namespace zb {

struct SBody {
  std::string name;
  uint32_t type = 2;  // 0 static, 1 kinematic, 2 dynamic (body.zig:8-15)
  float pos[3] = {0, 0, 0};
  float quat[4] = {0, 0, 0, 1};
  float mass = 1.0f;
  float inertia[3] = {0, 0, 0};
  int32_t parent = -1;
  float com[3] = {0, 0, 0};
};

struct SJoint {
  std::string name;
  uint32_t type = 1;  // 0 fixed, 1 revolute, 2 prismatic, 3 ball, 4 free, 5 universal
  uint32_t parent = 0, child = 0;
  float anchor_parent[3] = {0, 0, 0}, anchor_child[3] = {0, 0, 0};
  float axis[3] = {0, 0, 1}, axis2[3] = {0, 1, 0};
  float lower = -std::numeric_limits<float>::infinity();
  float upper = std::numeric_limits<float>::infinity();
  float damping = 0, stiffness = 0, armature = 0, ref = 0;
  bool limited = false;
};

struct SGeom {
  uint32_t type = 0;  // 0 sphere, 1 capsule, 2 box, 3 plane, 4 cylinder, 5 mesh, 6 heightfield
  uint32_t body = 0;
  float pos[3] = {0, 0, 0};
  float quat[4] = {0, 0, 0, 1};
  float size[3] = {1, 1, 1};
  float friction = 1.0f, restitution = 0.0f;
  uint32_t contype = 0, conaffinity = 0xFFFFFFFFu;
};

struct SActuator {
  uint32_t joint = 0;
  float ctrl_min = -1.0f, ctrl_max = 1.0f;
  float force_min = -std::numeric_limits<float>::infinity();
  float force_max = std::numeric_limits<float>::infinity();
  float gear = 1.0f, kp = 0.0f, kv = 0.0f;
};

struct SSensor {
  uint32_t type = 0, object = 0, dim = 1;
  float noise = 0.0f, cutoff = 0.0f;
};

struct Scene {
  std::vector<SBody> bodies;
  std::vector<SJoint> joints;
  std::vector<SGeom> geoms;
  std::vector<SActuator> actuators;
  std::vector<SSensor> sensors;
  std::unordered_map<std::string, uint32_t> joint_by_name;
  float timestep = 0.002f;
  float gravity[3] = {0.0f, 0.0f, -9.81f};
  // constants.zig:6-42 PhysicsConfig defaults
  float friction = 1.0f, restitution = 0.0f, baumgarte = 0.2f, slop = 0.005f;
  bool corrected = false;  // loaded with corrected semantics (frames, angles, sensors)
  uint32_t obs_dim() const;
};

// Parse MJCF text.  `base_dir` resolves <include file="..."/> (parser.zig:55-171).
// corrected = false reproduces the reference loader, quirks included.  corrected = true
// applies the MJCF compiler rules the reference skips:
//  * <compiler angle> (default "degree") converts hinge/ball ranges and euler angles, and
//    <compiler eulerseq> (default "xyz"; lower case = moving axes) orders euler rotations;
//  * body frames compose with the parent's rotation: pos_w = p_parent + R_parent pos,
//    q_w = q_parent q_local (local quats normalised);
//  * joint pos and axis are child-frame quantities: anchor_parent = pos + R_local jpos,
//    axis (kept in the parent frame, as the constraints read it) = normalise(R_local axis);
//  * geoms keep their orientation: quat / euler attributes, and fromto capsules and
//    cylinders turn local +z onto the segment (shortest arc); their centre is the midpoint;
//  * body inertia sums each geom's principal inertia rotated into the body frame (the
//    diagonal is kept: the step carries a diagonal inverse inertia) plus the parallel-axis
//    term of the geom centre;
//  * frame and site sensors resolve objname (objtype body/xbody) or site to their body; the
//    automatic sensors observe the first child of the world instead of the world.
bool load_mjcf(const std::string& text, const std::string& base_dir, Scene* out, std::string* err,
               bool corrected = false);
bool load_mjcf_file(const std::string& path, Scene* out, std::string* err, bool corrected = false);

}  // namespace zb
