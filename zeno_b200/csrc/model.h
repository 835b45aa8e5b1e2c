// Model building: Scene -> the read-only tables the step kernel uses, plus the
// reference-layout records (BodyDataGPU, JointDataGPU, GeomGPU, ActuatorDataGPU,
// SensorGPU, XPBDConstraint) exported for parity checks of the model itself.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "scene.h"
#include "zeno_types.h"

namespace zb {

struct HostModel {
  uint32_t B = 0, J = 0, A = 0, G = 0, S = 0, K = 0, obs_dim = 0, num_colors = 0;
  std::vector<DBody> bodies;
  std::vector<uint32_t> jf_list;
  std::vector<DJoint> joints;
  std::vector<DGeom> geoms;
  std::vector<DPair> pairs;
  // grid broad phase: per-geom distance-test radius, plane geoms, cell edge and buckets
  std::vector<float> geom_bound;
  std::vector<uint32_t> plane_geoms;
  float grid_inv_cell = 1.0f;
  uint32_t grid_buckets = 32;
  std::vector<DActuator> actuators;
  std::vector<DSensor> sensors;
  // Constraints the kernels solve: colour-sorted, without the angular limits no hinge angle
  // can reach (kcolor_ranges: their (start, count) per colour; K: their number).
  // color_ranges: the reference's ranges over every constraint (model parity tables).
  std::vector<DConstraint> constraints;
  std::vector<uint32_t> kcolor_ranges;
  std::vector<uint32_t> color_ranges;
  // Hinge groups (see hinge_groups in model.cpp): per group k0, k1, k2, kind (0 a single
  // constraint k0; 1 point k0 + axis k1; 2 point + axis + angle limit k2) in sweep order,
  // and for the general kernel the same groups by dependency level: jgroup_words holds
  // (k0 | k1 << 16, k2 | kind << 16) per group, level by level; jgroup_levels the start of
  // each level and the end (num_levels + 1 entries).
  std::vector<uint32_t> hinge_groups;
  std::vector<uint32_t> jgroup_words;
  std::vector<uint32_t> jgroup_levels;
  std::vector<uint32_t> subtree;
  std::vector<float> init_state;         // B*4 pos, B*4 quat, B*4 vel, B*4 angvel, J jpos, J jvel
  bool actuators_unique = true;
  bool corrected = false;  // corrected semantics: rotated geom frames and bounds, B->A normals
  // reference-layout records (byte blobs) for model parity checks
  std::vector<uint8_t> ref_bodies, ref_joints, ref_geoms, ref_actuators, ref_sensors, ref_constraints;
};

// Builds every table.  Fails (returns false, fills *err) for models the kernel cannot
// hold: more than 65535 bodies or geoms per environment (contact slots pack the body and
// geom indices into 16 bits each).  Whether an environment fits the step kernel's shared
// memory is decided when the world is created.
bool build_model(const Scene& sc, HostModel* m, std::string* err);

}  // namespace zb
