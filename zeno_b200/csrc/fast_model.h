// FModel: the whole model in one struct, passed to the environment-per-lane step kernel
// as a __grid_constant__ parameter.  Every lane of a warp runs the same model loop, so the
// loads are warp-uniform and the constant cache serves them as broadcasts.
//
// The struct has fixed capacities; pack_fast_model() reports models that do not fit (or
// that use features the kernel leaves to the general path) and World then runs the
// general kernel for them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace zb {

struct HostModel;

namespace fm {
constexpr uint32_t kB = 32, kJ = 32, kJF = 64, kK = 96, kG = 32, kP = 254, kH = 64, kA = 32, kS = 64;
constexpr uint32_t kNoHit = 127;  // hittable-index field of a candidate that never hits
constexpr uint32_t kNoPair = 255; // gg_pair entry for geom pairs that are not candidates
constexpr uint32_t kMaxSlots = 255;  // contact slots per env the per-slot byte fields can index
constexpr uint32_t kNoGroup = 0xFFu; // empty member of a constraint group
}  // namespace fm

struct FModel {
  // bodies
  float4 imi[fm::kB];     // 1/m, 1/Ixx, 1/Iyy, 1/Izz
  float4 com[fm::kB];     // centre-of-mass offset, body frame
  uint32_t body[fm::kB];  // type | jf_begin << 8 | jf_end << 16 | subtree size << 24
  uint8_t jf[fm::kJF];    // joint | 0x80 when the body is the joint's parent (joint order)
  // joints
  float4 j_ap[fm::kJ], j_ac[fm::kJ], j_axis[fm::kJ];
  uint32_t j_info[fm::kJ];  // type | parent << 8 | child << 16
  // constraints, colour-sorted (solving them one by one in this order equals solving
  // colour by colour: the constraints of one colour touch disjoint dynamic bodies)
  float4 c_aa[fm::kK], c_ab[fm::kK], c_at[fm::kK], c_lim[fm::kK];
  uint32_t c_info[fm::kK];  // body a | body b << 8 | type << 16
  // broad-phase candidates in emission order
  uint32_t p_info[fm::kP];  // ga | gb << 8 | hittable index << 16 (kNoHit) | key rank << 24
  uint32_t p_body[fm::kP];  // body a | body b << 8 | plane << 16
  float p_md2[fm::kP];      // ((r_a + r_b) + 0.1)^2
  // candidates whose geom types the narrow phase can report a contact for
  uint32_t h_pair[fm::kH];  // candidate index
  uint32_t h_info[fm::kH];  // type a | type b << 8 | body a << 16 | body b << 24
  float4 h_ga[fm::kH];      // geom a offset xyz, size[0]
  float4 h_gb[fm::kH];      // geom b offset xyz, size[0]
  float4 h_cax[fm::kH];     // capsule axis: +z rotated by the capsule's local quaternion (when one geom is a capsule)
  float h_hl[fm::kH];       // capsule half length (size[1])
  float4 h_sz[fm::kH];      // size[1], size[2] of geom a, size[1], size[2] of geom b
  float h_fr[fm::kH];       // combined friction sqrt(f_a * f_b)
  // geoms
  float4 g_ps[fm::kG];               // offset xyz, size[0]
  uint32_t g_body[fm::kG];
  uint8_t gg_pair[fm::kG * fm::kG];  // (ga, gb) -> candidate index, kNoPair otherwise
  // actuators
  uint32_t a_joint[fm::kA];
  float a_cmin[fm::kA], a_cmax[fm::kA], a_gear[fm::kA], a_fmin[fm::kA], a_fmax[fm::kA];
  // sensors
  uint32_t s_info[fm::kS];  // type | object << 8 | obs offset << 16
  uint32_t P, H, G;
  uint32_t n_capsule_plane;  // hittables [0, n) are capsule-plane pairs (reference narrow phase)
  uint32_t narrow_mode;  // 0: reference GPU narrow phase; 1: its CPU detectCollision
  // 1 when no two hittable candidates share a sort key (body pair): the warm-start match
  // of a hittable then reads only its own previous point, so one narrow-phase pass can
  // match and store (else a second pass stores once every match has read)
  uint32_t hit_keys_unique;
  // The tables read inside the substep loop, packed contiguously ("hot image"): the
  // kernel copies them into shared memory once per block, where warp-uniform reads are
  // broadcasts that never miss.  Byte offsets into the image (16-byte aligned sections):
  const uint4* hot;  // device copy of the image
  uint32_t hot_bytes;
  uint32_t o_imi, o_com, o_body, o_jf, o_jaxis, o_jinfo, o_caa, o_cab, o_cat, o_clim, o_cinfo;
  uint32_t o_pbody, o_pinfo, o_pmd2, o_gps, o_hinfo, o_hga, o_hgb, o_hcax, o_hhl, o_hfr, o_hpair, o_hsz;
  uint32_t o_gbody, o_ggpair;  // geom -> body (u32[G]), (ga, gb) -> candidate (u8[G * G])
  uint32_t o_gforce;           // float4[B], filled by each block: gravity * mass (zero when massless)
  uint32_t o_runs;             // u32[num_runs]: first constraint | count << 12 | type << 24
  uint32_t num_runs;
  // One iteration of the colour sweep for one lane per environment, as groups: a hinge's
  // point, axis and (when it acts) angle-limit constraints on one body pair, solved
  // together with the two bodies' poses kept in registers, or a single constraint.
  // k0 | k1 << 8 | k2 << 16 | kind << 24; kind 0: constraint k0 alone, 1: point k0 then
  // axis k1, 2: point k0, axis k1, limit k2.  The groups are a dependency-respecting order
  // of the sweep (hinge_groups in model.cpp).
  uint32_t o_groups;
  uint32_t num_groups;
  // The same groups by dependency level, for two lanes per environment (HostModel::
  // jgroup_levels): a level's groups touch disjoint dynamic bodies and are split across
  // the lanes.  u32[num_glv + 1] level starts, then the group words (packed as above) level
  // by level; num_glv 0 when a constraint index does not fit the packing (colour runs then).
  uint32_t o_glv, o_gwords;
  uint32_t num_glv;
};

// Fills *out and the hot image *hot (to be uploaded and linked through out->hot); false
// (with the reason in *why) when the model needs the general kernel.
bool pack_fast_model(const HostModel& h, uint32_t max_contacts, uint32_t narrow_mode, FModel* out,
                     std::vector<uint8_t>* hot, std::string* why);

}  // namespace zb
