// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle for the batched physics step.
// Nothing in the product (zeno_b200/, include/) may include or link this file.
//
// LITERAL mode of the oracle: one substep of one environment written the way the
// reference's Metal kernels write it (src/shaders/all_shaders.metal), statement by
// statement, in plain IEEE-754 single precision:
//   * +, -, *, / each correctly rounded, evaluated left to right as written; no fused
//     multiply-add anywhere (the file is compiled with -ffp-contract=off and calls no fmaf);
//   * length(v) = sqrtf(dot(v, v)), normalize-by-division v / length(v), and the MSL
//     builtins atan2 / asin / sqrt as libm's atan2f / asinf / sqrtf;
//   * dot(a, b) = a.x*b.x + a.y*b.y + a.z*b.z (+ a.w*b.w), cross(a, b) = a.yzx*b.zxy -
//     a.zxy*b.yzx, and quat_multiply / rotate_by_quat as written at all_shaders.metal:76-97;
//   * unsuffixed MSL literals (0.999, 0.5, 2.0, 1e-8 ...) are single precision, as Metal
//     has no double type.
// The file is compiled twice (Makefile): as written above, giving substep_env_literal,
// and with -ffp-contract=fast, giving substep_env_literal_contracted: the same expressions
// with products and sums fused into FMAs wherever the compiler chooses, one of the rewrites
// the Metal compiler's default fast-math compilation of the reference kernels makes.  The
// distance between the two is the spread of the reference's own source under two legitimate
// compilations, the yardstick for the canonical arithmetic's distance from either.
// It shares nothing with the canonical arithmetic of oracle_math.h (Newton-Raphson
// reciprocals, explicit FMAs, fitted arctangent) that the product kernel and the
// canonical oracle evaluate bit for bit; it exists to bound how far that canonical
// arithmetic lies from the reference's own arithmetic (the tolerance tests in tests/).
// Model set-up (loader, templates, colouring) and the host parts of World.step are the
// oracle's own, which are integer/table work pinned to the reference's known answers.
//
// Stages that race in the reference get the same serial order as the canonical oracle:
// broad-phase emission geom a ascending then b ascending; apply_joint_forces summed per
// body in joint order; solve_contacts slot by slot.  Only the reference semantics are
// restated (not the corrected-semantics mode); the extended narrow phases (modes 1, 2)
// call the oracle's restatement of the reference CPU collision code, whose arithmetic is
// already the Zig source's plain IEEE arithmetic.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "oracle_model.h"

#ifndef ZO_LITERAL_NS
#define ZO_LITERAL_NS lit
#endif

namespace zo {
namespace ZO_LITERAL_NS {

struct V3 {
  float x, y, z;
};
struct Q4 {
  float x, y, z, w;
};

inline V3 operator+(V3 a, V3 b) { return V3{a.x + b.x, a.y + b.y, a.z + b.z}; }
inline V3 operator-(V3 a, V3 b) { return V3{a.x - b.x, a.y - b.y, a.z - b.z}; }
inline V3 operator-(V3 a) { return V3{-a.x, -a.y, -a.z}; }
inline V3 operator*(V3 a, float s) { return V3{a.x * s, a.y * s, a.z * s}; }
inline V3 operator*(float s, V3 a) { return V3{s * a.x, s * a.y, s * a.z}; }
inline V3 operator*(V3 a, V3 b) { return V3{a.x * b.x, a.y * b.y, a.z * b.z}; }
inline V3 operator/(V3 a, float s) { return V3{a.x / s, a.y / s, a.z / s}; }
inline Q4 operator+(Q4 a, Q4 b) { return Q4{a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w}; }
inline Q4 operator-(Q4 a, Q4 b) { return Q4{a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w}; }
inline Q4 operator-(Q4 a) { return Q4{-a.x, -a.y, -a.z, -a.w}; }
inline Q4 operator*(Q4 a, float s) { return Q4{a.x * s, a.y * s, a.z * s, a.w * s}; }
inline Q4 operator/(Q4 a, float s) { return Q4{a.x / s, a.y / s, a.z / s, a.w / s}; }

inline float dot(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline float dot4(Q4 a, Q4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
inline float length(V3 a) { return std::sqrt(dot(a, a)); }
inline float length4(Q4 a) { return std::sqrt(dot4(a, a)); }
inline V3 cross(V3 a, V3 b) {
  return V3{a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}

// all_shaders.metal:76-83
inline Q4 quat_multiply(Q4 a, Q4 b) {
  return Q4{a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y, a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
            a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w, a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z};
}
// all_shaders.metal:85-87
inline Q4 quat_conjugate(Q4 q) { return Q4{-q.x, -q.y, -q.z, q.w}; }
// all_shaders.metal:89-94: v + 2.0 * (q.w * uv + uuv)
inline V3 rotate_by_quat(V3 v, Q4 q) {
  V3 qv{q.x, q.y, q.z};
  V3 uv = cross(qv, v);
  V3 uuv = cross(qv, uv);
  return v + 2.0f * (q.w * uv + uuv);
}
// all_shaders.metal:96-99
inline Q4 quat_normalize(Q4 q) {
  float len = length4(q);
  return len > 1e-8f ? q / len : Q4{0, 0, 0, 1};
}
inline Q4 qv(V3 v, float w) { return Q4{v.x, v.y, v.z, w}; }

inline V3 ld3(const float* p) { return V3{p[0], p[1], p[2]}; }
inline Q4 ld4(const float* p) { return Q4{p[0], p[1], p[2], p[3]}; }
inline void st3(float* p, V3 v) {
  p[0] = v.x;
  p[1] = v.y;
  p[2] = v.z;
}
inline void st4(float* p, Q4 v) {
  p[0] = v.x;
  p[1] = v.y;
  p[2] = v.z;
  p[3] = v.w;
}
inline void st3w0(float* p, V3 v) { st4(p, Q4{v.x, v.y, v.z, 0.0f}); }
inline float clampf(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }

inline uint32_t pair_key(uint32_t a, uint32_t b) {
  uint32_t lo = a < b ? a : b, hi = a < b ? b : a;
  return (lo << 16) | hi;
}

}  // namespace ZO_LITERAL_NS

// One substep of environment e, kernels in the dispatch order of stepOnce
// (src/world/world.zig:934-1293).
#ifndef ZO_LITERAL_FN
#define ZO_LITERAL_FN substep_env_literal
#endif
void ZO_LITERAL_FN(World* w, uint32_t e) {
  using namespace ZO_LITERAL_NS;
  const Params& P = w->params;
  const uint32_t B = w->B, J = w->J, A = w->A, G = w->G, M = w->M, K = w->K;
  const float dt = P.dt;
  float* pos = &w->pos[size_t(e) * B * 4];
  float* quat = &w->quat[size_t(e) * B * 4];
  float* vel = &w->vel[size_t(e) * B * 4];
  float* ang = &w->angvel[size_t(e) * B * 4];
  float* frc = &w->force[size_t(e) * B * 4];
  float* trq = &w->torque[size_t(e) * B * 4];
  const float* imi = &w->inv_mi[size_t(e) * B * 4];
  float* ppos = &w->prev_pos[size_t(e) * B * 4];
  float* pquat = &w->prev_quat[size_t(e) * B * 4];
  float* jt = &w->jtorque[size_t(e) * std::max(J, 1u)];
  const float* act = &w->actions[size_t(e) * std::max(A, 1u)];
  ContactRec* con = &w->contacts[size_t(e) * M];
  ContactRec* prev = &w->prev_contacts[size_t(e) * M];
  ConstraintRec* cst = K ? &w->constraints[size_t(e) * K] : nullptr;

  // warm_start_constraints (all_shaders.metal:1408-1426) with factor 0.8 (world.zig:477-478)
  for (uint32_t k = 0; k < K; k++) cst[k].state[0] = 0.8f * cst[k].state[1];

  // apply_actions (all_shaders.metal:196-229)
  for (uint32_t a = 0; a < A; a++) {
    const ActuatorRec& ar = w->actuators[a];
    uint32_t jid = uint32_t(ar.params[0]);
    float ctrl = act[a];
    ctrl = clampf(ctrl, ar.params[1], ar.params[2]);
    float torque = ctrl * ar.params[3];
    torque = clampf(torque, ar.params2[0], ar.params2[1]);
    jt[jid] = torque;
  }

  // compute_forces (all_shaders.metal:345-388)
  const V3 gravity{P.gravity[0], P.gravity[1], P.gravity[2]};
  for (uint32_t b = 0; b < B; b++) {
    Q4 inv_mi = ld4(&imi[b * 4]);
    float inv_mass = inv_mi.x;
    if (inv_mass < 1e-8f) {
      st4(&frc[b * 4], Q4{0, 0, 0, 0});
      st4(&trq[b * 4], Q4{0, 0, 0, 0});
      continue;
    }
    float mass = 1.0f / inv_mass;
    V3 force = gravity * mass;
    st3w0(&frc[b * 4], force);
    V3 com_world = rotate_by_quat(ld3(w->bodies[b].com_offset), ld4(&quat[b * 4]));
    st3w0(&trq[b * 4], cross(com_world, force));
  }

  // update_kinematic (all_shaders.metal:304-339): body type 1 only
  for (uint32_t b = 0; b < B; b++) {
    if (uint32_t(w->bodies[b].params[1]) != 1) continue;
    V3 p = ld3(&pos[b * 4]);
    p = p + ld3(&vel[b * 4]) * dt;
    st3w0(&pos[b * 4], p);
    V3 omega = ld3(&ang[b * 4]);
    Q4 q = ld4(&quat[b * 4]);
    Q4 dq = quat_multiply(qv(omega * dt * 0.5f, 0.0f), q);
    st4(&quat[b * 4], quat_normalize(q + dq));
  }

  // apply_joint_forces (all_shaders.metal:122-190); the atomic adds of one body are
  // summed in joint order (f_old + val, val = -component for body a)
  for (uint32_t j = 0; j < J; j++) {
    float applied = jt[j];
    if (std::fabs(applied) < 1e-6f) continue;
    const JointRec& jr = w->joints[j];
    uint32_t type = uint32_t(jr.params[0]);
    uint32_t ba = uint32_t(jr.params[1]), bb = uint32_t(jr.params[2]);
    V3 axis_world = rotate_by_quat(ld3(jr.axis), ld4(&quat[ba * 4]));
    V3 f = axis_world * applied;
    float* tgt = type == 2 ? frc : trq;
    if (ba > 0) {
      tgt[ba * 4 + 0] = tgt[ba * 4 + 0] + -f.x;
      tgt[ba * 4 + 1] = tgt[ba * 4 + 1] + -f.y;
      tgt[ba * 4 + 2] = tgt[ba * 4 + 2] + -f.z;
    }
    if (bb > 0) {
      tgt[bb * 4 + 0] = tgt[bb * 4 + 0] + f.x;
      tgt[bb * 4 + 1] = tgt[bb * 4 + 1] + f.y;
      tgt[bb * 4 + 2] = tgt[bb * 4 + 2] + f.z;
    }
  }

  // save_prev_state (all_shaders.metal:1900-1913)
  std::memcpy(ppos, pos, sizeof(float) * 4 * B);
  std::memcpy(pquat, quat, sizeof(float) * 4 * B);

  // integrate (all_shaders.metal:394-462)
  for (uint32_t b = 0; b < B; b++) {
    Q4 inv_mi = ld4(&imi[b * 4]);
    float inv_mass = inv_mi.x;
    if (inv_mass < 1e-8f) continue;
    V3 force = ld3(&frc[b * 4]);
    V3 v = ld3(&vel[b * 4]);
    V3 p = ld3(&pos[b * 4]);
    V3 accel = force * inv_mass;
    v = v + accel * dt;
    v = v * 0.999f;
    p = p + v * dt;
    st3w0(&vel[b * 4], v);
    st3w0(&pos[b * 4], p);
    V3 inv_inertia{inv_mi.y, inv_mi.z, inv_mi.w};
    V3 torque = ld3(&trq[b * 4]);
    V3 omega = ld3(&ang[b * 4]);
    Q4 q = ld4(&quat[b * 4]);
    omega = omega + inv_inertia * torque * dt;
    omega = omega * 0.999f;
    Q4 dq = quat_multiply(qv(omega * dt * 0.5f, 0.0f), q);
    q = q + dq;
    float qlen = length4(q);
    if (qlen > 1e-8f) q = q / qlen;
    else q = Q4{0, 0, 0, 1};
    st3w0(&ang[b * 4], omega);
    st4(&quat[b * 4], q);
  }

  // broad_phase, all pairs (all_shaders.metal:468-533)
  uint32_t& count = w->counts[e];
  for (uint32_t ga = 0; ga < G; ga++) {
    const GeomRec& A_ = w->geoms[ga];
    uint32_t body_a = A_.type_body[1];
    V3 pos_a = ld3(&pos[body_a * 4]) + ld3(A_.pos_size0);
    float radius_a = A_.pos_size0[3];
    uint32_t type_a = A_.type_body[0], group_a = A_.type_body[3], mask_a = A_.type_body[2];
    for (uint32_t gb = ga + 1; gb < G; gb++) {
      const GeomRec& B_ = w->geoms[gb];
      uint32_t body_b = B_.type_body[1];
      if (body_a == body_b) continue;
      uint32_t type_b = B_.type_body[0], group_b = B_.type_body[3], mask_b = B_.type_body[2];
      if ((group_a & mask_b) == 0 && (group_b & mask_a) == 0) continue;
      V3 pos_b = ld3(&pos[body_b * 4]) + ld3(B_.pos_size0);
      float radius_b = B_.pos_size0[3];
      bool is_plane_pair = type_a == 3 || type_b == 3;
      if (!is_plane_pair) {
        V3 diff = pos_b - pos_a;
        float dist_sq = dot(diff, diff);
        float min_dist = radius_a + radius_b + 0.1f;
        if (dist_sq >= min_dist * min_dist) continue;
      }
      uint32_t c = count++;
      if (c < M) {
        con[c].indices[0] = body_a;
        con[c].indices[1] = body_b;
        con[c].indices[2] = ga;
        con[c].indices[3] = gb;
      }
    }
  }

  // sort_contacts (all_shaders.metal:711-745)
  const uint32_t n = std::min(count, M);
  for (uint32_t i = 1; i < n; i++) {
    ContactRec key = con[i];
    uint32_t key_val = pair_key(key.indices[0], key.indices[1]);
    int j = int(i) - 1;
    while (j >= 0) {
      if (pair_key(con[j].indices[0], con[j].indices[1]) <= key_val) break;
      con[j + 1] = con[j];
      j--;
    }
    con[j + 1] = key;
  }

  // narrow_phase (all_shaders.metal:751-894)
  for (uint32_t i = 0; i < n; i++) {
    ContactRec& c = con[i];
    uint32_t body_a = c.indices[0], body_b = c.indices[1];
    const GeomRec& geom_a = w->geoms[c.indices[2]];
    const GeomRec& geom_b = w->geoms[c.indices[3]];
    if (w->narrow_mode >= 1) {  // the reference CPU collision code (already plain IEEE)
      float pt[3], nm[3], pen = 0.0f;
      bool hit = narrow_cpu(geom_a, &pos[body_a * 4], &quat[body_a * 4], geom_b, &pos[body_b * 4],
                            &quat[body_b * 4], pt, nm, &pen, w->narrow_mode == 2);
      if (hit) {
        float fr = std::sqrt(geom_a.params[2] * geom_b.params[2]);
        st4(c.position_pen, Q4{pt[0], pt[1], pt[2], pen});
        st4(c.normal_friction, Q4{nm[0], nm[1], nm[2], fr});
        st4(c.impulses, Q4{0, 0, 0, P.restitution});
      } else {
        c.position_pen[3] = -1.0f;
      }
      continue;
    }
    V3 pos_a = ld3(&pos[body_a * 4]) + ld3(geom_a.pos_size0);
    V3 pos_b = ld3(&pos[body_b * 4]) + ld3(geom_b.pos_size0);
    uint32_t type_a = geom_a.type_body[0], type_b = geom_b.type_body[0];
    V3 normal{0, 0, 0}, contact_point{0, 0, 0};
    float penetration = 0.0f;
    bool has_contact = false;
    if (type_a == 0 && type_b == 0) {
      float radius_a = geom_a.pos_size0[3], radius_b = geom_b.pos_size0[3];
      V3 diff = pos_b - pos_a;
      float dist = length(diff);
      float min_dist = radius_a + radius_b;
      if (dist < min_dist && dist > 1e-6f) {
        normal = diff / dist;
        penetration = min_dist - dist;
        contact_point = pos_a + normal * (radius_a - penetration * 0.5f);
        has_contact = true;
      }
    } else if ((type_a == 0 && type_b == 3) || (type_a == 3 && type_b == 0)) {
      V3 sphere_pos = type_a == 0 ? pos_a : pos_b;
      float sphere_radius = type_a == 0 ? geom_a.pos_size0[3] : geom_b.pos_size0[3];
      V3 plane_pos = type_a == 0 ? pos_b : pos_a;
      V3 plane_normal{0, 0, 1};
      float signed_dist = dot(sphere_pos - plane_pos, plane_normal);
      if (signed_dist < sphere_radius) {
        normal = plane_normal;
        penetration = sphere_radius - signed_dist;
        contact_point = sphere_pos - plane_normal * (signed_dist + penetration * 0.5f);
        has_contact = true;
        if (type_a == 3) normal = -normal;
      }
    } else if ((type_a == 1 && type_b == 3) || (type_a == 3 && type_b == 1)) {
      const GeomRec& cg = type_a == 1 ? geom_a : geom_b;
      V3 capsule_pos = type_a == 1 ? pos_a : pos_b;
      float capsule_radius = cg.pos_size0[3], capsule_half_len = cg.params[0];
      V3 plane_normal{0, 0, 1};
      V3 axis = rotate_by_quat(V3{0, 0, 1}, ld4(cg.quat));
      V3 p1 = capsule_pos - axis * capsule_half_len;
      V3 p2 = capsule_pos + axis * capsule_half_len;
      float d1 = p1.z - capsule_radius;
      float d2 = p2.z - capsule_radius;
      if (d1 < 0 || d2 < 0) {
        V3 deepest = d1 < d2 ? p1 : p2;
        float dist = std::fmin(d1, d2);
        normal = type_a == 1 ? plane_normal : -plane_normal;
        penetration = -dist;
        contact_point = deepest;
        contact_point.z = 0;
        has_contact = true;
      }
    }
    if (has_contact) {
      float combined_friction = std::sqrt(geom_a.params[2] * geom_b.params[2]);
      st4(c.position_pen, Q4{contact_point.x, contact_point.y, contact_point.z, penetration});
      st4(c.normal_friction, Q4{normal.x, normal.y, normal.z, combined_friction});
      st4(c.impulses, Q4{0, 0, 0, P.restitution});
    } else {
      c.position_pen[3] = -1.0f;
    }
  }

  // match_cached_contacts (all_shaders.metal:1483-1544)
  const uint32_t prev_count = w->prev_counts[e];
  for (uint32_t i = 0; i < n; i++) {
    ContactRec& c = con[i];
    if (c.position_pen[3] < 0) continue;
    uint32_t body_a = c.indices[0], body_b = c.indices[1];
    V3 p = ld3(c.position_pen);
    float best_dist_sq = 0.04f;
    int best_match = -1;
    for (uint32_t k = 0; k < prev_count && k < M; k++) {
      const ContactRec& q = prev[k];
      if (q.position_pen[3] < 0) continue;
      bool same_pair = (q.indices[0] == body_a && q.indices[1] == body_b) ||
                       (q.indices[0] == body_b && q.indices[1] == body_a);
      if (!same_pair) continue;
      V3 diff = ld3(q.position_pen) - p;
      float dist_sq = dot(diff, diff);
      if (dist_sq < best_dist_sq) {
        best_dist_sq = dist_sq;
        best_match = int(k);
      }
    }
    if (best_match >= 0) {
      c.impulses[0] = prev[best_match].impulses[0] * 0.8f;
      c.impulses[1] = prev[best_match].impulses[1] * 0.8f;
      c.impulses[2] = prev[best_match].impulses[2] * 0.8f;
    }
  }

  // solve_joints (all_shaders.metal:909-1399), colour by colour (world.zig:1163-1195).
  // Within a colour the constraints of one environment touch disjoint bodies, so the
  // per-thread order inside a colour does not change the result.
  for (uint32_t it = 0; it < P.contact_iterations; it++) {
    for (uint32_t col = 0; col < w->num_colors; col++) {
      const uint32_t off = w->color_ranges[2 * col], cnt = w->color_ranges[2 * col + 1];
      for (uint32_t li = 0; li < cnt; li++) {
        ConstraintRec& c = cst[off + li];
        const uint32_t type = c.indices[3] & 0xFF;
        if (type > 10) continue;
        const uint32_t ia = c.indices[0], ib = c.indices[1];
        const Q4 inv_mi_a = ld4(&imi[ia * 4]), inv_mi_b = ld4(&imi[ib * 4]);
        const V3 Ia{inv_mi_a.y, inv_mi_a.z, inv_mi_a.w}, Ib{inv_mi_b.y, inv_mi_b.z, inv_mi_b.w};
        const float inv_mass_a = inv_mi_a.x, inv_mass_b = inv_mi_b.x;
        const float inv_mass_sum = inv_mass_a + inv_mass_b;
        if (inv_mass_sum < 1e-8f) continue;
        const V3 pos_a = ld3(&pos[ia * 4]), pos_b = ld3(&pos[ib * 4]);
        const Q4 quat_a = ld4(&quat[ia * 4]), quat_b = ld4(&quat[ib * 4]);
        const float compliance = c.anchor_a[3];
        const float alpha_tilde = compliance / (dt * dt);
        if (type == 2) {  // positional (all_shaders.metal:979-1030)
          V3 r_a = rotate_by_quat(ld3(c.anchor_a), quat_a);
          V3 r_b = rotate_by_quat(ld3(c.anchor_b), quat_b);
          V3 diff = (pos_a + r_a) - (pos_b + r_b);
          float C = length(diff);
          if (C > 1e-6f) {
            V3 nn = diff / C;
            V3 rn_a = cross(r_a, nn), rn_b = cross(r_b, nn);
            float w_a = inv_mass_a + dot(rn_a * Ia, rn_a);
            float w_b = inv_mass_b + dot(rn_b * Ib, rn_b);
            float wsum = w_a + w_b;
            float lambda_prev = c.state[0];
            float d_lambda = (-C - alpha_tilde * lambda_prev) / (wsum + alpha_tilde);
            c.state[0] = lambda_prev + d_lambda;
            V3 impulse = d_lambda * nn;
            V3 rc_a = r_a - rotate_by_quat(ld3(w->bodies[ia].com_offset), quat_a);
            V3 rc_b = r_b - rotate_by_quat(ld3(w->bodies[ib].com_offset), quat_b);
            if (inv_mass_a > 0) {
              st3(&pos[ia * 4], ld3(&pos[ia * 4]) + impulse * inv_mass_a);
              V3 d_omega = cross(rc_a, impulse) * Ia;
              Q4 dq = quat_multiply(qv(d_omega, 0), quat_a) * 0.5f;
              st4(&quat[ia * 4], quat_normalize(quat_a + dq));
            }
            if (inv_mass_b > 0) {
              st3(&pos[ib * 4], ld3(&pos[ib * 4]) - impulse * inv_mass_b);
              V3 d_omega = cross(rc_b, impulse) * Ib;
              Q4 dq = quat_multiply(qv(d_omega, 0), quat_b) * 0.5f;
              st4(&quat[ib * 4], quat_normalize(quat_b - dq));
            }
          }
        } else if (type == 7) {  // weld, body b only (all_shaders.metal:1032-1113)
          V3 r_a = rotate_by_quat(ld3(c.anchor_a), quat_a);
          V3 r_b = rotate_by_quat(ld3(c.anchor_b), quat_b);
          V3 diff = (pos_a + r_a) - (pos_b + r_b);
          float C = length(diff);
          if (C > 1e-6f) {
            V3 nn = diff / C;
            V3 rn_b = cross(r_b, nn);
            float w_b = inv_mass_b + dot(rn_b * Ib, rn_b);
            if (w_b > 1e-8f) {
              float d_lambda = (-C) / (w_b + alpha_tilde);
              V3 impulse = d_lambda * nn;
              st3(&pos[ib * 4], ld3(&pos[ib * 4]) - impulse * inv_mass_b);
              V3 d_omega = cross(r_b, impulse) * Ib;
              Q4 dq = quat_multiply(qv(d_omega, 0), quat_b) * 0.5f;
              st4(&quat[ib * 4], quat_normalize(quat_b - dq));
            }
          }
          Q4 q_rel_target = ld4(c.axis_target);
          Q4 quat_a_upd = ld4(&quat[ia * 4]), quat_b_upd = ld4(&quat[ib * 4]);
          Q4 q_rel = quat_multiply(quat_conjugate(quat_a_upd), quat_b_upd);
          Q4 q_err = quat_multiply(q_rel, quat_conjugate(q_rel_target));
          if (q_err.w < 0) q_err = -q_err;
          V3 q_err_xyz{q_err.x, q_err.y, q_err.z};
          float sin_half_angle = length(q_err_xyz);
          if (sin_half_angle > 1e-6f) {
            V3 axis_rel = q_err_xyz / sin_half_angle;
            float angle = 2.0f * std::atan2(sin_half_angle, q_err.w);
            V3 axis_world = rotate_by_quat(axis_rel, quat_a_upd);
            float w_b = dot(axis_world * Ib, axis_world);
            if (w_b > 1e-8f) {
              float d_lambda_ang = angle / (w_b + alpha_tilde);
              V3 ang_impulse = d_lambda_ang * axis_world;
              if (inv_mass_b > 0) {
                V3 d_omega = ang_impulse * Ib;
                Q4 dq = quat_multiply(qv(d_omega, 0), quat_b_upd) * 0.5f;
                st4(&quat[ib * 4], quat_normalize(quat_b_upd - dq));
              }
            }
          }
        } else if (type == 3) {  // angular / hinge alignment (all_shaders.metal:1116-1187)
          Q4 quat_a_curr = ld4(&quat[ia * 4]), quat_b_curr = ld4(&quat[ib * 4]);
          V3 axis_a_world = rotate_by_quat(ld3(c.anchor_a), quat_a_curr);
          V3 axis_b_world = rotate_by_quat(ld3(c.anchor_b), quat_b_curr);
          V3 cross_ab = cross(axis_a_world, axis_b_world);
          float sin_angle = length(cross_ab);
          if (sin_angle > 1e-6f) {
            V3 nn = cross_ab / sin_angle;
            float ang_C = std::asin(clampf(sin_angle, -1.0f, 1.0f));
            float w_a = dot(nn * Ia, nn);
            float w_b = dot(nn * Ib, nn);
            float wsum = w_a + w_b;
            if (wsum > 1e-8f) {
              float d_lambda = -ang_C / (wsum + alpha_tilde);
              if (inv_mass_a > 0) {
                V3 d_omega_a = d_lambda * nn * Ia;
                Q4 dq = quat_multiply(qv(d_omega_a, 0), quat_a_curr) * 0.5f;
                st4(&quat[ia * 4], quat_normalize(quat_a_curr + dq));
              }
              if (inv_mass_b > 0) {
                V3 d_omega_b = -d_lambda * nn * Ib;
                Q4 dq = quat_multiply(qv(d_omega_b, 0), quat_b_curr) * 0.5f;
                st4(&quat[ib * 4], quat_normalize(quat_b_curr + dq));
              }
            }
          }
        } else if (type == 4) {  // angular limit (all_shaders.metal:1189-1240)
          V3 axis_local = ld3(c.anchor_a);
          float lower = c.limits[0], upper = c.limits[1];
          Q4 quat_a_curr = ld4(&quat[ia * 4]), quat_b_curr = ld4(&quat[ib * 4]);
          Q4 q_rel = quat_multiply(quat_conjugate(quat_a_curr), quat_b_curr);
          float sin_half = dot(V3{q_rel.x, q_rel.y, q_rel.z}, axis_local);
          float angle = 2.0f * std::atan2(sin_half, q_rel.w);
          float violation = 0.0f;
          if (angle < lower) violation = lower - angle;
          else if (angle > upper) violation = upper - angle;
          if (std::fabs(violation) > 1e-6f) {
            V3 axis_world = rotate_by_quat(axis_local, quat_a_curr);
            float w_a = dot(axis_world * Ia, axis_world);
            float w_b = dot(axis_world * Ib, axis_world);
            float wsum = w_a + w_b;
            if (wsum > 1e-8f) {
              float d_lambda = violation / (wsum + alpha_tilde);
              V3 ang_impulse = d_lambda * axis_world;
              if (inv_mass_a > 0) {
                V3 d_omega = ang_impulse * Ia;
                Q4 dq = quat_multiply(qv(d_omega, 0), quat_a_curr) * 0.5f;
                st4(&quat[ia * 4], quat_normalize(quat_a_curr + dq));
              }
              if (inv_mass_b > 0) {
                V3 d_omega = ang_impulse * Ib;
                Q4 dq = quat_multiply(qv(d_omega, 0), quat_b_curr) * 0.5f;
                st4(&quat[ib * 4], quat_normalize(quat_b_curr - dq));
              }
            }
          }
        } else if (type == 5) {  // linear limit (all_shaders.metal:1242-1296)
          V3 axis_local = ld3(c.anchor_a);
          float lower = c.limits[0], upper = c.limits[1];
          Q4 quat_a_curr = ld4(&quat[ia * 4]), quat_b_curr = ld4(&quat[ib * 4]);
          V3 r_a = rotate_by_quat(V3{0, 0, 0}, quat_a_curr);
          V3 r_b = rotate_by_quat(ld3(c.anchor_b), quat_b_curr);
          V3 axis_world = rotate_by_quat(axis_local, quat_a_curr);
          V3 diff = (pos_b + r_b) - (pos_a + r_a);
          float dist = dot(diff, axis_world);
          float violation = 0.0f;
          if (dist < lower) violation = lower - dist;
          else if (dist > upper) violation = upper - dist;
          if (std::fabs(violation) > 1e-6f) {
            V3 nn = violation > 0 ? axis_world : -axis_world;
            float abs_violation = std::fabs(violation);
            V3 rn_a = cross(r_a, nn), rn_b = cross(r_b, nn);
            float w_a = inv_mass_a + dot(rn_a * Ia, rn_a);
            float w_b = inv_mass_b + dot(rn_b * Ib, rn_b);
            float wsum = w_a + w_b;
            if (wsum > 1e-8f) {
              float d_lambda = abs_violation / (wsum + alpha_tilde);
              V3 impulse = d_lambda * nn;
              if (inv_mass_a > 0) st3(&pos[ia * 4], ld3(&pos[ia * 4]) - impulse * inv_mass_a);
              if (inv_mass_b > 0) st3(&pos[ib * 4], ld3(&pos[ib * 4]) + impulse * inv_mass_b);
            }
          }
        } else if (type == 10) {  // slider (all_shaders.metal:1298-1393)
          V3 r_a = rotate_by_quat(ld3(c.anchor_a), quat_a);
          V3 r_b = rotate_by_quat(ld3(c.anchor_b), quat_b);
          V3 diff = (pos_a + r_a) - (pos_b + r_b);
          V3 axis_world = rotate_by_quat(ld3(c.axis_target), quat_a);
          float along = dot(diff, axis_world);
          V3 perp = diff - along * axis_world;
          float perp_len = length(perp);
          if (perp_len > 1e-6f) {
            V3 nn = perp / perp_len;
            V3 rn_a = cross(r_a, nn), rn_b = cross(r_b, nn);
            float w_a = inv_mass_a + dot(rn_a * Ia, rn_a);
            float w_b = inv_mass_b + dot(rn_b * Ib, rn_b);
            float wsum = w_a + w_b;
            float d_lambda = (-perp_len) / (wsum + alpha_tilde);
            V3 impulse = d_lambda * nn;
            if (inv_mass_a > 0) {
              st3(&pos[ia * 4], ld3(&pos[ia * 4]) + impulse * inv_mass_a);
              V3 d_omega = cross(r_a, impulse) * Ia;
              Q4 dq = quat_multiply(qv(d_omega, 0), quat_a) * 0.5f;
              st4(&quat[ia * 4], quat_normalize(quat_a + dq));
            }
            if (inv_mass_b > 0) {
              st3(&pos[ib * 4], ld3(&pos[ib * 4]) - impulse * inv_mass_b);
              V3 d_omega = cross(r_b, impulse) * Ib;
              Q4 dq = quat_multiply(qv(d_omega, 0), quat_b) * 0.5f;
              st4(&quat[ib * 4], quat_normalize(quat_b - dq));
            }
          }
          Q4 q_rel_target = ld4(c.limits);
          Q4 quat_a_upd = ld4(&quat[ia * 4]), quat_b_upd = ld4(&quat[ib * 4]);
          Q4 q_rel = quat_multiply(quat_conjugate(quat_a_upd), quat_b_upd);
          Q4 q_err = quat_multiply(q_rel, quat_conjugate(q_rel_target));
          if (q_err.w < 0) q_err = -q_err;
          V3 q_err_xyz{q_err.x, q_err.y, q_err.z};
          float sin_half_angle = length(q_err_xyz);
          if (sin_half_angle > 1e-6f) {
            V3 axis_err = q_err_xyz / sin_half_angle;
            float angle_err = 2.0f * std::atan2(sin_half_angle, q_err.w);
            V3 axis_err_world = rotate_by_quat(axis_err, quat_a_upd);
            float w_a = dot(axis_err_world * Ia, axis_err_world);
            float w_b = dot(axis_err_world * Ib, axis_err_world);
            float wsum = w_a + w_b;
            if (wsum > 1e-8f) {
              float d_lambda_ang = angle_err / (wsum + alpha_tilde);
              V3 ang_impulse = d_lambda_ang * axis_err_world;
              if (inv_mass_a > 0) {
                V3 d_omega = ang_impulse * Ia;
                Q4 dq = quat_multiply(qv(d_omega, 0), quat_a_upd) * 0.5f;
                st4(&quat[ia * 4], quat_normalize(quat_a_upd + dq));
              }
              if (inv_mass_b > 0) {
                V3 d_omega = ang_impulse * Ib;
                Q4 dq = quat_multiply(qv(d_omega, 0), quat_b_upd) * 0.5f;
                st4(&quat[ib * 4], quat_normalize(quat_b_upd - dq));
              }
            }
          }
        }
      }
    }
  }

  // solve_contacts (all_shaders.metal:1644-1793), slot by slot
  for (uint32_t it = 0; it < P.contact_iterations; it++) {
    for (uint32_t i = 0; i < n; i++) {
      ContactRec& c = con[i];
      if (c.position_pen[3] < 0) continue;
      const uint32_t ia = c.indices[0], ib = c.indices[1];
      const Q4 inv_mi_a = ld4(&imi[ia * 4]), inv_mi_b = ld4(&imi[ib * 4]);
      const V3 Ia{inv_mi_a.y, inv_mi_a.z, inv_mi_a.w}, Ib{inv_mi_b.y, inv_mi_b.z, inv_mi_b.w};
      const float inv_mass_a = inv_mi_a.x, inv_mass_b = inv_mi_b.x;
      const float inv_mass_sum = inv_mass_a + inv_mass_b;
      if (inv_mass_sum < 1e-8f) continue;
      V3 normal = ld3(c.normal_friction);
      float penetration = c.position_pen[3];
      float friction = c.normal_friction[3];
      V3 contact_point = ld3(c.position_pen);
      V3 pos_a = ld3(&pos[ia * 4]), pos_b = ld3(&pos[ib * 4]);
      V3 r_a = contact_point - pos_a;
      V3 r_b = contact_point - pos_b;
      V3 omega_a = ld3(&ang[ia * 4]), omega_b = ld3(&ang[ib * 4]);
      V3 vel_a = ld3(&vel[ia * 4]) + cross(omega_a, r_a);
      V3 vel_b = ld3(&vel[ib * 4]) + cross(omega_b, r_b);
      V3 rel_vel = vel_a - vel_b;
      float vel_normal = dot(rel_vel, normal);
      V3 vel_tangent = rel_vel - vel_normal * normal;
      float tangent_speed = length(vel_tangent);
      V3 rn_a = cross(r_a, normal), rn_b = cross(r_b, normal);
      float w_n_a = inv_mass_a + dot(rn_a * Ia, rn_a);
      float w_n_b = inv_mass_b + dot(rn_b * Ib, rn_b);
      float w_normal = w_n_a + w_n_b;
      if (w_normal < 1e-8f) continue;
      float bias = P.baumgarte * std::fmax(penetration - P.slop, 0.0f) / dt;
      float restitution = c.impulses[3];
      float vel_restitution = vel_normal < -0.5f ? restitution * vel_normal : 0.0f;
      float j_n = (-(vel_normal + vel_restitution) + bias) / w_normal;
      j_n = std::fmax(j_n, 0.0f);
      V3 impulse_n = j_n * normal;
      float pos_correction = P.baumgarte * std::fmax(penetration - P.slop, 0.0f);
      if (inv_mass_a > 1e-8f) {
        st3(&vel[ia * 4], ld3(&vel[ia * 4]) + impulse_n * inv_mass_a);
        st3(&ang[ia * 4], ld3(&ang[ia * 4]) + cross(r_a, impulse_n) * Ia);
        float mass_ratio_a = inv_mass_a / inv_mass_sum;
        st3(&pos[ia * 4], ld3(&pos[ia * 4]) + pos_correction * mass_ratio_a * normal);
      }
      if (inv_mass_b > 1e-8f) {
        st3(&vel[ib * 4], ld3(&vel[ib * 4]) - impulse_n * inv_mass_b);
        st3(&ang[ib * 4], ld3(&ang[ib * 4]) - cross(r_b, impulse_n) * Ib);
        float mass_ratio_b = inv_mass_b / inv_mass_sum;
        st3(&pos[ib * 4], ld3(&pos[ib * 4]) - pos_correction * mass_ratio_b * normal);
      }
      float j_n_accumulated = c.impulses[0] + j_n;
      if (tangent_speed > 1e-6f && j_n_accumulated > 1e-6f) {
        V3 tangent = vel_tangent / tangent_speed;
        V3 rt_a = cross(r_a, tangent), rt_b = cross(r_b, tangent);
        float w_t_a = inv_mass_a + dot(rt_a * Ia, rt_a);
        float w_t_b = inv_mass_b + dot(rt_b * Ib, rt_b);
        float w_tangent = w_t_a + w_t_b;
        if (w_tangent > 1e-8f) {
          float j_t_desired = tangent_speed / w_tangent;
          float j_t_max = friction * j_n_accumulated;
          float j_t = std::fmin(j_t_desired, j_t_max);
          V3 impulse_t = j_t * tangent;
          if (inv_mass_a > 1e-8f) {
            st3(&vel[ia * 4], ld3(&vel[ia * 4]) - impulse_t * inv_mass_a);
            st3(&ang[ia * 4], ld3(&ang[ia * 4]) - cross(r_a, impulse_t) * Ia);
          }
          if (inv_mass_b > 1e-8f) {
            st3(&vel[ib * 4], ld3(&vel[ib * 4]) + impulse_t * inv_mass_b);
            st3(&ang[ib * 4], ld3(&ang[ib * 4]) + cross(r_b, impulse_t) * Ib);
          }
        }
      }
      c.impulses[0] = j_n;
    }
  }

  // xpbd_update_velocities (all_shaders.metal:1922-1961)
  for (uint32_t b = 0; b < B; b++) {
    if (imi[b * 4] < 1e-8f) continue;
    const float inv_dt = 1.0f / dt;
    st3w0(&vel[b * 4], (ld3(&pos[b * 4]) - ld3(&ppos[b * 4])) * inv_dt);
    Q4 dq = quat_multiply(ld4(&quat[b * 4]), quat_conjugate(ld4(&pquat[b * 4])));
    if (dq.w < 0) dq = -dq;
    st3w0(&ang[b * 4], 2.0f * V3{dq.x, dq.y, dq.z} * inv_dt);
  }

  // update_joint_states (all_shaders.metal:1550-1638)
  float* jp = &w->jpos[size_t(e) * std::max(J, 1u)];
  float* jv = &w->jvel[size_t(e) * std::max(J, 1u)];
  for (uint32_t j = 0; j < J; j++) {
    const JointRec& jr = w->joints[j];
    const uint32_t type = uint32_t(jr.params[0]);
    const uint32_t ia = uint32_t(jr.params[1]), ib = uint32_t(jr.params[2]);
    jp[j] = 0;
    jv[j] = 0;
    Q4 q_a = ld4(&quat[ia * 4]), q_b = ld4(&quat[ib * 4]);
    V3 p_a = ld3(&pos[ia * 4]), p_b = ld3(&pos[ib * 4]);
    V3 v_a = ld3(&vel[ia * 4]), v_b = ld3(&vel[ib * 4]);
    V3 w_a = ld3(&ang[ia * 4]), w_b = ld3(&ang[ib * 4]);
    if (type == 1) {
      V3 axis_local = ld3(jr.axis);
      V3 axis_world_a = rotate_by_quat(axis_local, q_a);
      Q4 q_rel = quat_multiply(quat_conjugate(q_a), q_b);
      float sin_half = dot(V3{q_rel.x, q_rel.y, q_rel.z}, axis_local);
      jp[j] = 2.0f * std::atan2(sin_half, q_rel.w);
      jv[j] = dot(w_b - w_a, axis_world_a);
    } else if (type == 2) {
      V3 axis_world_a = rotate_by_quat(ld3(jr.axis), q_a);
      V3 r_a = rotate_by_quat(ld3(jr.anchor_parent), q_a);
      V3 r_b = rotate_by_quat(ld3(jr.anchor_child), q_b);
      V3 diff = (p_b + r_b) - (p_a + r_a);
      jp[j] = dot(diff, axis_world_a);
      V3 v_pt_a = v_a + cross(w_a, r_a);
      V3 v_pt_b = v_b + cross(w_b, r_b);
      jv[j] = dot(v_pt_b - v_pt_a, axis_world_a);
    }
  }

  // read_sensors (all_shaders.metal:1799-1893)
  float* ob = &w->obs_buf[size_t(e) * std::max(w->obs, 1u)];
  for (uint32_t s = 0; s < w->S; s++) {
    const SensorRec& sr = w->sensors[s];
    const uint32_t type = sr.type_object[0], obj = sr.type_object[1];
    const uint32_t off = uint32_t(sr.params[3]);
    switch (type) {
      case 0: ob[off] = jp[obj]; break;
      case 1: ob[off] = jv[obj]; break;
      case 2: {
        V3 local_gravity = rotate_by_quat(gravity, quat_conjugate(ld4(&quat[obj * 4])));
        ob[off] = local_gravity.x;
        ob[off + 1] = local_gravity.y;
        ob[off + 2] = local_gravity.z;
        break;
      }
      case 3:
      case 10:
        for (int k = 0; k < 3; k++) ob[off + k] = ang[obj * 4 + k];
        break;
      case 7:
        for (int k = 0; k < 3; k++) ob[off + k] = pos[obj * 4 + k];
        break;
      case 8:
        for (int k = 0; k < 4; k++) ob[off + k] = quat[obj * 4 + k];
        break;
      case 9:
        for (int k = 0; k < 3; k++) ob[off + k] = vel[obj * 4 + k];
        break;
      default: break;
    }
  }

  // cache_contacts (all_shaders.metal:1454-1478)
  w->prev_counts[e] = count;
  for (uint32_t i = 0; i < n; i++) prev[i] = con[i];

  // store_lambda_prev (all_shaders.metal:1428-1444)
  for (uint32_t k = 0; k < K; k++) cst[k].state[1] = cst[k].state[0];
}

}  // namespace zo
