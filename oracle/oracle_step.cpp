// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle for the batched physics step.
// Nothing in the product (zeno_b200/, include/) may include or link this file.
//
// Single-threaded restatement of the reference world set-up and step:
//   World.init / uploadSceneData / initializeState    src/world/world.zig:215-691
//   joint decomposition                               src/physics/joint.zig:202-350
//   graph colouring, stable colour sort, ranges       src/physics/xpbd.zig:533-640
//   World.step / stepOnce (18 kernels per substep)    src/world/world.zig:694-792, 934-1293
//   MSL kernel bodies                                 src/shaders/all_shaders.metal (cited per stage)
//   stepSubset / reset                                world.zig:833-929, 1296-1314
// Stages that race in the reference are given the serial order the product also uses:
//   * broad-phase emission: geom a ascending, then b ascending (all_shaders.metal:468-533)
//   * apply_joint_forces float atomics: joints in index order (all_shaders.metal:122-190)
//   * solve_contacts: contact slots in slot order, one after another (all_shaders.metal:1644-1793)
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

#include "oracle_math.h"
#include "oracle_model.h"

namespace zo {
namespace {

// ---- world.zig:184-212 host quaternion helpers (plain products, no fusion) ----
void host_qconj(const float q[4], float o[4]) {
  o[0] = -q[0];
  o[1] = -q[1];
  o[2] = -q[2];
  o[3] = q[3];
}
void host_qmul(const float a[4], const float b[4], float o[4]) {
  float r[4] = {a[3] * b[0] + a[0] * b[3] + a[1] * b[2] - a[2] * b[1],
                a[3] * b[1] - a[0] * b[2] + a[1] * b[3] + a[2] * b[0],
                a[3] * b[2] + a[0] * b[1] - a[1] * b[0] + a[2] * b[3],
                a[3] * b[3] - a[0] * b[0] - a[1] * b[1] - a[2] * b[2]};
  std::memcpy(o, r, 16);
}
void host_rotate(const float v[3], const float q[4], float o[3]) {
  float qv[3] = {q[0], q[1], q[2]};
  float qw = q[3];
  float t[3] = {2.0f * (qv[1] * v[2] - qv[2] * v[1]), 2.0f * (qv[2] * v[0] - qv[0] * v[2]),
                2.0f * (qv[0] * v[1] - qv[1] * v[0])};
  float r[3] = {v[0] + qw * t[0] + (qv[1] * t[2] - qv[2] * t[1]),
                v[1] + qw * t[1] + (qv[2] * t[0] - qv[0] * t[2]),
                v[2] + qw * t[2] + (qv[0] * t[1] - qv[1] * t[0])};
  std::memcpy(o, r, 12);
}

enum PrimType { PDistance, PPoint, PHinge, PSlider, PCone, PAngLimit, PLinLimit, PWeld };
struct Prim {
  PrimType type;
  uint32_t a, b;
  float la[3], lb[3], axis[3];
  float damping = 0, lower = 0, upper = 0, target = 0;
};

// joint.zig:202-350 decomposeJoint
std::vector<Prim> decompose(const JointDef& j) {
  std::vector<Prim> out;
  auto mk = [&](PrimType t, const float* axis) {
    Prim p;
    p.type = t;
    p.a = j.parent;
    p.b = j.child;
    std::memcpy(p.la, j.anchor_parent, 12);
    std::memcpy(p.lb, j.anchor_child, 12);
    if (axis) std::memcpy(p.axis, axis, 12);
    else p.axis[0] = p.axis[1] = p.axis[2] = 0;
    return p;
  };
  switch (j.type) {
    case kFixed: out.push_back(mk(PWeld, nullptr)); break;
    case kRevolute: {
      out.push_back(mk(PPoint, nullptr));
      Prim h = mk(PHinge, j.axis);
      h.damping = j.damping;
      out.push_back(h);
      if (j.has_limits()) {
        Prim l = mk(PAngLimit, j.axis);
        l.lower = j.lower;
        l.upper = j.upper;
        out.push_back(l);
      }
      break;
    }
    case kPrismatic: {
      Prim s = mk(PSlider, j.axis);
      s.damping = j.damping;
      out.push_back(s);
      if (j.has_limits()) {
        Prim l = mk(PLinLimit, j.axis);
        l.lower = j.lower;
        l.upper = j.upper;
        out.push_back(l);
      }
      break;
    }
    case kBall: {
      out.push_back(mk(PPoint, nullptr));
      if (j.has_limits()) {
        Prim c = mk(PCone, j.axis);
        c.upper = j.upper;
        out.push_back(c);
      }
      break;
    }
    case kFree: break;
    case kUniversal:
      out.push_back(mk(PPoint, nullptr));
      out.push_back(mk(PHinge, j.axis));
      out.push_back(mk(PHinge, j.axis2));
      break;
  }
  return out;
}

ConstraintRec make_constraint(uint32_t type, uint32_t a, uint32_t b) {
  ConstraintRec c;
  std::memset(&c, 0, sizeof(c));
  c.indices[0] = a;
  c.indices[1] = b;
  c.indices[2] = 0;
  c.indices[3] = type;
  return c;
}

// world.zig:315-445 template construction (compliance is always 0, world.zig:323)
std::vector<ConstraintRec> build_templates(const Scene& sc) {
  std::vector<ConstraintRec> t;
  for (const JointDef& j : sc.joints) {
    for (const Prim& p : decompose(j)) {
      const float comp = 0.0f;
      switch (p.type) {
        case PPoint: {  // xpbd.zig:214-230
          ConstraintRec c = make_constraint(2, p.a, p.b);
          std::memcpy(c.anchor_a, p.la, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, p.lb, 12);
          t.push_back(c);
          break;
        }
        case PHinge: {
          float aw[3], qbi[4], ab[3];
          host_rotate(p.axis, sc.bodies[p.a].quat, aw);
          host_qconj(sc.bodies[p.b].quat, qbi);
          host_rotate(aw, qbi, ab);
          ConstraintRec c = make_constraint(3, p.a, p.b);  // xpbd.zig:233-251
          std::memcpy(c.anchor_a, p.axis, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, ab, 12);
          c.anchor_b[3] = p.damping;
          t.push_back(c);
          break;
        }
        case PWeld: {
          float qai[4], rel[4];
          host_qconj(sc.bodies[p.a].quat, qai);
          host_qmul(qai, sc.bodies[p.b].quat, rel);
          ConstraintRec c = make_constraint(7, p.a, p.b);  // xpbd.zig:293-312
          std::memcpy(c.anchor_a, p.la, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, p.lb, 12);
          std::memcpy(c.axis_target, rel, 16);
          t.push_back(c);
          break;
        }
        case PAngLimit:
        case PCone: {
          ConstraintRec c = make_constraint(4, p.a, p.b);  // xpbd.zig:254-271
          std::memcpy(c.anchor_a, p.axis, 12);
          c.anchor_a[3] = comp;
          c.limits[0] = p.type == PCone ? -p.upper : p.lower;
          c.limits[1] = p.upper;
          t.push_back(c);
          break;
        }
        case PLinLimit: {  // world.zig:383-394
          ConstraintRec c = make_constraint(5, p.a, p.b);
          std::memcpy(c.anchor_a, p.axis, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, p.lb, 12);
          c.limits[0] = p.lower;
          c.limits[1] = p.upper;
          t.push_back(c);
          break;
        }
        case PSlider: {  // world.zig:396-415
          float qai[4], rel[4];
          host_qconj(sc.bodies[p.a].quat, qai);
          host_qmul(qai, sc.bodies[p.b].quat, rel);
          ConstraintRec c = make_constraint(10, p.a, p.b);
          std::memcpy(c.anchor_a, p.la, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, p.lb, 12);
          c.anchor_b[3] = p.damping;
          std::memcpy(c.axis_target, p.axis, 12);
          std::memcpy(c.limits, rel, 16);
          t.push_back(c);
          break;
        }
        case PDistance: {  // xpbd.zig:315-331
          ConstraintRec c = make_constraint(8, p.a, p.b);
          std::memcpy(c.anchor_a, p.la, 12);
          c.anchor_a[3] = comp;
          std::memcpy(c.anchor_b, p.lb, 12);
          c.axis_target[3] = p.target;
          t.push_back(c);
          break;
        }
      }
    }
  }
  return t;
}

uint32_t color_of(const ConstraintRec& c) { return (c.indices[3] >> 8) & 0xFF; }

// xpbd.zig:533-605 greedy colouring over shared bodies (body 0 included)
uint32_t color_constraints(std::vector<ConstraintRec>& cs, uint32_t nb) {
  if (cs.empty()) return 0;
  std::vector<std::vector<uint32_t>> by_body(nb);
  for (uint32_t i = 0; i < cs.size(); i++) {
    uint32_t a = cs[i].indices[0], b = cs[i].indices[1];
    if (a < nb) by_body[a].push_back(i);
    if (b < nb && b != a) by_body[b].push_back(i);
  }
  uint32_t max_color = 0;
  for (uint32_t i = 0; i < cs.size(); i++) {
    bool used[256] = {false};
    uint32_t a = cs[i].indices[0], b = cs[i].indices[1];
    if (a < nb)
      for (uint32_t n : by_body[a])
        if (n < i) used[color_of(cs[n])] = true;
    if (b < nb && b != a)
      for (uint32_t n : by_body[b])
        if (n < i) used[color_of(cs[n])] = true;
    uint32_t col = 0;
    while (col < 255 && used[col]) col++;
    cs[i].indices[3] = (cs[i].indices[3] & 0xFF) | (col << 8);
    if (col > max_color) max_color = col;
  }
  return max_color + 1;
}

float* body4(std::vector<float>& v, uint32_t B, uint32_t e, uint32_t b) { return &v[(size_t(e) * B + b) * 4]; }
F4 ld4(const float* p) { return F4{p[0], p[1], p[2], p[3]}; }
F3 ld3(const float* p) { return F3{p[0], p[1], p[2]}; }
void st3(float* p, F3 v) {
  p[0] = v.x;
  p[1] = v.y;
  p[2] = v.z;
}
void st4(float* p, F4 v) {
  p[0] = v.x;
  p[1] = v.y;
  p[2] = v.z;
  p[3] = v.w;
}

uint32_t pair_key(uint32_t a, uint32_t b) {
  uint32_t lo = a < b ? a : b, hi = a < b ? b : a;
  return (lo << 16) | hi;
}

// ------------------------------------------------------------------------------------
// One substep for one environment (world.zig:934-1293), kernels in dispatch order.
// ------------------------------------------------------------------------------------
void substep_env(World* w, uint32_t e) {
  const Params& P = w->params;
  const uint32_t B = w->B, J = w->J, A = w->A, G = w->G, M = w->M, K = w->K;
  const float dt = P.dt;
  const F3 grav{P.gravity[0], P.gravity[1], P.gravity[2]};
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

  // warm_start_constraints (all_shaders.metal:1408-1426), factor 0.8 (world.zig:477-478)
  for (uint32_t k = 0; k < K; k++) cst[k].state[0] = 0.8f * cst[k].state[1];

  // apply_actions (all_shaders.metal:196-229); actuators in index order
  for (uint32_t a = 0; a < A; a++) {
    const ActuatorRec& ar = w->actuators[a];
    uint32_t jid = uint32_t(ar.params[0]);
    float ctrl = clampf(act[a], ar.params[1], ar.params[2]);
    float tq = ctrl * ar.params[3];
    tq = clampf(tq, ar.params2[0], ar.params2[1]);
    jt[jid] = tq;
  }

  // compute_forces (all_shaders.metal:345-388)
  for (uint32_t b = 0; b < B; b++) {
    float inv_m = imi[b * 4 + 0];
    if (inv_m < 1e-8f) {
      st4(&frc[b * 4], F4{0, 0, 0, 0});
      st4(&trq[b * 4], F4{0, 0, 0, 0});
      continue;
    }
    float m = rcp_r(inv_m);
    F3 f = mul(grav, m);
    st4(&frc[b * 4], F4{f.x, f.y, f.z, 0});
    F3 cw = rotate(ld3(w->bodies[b].com_offset), ld4(&quat[b * 4]));
    F3 t = cross(cw, f);
    st4(&trq[b * 4], F4{t.x, t.y, t.z, 0});
  }

  // update_kinematic (all_shaders.metal:304-339): body type 1 only
  for (uint32_t b = 0; b < B; b++) {
    if (uint32_t(w->bodies[b].params[1]) != 1) continue;
    F3 p = madd(ld3(&vel[b * 4]), dt, ld3(&pos[b * 4]));
    st4(&pos[b * 4], F4{p.x, p.y, p.z, 0});
    F3 om = ld3(&ang[b * 4]);
    F3 h = mul(mul(om, dt), 0.5f);
    F4 q = ld4(&quat[b * 4]);
    F4 dq = qmul(F4{h.x, h.y, h.z, 0.0f}, q);
    st4(&quat[b * 4], qnormalize(qmadd(dq, 1.0f, q)));
  }

  // apply_joint_forces (all_shaders.metal:122-190); float atomics -> joint order
  for (uint32_t j = 0; j < J; j++) {
    float tau = jt[j];
    if (std::fabs(tau) < 1e-6f) continue;
    const JointRec& jr = w->joints[j];
    uint32_t type = uint32_t(jr.params[0]);
    uint32_t ba = uint32_t(jr.params[1]), bb = uint32_t(jr.params[2]);
    F3 aw = rotate(ld3(jr.axis), ld4(&quat[ba * 4]));
    F3 f = mul(aw, tau);
    float* tgt = type == 2 ? frc : trq;
    if (ba > 0) st3(&tgt[ba * 4], sub(ld3(&tgt[ba * 4]), f));
    if (bb > 0) st3(&tgt[bb * 4], add(ld3(&tgt[bb * 4]), f));
  }

  // save_prev_state (all_shaders.metal:1900-1913)
  std::memcpy(ppos, pos, sizeof(float) * 4 * B);
  std::memcpy(pquat, quat, sizeof(float) * 4 * B);

  // integrate (all_shaders.metal:394-462)
  for (uint32_t b = 0; b < B; b++) {
    F4 mi = ld4(&imi[b * 4]);
    if (mi.x < 1e-8f) continue;
    F3 v = madd(mul(ld3(&frc[b * 4]), mi.x), dt, ld3(&vel[b * 4]));
    v = mul(v, 0.999f);
    F3 p = madd(v, dt, ld3(&pos[b * 4]));
    st4(&vel[b * 4], F4{v.x, v.y, v.z, 0});
    st4(&pos[b * 4], F4{p.x, p.y, p.z, 0});
    F3 om = madd(mulv(F3{mi.y, mi.z, mi.w}, ld3(&trq[b * 4])), dt, ld3(&ang[b * 4]));
    om = mul(om, 0.999f);
    F3 h = mul(mul(om, dt), 0.5f);
    F4 q = ld4(&quat[b * 4]);
    F4 dq = qmul(F4{h.x, h.y, h.z, 0.0f}, q);
    q = qmadd(dq, 1.0f, q);
    st4(&ang[b * 4], F4{om.x, om.y, om.z, 0});
    st4(&quat[b * 4], qnormalize(q));
  }

  // broad_phase O(n^2) (all_shaders.metal:468-533); G > 512 selects the spatial hash in
  // the reference (world.zig:534), whose pair set for non-plane pairs is the subset of
  // this one within the 27-cell neighbourhood; the oracle only restates the O(n^2) path.
  uint32_t& count = w->counts[e];
  // corrected semantics: geom offsets rotate with the body; bounding radius of the whole
  // geom (sphere r, capsule r + half length, box |half extents|, cylinder
  // sqrt(r^2 + half length^2))
  const bool corr = w->scene.corrected;
  if (corr) count = 0;  // corrected: the list is rebuilt every substep
  auto centre = [&](const GeomRec& g, uint32_t b) -> F3 {
    if (!corr) return add(ld3(&pos[b * 4]), ld3(g.pos_size0));
    float wp[3], wq[4];
    geom_world_pose(g, &pos[b * 4], &quat[b * 4], wp, wq);
    return F3{wp[0], wp[1], wp[2]};
  };
  auto bound = [&](const GeomRec& g) -> float {
    const float s0 = g.pos_size0[3], s1 = g.params[0], s2 = g.params[1];
    if (!corr) return s0;
    switch (g.type_body[0]) {
      case 1: return s0 + s1;
      case 2: return std::sqrt(s0 * s0 + s1 * s1 + s2 * s2);
      case 4: return std::sqrt(s0 * s0 + s1 * s1);
      default: return s0;
    }
  };
  for (uint32_t ga = 0; ga < G; ga++) {
    const GeomRec& A_ = w->geoms[ga];
    uint32_t ba = A_.type_body[1];
    F3 pa = centre(A_, ba);
    float ra = bound(A_);
    uint32_t ta = A_.type_body[0], grp_a = A_.type_body[3], msk_a = A_.type_body[2];
    for (uint32_t gb = ga + 1; gb < G; gb++) {
      const GeomRec& B_ = w->geoms[gb];
      uint32_t bb = B_.type_body[1];
      if (ba == bb) continue;
      uint32_t tb = B_.type_body[0], grp_b = B_.type_body[3], msk_b = B_.type_body[2];
      if ((grp_a & msk_b) == 0 && (grp_b & msk_a) == 0) continue;
      F3 pb = centre(B_, bb);
      float rb = bound(B_);
      bool plane = ta == 3 || tb == 3;
      if (!plane) {
        F3 d = sub(pb, pa);
        float dsq = dot(d, d);
        float md = (ra + rb) + 0.1f;
        if (dsq >= md * md) continue;
      }
      uint32_t c = count++;
      if (c < M) {
        con[c].indices[0] = ba;
        con[c].indices[1] = bb;
        con[c].indices[2] = ga;
        con[c].indices[3] = gb;
      }
    }
  }

  // sort_contacts (all_shaders.metal:711-745): stable insertion sort
  uint32_t n = std::min(count, M);
  for (uint32_t i = 1; i < n; i++) {
    ContactRec key = con[i];
    uint32_t kv = pair_key(key.indices[0], key.indices[1]);
    int j = int(i) - 1;
    while (j >= 0) {
      uint32_t jv = pair_key(con[j].indices[0], con[j].indices[1]);
      if (jv <= kv) break;
      con[j + 1] = con[j];
      j--;
    }
    con[j + 1] = key;
  }

  // narrow_phase (all_shaders.metal:751-894); extended modes: the reference's CPU
  // detectCollision (src/collision/narrow_phase.zig:28-136) on the same slots, mode 2
  // with GJK + EPA (src/collision/gjk.zig) for box-capsule pairs
  for (uint32_t i = 0; i < n; i++) {
    ContactRec& c = con[i];
    uint32_t ba = c.indices[0], bb = c.indices[1];
    const GeomRec& gA = w->geoms[c.indices[2]];
    const GeomRec& gB = w->geoms[c.indices[3]];
    if (w->narrow_mode >= 1) {
      float pt[3], nm[3], pen = 0.0f;
      bool hit;
      if (corr) {  // each geom placed by its own world frame; normals from B to A
        GeomRec ca = gA, cb = gB;
        float wpa[3], wqa[4], wpb[3], wqb[4];
        geom_world_pose(gA, &pos[ba * 4], &quat[ba * 4], wpa, wqa);
        geom_world_pose(gB, &pos[bb * 4], &quat[bb * 4], wpb, wqb);
        ca.pos_size0[0] = ca.pos_size0[1] = ca.pos_size0[2] = 0.0f;
        cb.pos_size0[0] = cb.pos_size0[1] = cb.pos_size0[2] = 0.0f;
        hit = narrow_cpu(ca, wpa, wqa, cb, wpb, wqb, pt, nm, &pen, w->narrow_mode == 2);
        if (hit && normal_a_to_b(gA.type_body[0], gB.type_body[0])) nm[0] = -nm[0], nm[1] = -nm[1], nm[2] = -nm[2];
      } else {
        hit = narrow_cpu(gA, &pos[ba * 4], &quat[ba * 4], gB, &pos[bb * 4], &quat[bb * 4], pt, nm, &pen,
                         w->narrow_mode == 2);
      }
      if (hit) {
        const float fr = std::sqrt(gA.params[2] * gB.params[2]);
        st4(c.position_pen, F4{pt[0], pt[1], pt[2], pen});
        st4(c.normal_friction, F4{nm[0], nm[1], nm[2], fr});
        st4(c.impulses, F4{0, 0, 0, P.restitution});
      } else {
        c.position_pen[3] = -1.0f;
      }
      continue;
    }
    F3 pa = add(ld3(&pos[ba * 4]), ld3(gA.pos_size0));
    F3 pb = add(ld3(&pos[bb * 4]), ld3(gB.pos_size0));
    uint32_t ta = gA.type_body[0], tb = gB.type_body[0];
    F3 normal{0, 0, 0}, point{0, 0, 0};
    float pen = 0;
    bool hit = false;
    if (ta == 0 && tb == 0) {
      float ra = gA.pos_size0[3], rb = gB.pos_size0[3];
      F3 d = sub(pb, pa);
      float dist;
      F3 nd = unit(d, &dist);
      float md = ra + rb;
      if (dist < md && dist > 1e-6f) {
        normal = nd;
        pen = md - dist;
        point = madd(normal, ra - pen * 0.5f, pa);
        hit = true;
      }
    } else if ((ta == 0 && tb == 3) || (ta == 3 && tb == 0)) {
      F3 sp = ta == 0 ? pa : pb;
      float sr = ta == 0 ? gA.pos_size0[3] : gB.pos_size0[3];
      F3 pp = ta == 0 ? pb : pa;
      F3 pn{0, 0, 1};
      float sd = dot(sub(sp, pp), pn);
      if (sd < sr) {
        normal = pn;
        pen = sr - sd;
        point = msub(pn, sd + pen * 0.5f, sp);
        hit = true;
        if (ta == 3) normal = neg(normal);
      }
    } else if ((ta == 1 && tb == 3) || (ta == 3 && tb == 1)) {
      const GeomRec& cg = ta == 1 ? gA : gB;
      F3 cp = ta == 1 ? pa : pb;
      float cr = cg.pos_size0[3], hl = cg.params[0];
      F3 axis = rotate(F3{0, 0, 1}, ld4(cg.quat));
      F3 p1 = msub(axis, hl, cp);
      F3 p2 = madd(axis, hl, cp);
      float d1 = p1.z - cr, d2 = p2.z - cr;
      if (d1 < 0 || d2 < 0) {
        F3 deep = d1 < d2 ? p1 : p2;
        float dist = std::fmin(d1, d2);
        normal = ta == 1 ? F3{0, 0, 1} : F3{0, 0, -1};
        pen = -dist;
        point = deep;
        point.z = 0;
        hit = true;
      }
    }
    if (hit) {
      float fr = std::sqrt(gA.params[2] * gB.params[2]);
      st4(c.position_pen, F4{point.x, point.y, point.z, pen});
      st4(c.normal_friction, F4{normal.x, normal.y, normal.z, fr});
      st4(c.impulses, F4{0, 0, 0, P.restitution});
    } else {
      c.position_pen[3] = -1.0f;
    }
  }

  // match_cached_contacts (all_shaders.metal:1483-1544)
  uint32_t pc = w->prev_counts[e];
  for (uint32_t i = 0; i < n; i++) {
    ContactRec& c = con[i];
    if (c.position_pen[3] < 0) continue;
    uint32_t ba = c.indices[0], bb = c.indices[1];
    F3 p = ld3(c.position_pen);
    float best = 0.04f;
    int match = -1;
    for (uint32_t k = 0; k < pc && k < M; k++) {
      const ContactRec& q = prev[k];
      if (q.position_pen[3] < 0) continue;
      bool same = (q.indices[0] == ba && q.indices[1] == bb) || (q.indices[0] == bb && q.indices[1] == ba);
      if (!same) continue;
      F3 d = sub(ld3(q.position_pen), p);
      float dsq = dot(d, d);
      if (dsq < best) {
        best = dsq;
        match = int(k);
      }
    }
    if (match >= 0) {
      c.impulses[0] = prev[match].impulses[0] * 0.8f;
      c.impulses[1] = prev[match].impulses[1] * 0.8f;
      c.impulses[2] = prev[match].impulses[2] * 0.8f;
    }
  }

  // solve_joints (all_shaders.metal:909-1399), colours in order (world.zig:1163-1195)
  const float alpha = 0.0f;  // compliance / dt^2 with compliance 0 (world.zig:323)
  for (uint32_t it = 0; it < P.contact_iterations; it++) {
    for (uint32_t col = 0; col < w->num_colors; col++) {
      uint32_t off = w->color_ranges[2 * col], cnt = w->color_ranges[2 * col + 1];
      for (uint32_t li = 0; li < cnt; li++) {
        ConstraintRec& c = cst[off + li];
        uint32_t type = c.indices[3] & 0xFF;
        if (type > 10) continue;
        uint32_t ia = c.indices[0], ib = c.indices[1];
        F4 mia = ld4(&imi[ia * 4]), mib = ld4(&imi[ib * 4]);
        F3 Ia{mia.y, mia.z, mia.w}, Ib{mib.y, mib.z, mib.w};
        float ima = mia.x, imb = mib.x;
        if (ima + imb < 1e-8f) continue;
        F3 pa = ld3(&pos[ia * 4]), pb = ld3(&pos[ib * 4]);
        F4 qa = ld4(&quat[ia * 4]), qb = ld4(&quat[ib * 4]);
        float lam = c.state[0];
        if (type == 2) {  // positional
          F3 ra = rotate(ld3(c.anchor_a), qa), rb = rotate(ld3(c.anchor_b), qb);
          F3 diff = sub(add(pa, ra), add(pb, rb));
          float C;
          F3 nn = unit(diff, &C);
          if (C > 1e-6f) {
            F3 rna = cross(ra, nn), rnb = cross(rb, nn);
            float wa = ima + dot(mulv(rna, Ia), rna);
            float wb = imb + dot(mulv(rnb, Ib), rnb);
            float wsum = wa + wb;
            float dl = div_r(std::fmaf(-alpha, lam, -C), wsum + alpha);
            c.state[0] = lam + dl;
            F3 imp = mul(nn, dl);
            F3 rca = sub(ra, rotate(ld3(w->bodies[ia].com_offset), qa));
            F3 rcb = sub(rb, rotate(ld3(w->bodies[ib].com_offset), qb));
            if (ima > 0) {
              st3(&pos[ia * 4], madd(imp, ima, pa));
              F3 dw = mulv(cross(rca, imp), Ia);
              F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qa);
              st4(&quat[ia * 4], qnormalize(qmadd(dq, 0.5f, qa)));
            }
            if (imb > 0) {
              st3(&pos[ib * 4], msub(imp, imb, pb));
              F3 dw = mulv(cross(rcb, imp), Ib);
              F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qb);
              st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qb)));
            }
          }
        } else if (type == 7) {  // weld (body b only)
          F3 ra = rotate(ld3(c.anchor_a), qa), rb = rotate(ld3(c.anchor_b), qb);
          F3 diff = sub(add(pa, ra), add(pb, rb));
          float C;
          F3 nn = unit(diff, &C);
          if (C > 1e-6f) {
            F3 rnb = cross(rb, nn);
            float wb = imb + dot(mulv(rnb, Ib), rnb);
            if (wb > 1e-8f) {
              float dl = div_r(-C, wb + alpha);
              F3 imp = mul(nn, dl);
              st3(&pos[ib * 4], msub(imp, imb, pb));
              F3 dw = mulv(cross(rb, imp), Ib);
              F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qb);
              st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qb)));
            }
          }
          F4 qau = ld4(&quat[ia * 4]), qbu = ld4(&quat[ib * 4]);
          F4 qrel = qmul(qconj(qau), qbu);
          F4 qerr = qmul(qrel, qconj(ld4(c.axis_target)));
          if (qerr.w < 0) qerr = qneg(qerr);
          F3 ev = xyz(qerr);
          float sh;
          F3 axr = unit(ev, &sh);
          if (sh > 1e-6f) {
            float ang_ = 2.0f * atan2_r(sh, qerr.w);
            F3 aw = rotate(axr, qau);
            float wb = dot(mulv(aw, Ib), aw);
            if (wb > 1e-8f) {
              float dl = div_r(ang_, wb + alpha);
              F3 ai = mul(aw, dl);
              if (imb > 0) {
                F3 dw = mulv(ai, Ib);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qbu);
                st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qbu)));
              }
            }
          }
        } else if (type == 3) {  // angular (hinge axis alignment)
          F3 aaw = rotate(ld3(c.anchor_a), qa), abw = rotate(ld3(c.anchor_b), qb);
          F3 cr = cross(aaw, abw);
          float sa;
          F3 nn = unit(cr, &sa);
          if (sa > 1e-6f) {
            float angC = asin_r(clampf(sa, -1.0f, 1.0f));
            float wa = dot(mulv(nn, Ia), nn), wb = dot(mulv(nn, Ib), nn);
            float wsum = wa + wb;
            if (wsum > 1e-8f) {
              float dl = div_r(-angC, wsum + alpha);
              if (ima > 0) {
                F3 dw = mulv(mul(nn, dl), Ia);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qa);
                st4(&quat[ia * 4], qnormalize(qmadd(dq, 0.5f, qa)));
              }
              if (imb > 0) {
                F3 dw = mulv(mul(nn, -dl), Ib);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qb);
                st4(&quat[ib * 4], qnormalize(qmadd(dq, 0.5f, qb)));
              }
            }
          }
        } else if (type == 4) {  // angular limit
          F3 axl = ld3(c.anchor_a);
          float lo = c.limits[0], hi = c.limits[1];
          F4 qrel = qmul(qconj(qa), qb);
          float sh = dot(xyz(qrel), axl);
          float angle = 2.0f * atan2_r(sh, qrel.w);
          float viol = 0.0f;
          if (angle < lo) viol = lo - angle;
          else if (angle > hi) viol = hi - angle;
          if (std::fabs(viol) > 1e-6f) {
            F3 aw = rotate(axl, qa);
            float wa = dot(mulv(aw, Ia), aw), wb = dot(mulv(aw, Ib), aw);
            float wsum = wa + wb;
            if (wsum > 1e-8f) {
              float dl = div_r(viol, wsum + alpha);
              F3 ai = mul(aw, dl);
              if (ima > 0) {
                F3 dw = mulv(ai, Ia);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qa);
                st4(&quat[ia * 4], qnormalize(qmadd(dq, 0.5f, qa)));
              }
              if (imb > 0) {
                F3 dw = mulv(ai, Ib);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qb);
                st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qb)));
              }
            }
          }
        } else if (type == 5) {  // linear limit
          F3 axl = ld3(c.anchor_a);
          float lo = c.limits[0], hi = c.limits[1];
          F3 ra = rotate(F3{0, 0, 0}, qa), rb = rotate(ld3(c.anchor_b), qb);
          F3 aw = rotate(axl, qa);
          F3 diff = sub(add(pb, rb), add(pa, ra));
          float dist = dot(diff, aw);
          float viol = 0.0f;
          if (dist < lo) viol = lo - dist;
          else if (dist > hi) viol = hi - dist;
          if (std::fabs(viol) > 1e-6f) {
            F3 nn = viol > 0 ? aw : neg(aw);
            float av = std::fabs(viol);
            F3 rna = cross(ra, nn), rnb = cross(rb, nn);
            float wa = ima + dot(mulv(rna, Ia), rna);
            float wb = imb + dot(mulv(rnb, Ib), rnb);
            float wsum = wa + wb;
            if (wsum > 1e-8f) {
              float dl = div_r(av, wsum + alpha);
              F3 imp = mul(nn, dl);
              if (ima > 0) st3(&pos[ia * 4], msub(imp, ima, pa));
              if (imb > 0) st3(&pos[ib * 4], madd(imp, imb, pb));
            }
          }
        } else if (type == 10) {  // slider
          F3 ra = rotate(ld3(c.anchor_a), qa), rb = rotate(ld3(c.anchor_b), qb);
          F3 diff = sub(add(pa, ra), add(pb, rb));
          F3 aw = rotate(ld3(c.axis_target), qa);
          float along = dot(diff, aw);
          F3 perp = msub(aw, along, diff);
          float pl;
          F3 nn = unit(perp, &pl);
          if (pl > 1e-6f) {
            F3 rna = cross(ra, nn), rnb = cross(rb, nn);
            float wa = ima + dot(mulv(rna, Ia), rna);
            float wb = imb + dot(mulv(rnb, Ib), rnb);
            float wsum = wa + wb;
            float dl = div_r(-pl, wsum + alpha);
            F3 imp = mul(nn, dl);
            if (ima > 0) {
              st3(&pos[ia * 4], madd(imp, ima, pa));
              F3 dw = mulv(cross(ra, imp), Ia);
              F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qa);
              st4(&quat[ia * 4], qnormalize(qmadd(dq, 0.5f, qa)));
            }
            if (imb > 0) {
              st3(&pos[ib * 4], msub(imp, imb, pb));
              F3 dw = mulv(cross(rb, imp), Ib);
              F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qb);
              st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qb)));
            }
          }
          F4 qau = ld4(&quat[ia * 4]), qbu = ld4(&quat[ib * 4]);
          F4 qrel = qmul(qconj(qau), qbu);
          F4 qerr = qmul(qrel, qconj(ld4(c.limits)));
          if (qerr.w < 0) qerr = qneg(qerr);
          F3 ev = xyz(qerr);
          float sh;
          F3 axe = unit(ev, &sh);
          if (sh > 1e-6f) {
            float ae = 2.0f * atan2_r(sh, qerr.w);
            F3 aw2 = rotate(axe, qau);
            float wa = dot(mulv(aw2, Ia), aw2), wb = dot(mulv(aw2, Ib), aw2);
            float wsum = wa + wb;
            if (wsum > 1e-8f) {
              float dl = div_r(ae, wsum + alpha);
              F3 ai = mul(aw2, dl);
              if (ima > 0) {
                F3 dw = mulv(ai, Ia);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qau);
                st4(&quat[ia * 4], qnormalize(qmadd(dq, 0.5f, qau)));
              }
              if (imb > 0) {
                F3 dw = mulv(ai, Ib);
                F4 dq = qmul(F4{dw.x, dw.y, dw.z, 0.0f}, qbu);
                st4(&quat[ib * 4], qnormalize(qmsub(dq, 0.5f, qbu)));
              }
            }
          }
        }
      }
    }
  }

  // solve_contacts (all_shaders.metal:1644-1793), slots in order
  for (uint32_t it = 0; it < P.contact_iterations; it++) {
    for (uint32_t i = 0; i < n; i++) {
      ContactRec& c = con[i];
      if (c.position_pen[3] < 0) continue;
      uint32_t ia = c.indices[0], ib = c.indices[1];
      F4 mia = ld4(&imi[ia * 4]), mib = ld4(&imi[ib * 4]);
      F3 Ia{mia.y, mia.z, mia.w}, Ib{mib.y, mib.z, mib.w};
      float ima = mia.x, imb = mib.x;
      float isum = ima + imb;
      if (isum < 1e-8f) continue;
      F3 nn = ld3(c.normal_friction);
      float pen = c.position_pen[3], fr = c.normal_friction[3];
      F3 cp = ld3(c.position_pen);
      F3 pa = ld3(&pos[ia * 4]), pb = ld3(&pos[ib * 4]);
      F3 ra = sub(cp, pa), rb = sub(cp, pb);
      F3 wa_ = ld3(&ang[ia * 4]), wb_ = ld3(&ang[ib * 4]);
      F3 va = add(ld3(&vel[ia * 4]), cross(wa_, ra));
      F3 vb = add(ld3(&vel[ib * 4]), cross(wb_, rb));
      F3 rv = sub(va, vb);
      float vn = dot(rv, nn);
      F3 vt = msub(nn, vn, rv);
      float ts;
      F3 tt = unit(vt, &ts);
      F3 rna = cross(ra, nn), rnb = cross(rb, nn);
      float wna = ima + dot(mulv(rna, Ia), rna);
      float wnb = imb + dot(mulv(rnb, Ib), rnb);
      float wn = wna + wnb;
      if (wn < 1e-8f) continue;
      float excess = std::fmax(pen - P.slop, 0.0f);
      float bias = div_r(P.baumgarte * excess, dt);
      float rest = c.impulses[3];
      float vrest = vn < -0.5f ? rest * vn : 0.0f;
      float jn = div_r(-(vn + vrest) + bias, wn);
      jn = std::fmax(jn, 0.0f);
      F3 in_ = mul(nn, jn);
      float pcorr = P.baumgarte * excess;
      if (ima > 1e-8f) {
        st3(&vel[ia * 4], madd(in_, ima, ld3(&vel[ia * 4])));
        st3(&ang[ia * 4], add(ld3(&ang[ia * 4]), mulv(cross(ra, in_), Ia)));
        float mr = div_r(ima, isum);
        st3(&pos[ia * 4], madd(nn, pcorr * mr, ld3(&pos[ia * 4])));
      }
      if (imb > 1e-8f) {
        st3(&vel[ib * 4], msub(in_, imb, ld3(&vel[ib * 4])));
        st3(&ang[ib * 4], sub(ld3(&ang[ib * 4]), mulv(cross(rb, in_), Ib)));
        float mr = div_r(imb, isum);
        st3(&pos[ib * 4], msub(nn, pcorr * mr, ld3(&pos[ib * 4])));
      }
      float jacc = c.impulses[0] + jn;
      if (ts > 1e-6f && jacc > 1e-6f) {
        F3 rta = cross(ra, tt), rtb = cross(rb, tt);
        float wta = ima + dot(mulv(rta, Ia), rta);
        float wtb = imb + dot(mulv(rtb, Ib), rtb);
        float wt = wta + wtb;
        if (wt > 1e-8f) {
          float jdes = div_r(ts, wt);
          float jmax = fr * jacc;
          float jt_ = std::fmin(jdes, jmax);
          F3 it_ = mul(tt, jt_);
          if (ima > 1e-8f) {
            st3(&vel[ia * 4], msub(it_, ima, ld3(&vel[ia * 4])));
            st3(&ang[ia * 4], sub(ld3(&ang[ia * 4]), mulv(cross(ra, it_), Ia)));
          }
          if (imb > 1e-8f) {
            st3(&vel[ib * 4], madd(it_, imb, ld3(&vel[ib * 4])));
            st3(&ang[ib * 4], add(ld3(&ang[ib * 4]), mulv(cross(rb, it_), Ib)));
          }
        }
      }
      c.impulses[0] = jn;
    }
  }

  // xpbd_update_velocities (all_shaders.metal:1922-1961)
  const float inv_dt = 1.0f / dt;
  for (uint32_t b = 0; b < B; b++) {
    if (imi[b * 4] < 1e-8f) continue;
    F3 v = mul(sub(ld3(&pos[b * 4]), ld3(&ppos[b * 4])), inv_dt);
    st4(&vel[b * 4], F4{v.x, v.y, v.z, 0});
    F4 dq = qmul(ld4(&quat[b * 4]), qconj(ld4(&pquat[b * 4])));
    if (dq.w < 0) dq = qneg(dq);
    F3 om = mul(mul(xyz(dq), 2.0f), inv_dt);
    st4(&ang[b * 4], F4{om.x, om.y, om.z, 0});
  }

  // update_joint_states (all_shaders.metal:1550-1638)
  float* jp = &w->jpos[size_t(e) * std::max(J, 1u)];
  float* jv = &w->jvel[size_t(e) * std::max(J, 1u)];
  for (uint32_t j = 0; j < J; j++) {
    const JointRec& jr = w->joints[j];
    uint32_t type = uint32_t(jr.params[0]);
    uint32_t ia = uint32_t(jr.params[1]), ib = uint32_t(jr.params[2]);
    jp[j] = 0;
    jv[j] = 0;
    F4 qa = ld4(&quat[ia * 4]), qb = ld4(&quat[ib * 4]);
    F3 pa = ld3(&pos[ia * 4]), pb = ld3(&pos[ib * 4]);
    F3 va = ld3(&vel[ia * 4]), vb = ld3(&vel[ib * 4]);
    F3 wa_ = ld3(&ang[ia * 4]), wb_ = ld3(&ang[ib * 4]);
    if (type == 1) {
      F3 axl = ld3(jr.axis);
      F3 aw = rotate(axl, qa);
      F4 qrel = qmul(qconj(qa), qb);
      float sh = dot(xyz(qrel), axl);
      jp[j] = 2.0f * atan2_r(sh, qrel.w);
      jv[j] = dot(sub(wb_, wa_), aw);
    } else if (type == 2) {
      F3 aw = rotate(ld3(jr.axis), qa);
      F3 ra = rotate(ld3(jr.anchor_parent), qa), rb = rotate(ld3(jr.anchor_child), qb);
      F3 diff = sub(add(pb, rb), add(pa, ra));
      jp[j] = dot(diff, aw);
      F3 vpa = add(va, cross(wa_, ra)), vpb = add(vb, cross(wb_, rb));
      jv[j] = dot(sub(vpb, vpa), aw);
    }
  }

  // read_sensors (all_shaders.metal:1799-1893)
  float* ob = &w->obs_buf[size_t(e) * std::max(w->obs, 1u)];
  for (uint32_t s = 0; s < w->S; s++) {
    const SensorRec& sr = w->sensors[s];
    uint32_t type = sr.type_object[0], obj = sr.type_object[1];
    uint32_t off = uint32_t(sr.params[3]);
    switch (type) {
      case 0: ob[off] = jp[obj]; break;
      case 1: ob[off] = jv[obj]; break;
      case 2: {
        F3 lg = rotate(grav, qconj(ld4(&quat[obj * 4])));
        ob[off] = lg.x;
        ob[off + 1] = lg.y;
        ob[off + 2] = lg.z;
        break;
      }
      case 3:
      case 10:
        ob[off] = ang[obj * 4];
        ob[off + 1] = ang[obj * 4 + 1];
        ob[off + 2] = ang[obj * 4 + 2];
        break;
      case 7:
        ob[off] = pos[obj * 4];
        ob[off + 1] = pos[obj * 4 + 1];
        ob[off + 2] = pos[obj * 4 + 2];
        break;
      case 8:
        for (int k = 0; k < 4; k++) ob[off + k] = quat[obj * 4 + k];
        break;
      case 9:
        ob[off] = vel[obj * 4];
        ob[off + 1] = vel[obj * 4 + 1];
        ob[off + 2] = vel[obj * 4 + 2];
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

}  // namespace

bool world_init(World* w, const Scene& scene, const Config& cfg) {
  w->scene = scene;
  w->cfg = cfg;
  w->narrow_mode = scene.corrected ? 2u : 0u;  // corrected semantics: CPU routines + GJK
  w->timestep = cfg.timestep > 0 ? cfg.timestep : scene.timestep;  // main.zig:153
  const uint32_t E = cfg.num_envs;
  w->E = E;
  w->B = uint32_t(scene.bodies.size());
  w->J = uint32_t(scene.joints.size());
  w->A = uint32_t(scene.actuators.size());
  w->G = uint32_t(scene.geoms.size());
  w->S = uint32_t(scene.sensors.size());
  w->M = cfg.max_contacts_per_env;
  w->obs = scene.obs_dim();
  const uint32_t B = w->B, J = w->J, A = w->A;

  // uploadSceneData (world.zig:617-660)
  w->bodies.clear();
  for (const BodyDef& bd : scene.bodies) {
    BodyRec r;
    std::memset(&r, 0, sizeof(r));
    float ii[3];
    bd.inv_inertia(ii);
    r.position[0] = bd.pos[0];
    r.position[1] = bd.pos[1];
    r.position[2] = bd.pos[2];
    std::memcpy(r.quaternion, bd.quat, 16);
    r.inv_mass_inertia[0] = bd.inv_mass();
    r.inv_mass_inertia[1] = ii[0];
    r.inv_mass_inertia[2] = ii[1];
    r.inv_mass_inertia[3] = ii[2];
    r.params[0] = float(bd.parent);
    r.params[1] = float(uint32_t(bd.type));
    r.params[2] = 1.0f;  // gravity_scale default
    r.params[3] = 0.0f;  // linear_damping default
    std::memcpy(r.com_offset, bd.com, 12);
    w->bodies.push_back(r);
  }
  w->joints.clear();
  for (const JointDef& jd : scene.joints) {
    JointRec r;
    std::memset(&r, 0, sizeof(r));
    std::memcpy(r.anchor_parent, jd.anchor_parent, 12);
    std::memcpy(r.anchor_child, jd.anchor_child, 12);
    std::memcpy(r.axis, jd.axis, 12);
    r.params[0] = float(uint32_t(jd.type));
    r.params[1] = float(jd.parent);
    r.params[2] = float(jd.child);
    r.params[3] = jd.lower;
    r.params2[0] = jd.upper;
    r.params2[1] = jd.damping;
    r.params2[2] = jd.stiffness;
    r.params2[3] = jd.ref;
    w->joints.push_back(r);
  }
  w->geoms.clear();
  for (const GeomDef& g : scene.geoms) {
    GeomRec r;
    r.type_body[0] = g.type;
    r.type_body[1] = g.body;
    r.type_body[2] = g.conaffinity;
    r.type_body[3] = g.contype;
    r.pos_size0[0] = g.pos[0];
    r.pos_size0[1] = g.pos[1];
    r.pos_size0[2] = g.pos[2];
    r.pos_size0[3] = g.size[0];
    std::memcpy(r.quat, g.quat, 16);
    r.params[0] = g.size[1];
    r.params[1] = g.size[2];
    r.params[2] = g.friction;
    r.params[3] = g.restitution;
    w->geoms.push_back(r);
  }
  w->actuators.clear();
  for (const ActuatorDef& a : scene.actuators) {
    ActuatorRec r;
    r.params[0] = float(a.joint);
    r.params[1] = a.ctrl_min;
    r.params[2] = a.ctrl_max;
    r.params[3] = a.gear;
    r.params2[0] = a.force_min;
    r.params2[1] = a.force_max;
    r.params2[2] = a.kp;
    r.params2[3] = a.kv;
    w->actuators.push_back(r);
  }
  w->sensors.clear();
  uint32_t off = 0;
  for (const SensorDef& s : scene.sensors) {
    SensorRec r;
    r.type_object[0] = s.type;
    r.type_object[1] = s.object;
    r.type_object[2] = s.dim;
    r.type_object[3] = 0;
    r.params[0] = s.noise;
    r.params[1] = s.cutoff;
    r.params[2] = float(s.dim);
    r.params[3] = float(off);
    off += s.dim;
    w->sensors.push_back(r);
  }

  // constraints: templates, colouring, stable sort, ranges, replicate (world.zig:315-501)
  w->templ = build_templates(scene);
  w->K = uint32_t(w->templ.size());
  w->num_colors = 0;
  w->color_ranges.clear();
  if (w->K > 0) {
    w->num_colors = color_constraints(w->templ, B);
    std::stable_sort(w->templ.begin(), w->templ.end(),
                     [](const ConstraintRec& a, const ConstraintRec& b) { return color_of(a) < color_of(b); });
    w->color_ranges.assign(2 * w->num_colors, 0);
    uint32_t cur = color_of(w->templ[0]), start = 0;
    for (uint32_t i = 0; i < w->K; i++) {
      uint32_t c = color_of(w->templ[i]);
      if (c != cur) {
        w->color_ranges[2 * cur] = start;
        w->color_ranges[2 * cur + 1] = i - start;
        cur = c;
        start = i;
      }
    }
    w->color_ranges[2 * cur] = start;
    w->color_ranges[2 * cur + 1] = w->K - start;
  }
  w->constraints.assign(size_t(E) * w->K, ConstraintRec{});
  for (uint32_t e = 0; e < E; e++)
    for (uint32_t k = 0; k < w->K; k++) {
      ConstraintRec c = w->templ[k];
      c.indices[2] = e;
      w->constraints[size_t(e) * w->K + k] = c;
    }

  // SimParams (world.zig:510-531)
  Params& P = w->params;
  P.num_envs = E;
  P.num_bodies = B;
  P.num_joints = J;
  P.num_actuators = A;
  P.num_geoms = w->G;
  P.num_sensors = w->S;
  P.max_contacts = w->M;
  P.contact_iterations = cfg.contact_iterations;
  P.dt = w->timestep / float(cfg.substeps);
  std::memcpy(P.gravity, scene.gravity, 12);
  P.friction = scene.friction;
  P.restitution = scene.restitution;
  P.baumgarte = scene.baumgarte;
  P.slop = scene.slop;
  P.obs_dim = w->obs;

  // State.init (state.zig:56-117): every buffer starts zeroed
  const size_t nb4 = size_t(E) * B * 4;
  for (auto* v : {&w->pos, &w->vel, &w->acc, &w->angvel, &w->quat, &w->force, &w->torque, &w->inv_mi,
                  &w->prev_pos, &w->prev_quat, &w->prev_vel})
    v->assign(nb4, 0.0f);
  w->jpos.assign(size_t(E) * std::max(J, 1u), 0.0f);
  w->jvel.assign(size_t(E) * std::max(J, 1u), 0.0f);
  w->jtorque.assign(size_t(E) * std::max(J, 1u), 0.0f);
  w->actions.assign(size_t(E) * std::max(A, 1u), 0.0f);
  w->obs_buf.assign(size_t(E) * std::max(w->obs, 1u), 0.0f);
  w->rewards.assign(E, 0.0f);
  w->dones.assign(E, 0);
  ContactRec zc;
  std::memset(&zc, 0, sizeof(zc));
  w->contacts.assign(size_t(E) * w->M, zc);
  w->prev_contacts.assign(size_t(E) * w->M, zc);
  w->counts.assign(E, 0);
  w->prev_counts.assign(E, 0);
  w->episode.assign(E, 0);
  w->subtree.assign(B, 1u);
  for (uint32_t b = B; b-- > 1;) {
    int32_t par = scene.bodies[b].parent;
    if (par >= 0) w->subtree[uint32_t(par)] += w->subtree[b];
  }

  // initializeState (world.zig:663-691)
  for (uint32_t e = 0; e < E; e++)
    for (uint32_t b = 0; b < B; b++) {
      const BodyRec& r = w->bodies[b];
      float* p = body4(w->pos, B, e, b);
      p[0] = r.position[0];
      p[1] = r.position[1];
      p[2] = r.position[2];
      p[3] = 0;
      std::memcpy(body4(w->quat, B, e, b), r.quaternion, 16);
      std::memcpy(body4(w->inv_mi, B, e, b), r.inv_mass_inertia, 16);
    }
  // InitialState.capture (state.zig:358-388), env 0
  w->init_pos.assign(w->pos.begin(), w->pos.begin() + B * 4);
  w->init_quat.assign(w->quat.begin(), w->quat.begin() + B * 4);
  w->init_vel.assign(w->vel.begin(), w->vel.begin() + B * 4);
  w->init_angvel.assign(w->angvel.begin(), w->angvel.begin() + B * 4);
  w->init_jpos.assign(w->jpos.begin(), w->jpos.begin() + J);
  w->init_jvel.assign(w->jvel.begin(), w->jvel.begin() + J);
  w->adaptive_substeps = cfg.substeps;
  return true;
}

// The substep in the world's arithmetic mode.
void substep(World* w, uint32_t e) {
  if (w->arithmetic == 1) substep_env_literal(w, e);
  else if (w->arithmetic == 2) substep_env_literal_contracted(w, e);
  else substep_env(w, e);
}

// World.step (world.zig:694-792) for all environments.  Environments never share
// mutable state, so `threads` > 1 splits them across host threads (same results).
void world_step(World* w, const float* actions, uint32_t substeps, uint32_t threads) {
  const uint32_t E = w->E, B = w->B;
  if (actions) std::memcpy(w->actions.data(), actions, sizeof(float) * size_t(E) * w->A);
  uint32_t ns = substeps == 0 ? w->adaptive_substeps : substeps;
  w->params.dt = w->timestep / float(std::max(ns, 1u));
  w->prev_vel = w->vel;
  if (threads <= 1) {
    for (uint32_t s = 0; s < ns; s++)
      for (uint32_t e = 0; e < E; e++) substep(w, e);
  } else {
    std::vector<std::thread> pool;
    for (uint32_t t = 0; t < threads; t++)
      pool.emplace_back([w, t, threads, E, ns]() {
        const uint32_t e0 = uint32_t(uint64_t(E) * t / threads), e1 = uint32_t(uint64_t(E) * (t + 1) / threads);
        for (uint32_t e = e0; e < e1; e++)
          for (uint32_t s = 0; s < ns; s++) substep(w, e);
      });
    for (auto& th : pool) th.join();
  }
  float inv_step = w->timestep > 0 ? 1.0f / w->timestep : 0.0f;
  for (size_t i = 0; i < size_t(E) * B; i++) {
    w->acc[i * 4 + 0] = (w->vel[i * 4 + 0] - w->prev_vel[i * 4 + 0]) * inv_step;
    w->acc[i * 4 + 1] = (w->vel[i * 4 + 1] - w->prev_vel[i * 4 + 1]) * inv_step;
    w->acc[i * 4 + 2] = (w->vel[i * 4 + 2] - w->prev_vel[i * 4 + 2]) * inv_step;
    w->acc[i * 4 + 3] = 0;
  }
  world_apply_task(w, nullptr);
}

// World.stepSubset (world.zig:833-929): step everything, restore the unmasked envs'
// public buffers.  Internal caches (prev contacts, lambdas) keep the stepped values.
int world_step_subset(World* w, const float* actions, const uint8_t* mask, uint32_t substeps) {
  const uint32_t E = w->E, B = w->B, J = w->J, M = w->M, O = w->obs;
  uint32_t active = 0;
  for (uint32_t e = 0; e < E; e++) active += mask[e] != 0;
  if (active == 0) return 0;
  if (active == E) {
    world_step(w, actions, substeps);
    return 0;
  }
  World snap_src = *w;  // copy of the public buffers before the step
  const uint32_t ns = substeps == 0 ? w->adaptive_substeps : substeps;
  std::memcpy(w->actions.data(), actions, sizeof(float) * size_t(E) * w->A);
  w->params.dt = w->timestep / float(std::max(ns, 1u));
  w->prev_vel = w->vel;
  for (uint32_t s = 0; s < ns; s++)
    for (uint32_t e = 0; e < E; e++) substep(w, e);
  float inv_step = w->timestep > 0 ? 1.0f / w->timestep : 0.0f;
  for (size_t i = 0; i < size_t(E) * B; i++) {
    for (int k = 0; k < 3; k++) w->acc[i * 4 + k] = (w->vel[i * 4 + k] - w->prev_vel[i * 4 + k]) * inv_step;
    w->acc[i * 4 + 3] = 0;
  }
  world_apply_task(w, mask);
  for (uint32_t e = 0; e < E; e++) {
    if (mask[e]) continue;
    size_t b0 = size_t(e) * B * 4, b1 = b0 + size_t(B) * 4;
    for (auto pr : {std::make_pair(&w->pos, &snap_src.pos), std::make_pair(&w->quat, &snap_src.quat),
                    std::make_pair(&w->vel, &snap_src.vel), std::make_pair(&w->acc, &snap_src.acc),
                    std::make_pair(&w->angvel, &snap_src.angvel)})
      std::copy(pr.second->begin() + b0, pr.second->begin() + b1, pr.first->begin() + b0);
    if (J > 0) {
      size_t j0 = size_t(e) * J, j1 = j0 + J;
      std::copy(snap_src.jpos.begin() + j0, snap_src.jpos.begin() + j1, w->jpos.begin() + j0);
      std::copy(snap_src.jvel.begin() + j0, snap_src.jvel.begin() + j1, w->jvel.begin() + j0);
      std::copy(snap_src.jtorque.begin() + j0, snap_src.jtorque.begin() + j1, w->jtorque.begin() + j0);
    }
    if (O > 0) {
      size_t o0 = size_t(e) * O, o1 = o0 + O;
      std::copy(snap_src.obs_buf.begin() + o0, snap_src.obs_buf.begin() + o1, w->obs_buf.begin() + o0);
    }
    w->rewards[e] = snap_src.rewards[e];
    w->dones[e] = snap_src.dones[e];
    w->counts[e] = snap_src.counts[e];
    for (uint32_t i = 0; i < M; i++) w->contacts[size_t(e) * M + i] = snap_src.contacts[size_t(e) * M + i];
  }
  return 0;
}

// World.reset (world.zig:1296-1314)
void world_reset(World* w, const uint8_t* mask) {
  const uint32_t B = w->B, J = w->J;
  for (uint32_t e = 0; e < w->E; e++) {
    if (mask && !mask[e]) continue;
    std::copy(w->init_pos.begin(), w->init_pos.end(), w->pos.begin() + size_t(e) * B * 4);
    std::copy(w->init_quat.begin(), w->init_quat.end(), w->quat.begin() + size_t(e) * B * 4);
    std::copy(w->init_vel.begin(), w->init_vel.end(), w->vel.begin() + size_t(e) * B * 4);
    std::copy(w->init_angvel.begin(), w->init_angvel.end(), w->angvel.begin() + size_t(e) * B * 4);
    std::copy(w->init_jpos.begin(), w->init_jpos.end(), w->jpos.begin() + size_t(e) * J);
    std::copy(w->init_jvel.begin(), w->init_jvel.end(), w->jvel.begin() + size_t(e) * J);
  }
  std::fill(w->counts.begin(), w->counts.end(), 0u);
}

// ---------------------------------------------------------------------------------
// Episode task extension (no reference counterpart: the reference never writes rewards
// or dones, state.zig:93-94).  Counter-based random numbers from the splitmix64 mixer
// (the same mixer the reference uses to seed its unused RNG buffer, state.zig:218-240).
// ---------------------------------------------------------------------------------
static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// uniform in [-1, 1): 24 random bits, exact in float
static float task_uniform(uint64_t seed, uint64_t env, uint32_t episode, uint32_t k) {
  uint64_t h = mix64(mix64(mix64(seed) ^ env) ^ ((uint64_t(episode) << 32) | k));
  float u = float(uint32_t(h >> 40)) * (1.0f / 16777216.0f);
  return 2.0f * u - 1.0f;
}

void world_reset_env_noise(World* w, uint32_t e) {
  const uint32_t B = w->B, J = w->J;
  float* pos = &w->pos[size_t(e) * B * 4];
  float* quat = &w->quat[size_t(e) * B * 4];
  std::copy(w->init_pos.begin(), w->init_pos.end(), pos);
  std::copy(w->init_quat.begin(), w->init_quat.end(), quat);
  std::copy(w->init_vel.begin(), w->init_vel.end(), w->vel.begin() + size_t(e) * B * 4);
  std::copy(w->init_angvel.begin(), w->init_angvel.end(), w->angvel.begin() + size_t(e) * B * 4);
  std::copy(w->init_jpos.begin(), w->init_jpos.end(), w->jpos.begin() + size_t(e) * J);
  std::copy(w->init_jvel.begin(), w->init_jvel.end(), w->jvel.begin() + size_t(e) * J);
  const Task& t = w->task;
  const uint64_t genv = uint64_t(e) + w->task_env_offset;
  const uint32_t ep = w->episode[e];
  if (t.noise != 0.0f) {
    uint32_t rb = t.body;
    for (int k = 0; k < 3; k++) pos[rb * 4 + k] += t.noise * task_uniform(t.seed, genv, ep, uint32_t(k));
    // hinge-angle noise: rotate each hinge child's subtree (bodies are stored in
    // depth-first order, so a subtree is a contiguous index range) about the joint
    // anchor by ~theta; the rotation quaternion is normalize(axis*theta/2, 1).
    for (uint32_t j = 0; j < J; j++) {
      const JointRec& jr = w->joints[j];
      if (uint32_t(jr.params[0]) != 1) continue;
      float th = t.noise * task_uniform(t.seed, genv, ep, 3u + j);
      uint32_t pa = uint32_t(jr.params[1]), ch = uint32_t(jr.params[2]);
      F4 qp = ld4(&quat[pa * 4]);
      F3 anchor = add(ld3(&pos[pa * 4]), rotate(ld3(jr.anchor_parent), qp));
      F3 ax = rotate(ld3(jr.axis), qp);
      float al = length(ax);
      if (!(al > 1e-8f)) continue;
      F3 h = mul(ax, div_r(0.5f * th, al));
      F4 qr = qnormalize(F4{h.x, h.y, h.z, 1.0f});
      for (uint32_t d = ch; d < ch + w->subtree[ch]; d++) {
        F3 rel = sub(ld3(&pos[d * 4]), anchor);
        st3(&pos[d * 4], add(anchor, rotate(rel, qr)));
        st4(&quat[d * 4], qnormalize(qmul(qr, ld4(&quat[d * 4]))));
      }
    }
  }
  w->counts[e] = 0;
  w->episode[e] = ep + 1;
}

void world_apply_task(World* w, const uint8_t* mask) {
  const Task& t = w->task;
  if (!t.enabled) return;
  const uint32_t B = w->B, A = w->A;
  for (uint32_t e = 0; e < w->E; e++) {
    if (mask && !mask[e]) continue;
    const float* p = &w->pos[(size_t(e) * B + t.body) * 4];
    const float* v = &w->vel[(size_t(e) * B + t.body) * 4];
    float z = p[2];
    bool done = !(z >= t.z_min && z <= t.z_max);
    float ctrl = 0.0f;
    for (uint32_t a = 0; a < A; a++) {
      float u = w->actions[size_t(e) * A + a];
      ctrl = std::fmaf(u, u, ctrl);
    }
    float r = std::fmaf(t.forward_weight, v[0], t.alive_bonus);
    r = std::fmaf(-t.ctrl_cost, ctrl, r);
    w->rewards[e] = r;
    w->dones[e] = done ? 1 : 0;
    if (done && t.auto_reset) world_reset_env_noise(w, e);
  }
}

}  // namespace zo
