// Scene -> kernel tables.
//   inverse mass / inertia            src/physics/body.zig:53-75
//   joint decomposition               src/physics/joint.zig:202-350
//   constraint templates              src/world/world.zig:315-445 (compliance 0, :323)
//   greedy colouring, stable sort     src/physics/xpbd.zig:533-640
//   GPU record layouts                world.zig:1573-1637, primitives.zig:424-441, sensors.zig:142-160
#include <algorithm>
#include <cmath>
#include <bitset>
#include <cstring>

#include "model.h"

namespace zb {
namespace {

// world.zig:184-212 (host side, plain products)
void hq_conj(const float q[4], float o[4]) { o[0] = -q[0], o[1] = -q[1], o[2] = -q[2], o[3] = q[3]; }
void hq_mul(const float a[4], const float b[4], float o[4]) {
  const float x = a[3] * b[0] + a[0] * b[3] + a[1] * b[2] - a[2] * b[1];
  const float y = a[3] * b[1] - a[0] * b[2] + a[1] * b[3] + a[2] * b[0];
  const float z = a[3] * b[2] + a[0] * b[1] - a[1] * b[0] + a[2] * b[3];
  const float w = a[3] * b[3] - a[0] * b[0] - a[1] * b[1] - a[2] * b[2];
  o[0] = x, o[1] = y, o[2] = z, o[3] = w;
}
void hq_rot(const float v[3], const float q[4], float o[3]) {
  const float t0 = 2.0f * (q[1] * v[2] - q[2] * v[1]);
  const float t1 = 2.0f * (q[2] * v[0] - q[0] * v[2]);
  const float t2 = 2.0f * (q[0] * v[1] - q[1] * v[0]);
  const float r0 = v[0] + q[3] * t0 + (q[1] * t2 - q[2] * t1);
  const float r1 = v[1] + q[3] * t1 + (q[2] * t0 - q[0] * t2);
  const float r2 = v[2] + q[3] * t2 + (q[0] * t1 - q[1] * t0);
  o[0] = r0, o[1] = r1, o[2] = r2;
}

float inv_mass_of(const SBody& b) {
  if (b.type == 0 || b.type == 1 || b.mass <= 0.0f) return 0.0f;
  return 1.0f / b.mass;
}
void inv_inertia_of(const SBody& b, float o[3]) {
  for (int i = 0; i < 3; ++i) o[i] = (b.type == 0 || b.type == 1) ? 0.0f : (b.inertia[i] > 1e-6f ? 1.0f / b.inertia[i] : 0.0f);
}

// One XPBDConstraint in the reference byte layout (xpbd.zig:50-76).
struct RefConstraint {
  uint32_t indices[4];
  float anchor_a[4], anchor_b[4], axis_target[4], limits[4], state[4];
};
static_assert(sizeof(RefConstraint) == 96, "XPBDConstraint");

RefConstraint blank(uint32_t type, uint32_t a, uint32_t b) {
  RefConstraint c;
  std::memset(&c, 0, sizeof(c));
  c.indices[0] = a, c.indices[1] = b, c.indices[3] = type;
  return c;
}
void put3(float* d, const float* s, float w) { d[0] = s[0], d[1] = s[1], d[2] = s[2], d[3] = w; }

// Constraint templates in joint order (joint.zig decomposition, world.zig construction).
std::vector<RefConstraint> templates(const Scene& sc) {
  std::vector<RefConstraint> out;
  const float zero3[3] = {0, 0, 0};
  for (const SJoint& j : sc.joints) {
    const bool lim = j.limited && j.lower < j.upper;
    const float* qa = sc.bodies[j.parent].quat;
    const float* qb = sc.bodies[j.child].quat;
    auto point = [&]() {
      RefConstraint c = blank(2, j.parent, j.child);
      put3(c.anchor_a, j.anchor_parent, 0.0f);
      put3(c.anchor_b, j.anchor_child, 0.0f);
      out.push_back(c);
    };
    auto hinge = [&](const float* axis, float damping) {
      float aw[3], qbi[4], ab[3];
      hq_rot(axis, qa, aw);
      hq_conj(qb, qbi);
      hq_rot(aw, qbi, ab);
      RefConstraint c = blank(3, j.parent, j.child);
      put3(c.anchor_a, axis, 0.0f);
      put3(c.anchor_b, ab, damping);
      out.push_back(c);
    };
    auto rel_quat = [&](float r[4]) {
      float qai[4];
      hq_conj(qa, qai);
      hq_mul(qai, qb, r);
    };
    switch (j.type) {
      case 0: {  // fixed -> weld
        RefConstraint c = blank(7, j.parent, j.child);
        put3(c.anchor_a, j.anchor_parent, 0.0f);
        put3(c.anchor_b, j.anchor_child, 0.0f);
        rel_quat(c.axis_target);
        out.push_back(c);
        break;
      }
      case 1:  // revolute -> point, hinge, [angular limit]
        point();
        hinge(j.axis, j.damping);
        if (lim) {
          RefConstraint c = blank(4, j.parent, j.child);
          put3(c.anchor_a, j.axis, 0.0f);
          c.limits[0] = j.lower, c.limits[1] = j.upper;
          out.push_back(c);
        }
        break;
      case 2: {  // prismatic -> slider, [linear limit]
        RefConstraint c = blank(10, j.parent, j.child);
        put3(c.anchor_a, j.anchor_parent, 0.0f);
        put3(c.anchor_b, j.anchor_child, j.damping);
        put3(c.axis_target, j.axis, 0.0f);
        rel_quat(c.limits);
        out.push_back(c);
        if (lim) {
          RefConstraint l = blank(5, j.parent, j.child);
          put3(l.anchor_a, j.axis, 0.0f);
          put3(l.anchor_b, j.anchor_child, 0.0f);
          l.limits[0] = j.lower, l.limits[1] = j.upper;
          out.push_back(l);
        }
        break;
      }
      case 3:  // ball -> point, [cone limit as symmetric angular limit]
        point();
        if (lim) {
          RefConstraint c = blank(4, j.parent, j.child);
          put3(c.anchor_a, j.axis, 0.0f);
          c.limits[0] = -j.upper, c.limits[1] = j.upper;
          out.push_back(c);
        }
        break;
      case 5:  // universal -> point, hinge(axis), hinge(axis2)
        point();
        hinge(j.axis, 0.0f);
        hinge(j.axis2, 0.0f);
        break;
      default: break;  // free: no constraint
    }
    (void)zero3;
  }
  return out;
}

// Greedy colouring: each constraint takes the smallest colour not used by an earlier
// constraint that shares one of its bodies (body 0 included).
uint32_t colour(std::vector<RefConstraint>& cs, uint32_t nb) {
  if (cs.empty()) return 0;
  std::vector<std::bitset<256>> used(nb);
  uint32_t ncol = 0;
  for (RefConstraint& c : cs) {
    const uint32_t a = c.indices[0], b = c.indices[1];
    std::bitset<256> taken;
    if (a < nb) taken |= used[a];
    if (b < nb && b != a) taken |= used[b];
    uint32_t col = 0;
    while (col < 255 && taken[col]) ++col;
    c.indices[3] = (c.indices[3] & 0xFFu) | (col << 8);
    if (a < nb) used[a].set(col);
    if (b < nb) used[b].set(col);
    ncol = std::max(ncol, col + 1);
  }
  return ncol;
}

// Radius of a sphere around the geom centre that holds the whole geom (corrected broad
// phase): sphere r, capsule r + half length, box |half extents|, cylinder
// sqrt(r^2 + half length^2); other types keep size[0].
float bound_radius(const SGeom& g) {
  switch (g.type) {
    case 1: return g.size[0] + g.size[1];
    case 2: return std::sqrt(g.size[0] * g.size[0] + g.size[1] * g.size[1] + g.size[2] * g.size[2]);
    case 4: return std::sqrt(g.size[0] * g.size[0] + g.size[1] * g.size[1]);
    default: return g.size[0];
  }
}

template <class T>
void blob(std::vector<uint8_t>& dst, const std::vector<T>& v) {
  dst.resize(v.size() * sizeof(T));
  if (!v.empty()) std::memcpy(dst.data(), v.data(), dst.size());
}

}  // namespace

// Hinge groups.  Solving the colour-sorted constraints one by one is the reference's
// colour-by-colour sweep; two constraints with no dynamic body in common commute exactly
// (each reads and writes only its own two bodies; static bodies are never written), so
// moving a constraint forward past constraints that share no dynamic body with it leaves
// every pose bit-identical.  Walking the sweep, each unplaced point constraint (type 2)
// pulls forward the axis constraint (3) and then the angle limit (4) of the same body
// pair, when every unplaced constraint in between shares no dynamic body with them; a
// group is then solved with the pair's poses held in registers.  Levels (general kernel):
// a group's level is one more than the highest level of the earlier groups it shares a
// dynamic body with, so the groups of a level touch disjoint dynamic bodies and can be
// solved side by side, and every body sees its groups in sweep order.
static void hinge_groups(HostModel* hp) {
  HostModel& h = *hp;
  const uint32_t K = uint32_t(h.constraints.size());
  auto dyn = [&](uint32_t b) { return h.bodies[b].inv_mass_inertia[0] > 0.0f; };
  auto type = [&](uint32_t k) { return h.constraints[k].type & 0xFFu; };
  auto shares = [&](uint32_t i, uint32_t j) {
    const DConstraint &a = h.constraints[i], &b = h.constraints[j];
    return (dyn(a.body_a) && (a.body_a == b.body_a || a.body_a == b.body_b)) ||
           (dyn(a.body_b) && (a.body_b == b.body_a || a.body_b == b.body_b));
  };
  constexpr uint32_t kNone = 0xFFFFFFFFu;
  std::vector<uint8_t> placed(K, 0);
  auto pull = [&](uint32_t i, uint32_t want) -> uint32_t {  // next movable constraint of type want on i's pair
    const DConstraint& c = h.constraints[i];
    for (uint32_t j = i + 1; j < K; ++j) {
      if (placed[j]) continue;
      const DConstraint& d = h.constraints[j];
      if (type(j) == want && d.body_a == c.body_a && d.body_b == c.body_b) {
        for (uint32_t x = i + 1; x < j; ++x)
          if (!placed[x] && shares(x, j)) return kNone;
        return j;
      }
      if (shares(j, i)) return kNone;  // an earlier constraint on a body of the pair comes first
    }
    return kNone;
  };
  h.hinge_groups.clear();
  for (uint32_t i = 0; i < K; ++i) {
    if (placed[i]) continue;
    placed[i] = 1;
    uint32_t k1 = i, k2 = i, kind = 0;
    if (type(i) == 2u) {
      const uint32_t j = pull(i, 3u);
      if (j != kNone) {
        placed[j] = 1;
        const uint32_t l = pull(j, 4u);
        if (l != kNone) placed[l] = 1;
        k1 = j, k2 = l != kNone ? l : i, kind = l != kNone ? 2u : 1u;
      }
    }
    h.hinge_groups.insert(h.hinge_groups.end(), {i, k1, k2, kind});
  }
  // levels (constraint indices packed in 16 bits)
  h.jgroup_words.clear();
  h.jgroup_levels.clear();
  if (K > 0xFFFFu) return;
  const uint32_t NG = uint32_t(h.hinge_groups.size() / 4);
  std::vector<uint32_t> level(NG, 0), body_level(h.B, 0);  // body_level: highest level + 1 so far
  uint32_t num_levels = 0;
  for (uint32_t g = 0; g < NG; ++g) {
    const DConstraint& c = h.constraints[h.hinge_groups[4 * g]];
    uint32_t lv = 0;
    if (dyn(c.body_a)) lv = std::max(lv, body_level[c.body_a]);
    if (dyn(c.body_b)) lv = std::max(lv, body_level[c.body_b]);
    level[g] = lv;
    if (dyn(c.body_a)) body_level[c.body_a] = lv + 1;
    if (dyn(c.body_b)) body_level[c.body_b] = lv + 1;
    num_levels = std::max(num_levels, lv + 1);
  }
  h.jgroup_levels.assign(1, 0u);
  for (uint32_t lv = 0; lv < num_levels; ++lv) {
    for (uint32_t g = 0; g < NG; ++g) {
      if (level[g] != lv) continue;
      const uint32_t* q = &h.hinge_groups[4 * g];
      h.jgroup_words.push_back(q[0] | (q[1] << 16));
      h.jgroup_words.push_back(q[2] | (q[3] << 16));
    }
    h.jgroup_levels.push_back(uint32_t(h.jgroup_words.size() / 2));
  }
}

bool build_model(const Scene& sc, HostModel* m, std::string* err) {
  HostModel h;
  h.corrected = sc.corrected;
  h.B = uint32_t(sc.bodies.size());
  h.J = uint32_t(sc.joints.size());
  h.A = uint32_t(sc.actuators.size());
  h.G = uint32_t(sc.geoms.size());
  h.S = uint32_t(sc.sensors.size());
  h.obs_dim = sc.obs_dim();
  if (h.B > 65535 || h.G > 65535) {
    if (err) *err = "more than 65535 bodies or geoms per environment";
    return false;
  }

  // bodies + joint-force incidence lists (joint order; body 0 never receives a wrench)
  h.bodies.resize(h.B);
  for (uint32_t b = 0; b < h.B; ++b) {
    const SBody& sb = sc.bodies[b];
    DBody& d = h.bodies[b];
    std::memset(&d, 0, sizeof(d));
    d.inv_mass_inertia[0] = inv_mass_of(sb);
    inv_inertia_of(sb, &d.inv_mass_inertia[1]);
    std::memcpy(d.com, sb.com, 12);
    d.type = sb.type;
    d.jf_begin = uint32_t(h.jf_list.size());
    if (b > 0)
      for (uint32_t j = 0; j < h.J; ++j) {
        if (sc.joints[j].parent == b) h.jf_list.push_back(j | 0x80000000u);
        else if (sc.joints[j].child == b) h.jf_list.push_back(j);
      }
    d.jf_end = uint32_t(h.jf_list.size());
  }
  h.subtree.assign(h.B, 1u);
  for (uint32_t b = h.B; b-- > 1;)
    if (sc.bodies[b].parent >= 0) h.subtree[uint32_t(sc.bodies[b].parent)] += h.subtree[b];

  for (const SJoint& sj : sc.joints) {
    DJoint d;
    std::memset(&d, 0, sizeof(d));
    put3(d.anchor_parent, sj.anchor_parent, 0.0f);
    put3(d.anchor_child, sj.anchor_child, 0.0f);
    put3(d.axis, sj.axis, 0.0f);
    d.type = sj.type, d.parent = sj.parent, d.child = sj.child;
    h.joints.push_back(d);
  }
  for (const SGeom& sg : sc.geoms) {
    DGeom d;
    put3(d.pos_size0, sg.pos, sg.size[0]);
    std::memcpy(d.quat, sg.quat, 16);
    d.size12_fr_rest[0] = sg.size[1], d.size12_fr_rest[1] = sg.size[2];
    d.size12_fr_rest[2] = sg.friction, d.size12_fr_rest[3] = sg.restitution;
    d.type = sg.type, d.body = sg.body, d.contype = sg.contype, d.conaffinity = sg.conaffinity;
    h.geoms.push_back(d);
  }
  // distance-test radius per geom (size[0] in the reference; the whole-geom bound under
  // corrected semantics) and the grid parameters: the cell edge exceeds every non-plane
  // pair's distance bound (r_a + r_b) + 0.1 by 0.1 %, so pairs that pass the test lie in
  // neighbouring cells; buckets: a power of two >= the grid geoms (and >= 32)
  float r_max = 0.0f;
  uint32_t n_grid = 0;
  for (uint32_t g = 0; g < h.G; ++g) {
    const SGeom& sg = sc.geoms[g];
    const float r = sc.corrected ? bound_radius(sg) : sg.size[0];
    h.geom_bound.push_back(r);
    if (sg.type == 3) {
      h.plane_geoms.push_back(g);
    } else {
      ++n_grid;
      if (r > r_max) r_max = r;
    }
  }
  {
    const double cell = (2.0 * double(r_max) + 0.1) * 1.001;
    h.grid_inv_cell = float(1.0 / cell);
    uint32_t nb = 32;
    while (nb < n_grid) nb <<= 1;
    h.grid_buckets = nb;
  }
  // broad-phase candidates: static filters of all_shaders.metal:494-507, emission order
  for (uint32_t a = 0; a < h.G; ++a)
    for (uint32_t b = a + 1; b < h.G; ++b) {
      const SGeom &ga = sc.geoms[a], &gb = sc.geoms[b];
      if (ga.body == gb.body) continue;
      if ((ga.contype & gb.conaffinity) == 0 && (gb.contype & ga.conaffinity) == 0) continue;
      const float md = (sc.corrected ? bound_radius(ga) + bound_radius(gb) : ga.size[0] + gb.size[0]) + 0.1f;
      h.pairs.push_back(DPair{a, b, md * md, (ga.type == 3 || gb.type == 3) ? 1u : 0u});
    }
  std::vector<uint32_t> seen(h.J, 0);
  for (const SActuator& sa : sc.actuators) {
    DActuator d;
    std::memset(&d, 0, sizeof(d));
    d.joint = sa.joint;
    d.ctrl_min = sa.ctrl_min, d.ctrl_max = sa.ctrl_max, d.gear = sa.gear;
    d.force_min = sa.force_min, d.force_max = sa.force_max;
    h.actuators.push_back(d);
    if (sa.joint < h.J && seen[sa.joint]++) h.actuators_unique = false;
  }
  uint32_t off = 0;
  for (const SSensor& ss : sc.sensors) {
    h.sensors.push_back(DSensor{ss.type, ss.object, off, ss.dim});
    off += ss.dim;
  }

  // constraints: templates -> colours -> stable sort by colour -> ranges
  std::vector<RefConstraint> tc = templates(sc);
  h.K = uint32_t(tc.size());
  h.num_colors = colour(tc, h.B);
  std::stable_sort(tc.begin(), tc.end(), [](const RefConstraint& x, const RefConstraint& y) {
    return ((x.indices[3] >> 8) & 0xFFu) < ((y.indices[3] >> 8) & 0xFFu);
  });
  h.color_ranges.assign(2 * h.num_colors, 0u);
  for (uint32_t i = 0; i < h.K; ++i) {
    const uint32_t c = (tc[i].indices[3] >> 8) & 0xFFu;
    if (h.color_ranges[2 * c + 1] == 0) h.color_ranges[2 * c] = i;
    h.color_ranges[2 * c + 1]++;
  }
  // Kernel copy.  An angular limit (type 4) whose range contains [-6.29, 6.29] never acts:
  // the hinge angle is 2 atan2(.), within 2 pi in magnitude, so the violation is always 0
  // (a NaN angle compares false as well) and the constraint changes nothing.  The
  // reference's raw-radian MJCF ranges (Ant hips +-30, every Humanoid limit) are of this
  // kind; dropping them from the colour runs leaves every other constraint's order and
  // every result unchanged.
  h.kcolor_ranges.assign(2 * h.num_colors, 0u);
  for (uint32_t i = 0; i < uint32_t(tc.size()); ++i) {
    const RefConstraint& r = tc[i];
    const uint32_t type = r.indices[3] & 0xFFu;
    if (type == 4 && r.limits[0] < -6.29f && r.limits[1] > 6.29f) continue;
    DConstraint d;
    std::memset(&d, 0, sizeof(d));
    d.body_a = r.indices[0], d.body_b = r.indices[1], d.type = r.indices[3];
    std::memcpy(d.anchor_a, r.anchor_a, 16);
    std::memcpy(d.anchor_b, r.anchor_b, 16);
    std::memcpy(d.axis_target, r.axis_target, 16);
    std::memcpy(d.limits, r.limits, 16);
    const uint32_t c = (r.indices[3] >> 8) & 0xFFu;
    if (h.kcolor_ranges[2 * c + 1] == 0) h.kcolor_ranges[2 * c] = uint32_t(h.constraints.size());
    h.kcolor_ranges[2 * c + 1]++;
    h.constraints.push_back(d);
  }
  h.K = uint32_t(h.constraints.size());
  blob(h.ref_constraints, tc);
  hinge_groups(&h);

  // initial-state template (world.zig:663-691, env 0; state.zig:358-388)
  h.init_state.assign(16 * h.B + 2 * h.J, 0.0f);
  for (uint32_t b = 0; b < h.B; ++b) {
    const SBody& sb = sc.bodies[b];
    std::memcpy(&h.init_state[4 * b], sb.pos, 12);
    std::memcpy(&h.init_state[4 * (h.B + b)], sb.quat, 16);
  }

  // reference-layout records for parity checks of the model tables
  struct RB { float position[4], quaternion[4], inv_mass_inertia[4], params[4], com_offset[4]; };
  struct RJ { float anchor_parent[4], anchor_child[4], axis[4], params[4], params2[4]; };
  struct RG { uint32_t type_body[4]; float pos_size0[4], quat[4], params[4]; };
  struct RA { float params[4], params2[4]; };
  struct RS { uint32_t type_object[4]; float params[4]; };
  std::vector<RB> rb;
  for (uint32_t b = 0; b < h.B; ++b) {
    const SBody& sb = sc.bodies[b];
    RB r;
    put3(r.position, sb.pos, 0.0f);
    std::memcpy(r.quaternion, sb.quat, 16);
    std::memcpy(r.inv_mass_inertia, h.bodies[b].inv_mass_inertia, 16);
    r.params[0] = float(sb.parent), r.params[1] = float(sb.type), r.params[2] = 1.0f, r.params[3] = 0.0f;
    put3(r.com_offset, sb.com, 0.0f);
    rb.push_back(r);
  }
  std::vector<RJ> rj;
  for (const SJoint& sj : sc.joints) {
    RJ r;
    put3(r.anchor_parent, sj.anchor_parent, 0.0f);
    put3(r.anchor_child, sj.anchor_child, 0.0f);
    put3(r.axis, sj.axis, 0.0f);
    r.params[0] = float(sj.type), r.params[1] = float(sj.parent), r.params[2] = float(sj.child), r.params[3] = sj.lower;
    r.params2[0] = sj.upper, r.params2[1] = sj.damping, r.params2[2] = sj.stiffness, r.params2[3] = sj.ref;
    rj.push_back(r);
  }
  std::vector<RG> rg;
  for (const SGeom& sg : sc.geoms) {
    RG r;
    r.type_body[0] = sg.type, r.type_body[1] = sg.body, r.type_body[2] = sg.conaffinity, r.type_body[3] = sg.contype;
    put3(r.pos_size0, sg.pos, sg.size[0]);
    std::memcpy(r.quat, sg.quat, 16);
    r.params[0] = sg.size[1], r.params[1] = sg.size[2], r.params[2] = sg.friction, r.params[3] = sg.restitution;
    rg.push_back(r);
  }
  std::vector<RA> ra;
  for (const SActuator& sa : sc.actuators) {
    RA r;
    r.params[0] = float(sa.joint), r.params[1] = sa.ctrl_min, r.params[2] = sa.ctrl_max, r.params[3] = sa.gear;
    r.params2[0] = sa.force_min, r.params2[1] = sa.force_max, r.params2[2] = sa.kp, r.params2[3] = sa.kv;
    ra.push_back(r);
  }
  std::vector<RS> rs;
  off = 0;
  for (const SSensor& ss : sc.sensors) {
    RS r;
    r.type_object[0] = ss.type, r.type_object[1] = ss.object, r.type_object[2] = ss.dim, r.type_object[3] = 0;
    r.params[0] = ss.noise, r.params[1] = ss.cutoff, r.params[2] = float(ss.dim), r.params[3] = float(off);
    off += ss.dim;
    rs.push_back(r);
  }
  blob(h.ref_bodies, rb);
  blob(h.ref_joints, rj);
  blob(h.ref_geoms, rg);
  blob(h.ref_actuators, ra);
  blob(h.ref_sensors, rs);
  *m = std::move(h);
  return true;
}

}  // namespace zb
