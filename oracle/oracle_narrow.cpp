// TEST INFRASTRUCTURE ONLY -- restatement of the reference's CPU collision routines
// (src/collision/narrow_phase.zig, detectCollision and the primitive pairs it dispatches
// to), used by the oracle when a world selects the extended narrow phase.
//
// Semantics kept from the reference code:
//  * a geom is placed by its body transform: centre = R(q_body) * local_pos + body_pos
//    (getWorldCenter, primitives.zig:413-415); capsule axes, box axes and plane normals
//    come from the body quaternion only (the geom's own local quaternion is not applied);
//  * boxes are centred on the body origin in sphereBox / boxPlane (they use the body
//    transform, not the geom centre), but on the geom centre in boxBox;
//  * box-capsule pairs, plane-plane pairs and every pair with a cylinder, mesh or
//    heightfield report no contact (no primitive routine, or outside this build's scope);
//  * narrow-phase mode 2 adds one extension: box-capsule pairs go through the reference's
//    GJK + EPA (src/collision/gjk.zig, which the reference itself runs only for meshes),
//    on the sphere / capsule / box support maps of that file, and the contact is built as
//    meshPrimitiveCollision builds it.
// Arithmetic follows the Zig source literally: plain IEEE-754 single-precision +, -, *,
// / and sqrt, evaluated left to right as written (Zig's default float mode contracts
// nothing); the oracle is compiled with -ffp-contract=off for the same reason.
#include <cmath>
#include <limits>
#include <utility>

#include "oracle_model.h"

namespace zo {
namespace {

constexpr float kEps = 1e-6f;  // constants.EPSILON (src/physics/constants.zig:13)

struct P3 {
  float x, y, z;
};
inline P3 p3(const float* v) { return P3{v[0], v[1], v[2]}; }
inline P3 add(P3 a, P3 b) { return P3{a.x + b.x, a.y + b.y, a.z + b.z}; }
inline P3 sub(P3 a, P3 b) { return P3{a.x - b.x, a.y - b.y, a.z - b.z}; }
inline P3 scl(P3 v, float s) { return P3{v.x * s, v.y * s, v.z * s}; }
inline float dot(P3 a, P3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline P3 cross(P3 a, P3 b) { return P3{a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
inline float clampf(float v, float lo, float hi) { return std::fmax(lo, std::fmin(v, hi)); }

struct Quat {
  float x, y, z, w;
};
// rotateByQuat (src/physics/body.zig:254-264): v + 2 (w (q x v) + q x (q x v))
inline P3 rot(P3 v, Quat q) {
  const P3 qv{q.x, q.y, q.z};
  const P3 uv = cross(qv, v);
  const P3 uuv = cross(qv, uv);
  return P3{v.x + 2.0f * (q.w * uv.x + uuv.x), v.y + 2.0f * (q.w * uv.y + uuv.y), v.z + 2.0f * (q.w * uv.z + uuv.z)};
}
struct Xf {  // body.Transform
  P3 p;
  Quat q;
  P3 point(P3 v) const { return add(rot(v, q), p); }  // transformPoint
  P3 vec(P3 v) const { return rot(v, q); }            // transformVector
  Xf inverse() const {                                 // inverse()
    const Quat iq{-q.x, -q.y, -q.z, q.w};
    return Xf{rot(P3{-p.x, -p.y, -p.z}, iq), iq};
  }
};

struct Res {
  P3 point, normal;
  float pen;
};

// -------------------------------------------------------------- helpers (narrow_phase.zig)
P3 closest_on_segment(P3 point, P3 s, P3 e) {
  const P3 seg = sub(e, s);
  const float len_sq = dot(seg, seg);
  if (len_sq < kEps) return s;
  const float t = clampf(dot(sub(point, s), seg) / len_sq, 0.0f, 1.0f);
  return add(s, scl(seg, t));
}

void closest_between_segments(P3 a1, P3 a2, P3 b1, P3 b2, P3* pa, P3* pb) {
  const P3 d1 = sub(a2, a1), d2 = sub(b2, b1), r = sub(a1, b1);
  const float a = dot(d1, d1), e = dot(d2, d2), f = dot(d2, r);
  float s = 0.0f, t = 0.0f;
  if (a < kEps && e < kEps) {
    *pa = a1, *pb = b1;
    return;
  }
  if (a < kEps) {
    t = clampf(f / e, 0.0f, 1.0f);
  } else {
    const float c = dot(d1, r);
    if (e < kEps) {
      s = clampf(-c / a, 0.0f, 1.0f);
    } else {
      const float b = dot(d1, d2);
      const float denom = a * e - b * b;
      if (denom != 0.0f) s = clampf((b * f - c * e) / denom, 0.0f, 1.0f);
      t = (b * s + f) / e;
      if (t < 0.0f) {
        t = 0.0f;
        s = clampf(-c / a, 0.0f, 1.0f);
      } else if (t > 1.0f) {
        t = 1.0f;
        s = clampf((b - c) / a, 0.0f, 1.0f);
      }
    }
  }
  *pa = add(a1, scl(d1, s));
  *pb = add(b1, scl(d2, t));
}

P3 box_face_normal(P3 p, P3 h) {  // the face with the largest distance, as written
  const float pc[3] = {p.x, p.y, p.z}, hc[3] = {h.x, h.y, h.z};
  float max_dist = -std::numeric_limits<float>::infinity();
  float n[3] = {0.0f, 0.0f, 1.0f};
  for (int i = 0; i < 3; ++i) {
    const float d_pos = hc[i] - pc[i], d_neg = hc[i] + pc[i];
    if (d_pos > max_dist) {
      max_dist = d_pos;
      n[0] = n[1] = n[2] = 0.0f;
      n[i] = 1.0f;
    }
    if (d_neg > max_dist) {
      max_dist = d_neg;
      n[0] = n[1] = n[2] = 0.0f;
      n[i] = -1.0f;
    }
  }
  return P3{n[0], n[1], n[2]};
}

// testAxis: overlap on `axis`, or false when it separates
bool test_axis(P3 axis, P3 d, const P3* axa, P3 ha, const P3* axb, P3 hb, float* overlap) {
  const float proj_a = ha.x * std::fabs(dot(axis, axa[0])) + ha.y * std::fabs(dot(axis, axa[1])) +
                       ha.z * std::fabs(dot(axis, axa[2]));
  const float proj_b = hb.x * std::fabs(dot(axis, axb[0])) + hb.y * std::fabs(dot(axis, axb[1])) +
                       hb.z * std::fabs(dot(axis, axb[2]));
  const float dist = std::fabs(dot(d, axis));
  if (dist > proj_a + proj_b) return false;
  *overlap = proj_a + proj_b - dist;
  return true;
}

// ------------------------------------------------------------------ primitive pairs
bool sphere_sphere(P3 pa, float ra, P3 pb, float rb, Res* o) {
  const P3 diff = sub(pb, pa);
  const float dist_sq = dot(diff, diff), min_dist = ra + rb;
  if (dist_sq >= min_dist * min_dist) return false;
  const float dist = std::sqrt(dist_sq);
  const P3 n = dist > kEps ? scl(diff, 1.0f / dist) : P3{0.0f, 0.0f, 1.0f};
  const float pen = min_dist - dist;
  *o = Res{add(pa, scl(n, ra - pen * 0.5f)), n, pen};
  return true;
}

bool sphere_capsule(P3 sp, float sr, P3 cp, float cr, float hl, const Xf& ct, Res* o) {
  const P3 axis = ct.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 p1 = sub(cp, scl(axis, hl)), p2 = add(cp, scl(axis, hl));
  const P3 closest = closest_on_segment(sp, p1, p2);
  const P3 diff = sub(sp, closest);
  const float dist_sq = dot(diff, diff), min_dist = sr + cr;
  if (dist_sq >= min_dist * min_dist) return false;
  const float dist = std::sqrt(dist_sq);
  const P3 n = dist > kEps ? scl(diff, 1.0f / dist) : P3{0.0f, 0.0f, 1.0f};
  const float pen = min_dist - dist;
  *o = Res{add(closest, scl(n, cr - pen * 0.5f)), n, pen};
  return true;
}

bool sphere_plane(P3 sp, float sr, P3 plane_local, float plane_off, const Xf& pt, Res* o) {
  const P3 n = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 plane_point = pt.point(plane_local);
  const float sd = dot(sub(sp, plane_point), n) - plane_off;
  if (sd >= sr) return false;
  const float pen = sr - sd;
  *o = Res{sub(sp, scl(n, sd + pen * 0.5f)), n, pen};
  return true;
}

bool sphere_box(P3 sp, float sr, P3 half, const Xf& bt, Res* o) {
  const Xf inv = bt.inverse();
  const P3 ls = inv.point(sp);
  const P3 cl{clampf(ls.x, -half.x, half.x), clampf(ls.y, -half.y, half.y), clampf(ls.z, -half.z, half.z)};
  const P3 diff = sub(ls, cl);
  const float dist_sq = dot(diff, diff);
  if (dist_sq >= sr * sr) return false;
  const float dist = std::sqrt(dist_sq);
  const P3 ln = dist > kEps ? scl(diff, 1.0f / dist) : box_face_normal(ls, half);
  const P3 wc = bt.point(cl);
  const P3 n = bt.vec(ln);
  const float pen = sr - dist;
  *o = Res{add(wc, scl(n, pen * 0.5f)), n, pen};
  return true;
}

bool capsule_capsule(P3 pa, float ra, float hla, const Xf& ta, P3 pb, float rb, float hlb, const Xf& tb, Res* o) {
  const P3 axa = ta.vec(P3{0.0f, 0.0f, 1.0f}), axb = tb.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 a1 = sub(pa, scl(axa, hla)), a2 = add(pa, scl(axa, hla));
  const P3 b1 = sub(pb, scl(axb, hlb)), b2 = add(pb, scl(axb, hlb));
  P3 ca, cb;
  closest_between_segments(a1, a2, b1, b2, &ca, &cb);
  const P3 diff = sub(cb, ca);
  const float dist_sq = dot(diff, diff), min_dist = ra + rb;
  if (dist_sq >= min_dist * min_dist) return false;
  const float dist = std::sqrt(dist_sq);
  const P3 n = dist > kEps ? scl(diff, 1.0f / dist) : P3{0.0f, 0.0f, 1.0f};
  const float pen = min_dist - dist;
  const P3 paw = add(ca, scl(n, ra)), pbw = sub(cb, scl(n, rb));
  *o = Res{scl(add(paw, pbw), 0.5f), n, pen};
  return true;
}

bool capsule_plane(P3 cp, float r, float hl, const Xf& ct, P3 plane_local, const Xf& pt, Res* o) {
  const P3 axis = ct.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pn = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pp = pt.point(plane_local);
  const P3 p1 = sub(cp, scl(axis, hl)), p2 = add(cp, scl(axis, hl));
  const float d1 = dot(sub(p1, pp), pn) - r, d2 = dot(sub(p2, pp), pn) - r;
  if (d1 >= 0.0f && d2 >= 0.0f) return false;
  const P3 deepest = d1 < d2 ? p1 : p2;
  const float dist = std::fmin(d1, d2);
  *o = Res{sub(deepest, scl(pn, dist * 0.5f + r)), pn, -dist};
  return true;
}

bool box_plane(P3 half, const Xf& bt, P3 plane_local, const Xf& pt, Res* o) {
  const P3 pn = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pp = pt.point(plane_local);
  const float hx = half.x, hy = half.y, hz = half.z;
  const P3 corners[8] = {{-hx, -hy, -hz}, {hx, -hy, -hz}, {-hx, hy, -hz}, {hx, hy, -hz},
                         {-hx, -hy, hz},  {hx, -hy, hz},  {-hx, hy, hz},  {hx, hy, hz}};
  float min_dist = std::numeric_limits<float>::infinity();
  P3 deepest{0.0f, 0.0f, 0.0f};
  for (const P3& c : corners) {
    const P3 wc = bt.point(c);
    const float dist = dot(sub(wc, pp), pn);
    if (dist < min_dist) {
      min_dist = dist;
      deepest = wc;
    }
  }
  if (min_dist >= 0.0f) return false;
  *o = Res{deepest, pn, -min_dist};
  return true;
}

bool box_box(P3 pa, P3 ha, const Xf& ta, P3 pb, P3 hb, const Xf& tb, Res* o) {
  const P3 axa[3] = {ta.vec(P3{1.0f, 0.0f, 0.0f}), ta.vec(P3{0.0f, 1.0f, 0.0f}), ta.vec(P3{0.0f, 0.0f, 1.0f})};
  const P3 axb[3] = {tb.vec(P3{1.0f, 0.0f, 0.0f}), tb.vec(P3{0.0f, 1.0f, 0.0f}), tb.vec(P3{0.0f, 0.0f, 1.0f})};
  const P3 d = sub(pb, pa);
  float min_overlap = std::numeric_limits<float>::infinity(), ov = 0.0f;
  P3 best{0.0f, 0.0f, 1.0f};
  for (int i = 0; i < 3; ++i) {
    if (!test_axis(axa[i], d, axa, ha, axb, hb, &ov)) return false;
    if (ov < min_overlap) min_overlap = ov, best = axa[i];
  }
  for (int i = 0; i < 3; ++i) {
    if (!test_axis(axb[i], d, axa, ha, axb, hb, &ov)) return false;
    if (ov < min_overlap) min_overlap = ov, best = axb[i];
  }
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      const P3 ea = cross(axa[i], axb[j]);
      const float len = std::sqrt(dot(ea, ea));
      if (len < kEps) continue;
      const P3 nrm = scl(ea, 1.0f / len);
      if (!test_axis(nrm, d, axa, ha, axb, hb, &ov)) return false;
      if (ov < min_overlap) min_overlap = ov, best = nrm;
    }
  if (dot(best, d) < 0.0f) best = scl(best, -1.0f);
  *o = Res{add(pa, scl(d, 0.5f)), best, min_overlap};
  return true;
}

Res flip(Res r) { return Res{r.point, scl(r.normal, -1.0f), r.pen}; }

// ---- GJK + EPA (src/collision/gjk.zig) on the sphere, capsule and box support maps ----
constexpr float kGjkTol = 1e-6f;  // GJK_TOLERANCE (gjk.zig:17)
constexpr float kEpaTol = 1e-4f;  // EPA_TOLERANCE (gjk.zig:19)
constexpr int kGjkIters = 64;     // GJK_MAX_ITERATIONS
constexpr int kEpaIters = 64;     // EPA_MAX_ITERATIONS
constexpr int kEpaFaces = 128;    // EPA_MAX_FACES
constexpr int kEpaEdges = 256;    // horizon edge list (addEdge)
// EPA starts from 4 vertices and adds at most one per iteration, so its 256-entry vertex
// array never holds more than 4 + 64.
constexpr int kEpaVerts = 4 + kEpaIters;

struct Shape {  // ConvexShape: geom type 0 sphere, 1 capsule, 2 box; body transform
  uint32_t type;
  P3 local;  // geom local position
  P3 size;   // size[0..2]: radius / half length, or box half extents
  Xf xf;
};

inline P3 neg(P3 v) { return P3{-v.x, -v.y, -v.z}; }
// safeNormalize (gjk.zig:661-665)
inline P3 safe_normalize(P3 v) {
  const float len = std::sqrt(dot(v, v));
  if (len < kGjkTol) return P3{0.0f, 0.0f, 1.0f};
  return scl(v, 1.0f / len);
}
inline P3 triple(P3 a, P3 b, P3 c) { return cross(cross(a, b), c); }  // tripleProduct
// perpendicular (gjk.zig:673-679)
inline P3 perpendicular(P3 v) {
  if (std::fabs(v.x) < std::fabs(v.y)) return safe_normalize(cross(v, P3{1.0f, 0.0f, 0.0f}));
  return safe_normalize(cross(v, P3{0.0f, 1.0f, 0.0f}));
}

// sphereSupport / capsuleSupport / boxSupport (gjk.zig:70-120).  The box support point is
// taken about the body origin (transformPoint of the corner), as written.
P3 support(const Shape& s, P3 dir) {
  if (s.type == 0) {
    const P3 c = s.xf.point(s.local);
    return add(c, scl(safe_normalize(dir), s.size.x));
  }
  if (s.type == 1) {
    const P3 c = s.xf.point(s.local);
    const P3 axis = s.xf.vec(P3{0.0f, 0.0f, 1.0f});
    const P3 n = safe_normalize(dir);
    const float d = dot(axis, dir);
    const P3 e = d >= 0.0f ? add(c, scl(axis, s.size.y)) : sub(c, scl(axis, s.size.y));
    return add(e, scl(n, s.size.x));
  }
  const P3 ld = s.xf.inverse().vec(dir);
  const P3 corner{ld.x >= 0.0f ? s.size.x : -s.size.x, ld.y >= 0.0f ? s.size.y : -s.size.y,
                  ld.z >= 0.0f ? s.size.z : -s.size.z};
  return s.xf.point(corner);
}

struct MinkPoint {
  P3 p, sa, sb;
};
// minkowskiSupport (gjk.zig:137-149): support of A - B
inline MinkPoint mink(const Shape& A, const Shape& B, P3 dir) {
  const P3 sa = support(A, dir), sb = support(B, neg(dir));
  return MinkPoint{sub(sa, sb), sa, sb};
}

struct Simplex {
  P3 s[4], sa[4], sb[4];
  uint32_t n;
};

// doSimplex2 (gjk.zig:226-253); the support points are left as they are, as written.
void simplex2(Simplex& x, P3& dir) {
  const P3 a = x.s[1], b = x.s[0];
  const P3 ab = sub(b, a), ao = neg(a);
  if (dot(ab, ao) > 0.0f) {
    dir = triple(ab, ao, ab);
    if (dot(dir, dir) < kGjkTol) dir = perpendicular(ab);
  } else {
    x.s[0] = a;
    x.n = 1;
    dir = ao;
  }
}

// doSimplex3 (gjk.zig:256-339)
void simplex3(Simplex& x, P3& dir) {
  const P3 a = x.s[2], b = x.s[1], c = x.s[0];
  const P3 ab = sub(b, a), ac = sub(c, a), ao = neg(a);
  const P3 abc = cross(ab, ac);
  if (dot(cross(ab, abc), ao) > 0.0f) {
    if (dot(ab, ao) > 0.0f) {
      x.s[0] = b, x.s[1] = a;
      x.sa[0] = x.sa[1], x.sb[0] = x.sb[1];
      x.sa[1] = x.sa[2], x.sb[1] = x.sb[2];
      x.n = 2;
      dir = triple(ab, ao, ab);
      if (dot(dir, dir) < kGjkTol) dir = perpendicular(ab);
    } else {
      x.s[0] = a;
      x.sa[0] = x.sa[2], x.sb[0] = x.sb[2];
      x.n = 1;
      dir = ao;
    }
    return;
  }
  if (dot(cross(abc, ac), ao) > 0.0f) {
    if (dot(ac, ao) > 0.0f) {
      x.s[0] = c, x.s[1] = a;
      x.sa[1] = x.sa[2], x.sb[1] = x.sb[2];
      x.n = 2;
      dir = triple(ac, ao, ac);
      if (dot(dir, dir) < kGjkTol) dir = perpendicular(ac);
    } else {
      x.s[0] = a;
      x.sa[0] = x.sa[2], x.sb[0] = x.sb[2];
      x.n = 1;
      dir = ao;
    }
    return;
  }
  if (dot(abc, ao) > 0.0f) {
    dir = abc;
  } else {
    std::swap(x.s[0], x.s[1]);
    std::swap(x.sa[0], x.sa[1]);
    std::swap(x.sb[0], x.sb[1]);
    dir = neg(abc);
  }
}

// doSimplex4 (gjk.zig:342-413).  The support copies run in the written order: in the ADB
// case slot 1 receives the already overwritten slot 0 (b), as in the reference.
bool simplex4(Simplex& x, P3& dir) {
  const P3 a = x.s[3], b = x.s[2], c = x.s[1], d = x.s[0];
  const P3 ab = sub(b, a), ac = sub(c, a), ad = sub(d, a), ao = neg(a);
  const P3 abc = cross(ab, ac), acd = cross(ac, ad), adb = cross(ad, ab);
  if (dot(abc, ao) > 0.0f) {
    x.s[0] = c, x.s[1] = b, x.s[2] = a;
    x.sa[0] = x.sa[1], x.sb[0] = x.sb[1];
    x.sa[1] = x.sa[2], x.sb[1] = x.sb[2];
    x.sa[2] = x.sa[3], x.sb[2] = x.sb[3];
    x.n = 3;
    dir = abc;
    return false;
  }
  if (dot(acd, ao) > 0.0f) {
    x.s[0] = d, x.s[1] = c, x.s[2] = a;
    x.sa[2] = x.sa[3], x.sb[2] = x.sb[3];
    x.n = 3;
    dir = acd;
    return false;
  }
  if (dot(adb, ao) > 0.0f) {
    x.s[0] = b, x.s[1] = d, x.s[2] = a;
    x.sa[0] = x.sa[2], x.sb[0] = x.sb[2];
    x.sa[1] = x.sa[0], x.sb[1] = x.sb[0];
    x.sa[2] = x.sa[3], x.sb[2] = x.sb[3];
    x.n = 3;
    dir = adb;
    return false;
  }
  return true;
}

// gjk (gjk.zig:152-223)
bool gjk(const Shape& A, const Shape& B, Simplex& x) {
  P3 dir = sub(B.xf.point(B.local), A.xf.point(A.local));
  if (dot(dir, dir) < kGjkTol) dir = P3{1.0f, 0.0f, 0.0f};
  const MinkPoint first = mink(A, B, dir);
  x.s[0] = first.p, x.sa[0] = first.sa, x.sb[0] = first.sb;
  x.n = 1;
  dir = neg(first.p);
  for (int it = 0; it < kGjkIters; ++it) {
    const MinkPoint m = mink(A, B, dir);
    if (dot(m.p, dir) < -kGjkTol) return false;
    const uint32_t i = x.n;
    x.s[i] = m.p, x.sa[i] = m.sa, x.sb[i] = m.sb;
    x.n += 1;
    if (x.n == 2) simplex2(x, dir);
    else if (x.n == 3) simplex3(x, dir);
    else if (simplex4(x, dir)) return true;
  }
  return false;
}

struct Face {
  uint32_t i0, i1, i2;
  P3 n;
  float d;
};

// faceNormal (gjk.zig:600-604)
inline P3 face_normal(P3 a, P3 b, P3 c) { return safe_normalize(cross(sub(b, a), sub(c, a))); }

// barycentricOriginProjection (gjk.zig:607-638)
void barycentric(P3 a, P3 b, P3 c, float out[3]) {
  const float third = 1.0f / 3.0f;
  const P3 ab = sub(b, a), ac = sub(c, a), ao = neg(a);
  const float d00 = dot(ab, ab), d01 = dot(ab, ac), d11 = dot(ac, ac), d20 = dot(ao, ab), d21 = dot(ao, ac);
  const float denom = d00 * d11 - d01 * d01;
  if (std::fabs(denom) < kGjkTol) {
    out[0] = out[1] = out[2] = third;
    return;
  }
  const float v = (d11 * d20 - d01 * d21) / denom;
  const float w = (d00 * d21 - d01 * d20) / denom;
  const float u = 1.0f - v - w;
  const float cu = clampf(u, 0.0f, 1.0f), cv = clampf(v, 0.0f, 1.0f), cw = clampf(w, 0.0f, 1.0f);
  const float total = cu + cv + cw;
  if (total < kGjkTol) {
    out[0] = out[1] = out[2] = third;
    return;
  }
  out[0] = cu / total, out[1] = cv / total, out[2] = cw / total;
}

// addEdge (gjk.zig:577-597): a reversed duplicate cancels, else append while room remains.
void add_edge(uint32_t (*edges)[2], uint32_t& ne, uint32_t a, uint32_t b) {
  for (uint32_t i = 0; i < ne; ++i)
    if (edges[i][0] == b && edges[i][1] == a) {
      edges[i][0] = edges[ne - 1][0], edges[i][1] = edges[ne - 1][1];
      ne -= 1;
      return;
    }
  if (ne < uint32_t(kEpaEdges)) edges[ne][0] = a, edges[ne][1] = b, ne += 1;
}

// epa (gjk.zig:424-574): contact normal (A to B), depth and the witness points on A and B.
bool epa(const Shape& A, const Shape& B, const Simplex& x, P3* normal, float* depth, P3* pa, P3* pb) {
  if (x.n < 4) return false;
  P3 v[kEpaVerts], va[kEpaVerts], vb[kEpaVerts];
  uint32_t nv = 4;
  for (int i = 0; i < 4; ++i) v[i] = x.s[i], va[i] = x.sa[i], vb[i] = x.sb[i];
  Face f[kEpaFaces];
  uint32_t nf = 0;
  static const uint32_t tet[4][3] = {{0, 1, 2}, {0, 3, 1}, {0, 2, 3}, {1, 3, 2}};
  for (const auto& t : tet) {
    const P3 n = face_normal(v[t[0]], v[t[1]], v[t[2]]);
    const float d = dot(n, v[t[0]]);
    if (d < 0.0f) f[nf++] = Face{t[0], t[2], t[1], neg(n), -d};
    else f[nf++] = Face{t[0], t[1], t[2], n, d};
  }
  auto finish = [&](uint32_t k, float dist) {
    const Face& fc = f[k];
    float w[3];
    barycentric(v[fc.i0], v[fc.i1], v[fc.i2], w);
    *pa = add(add(scl(va[fc.i0], w[0]), scl(va[fc.i1], w[1])), scl(va[fc.i2], w[2]));
    *pb = add(add(scl(vb[fc.i0], w[0]), scl(vb[fc.i1], w[1])), scl(vb[fc.i2], w[2]));
    *normal = fc.n;
    *depth = dist;
  };
  auto closest = [&](float* dist) {
    uint32_t k = 0;
    float best = std::numeric_limits<float>::infinity();
    for (uint32_t i = 0; i < nf; ++i)
      if (f[i].d < best) best = f[i].d, k = i;
    *dist = best;
    return k;
  };
  for (int it = 0; it < kEpaIters; ++it) {
    float cd;
    const uint32_t k = closest(&cd);
    const P3 dir = f[k].n;
    const MinkPoint m = mink(A, B, dir);
    if (dot(m.p, dir) - cd < kEpaTol) {
      finish(k, cd);
      return true;
    }
    const uint32_t ni = nv;
    v[nv] = m.p, va[nv] = m.sa, vb[nv] = m.sb;
    nv += 1;
    uint32_t edges[kEpaEdges][2];
    uint32_t ne = 0;
    for (uint32_t i = 0; i < nf;) {
      if (dot(f[i].n, sub(m.p, v[f[i].i0])) > 0.0f) {
        add_edge(edges, ne, f[i].i0, f[i].i1);
        add_edge(edges, ne, f[i].i1, f[i].i2);
        add_edge(edges, ne, f[i].i2, f[i].i0);
        f[i] = f[nf - 1];
        nf -= 1;
      } else {
        i += 1;
      }
    }
    for (uint32_t e = 0; e < ne; ++e) {
      if (nf >= uint32_t(kEpaFaces)) break;
      const uint32_t e0 = edges[e][0], e1 = edges[e][1];
      const P3 n = face_normal(v[e0], v[e1], v[ni]);
      const float d = dot(n, v[e0]);
      if (d < 0.0f) f[nf++] = Face{e1, e0, ni, neg(n), -d};
      else f[nf++] = Face{e0, e1, ni, n, d};
    }
    if (nf == 0) break;
  }
  if (nf == 0) return false;
  float cd;
  const uint32_t k = closest(&cd);
  finish(k, cd);
  return true;
}

// The contact the reference builds from GJK + EPA (meshPrimitiveCollision,
// narrow_phase.zig:693-747): point = midpoint of the witness points, normal = EPA normal
// (A to B), penetration = EPA depth.
bool gjk_contact(const Shape& A, const Shape& B, Res* o) {
  Simplex x{};
  if (!gjk(A, B, x)) return false;
  P3 n, pa, pb;
  float depth;
  if (!epa(A, B, x, &n, &depth, &pa, &pb)) return false;
  *o = Res{scl(add(pa, pb), 0.5f), n, depth};
  return true;
}

}  // namespace

// detectCollision (narrow_phase.zig:28-136) for the primitive geoms.  Geom types: 0 sphere,
// 1 capsule, 2 box, 3 plane; anything else reports no contact.
bool narrow_cpu(const GeomRec& ga, const float* bpa, const float* bqa, const GeomRec& gb, const float* bpb,
                const float* bqb, float point[3], float normal[3], float* pen, bool gjk_pairs) {
  const Xf ta{p3(bpa), Quat{bqa[0], bqa[1], bqa[2], bqa[3]}};
  const Xf tb{p3(bpb), Quat{bqb[0], bqb[1], bqb[2], bqb[3]}};
  const P3 la = p3(ga.pos_size0), lb = p3(gb.pos_size0);
  const P3 pa = ta.point(la), pb = tb.point(lb);  // getWorldCenter
  const float ra = ga.pos_size0[3], rb = gb.pos_size0[3];
  const float hla = ga.params[0], hlb = gb.params[0];  // size[1]
  const P3 sza{ga.pos_size0[3], ga.params[0], ga.params[1]}, szb{gb.pos_size0[3], gb.params[0], gb.params[1]};
  const uint32_t ka = ga.type_body[0], kb = gb.type_body[0];
  Res r{};
  bool hit = false;
  if (ka == 0) {
    if (kb == 0) hit = sphere_sphere(pa, ra, pb, rb, &r);
    else if (kb == 1) hit = sphere_capsule(pa, ra, pb, rb, hlb, tb, &r);
    else if (kb == 2) hit = sphere_box(pa, ra, szb, tb, &r);
    else if (kb == 3) hit = sphere_plane(pa, ra, lb, rb, tb, &r);
  } else if (gjk_pairs && ((ka == 1 && kb == 2) || (ka == 2 && kb == 1))) {
    const Shape A{ka, la, sza, ta}, B{kb, lb, szb, tb};
    hit = gjk_contact(A, B, &r);
  } else if (ka == 1) {
    if (kb == 0) {
      hit = sphere_capsule(pb, rb, pa, ra, hla, ta, &r);
      if (hit) r = flip(r);
    } else if (kb == 1) {
      hit = capsule_capsule(pa, ra, hla, ta, pb, rb, hlb, tb, &r);
    } else if (kb == 3) {
      hit = capsule_plane(pa, ra, hla, ta, lb, tb, &r);
    }
  } else if (ka == 2) {
    if (kb == 0) {
      hit = sphere_box(pb, rb, sza, ta, &r);
      if (hit) r = flip(r);
    } else if (kb == 2) {
      hit = box_box(pa, sza, ta, pb, szb, tb, &r);
    } else if (kb == 3) {
      hit = box_plane(sza, ta, lb, tb, &r);
    }
  } else if (ka == 3) {
    if (kb == 0) hit = sphere_plane(pb, rb, la, ra, ta, &r);
    else if (kb == 1) hit = capsule_plane(pb, rb, hlb, tb, la, ta, &r);
    else if (kb == 2) hit = box_plane(szb, tb, la, ta, &r);
    if (hit) r = flip(r);
  }
  if (!hit) return false;
  point[0] = r.point.x, point[1] = r.point.y, point[2] = r.point.z;
  normal[0] = r.normal.x, normal[1] = r.normal.y, normal[2] = r.normal.z;
  *pen = r.pen;
  return true;
}

// Corrected semantics: a geom's world frame, body pose (x) geom local pose: centre =
// transformPoint(local position), orientation = quatMultiply(body quat, geom quat), both
// in written order with plain IEEE operations.
void geom_world_pose(const GeomRec& g, const float* bp, const float* bq, float wp[3], float wq[4]) {
  const Xf t{p3(bp), Quat{bq[0], bq[1], bq[2], bq[3]}};
  const P3 c = t.point(p3(g.pos_size0));
  wp[0] = c.x, wp[1] = c.y, wp[2] = c.z;
  const float* b = g.quat;
  wq[0] = bq[3] * b[0] + bq[0] * b[3] + bq[1] * b[2] - bq[2] * b[1];
  wq[1] = bq[3] * b[1] - bq[0] * b[2] + bq[1] * b[3] + bq[2] * b[0];
  wq[2] = bq[3] * b[2] + bq[0] * b[1] - bq[1] * b[0] + bq[2] * b[3];
  wq[3] = bq[3] * b[3] - bq[0] * b[0] - bq[1] * b[1] - bq[2] * b[2];
}

// The type pairs whose routines return the normal from A to B (sphere-sphere,
// capsule-capsule, box-box; GJK's box-capsule).  The others, and all plane pairs, return
// it from B to A, the direction solve_contacts pushes body A along.
bool normal_a_to_b(uint32_t ta, uint32_t tb) {
  return (ta == tb && ta <= 2) || (ta == 1 && tb == 2) || (ta == 2 && tb == 1);
}

// gjk then epa on two free-standing shapes (types 0 sphere, 1 capsule, 2 box), for the
// reference's own GJK / EPA unit tests (gjk.zig:712-826).  Returns 0 when GJK finds no
// intersection, 1 when it does but EPA gives no result, 2 with out = EPA normal xyz,
// depth, witness point on A xyz, witness point on B xyz.
int gjk_epa_query(const GeomRec& ga, const float* bpa, const float* bqa, const GeomRec& gb, const float* bpb,
                  const float* bqb, float out[10]) {
  const Xf ta{p3(bpa), Quat{bqa[0], bqa[1], bqa[2], bqa[3]}};
  const Xf tb{p3(bpb), Quat{bqb[0], bqb[1], bqb[2], bqb[3]}};
  const Shape A{ga.type_body[0], p3(ga.pos_size0), P3{ga.pos_size0[3], ga.params[0], ga.params[1]}, ta};
  const Shape B{gb.type_body[0], p3(gb.pos_size0), P3{gb.pos_size0[3], gb.params[0], gb.params[1]}, tb};
  Simplex x{};
  if (!gjk(A, B, x)) return 0;
  P3 n, pa, pb;
  float depth;
  if (!epa(A, B, x, &n, &depth, &pa, &pb)) return 1;
  const float v[10] = {n.x, n.y, n.z, depth, pa.x, pa.y, pa.z, pb.x, pb.y, pb.z};
  for (int i = 0; i < 10; ++i) out[i] = v[i];
  return 2;
}

}  // namespace zo
