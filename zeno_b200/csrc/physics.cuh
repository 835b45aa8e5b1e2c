// Per-constraint and per-contact physics shared by both step kernels.
//
// The functions are templated on two small accessor types so that the same arithmetic
// runs on any layout:
//   S (body state):  float4& pos(b), quat(b), vel(b), ang(b)
//   M (model):       float4 imi(b) (1/m, 1/Ixx, 1/Iyy, 1/Izz), float4 com(b),
//                    ConstraintV constraint(k)
// Every expression keeps the canonical evaluation order of devmath.cuh, so the two
// kernels produce bit-identical results.
#pragma once
#include "devmath.cuh"

namespace zb {

struct ConstraintV {
  uint32_t a, b, type;
  float4 aa, ab, at, lim;  // anchor a, anchor b, axis / weld target, limits / slider target
};

// ------------------------------------------------------------------------------------
// XPBD joint constraints (solve_joints, all_shaders.metal:909-1399).  The multiplier is
// not tracked: with compliance 0, alpha~ = 0 and dlambda = -C / w exactly.
//
// cons_math<T> applies one constraint of type T to the poses of its two bodies held in
// registers (pa/pb keep their w component); solve_constraint loads them, dispatches on
// the type and stores them back.
// ------------------------------------------------------------------------------------
template <int T, class M>
__device__ __forceinline__ void cons_math(const M& m, const ConstraintV& c, float4 mia, float4 mib, float4& pa4,
                                          float4& qa, float4& pb4, float4& qb) {
  // Each correction is computed unconditionally and kept with a select when the
  // reference's guard holds; a discarded value is never stored, so the results equal the
  // branching form while the dependency chain stays free of branches.
  const V3 Ia{mia.y, mia.z, mia.w}, Ib{mib.y, mib.z, mib.w};
  const float ima = mia.x, imb = mib.x;
  const V3 pa = v3(pa4), pb = v3(pb4);
  const V3 aa = v3(c.aa), ab = v3(c.ab);
  if (T == 2) {  // positional
    const V3 ra = rotate(aa, qa), rb = rotate(ab, qb);
    const V3 diff = (pa + ra) - (pb + rb);
    float C;
    const V3 n = unit(diff, C);
    const V3 rna = cross(ra, n), rnb = cross(rb, n);
    const float wa = ima + dot(hadamard(rna, Ia), rna);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const float dl = div_(-C, wa + wb);
    const V3 imp = n * dl;
    const V3 rca = ra - rotate(v3(m.com(c.a)), qa), rcb = rb - rotate(v3(m.com(c.b)), qb);
    const bool ok = C > 1e-6f;
    const bool ua = ok && ima > 0.0f, ub = ok && imb > 0.0f;
    const float4 pa_n = with_w(madd(imp, ima, pa), pa4.w);
    const float4 qa_n = qnormalize(qmadd(qmul_v(hadamard(cross(rca, imp), Ia), qa), 0.5f, qa));
    const float4 pb_n = with_w(msub(imp, imb, pb), pb4.w);
    const float4 qb_n = qnormalize(qmsub(qmul_v(hadamard(cross(rcb, imp), Ib), qb), 0.5f, qb));
    pa4 = sel4(ua, pa_n, pa4);
    qa = sel4(ua, qa_n, qa);
    pb4 = sel4(ub, pb_n, pb4);
    qb = sel4(ub, qb_n, qb);
  } else if (T == 7) {  // weld: corrections on body b only
    const V3 ra = rotate(aa, qa), rb = rotate(ab, qb);
    const V3 diff = (pa + ra) - (pb + rb);
    float C;
    const V3 n = unit(diff, C);
    const V3 rnb = cross(rb, n);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const V3 imp = n * div_(-C, wb);
    const bool u1 = C > 1e-6f && wb > 1e-8f;
    pb4 = sel4(u1, with_w(msub(imp, imb, pb), pb4.w), pb4);
    qb = sel4(u1, qnormalize(qmsub(qmul_v(hadamard(cross(rb, imp), Ib), qb), 0.5f, qb)), qb);
    const float4 qau = qa, qbu = qb;
    float4 qerr = qmul(qmul(qconj(qau), qbu), qconj(c.at));
    qerr = sel4(qerr.w < 0.0f, qneg(qerr), qerr);
    const V3 ev = xyz(qerr);
    float sh;
    const V3 axr = unit(ev, sh);
    const float ang = 2.0f * atan2r(sh, qerr.w);
    const V3 aw = rotate(axr, qau);
    const float w2 = dot(hadamard(aw, Ib), aw);
    const V3 ai = aw * div_(ang, w2);
    const bool u2 = sh > 1e-6f && w2 > 1e-8f && imb > 0.0f;
    qb = sel4(u2, qnormalize(qmsub(qmul_v(hadamard(ai, Ib), qbu), 0.5f, qbu)), qb);
  } else if (T == 3) {  // angular: keep hinge axes parallel
    const V3 aaw = rotate(aa, qa), abw = rotate(ab, qb);
    const V3 cr = cross(aaw, abw);
    float sa;
    const V3 n = unit(cr, sa);
    const float angC = asinr(clampf(sa, -1.0f, 1.0f));
    const float w = dot(hadamard(n, Ia), n) + dot(hadamard(n, Ib), n);
    const float dl = div_(-angC, w);
    const bool ok = sa > 1e-6f && w > 1e-8f;
    const float4 qa_n = qnormalize(qmadd(qmul_v(hadamard(n * dl, Ia), qa), 0.5f, qa));
    const float4 qb_n = qnormalize(qmadd(qmul_v(hadamard(n * (-dl), Ib), qb), 0.5f, qb));
    qa = sel4(ok && ima > 0.0f, qa_n, qa);
    qb = sel4(ok && imb > 0.0f, qb_n, qb);
  } else if (T == 4) {  // angular limit
    const float lo = c.lim.x, hi = c.lim.y;
    const float4 qrel = qmul(qconj(qa), qb);
    const float angle = 2.0f * atan2r(dot(xyz(qrel), aa), qrel.w);
    float viol = 0.0f;
    if (angle < lo) viol = lo - angle;
    else if (angle > hi) viol = hi - angle;
    if (fabsf(viol) > 1e-6f) {  // rarely taken: keep the branch, skip the work
      const V3 aw = rotate(aa, qa);
      const float w = dot(hadamard(aw, Ia), aw) + dot(hadamard(aw, Ib), aw);
      const V3 ai = aw * div_(viol, w);
      const bool ok = w > 1e-8f;
      const float4 qa_n = qnormalize(qmadd(qmul_v(hadamard(ai, Ia), qa), 0.5f, qa));
      const float4 qb_n = qnormalize(qmsub(qmul_v(hadamard(ai, Ib), qb), 0.5f, qb));
      qa = sel4(ok && ima > 0.0f, qa_n, qa);
      qb = sel4(ok && imb > 0.0f, qb_n, qb);
    }
  } else if (T == 5) {  // linear limit
    const float lo = c.lim.x, hi = c.lim.y;
    const V3 ra = rotate(v3(0.0f, 0.0f, 0.0f), qa), rb = rotate(ab, qb);
    const V3 aw = rotate(aa, qa);
    const float dist = dot((pb + rb) - (pa + ra), aw);
    float viol = 0.0f;
    if (dist < lo) viol = lo - dist;
    else if (dist > hi) viol = hi - dist;
    if (fabsf(viol) > 1e-6f) {
      const V3 n = viol > 0.0f ? aw : -aw;
      const V3 rna = cross(ra, n), rnb = cross(rb, n);
      const float wa = ima + dot(hadamard(rna, Ia), rna);
      const float wb = imb + dot(hadamard(rnb, Ib), rnb);
      const float w = wa + wb;
      const V3 imp = n * div_(fabsf(viol), w);
      const bool ok = w > 1e-8f;
      pa4 = sel4(ok && ima > 0.0f, with_w(msub(imp, ima, pa), pa4.w), pa4);
      pb4 = sel4(ok && imb > 0.0f, with_w(madd(imp, imb, pb), pb4.w), pb4);
    }
  } else if (T == 10) {  // slider: perpendicular lock + relative-orientation weld
    const V3 ra = rotate(aa, qa), rb = rotate(ab, qb);
    const V3 diff = (pa + ra) - (pb + rb);
    const V3 aw = rotate(v3(c.at), qa);
    const V3 perp = msub(aw, dot(diff, aw), diff);
    float pl;
    const V3 n = unit(perp, pl);
    const V3 rna = cross(ra, n), rnb = cross(rb, n);
    const float wa = ima + dot(hadamard(rna, Ia), rna);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const V3 imp = n * div_(-pl, wa + wb);
    const bool ok = pl > 1e-6f;
    const float4 qa0 = qa, qb0 = qb;
    const bool ua = ok && ima > 0.0f, ub = ok && imb > 0.0f;
    pa4 = sel4(ua, with_w(madd(imp, ima, pa), pa4.w), pa4);
    qa = sel4(ua, qnormalize(qmadd(qmul_v(hadamard(cross(ra, imp), Ia), qa0), 0.5f, qa0)), qa);
    pb4 = sel4(ub, with_w(msub(imp, imb, pb), pb4.w), pb4);
    qb = sel4(ub, qnormalize(qmsub(qmul_v(hadamard(cross(rb, imp), Ib), qb0), 0.5f, qb0)), qb);
    const float4 qau = qa, qbu = qb;
    float4 qerr = qmul(qmul(qconj(qau), qbu), qconj(c.lim));
    qerr = sel4(qerr.w < 0.0f, qneg(qerr), qerr);
    const V3 ev = xyz(qerr);
    float sh;
    const V3 axe = unit(ev, sh);
    const float ae = 2.0f * atan2r(sh, qerr.w);
    const V3 aw2 = rotate(axe, qau);
    const float w = dot(hadamard(aw2, Ia), aw2) + dot(hadamard(aw2, Ib), aw2);
    const V3 ai = aw2 * div_(ae, w);
    const bool ok2 = sh > 1e-6f && w > 1e-8f;
    qa = sel4(ok2 && ima > 0.0f, qnormalize(qmadd(qmul_v(hadamard(ai, Ia), qau), 0.5f, qau)), qa);
    qb = sel4(ok2 && imb > 0.0f, qnormalize(qmsub(qmul_v(hadamard(ai, Ib), qbu), 0.5f, qbu)), qb);
  }
}

template <int T, class M, class S>
__device__ __forceinline__ void solve_typed(const M& m, const ConstraintV& c, S& s) {
  const float4 mia = m.imi(c.a), mib = m.imi(c.b);
  if (mia.x + mib.x < 1e-8f) return;
  float4 pa = s.pos(c.a), qa = s.quat(c.a), pb = s.pos(c.b), qb = s.quat(c.b);
  cons_math<T>(m, c, mia, mib, pa, qa, pb, qb);
  s.pos(c.a) = pa;
  s.quat(c.a) = qa;
  s.pos(c.b) = pb;
  s.quat(c.b) = qb;
}

// A hinge's constraints on one body pair -- point (c0), axis (c1) and, when `limit`, angle
// limit (c2) -- in that order, with the two poses kept in registers between them.
template <class M, class S>
__device__ __forceinline__ void solve_hinge(const M& m, const ConstraintV& c0, const ConstraintV& c1,
                                            const ConstraintV& c2, bool limit, S& s) {
  const float4 mia = m.imi(c0.a), mib = m.imi(c0.b);
  if (mia.x + mib.x < 1e-8f) return;
  float4 pa = s.pos(c0.a), qa = s.quat(c0.a), pb = s.pos(c0.b), qb = s.quat(c0.b);
  cons_math<2>(m, c0, mia, mib, pa, qa, pb, qb);
  cons_math<3>(m, c1, mia, mib, pa, qa, pb, qb);
  if (limit) cons_math<4>(m, c2, mia, mib, pa, qa, pb, qb);
  s.pos(c0.a) = pa;
  s.quat(c0.a) = qa;
  s.pos(c0.b) = pb;
  s.quat(c0.b) = qb;
}

// One constraint of any type, in place.
template <class M, class S>
__device__ __forceinline__ void solve_constraint(const M& m, const ConstraintV& c, S& s) {
  switch (c.type) {
    case 2: solve_typed<2>(m, c, s); break;
    case 3: solve_typed<3>(m, c, s); break;
    case 4: solve_typed<4>(m, c, s); break;
    case 5: solve_typed<5>(m, c, s); break;
    case 7: solve_typed<7>(m, c, s); break;
    case 10: solve_typed<10>(m, c, s); break;
    default: break;
  }
}

// ------------------------------------------------------------------------------------
// Contact solve for one slot (solve_contacts, all_shaders.metal:1644-1793).
// cpp = (point, penetration), cnf = (normal, friction); jx is the slot's accumulated
// normal impulse (impulses[0]), rest its restitution (impulses[3]).
// ------------------------------------------------------------------------------------
template <class M, class S>
__device__ __forceinline__ void solve_contact(const M& m, float4 cpp, float4 cnf, float& jx, float rest, uint32_t ia,
                                              uint32_t ib, S& s, float dt, float baumgarte, float slop) {
  const float4 mia = m.imi(ia);
  const float4 mib = m.imi(ib);
  const V3 Ia{mia.y, mia.z, mia.w}, Ib{mib.y, mib.z, mib.w};
  const float ima = mia.x, imb = mib.x;
  const float isum = ima + imb;
  if (isum < 1e-8f) return;
  const V3 n = xyz(cnf);
  const float pen = cpp.w, fr = cnf.w;
  const V3 cp = xyz(cpp);
  const V3 ra = cp - v3(s.pos(ia)), rb = cp - v3(s.pos(ib));
  const V3 va = v3(s.vel(ia)) + cross(v3(s.ang(ia)), ra);
  const V3 vb = v3(s.vel(ib)) + cross(v3(s.ang(ib)), rb);
  const V3 rv = va - vb;
  const float vn = dot(rv, n);
  const V3 vt = msub(n, vn, rv);
  float ts;
  const V3 t = unit(vt, ts);
  const V3 rna = cross(ra, n), rnb = cross(rb, n);
  const float wn = (ima + dot(hadamard(rna, Ia), rna)) + (imb + dot(hadamard(rnb, Ib), rnb));
  if (wn < 1e-8f) return;
  const float excess = fmaxf(pen - slop, 0.0f);
  const float bias = div_(baumgarte * excess, dt);
  const float vrest = vn < -0.5f ? rest * vn : 0.0f;
  const float jn = fmaxf(div_(-(vn + vrest) + bias, wn), 0.0f);
  const V3 in_ = n * jn;
  const float pcorr = baumgarte * excess;
  if (ima > 1e-8f) {
    s.vel(ia) = with_w(madd(in_, ima, v3(s.vel(ia))), s.vel(ia).w);
    s.ang(ia) = with_w(v3(s.ang(ia)) + hadamard(cross(ra, in_), Ia), s.ang(ia).w);
    s.pos(ia) = with_w(madd(n, pcorr * div_(ima, isum), v3(s.pos(ia))), s.pos(ia).w);
  }
  if (imb > 1e-8f) {
    s.vel(ib) = with_w(msub(in_, imb, v3(s.vel(ib))), s.vel(ib).w);
    s.ang(ib) = with_w(v3(s.ang(ib)) - hadamard(cross(rb, in_), Ib), s.ang(ib).w);
    s.pos(ib) = with_w(msub(n, pcorr * div_(imb, isum), v3(s.pos(ib))), s.pos(ib).w);
  }
  const float jacc = jx + jn;
  if (ts > 1e-6f && jacc > 1e-6f) {
    const V3 rta = cross(ra, t), rtb = cross(rb, t);
    const float wt = (ima + dot(hadamard(rta, Ia), rta)) + (imb + dot(hadamard(rtb, Ib), rtb));
    if (wt > 1e-8f) {
      const float jt = fminf(div_(ts, wt), fr * jacc);
      const V3 it = t * jt;
      if (ima > 1e-8f) {
        s.vel(ia) = with_w(msub(it, ima, v3(s.vel(ia))), s.vel(ia).w);
        s.ang(ia) = with_w(v3(s.ang(ia)) - hadamard(cross(ra, it), Ia), s.ang(ia).w);
      }
      if (imb > 1e-8f) {
        s.vel(ib) = with_w(madd(it, imb, v3(s.vel(ib))), s.vel(ib).w);
        s.ang(ib) = with_w(v3(s.ang(ib)) + hadamard(cross(rb, it), Ib), s.ang(ib).w);
      }
    }
  }
  jx = jn;
}

// ------------------------------------------------------------------------------------
// Narrow phase for one geom pair (narrow_phase, all_shaders.metal:751-894): sphere-
// sphere, sphere-plane and capsule-plane; every other type pair reports no contact.
// pa, pb: body position + unrotated geom offset; ra, rb: size[0]; hl, cq: half length
// and local quaternion of the capsule when one of the two geoms is a capsule.
// ------------------------------------------------------------------------------------
// Axis of a capsule geom: +z rotated by the geom's local quaternion (all_shaders.metal:
// 858-860 uses the geom quaternion, not the body's).
__device__ __forceinline__ V3 capsule_axis(float4 cq) { return rotate(v3(0.0f, 0.0f, 1.0f), cq); }

// Capsule-plane contact (the capsule's geom-frame axis, see capsule_axis): the deeper of
// the two segment ends below the plane z = 0 (the plane position is not used).
// capsule_a: the capsule is geom A (normal +z), else geom B (normal -z).
__device__ __forceinline__ bool capsule_plane(V3 cpos, float cr, float hl, V3 axis, bool capsule_a, V3& point,
                                              V3& normal, float& pen) {
  const V3 p1 = msub(axis, hl, cpos), p2 = madd(axis, hl, cpos);
  const float d1 = p1.z - cr, d2 = p2.z - cr;
  point = d1 < d2 ? p1 : p2;
  point.z = 0.0f;
  pen = -fminf(d1, d2);
  normal = capsule_a ? v3(0.0f, 0.0f, 1.0f) : v3(0.0f, 0.0f, -1.0f);
  return d1 < 0.0f || d2 < 0.0f;
}

__device__ __forceinline__ bool narrow_core(uint32_t ta, uint32_t tb, V3 pa, V3 pb, float ra, float rb, float hl,
                                            V3 caxis, V3& point, V3& normal, float& pen) {
  if (ta == 0 && tb == 0) {
    const V3 d = pb - pa;
    float dist;
    const V3 nd = unit(d, dist);
    const float md = ra + rb;
    if (dist < md && dist > 1e-6f) {
      normal = nd;
      pen = md - dist;
      point = madd(normal, ra - pen * 0.5f, pa);
      return true;
    }
  } else if ((ta == 0 && tb == 3) || (ta == 3 && tb == 0)) {
    const V3 sp = ta == 0 ? pa : pb, pp = ta == 0 ? pb : pa;
    const float sr = ta == 0 ? ra : rb;
    const V3 pn{0.0f, 0.0f, 1.0f};
    const float sd = dot(sp - pp, pn);
    if (sd < sr) {
      normal = ta == 3 ? -pn : pn;
      pen = sr - sd;
      point = msub(pn, sd + pen * 0.5f, sp);
      return true;
    }
  } else if ((ta == 1 && tb == 3) || (ta == 3 && tb == 1)) {
    return capsule_plane(ta == 1 ? pa : pb, ta == 1 ? ra : rb, hl, caxis, ta == 1, point, normal, pen);
  }
  return false;
}

// True for the type pairs narrow_core can report a contact for.
__host__ __device__ inline bool narrow_supported(uint32_t ta, uint32_t tb) {
  return (ta == 0 && tb == 0) || (ta == 0 && tb == 3) || (ta == 3 && tb == 0) || (ta == 1 && tb == 3) ||
         (ta == 3 && tb == 1);
}

// ------------------------------------------------------------------------------------
// Extended narrow phase: the reference's CPU collision routines (src/collision/
// narrow_phase.zig, detectCollision and the primitive pairs it dispatches to), selected
// per world with zeno_world_set_narrow_phase(1).  Geoms are placed by their body's pose
// (centre = R(q_body) local_pos + body_pos); capsule/box axes and plane normals come from
// the body quaternion.  Box-capsule, plane-plane and cylinder/mesh/heightfield pairs report
// no contact.  The arithmetic is the Zig source's: plain single-precision +, -, *, /,
// sqrt, left to right as written, no fused multiply-adds (the file is compiled with
// -fmad=false).
// ------------------------------------------------------------------------------------
namespace cpu_narrow {

constexpr float kEps = 1e-6f;  // constants.EPSILON

struct P3 {
  float x, y, z;
};
__device__ __forceinline__ P3 add(P3 a, P3 b) { return P3{a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ P3 sub(P3 a, P3 b) { return P3{a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ P3 scl(P3 v, float s) { return P3{v.x * s, v.y * s, v.z * s}; }
__device__ __forceinline__ float dot(P3 a, P3 b) { return __fadd_rn(__fadd_rn(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)), __fmul_rn(a.z, b.z)); }
__device__ __forceinline__ P3 cross(P3 a, P3 b) {
  return P3{__fsub_rn(__fmul_rn(a.y, b.z), __fmul_rn(a.z, b.y)), __fsub_rn(__fmul_rn(a.z, b.x), __fmul_rn(a.x, b.z)),
            __fsub_rn(__fmul_rn(a.x, b.y), __fmul_rn(a.y, b.x))};
}
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fmaxf(lo, fminf(v, hi)); }
// rotateByQuat (src/physics/body.zig:254-264)
__device__ __forceinline__ P3 rot(P3 v, float4 q) {
  const P3 qv{q.x, q.y, q.z};
  const P3 uv = cross(qv, v);
  const P3 uuv = cross(qv, uv);
  return P3{__fadd_rn(v.x, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(q.w, uv.x), uuv.x))),
            __fadd_rn(v.y, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(q.w, uv.y), uuv.y))),
            __fadd_rn(v.z, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(q.w, uv.z), uuv.z)))};
}
struct Xf {  // body.Transform
  P3 p;
  float4 q;
  __device__ __forceinline__ P3 point(P3 v) const { return add(rot(v, q), p); }
  __device__ __forceinline__ P3 vec(P3 v) const { return rot(v, q); }
  __device__ __forceinline__ Xf inverse() const {
    const float4 iq = make_float4(-q.x, -q.y, -q.z, q.w);
    return Xf{rot(P3{-p.x, -p.y, -p.z}, iq), iq};
  }
};
struct Res {
  P3 point, normal;
  float pen;
};

__device__ __forceinline__ P3 closest_on_segment(P3 point, P3 s, P3 e) {
  const P3 seg = sub(e, s);
  const float len_sq = dot(seg, seg);
  if (len_sq < kEps) return s;
  const float t = clampf(__fdiv_rn(dot(sub(point, s), seg), len_sq), 0.0f, 1.0f);
  return add(s, scl(seg, t));
}

__device__ __forceinline__ void closest_between_segments(P3 a1, P3 a2, P3 b1, P3 b2, P3& pa, P3& pb) {
  const P3 d1 = sub(a2, a1), d2 = sub(b2, b1), r = sub(a1, b1);
  const float a = dot(d1, d1), e = dot(d2, d2), f = dot(d2, r);
  float s = 0.0f, t = 0.0f;
  if (a < kEps && e < kEps) {
    pa = a1, pb = b1;
    return;
  }
  if (a < kEps) {
    t = clampf(__fdiv_rn(f, e), 0.0f, 1.0f);
  } else {
    const float c = dot(d1, r);
    if (e < kEps) {
      s = clampf(__fdiv_rn(-c, a), 0.0f, 1.0f);
    } else {
      const float b = dot(d1, d2);
      const float denom = __fsub_rn(__fmul_rn(a, e), __fmul_rn(b, b));
      if (denom != 0.0f) s = clampf(__fdiv_rn(__fsub_rn(__fmul_rn(b, f), __fmul_rn(c, e)), denom), 0.0f, 1.0f);
      t = __fdiv_rn(__fadd_rn(__fmul_rn(b, s), f), e);
      if (t < 0.0f) {
        t = 0.0f;
        s = clampf(__fdiv_rn(-c, a), 0.0f, 1.0f);
      } else if (t > 1.0f) {
        t = 1.0f;
        s = clampf(__fdiv_rn(__fsub_rn(b, c), a), 0.0f, 1.0f);
      }
    }
  }
  pa = add(a1, scl(d1, s));
  pb = add(b1, scl(d2, t));
}

__device__ __forceinline__ P3 box_face_normal(P3 p, P3 h) {  // the face with the largest distance, as written
  const float pc[3] = {p.x, p.y, p.z}, hc[3] = {h.x, h.y, h.z};
  float max_dist = -__int_as_float(0x7f800000);
  float n[3] = {0.0f, 0.0f, 1.0f};
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float d_pos = __fsub_rn(hc[i], pc[i]), d_neg = __fadd_rn(hc[i], pc[i]);
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

__device__ __forceinline__ bool test_axis(P3 axis, P3 d, const P3* axa, P3 ha, const P3* axb, P3 hb, float& overlap) {
  const float proj_a = __fadd_rn(__fadd_rn(__fmul_rn(ha.x, fabsf(dot(axis, axa[0]))), __fmul_rn(ha.y, fabsf(dot(axis, axa[1])))),
                                 __fmul_rn(ha.z, fabsf(dot(axis, axa[2]))));
  const float proj_b = __fadd_rn(__fadd_rn(__fmul_rn(hb.x, fabsf(dot(axis, axb[0]))), __fmul_rn(hb.y, fabsf(dot(axis, axb[1])))),
                                 __fmul_rn(hb.z, fabsf(dot(axis, axb[2]))));
  const float dist = fabsf(dot(d, axis));
  const float sum = __fadd_rn(proj_a, proj_b);
  if (dist > sum) return false;
  overlap = __fsub_rn(sum, dist);
  return true;
}

__device__ __forceinline__ bool sphere_sphere(P3 pa, float ra, P3 pb, float rb, Res& o) {
  const P3 diff = sub(pb, pa);
  const float dist_sq = dot(diff, diff), min_dist = __fadd_rn(ra, rb);
  if (dist_sq >= __fmul_rn(min_dist, min_dist)) return false;
  const float dist = __fsqrt_rn(dist_sq);
  const P3 n = dist > kEps ? scl(diff, __fdiv_rn(1.0f, dist)) : P3{0.0f, 0.0f, 1.0f};
  const float pen = __fsub_rn(min_dist, dist);
  o = Res{add(pa, scl(n, __fsub_rn(ra, __fmul_rn(pen, 0.5f)))), n, pen};
  return true;
}

__device__ __forceinline__ bool sphere_capsule(P3 sp, float sr, P3 cp, float cr, float hl, const Xf& ct, Res& o) {
  const P3 axis = ct.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 p1 = sub(cp, scl(axis, hl)), p2 = add(cp, scl(axis, hl));
  const P3 closest = closest_on_segment(sp, p1, p2);
  const P3 diff = sub(sp, closest);
  const float dist_sq = dot(diff, diff), min_dist = __fadd_rn(sr, cr);
  if (dist_sq >= __fmul_rn(min_dist, min_dist)) return false;
  const float dist = __fsqrt_rn(dist_sq);
  const P3 n = dist > kEps ? scl(diff, __fdiv_rn(1.0f, dist)) : P3{0.0f, 0.0f, 1.0f};
  const float pen = __fsub_rn(min_dist, dist);
  o = Res{add(closest, scl(n, __fsub_rn(cr, __fmul_rn(pen, 0.5f)))), n, pen};
  return true;
}

__device__ __forceinline__ bool sphere_plane(P3 sp, float sr, P3 plane_local, float plane_off, const Xf& pt, Res& o) {
  const P3 n = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 plane_point = pt.point(plane_local);
  const float sd = __fsub_rn(dot(sub(sp, plane_point), n), plane_off);
  if (sd >= sr) return false;
  const float pen = __fsub_rn(sr, sd);
  o = Res{sub(sp, scl(n, __fadd_rn(sd, __fmul_rn(pen, 0.5f)))), n, pen};
  return true;
}

__device__ __forceinline__ bool sphere_box(P3 sp, float sr, P3 half, const Xf& bt, Res& o) {
  const Xf inv = bt.inverse();
  const P3 ls = inv.point(sp);
  const P3 cl{clampf(ls.x, -half.x, half.x), clampf(ls.y, -half.y, half.y), clampf(ls.z, -half.z, half.z)};
  const P3 diff = sub(ls, cl);
  const float dist_sq = dot(diff, diff);
  if (dist_sq >= __fmul_rn(sr, sr)) return false;
  const float dist = __fsqrt_rn(dist_sq);
  const P3 ln = dist > kEps ? scl(diff, __fdiv_rn(1.0f, dist)) : box_face_normal(ls, half);
  const P3 wc = bt.point(cl);
  const P3 n = bt.vec(ln);
  const float pen = __fsub_rn(sr, dist);
  o = Res{add(wc, scl(n, __fmul_rn(pen, 0.5f))), n, pen};
  return true;
}

__device__ __forceinline__ bool capsule_capsule(P3 pa, float ra, float hla, const Xf& ta, P3 pb, float rb, float hlb,
                                                const Xf& tb, Res& o) {
  const P3 axa = ta.vec(P3{0.0f, 0.0f, 1.0f}), axb = tb.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 a1 = sub(pa, scl(axa, hla)), a2 = add(pa, scl(axa, hla));
  const P3 b1 = sub(pb, scl(axb, hlb)), b2 = add(pb, scl(axb, hlb));
  P3 ca, cb;
  closest_between_segments(a1, a2, b1, b2, ca, cb);
  const P3 diff = sub(cb, ca);
  const float dist_sq = dot(diff, diff), min_dist = __fadd_rn(ra, rb);
  if (dist_sq >= __fmul_rn(min_dist, min_dist)) return false;
  const float dist = __fsqrt_rn(dist_sq);
  const P3 n = dist > kEps ? scl(diff, __fdiv_rn(1.0f, dist)) : P3{0.0f, 0.0f, 1.0f};
  const float pen = __fsub_rn(min_dist, dist);
  const P3 paw = add(ca, scl(n, ra)), pbw = sub(cb, scl(n, rb));
  o = Res{scl(add(paw, pbw), 0.5f), n, pen};
  return true;
}

__device__ __forceinline__ bool capsule_plane(P3 cp, float r, float hl, const Xf& ct, P3 plane_local, const Xf& pt,
                                              Res& o) {
  const P3 axis = ct.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pn = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pp = pt.point(plane_local);
  const P3 p1 = sub(cp, scl(axis, hl)), p2 = add(cp, scl(axis, hl));
  const float d1 = __fsub_rn(dot(sub(p1, pp), pn), r), d2 = __fsub_rn(dot(sub(p2, pp), pn), r);
  if (d1 >= 0.0f && d2 >= 0.0f) return false;
  const P3 deepest = d1 < d2 ? p1 : p2;
  const float dist = fminf(d1, d2);
  o = Res{sub(deepest, scl(pn, __fadd_rn(__fmul_rn(dist, 0.5f), r))), pn, -dist};
  return true;
}

__device__ __forceinline__ bool box_plane(P3 half, const Xf& bt, P3 plane_local, const Xf& pt, Res& o) {
  const P3 pn = pt.vec(P3{0.0f, 0.0f, 1.0f});
  const P3 pp = pt.point(plane_local);
  float min_dist = __int_as_float(0x7f800000);
  P3 deepest{0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // corner order of boxPlane: x fastest, then y, then z
    const P3 corner{(c & 1) ? half.x : -half.x, (c & 2) ? half.y : -half.y, (c & 4) ? half.z : -half.z};
    const P3 wc = bt.point(corner);
    const float dist = dot(sub(wc, pp), pn);
    if (dist < min_dist) {
      min_dist = dist;
      deepest = wc;
    }
  }
  if (min_dist >= 0.0f) return false;
  o = Res{deepest, pn, -min_dist};
  return true;
}

__device__ __forceinline__ bool box_box(P3 pa, P3 ha, const Xf& ta, P3 pb, P3 hb, const Xf& tb, Res& o) {
  const P3 axa[3] = {ta.vec(P3{1.0f, 0.0f, 0.0f}), ta.vec(P3{0.0f, 1.0f, 0.0f}), ta.vec(P3{0.0f, 0.0f, 1.0f})};
  const P3 axb[3] = {tb.vec(P3{1.0f, 0.0f, 0.0f}), tb.vec(P3{0.0f, 1.0f, 0.0f}), tb.vec(P3{0.0f, 0.0f, 1.0f})};
  const P3 d = sub(pb, pa);
  float min_overlap = __int_as_float(0x7f800000), ov = 0.0f;
  P3 best{0.0f, 0.0f, 1.0f};
  for (int i = 0; i < 3; ++i) {
    if (!test_axis(axa[i], d, axa, ha, axb, hb, ov)) return false;
    if (ov < min_overlap) min_overlap = ov, best = axa[i];
  }
  for (int i = 0; i < 3; ++i) {
    if (!test_axis(axb[i], d, axa, ha, axb, hb, ov)) return false;
    if (ov < min_overlap) min_overlap = ov, best = axb[i];
  }
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      const P3 ea = cross(axa[i], axb[j]);
      const float len = __fsqrt_rn(dot(ea, ea));
      if (len < kEps) continue;
      const P3 nrm = scl(ea, __fdiv_rn(1.0f, len));
      if (!test_axis(nrm, d, axa, ha, axb, hb, ov)) return false;
      if (ov < min_overlap) min_overlap = ov, best = nrm;
    }
  if (dot(best, d) < 0.0f) best = scl(best, -1.0f);
  o = Res{add(pa, scl(d, 0.5f)), best, min_overlap};
  return true;
}

// ---- GJK + EPA (src/collision/gjk.zig) on the sphere, capsule and box support maps ----
// Used by narrow-phase mode 2 for box-capsule pairs; the reference runs this code only for
// meshes.  Arithmetic as in the rest of this namespace: IEEE operations in written order.
constexpr float kGjkTol = 1e-6f;  // GJK_TOLERANCE
constexpr float kEpaTol = 1e-4f;  // EPA_TOLERANCE
constexpr int kGjkIters = 64, kEpaIters = 64, kEpaFaces = 128, kEpaEdges = 256;
constexpr int kEpaVerts = 4 + kEpaIters;  // 4 start vertices + at most one per iteration

struct Shape {  // ConvexShape: type 0 sphere, 1 capsule, 2 box; body transform
  uint32_t type;
  P3 local, size;
  Xf xf;
};
__device__ __forceinline__ P3 neg(P3 v) { return P3{-v.x, -v.y, -v.z}; }
__device__ __forceinline__ P3 safe_normalize(P3 v) {  // safeNormalize
  const float len = __fsqrt_rn(dot(v, v));
  if (len < kGjkTol) return P3{0.0f, 0.0f, 1.0f};
  return scl(v, __fdiv_rn(1.0f, len));
}
__device__ __forceinline__ P3 triple(P3 a, P3 b, P3 c) { return cross(cross(a, b), c); }
__device__ __forceinline__ P3 perpendicular(P3 v) {
  if (fabsf(v.x) < fabsf(v.y)) return safe_normalize(cross(v, P3{1.0f, 0.0f, 0.0f}));
  return safe_normalize(cross(v, P3{0.0f, 1.0f, 0.0f}));
}
// sphereSupport / capsuleSupport / boxSupport (box corner about the body origin, as written)
__device__ __forceinline__ P3 support(const Shape& s, P3 dir) {
  if (s.type == 0) return add(s.xf.point(s.local), scl(safe_normalize(dir), s.size.x));
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
__device__ __forceinline__ MinkPoint mink(const Shape& A, const Shape& B, P3 dir) {
  const P3 sa = support(A, dir), sb = support(B, neg(dir));
  return MinkPoint{sub(sa, sb), sa, sb};
}
struct Simplex {
  P3 s[4], sa[4], sb[4];
  uint32_t n;
};
// doSimplex2: support points left as they are, as written
__device__ __forceinline__ void simplex2(Simplex& x, P3& dir) {
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
__device__ __forceinline__ void simplex3(Simplex& x, P3& dir) {
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
    P3 t = x.s[0];
    x.s[0] = x.s[1], x.s[1] = t;
    t = x.sa[0], x.sa[0] = x.sa[1], x.sa[1] = t;
    t = x.sb[0], x.sb[0] = x.sb[1], x.sb[1] = t;
    dir = neg(abc);
  }
}
// doSimplex4: support copies in the written order (the ADB case copies slot 0 after it was
// overwritten, as in the reference)
__device__ __forceinline__ bool simplex4(Simplex& x, P3& dir) {
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
__device__ __forceinline__ bool gjk(const Shape& A, const Shape& B, Simplex& x) {
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
// Two 16-byte words, so that the removal pass reads a face with two vector loads: the
// outward normal and distance, then the face's first vertex (a copy of v[i0], which the
// visibility test reads) and the vertex indices.
struct alignas(16) Face {
  P3 n;
  float d;
  P3 v0;
  uint32_t idx;  // vertex indices i0 | i1 << 8 | i2 << 16
};
__device__ __forceinline__ uint32_t fidx(uint32_t i0, uint32_t i1, uint32_t i2) { return i0 | (i1 << 8) | (i2 << 16); }
__device__ __forceinline__ P3 face_normal(P3 a, P3 b, P3 c) { return safe_normalize(cross(sub(b, a), sub(c, a))); }
__device__ __forceinline__ void barycentric(P3 a, P3 b, P3 c, float& w0, float& w1, float& w2) {
  const float third = 1.0f / 3.0f;
  const P3 ab = sub(b, a), ac = sub(c, a), ao = neg(a);
  const float d00 = dot(ab, ab), d01 = dot(ab, ac), d11 = dot(ac, ac), d20 = dot(ao, ab), d21 = dot(ao, ac);
  const float denom = __fsub_rn(__fmul_rn(d00, d11), __fmul_rn(d01, d01));
  if (fabsf(denom) < kGjkTol) {
    w0 = w1 = w2 = third;
    return;
  }
  const float v = __fdiv_rn(__fsub_rn(__fmul_rn(d11, d20), __fmul_rn(d01, d21)), denom);
  const float w = __fdiv_rn(__fsub_rn(__fmul_rn(d00, d21), __fmul_rn(d01, d20)), denom);
  const float u = __fsub_rn(__fsub_rn(1.0f, v), w);
  const float cu = clampf(u, 0.0f, 1.0f), cv = clampf(v, 0.0f, 1.0f), cw = clampf(w, 0.0f, 1.0f);
  const float total = __fadd_rn(__fadd_rn(cu, cv), cw);
  if (total < kGjkTol) {
    w0 = w1 = w2 = third;
    return;
  }
  w0 = __fdiv_rn(cu, total), w1 = __fdiv_rn(cv, total), w2 = __fdiv_rn(cw, total);
}
// addEdge: a reversed duplicate cancels, else append while room remains (edge = a | b << 8)
__device__ __forceinline__ void add_edge(uint16_t* edges, uint32_t& ne, uint32_t a, uint32_t b) {
  const uint16_t rev = uint16_t(b | (a << 8));
  for (uint32_t i = 0; i < ne; ++i)
    if (edges[i] == rev) {
      edges[i] = edges[ne - 1];
      ne -= 1;
      return;
    }
  if (ne < uint32_t(kEpaEdges)) edges[ne++] = uint16_t(a | (b << 8));
}
// gjk, then epa, then the contact as meshPrimitiveCollision builds it (narrow_phase.zig:
// 693-747): midpoint of the witness points, EPA normal (A to B), EPA depth.
static __device__ __noinline__ bool gjk_contact(const Shape& A, const Shape& B, Res& o) {
  Simplex x;
  if (!gjk(A, B, x)) return false;
  if (x.n < 4) return false;
  P3 v[kEpaVerts], va[kEpaVerts], vb[kEpaVerts];
  Face f[kEpaFaces];
  uint16_t edges[kEpaEdges];
  uint32_t nv = 4, nf = 0;
  for (int i = 0; i < 4; ++i) v[i] = x.s[i], va[i] = x.sa[i], vb[i] = x.sb[i];
  // The closest face (the first position holding the smallest distance) is tracked as
  // the polytope changes rather than searched for at the top of each iteration: a face
  // the removal pass keeps stays at the position where the pass tested it, and positions
  // are settled in increasing order (kept faces, then appended ones), so a strict-less
  // scan in settling order picks the same face as a scan of the array.
  uint32_t k = 0;
  float cd = __int_as_float(0x7f800000);
  const uint8_t tf[4][3] = {{0, 1, 2}, {0, 3, 1}, {0, 2, 3}, {1, 3, 2}};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t i0 = tf[t][0], i1 = tf[t][1], i2 = tf[t][2];
    const P3 n = face_normal(v[i0], v[i1], v[i2]);
    const float d = dot(n, v[i0]);
    if (d < 0.0f) f[nf] = Face{neg(n), -d, v[i0], fidx(i0, i2, i1)};
    else f[nf] = Face{n, d, v[i0], fidx(i0, i1, i2)};
    if (f[nf].d < cd) cd = f[nf].d, k = nf;
    nf += 1;
  }
  bool done = false;
  for (int it = 0; it < kEpaIters; ++it) {
    const P3 dir = f[k].n;
    const MinkPoint m = mink(A, B, dir);
    if (__fsub_rn(dot(m.p, dir), cd) < kEpaTol) {
      done = true;
      break;
    }
    const uint32_t ni = nv;
    v[nv] = m.p, va[nv] = m.sa, vb[nv] = m.sb;
    nv += 1;
    uint32_t ne = 0;
    k = 0;
    cd = __int_as_float(0x7f800000);
    for (uint32_t i = 0; i < nf;) {
      const Face fc = f[i];
      const uint32_t fi = fc.idx;
      if (dot(fc.n, sub(m.p, fc.v0)) > 0.0f) {
        add_edge(edges, ne, fi & 0xFFu, (fi >> 8) & 0xFFu);
        add_edge(edges, ne, (fi >> 8) & 0xFFu, fi >> 16);
        add_edge(edges, ne, fi >> 16, fi & 0xFFu);
        f[i] = f[nf - 1];
        nf -= 1;
      } else {
        if (fc.d < cd) cd = fc.d, k = i;  // kept: position i is final
        i += 1;
      }
    }
    for (uint32_t e = 0; e < ne; ++e) {
      if (nf >= uint32_t(kEpaFaces)) break;
      const uint32_t e0 = edges[e] & 0xFFu, e1 = edges[e] >> 8;
      const P3 n = face_normal(v[e0], v[e1], v[ni]);
      const float d = dot(n, v[e0]);
      if (d < 0.0f) f[nf] = Face{neg(n), -d, v[e1], fidx(e1, e0, ni)};
      else f[nf] = Face{n, d, v[e0], fidx(e0, e1, ni)};
      if (f[nf].d < cd) cd = f[nf].d, k = nf;
      nf += 1;
    }
    if (nf == 0) break;
  }
  // not converged: the closest face of the current polytope, as tracked
  if (!done && nf == 0) return false;
  const uint32_t fi = f[k].idx, i0 = fi & 0xFFu, i1 = (fi >> 8) & 0xFFu, i2 = fi >> 16;
  float w0, w1, w2;
  barycentric(v[i0], v[i1], v[i2], w0, w1, w2);
  const P3 pa = add(add(scl(va[i0], w0), scl(va[i1], w1)), scl(va[i2], w2));
  const P3 pb = add(add(scl(vb[i0], w0), scl(vb[i1], w1)), scl(vb[i2], w2));
  o = Res{scl(add(pa, pb), 0.5f), f[k].n, cd};
  return true;
}

}  // namespace cpu_narrow

// ---- corrected semantics ----
// quatMultiply (src/physics/body.zig:238-245) in written order, plain IEEE operations.
__device__ __forceinline__ float4 qmul_ref(float4 a, float4 b) {
  return make_float4(a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y, a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
                     a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w, a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z);
}
// World centre of a geom (transformPoint of its local position by the body pose).
__device__ __forceinline__ V3 geom_centre(float4 bp, float4 bq, float4 local) {
  using namespace cpu_narrow;
  const P3 c = Xf{P3{bp.x, bp.y, bp.z}, bq}.point(P3{local.x, local.y, local.z});
  return V3{c.x, c.y, c.z};
}
// The routines that return normals from A to B (sphere-sphere, capsule-capsule, box-box,
// and GJK's box-capsule; the others and every plane pair point from B to A).  Corrected
// semantics negate these, so that every normal points from B to A, the direction
// solve_contacts (all_shaders.metal:1731-1745) pushes A along.
__host__ __device__ inline bool normal_a_to_b(uint32_t ta, uint32_t tb) {
  return (ta == tb && ta <= 2u) || (ta == 1u && tb == 2u) || (ta == 2u && tb == 1u);
}

// True for the type pairs narrow_cpu can report a contact for (types 0 sphere, 1 capsule,
// 2 box, 3 plane; no plane-plane; box-capsule only with GJK + EPA, mode 2).
__host__ __device__ inline bool narrow_cpu_supported(uint32_t ta, uint32_t tb, bool gjk_pairs = false) {
  if (ta > 3 || tb > 3) return false;
  if ((ta == 1 && tb == 2) || (ta == 2 && tb == 1)) return gjk_pairs;
  return !(ta == 3 && tb == 3);
}

// detectCollision (narrow_phase.zig:28-136).  la/lb: geom local position, size[0]; sa/sb:
// size[1], size[2]; bpa/bpb, bqa/bqb: body position and quaternion.
__device__ __forceinline__ bool narrow_cpu(uint32_t ka, uint32_t kb, float4 la, float2 sa, float4 lb, float2 sb,
                                           float4 bpa, float4 bqa, float4 bpb, float4 bqb, V3& point, V3& normal,
                                           float& pen, bool gjk_pairs = false) {
  using namespace cpu_narrow;
  const Xf ta{P3{bpa.x, bpa.y, bpa.z}, bqa}, tb{P3{bpb.x, bpb.y, bpb.z}, bqb};
  const P3 lpa{la.x, la.y, la.z}, lpb{lb.x, lb.y, lb.z};
  const P3 pa = ta.point(lpa), pb = tb.point(lpb);
  const float ra = la.w, rb = lb.w;
  const P3 sza{la.w, sa.x, sa.y}, szb{lb.w, sb.x, sb.y};
  Res r{};
  bool hit = false, flip = false;
  if (gjk_pairs && ((ka == 1 && kb == 2) || (ka == 2 && kb == 1))) {
    hit = gjk_contact(Shape{ka, lpa, sza, ta}, Shape{kb, lpb, szb, tb}, r);
  } else if (ka == 0) {
    if (kb == 0) hit = sphere_sphere(pa, ra, pb, rb, r);
    else if (kb == 1) hit = sphere_capsule(pa, ra, pb, rb, sb.x, tb, r);
    else if (kb == 2) hit = sphere_box(pa, ra, szb, tb, r);
    else if (kb == 3) hit = sphere_plane(pa, ra, lpb, rb, tb, r);
  } else if (ka == 1) {
    if (kb == 0) hit = sphere_capsule(pb, rb, pa, ra, sa.x, ta, r), flip = true;
    else if (kb == 1) hit = capsule_capsule(pa, ra, sa.x, ta, pb, rb, sb.x, tb, r);
    else if (kb == 3) hit = capsule_plane(pa, ra, sa.x, ta, lpb, tb, r);
  } else if (ka == 2) {
    if (kb == 0) hit = sphere_box(pb, rb, sza, ta, r), flip = true;
    else if (kb == 2) hit = box_box(pa, sza, ta, pb, szb, tb, r);
    else if (kb == 3) hit = box_plane(sza, ta, lpb, tb, r);
  } else if (ka == 3) {
    flip = true;
    if (kb == 0) hit = sphere_plane(pb, rb, lpa, ra, ta, r);
    else if (kb == 1) hit = capsule_plane(pb, rb, sb.x, tb, lpa, ta, r);
    else if (kb == 2) hit = box_plane(szb, tb, lpa, ta, r);
  }
  if (!hit) return false;
  if (flip) r.normal = scl(r.normal, -1.0f);
  point = V3{r.point.x, r.point.y, r.point.z};
  normal = V3{r.normal.x, r.normal.y, r.normal.z};
  pen = r.pen;
  return true;
}

}  // namespace zb
