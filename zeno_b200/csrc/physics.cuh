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
    const float C = len(diff);
    const V3 n = diff * rcp_(C);
    const V3 rna = cross(ra, n), rnb = cross(rb, n);
    const float wa = ima + dot(hadamard(rna, Ia), rna);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const float dl = __fdiv_rn(-C, wa + wb);
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
    const float C = len(diff);
    const V3 n = diff * rcp_(C);
    const V3 rnb = cross(rb, n);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const V3 imp = n * __fdiv_rn(-C, wb);
    const bool u1 = C > 1e-6f && wb > 1e-8f;
    pb4 = sel4(u1, with_w(msub(imp, imb, pb), pb4.w), pb4);
    qb = sel4(u1, qnormalize(qmsub(qmul_v(hadamard(cross(rb, imp), Ib), qb), 0.5f, qb)), qb);
    const float4 qau = qa, qbu = qb;
    float4 qerr = qmul(qmul(qconj(qau), qbu), qconj(c.at));
    qerr = sel4(qerr.w < 0.0f, qneg(qerr), qerr);
    const V3 ev = xyz(qerr);
    const float sh = len(ev);
    const V3 axr = ev * rcp_(sh);
    const float ang = 2.0f * atan2r(sh, qerr.w);
    const V3 aw = rotate(axr, qau);
    const float w2 = dot(hadamard(aw, Ib), aw);
    const V3 ai = aw * __fdiv_rn(ang, w2);
    const bool u2 = sh > 1e-6f && w2 > 1e-8f && imb > 0.0f;
    qb = sel4(u2, qnormalize(qmsub(qmul_v(hadamard(ai, Ib), qbu), 0.5f, qbu)), qb);
  } else if (T == 3) {  // angular: keep hinge axes parallel
    const V3 aaw = rotate(aa, qa), abw = rotate(ab, qb);
    const V3 cr = cross(aaw, abw);
    const float sa = len(cr);
    const V3 n = cr * rcp_(sa);
    const float angC = asinr(clampf(sa, -1.0f, 1.0f));
    const float w = dot(hadamard(n, Ia), n) + dot(hadamard(n, Ib), n);
    const float dl = __fdiv_rn(-angC, w);
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
      const V3 ai = aw * __fdiv_rn(viol, w);
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
      const V3 imp = n * __fdiv_rn(fabsf(viol), w);
      const bool ok = w > 1e-8f;
      pa4 = sel4(ok && ima > 0.0f, with_w(msub(imp, ima, pa), pa4.w), pa4);
      pb4 = sel4(ok && imb > 0.0f, with_w(madd(imp, imb, pb), pb4.w), pb4);
    }
  } else if (T == 10) {  // slider: perpendicular lock + relative-orientation weld
    const V3 ra = rotate(aa, qa), rb = rotate(ab, qb);
    const V3 diff = (pa + ra) - (pb + rb);
    const V3 aw = rotate(v3(c.at), qa);
    const V3 perp = msub(aw, dot(diff, aw), diff);
    const float pl = len(perp);
    const V3 n = perp * rcp_(pl);
    const V3 rna = cross(ra, n), rnb = cross(rb, n);
    const float wa = ima + dot(hadamard(rna, Ia), rna);
    const float wb = imb + dot(hadamard(rnb, Ib), rnb);
    const V3 imp = n * __fdiv_rn(-pl, wa + wb);
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
    const float sh = len(ev);
    const V3 axe = ev * rcp_(sh);
    const float ae = 2.0f * atan2r(sh, qerr.w);
    const V3 aw2 = rotate(axe, qau);
    const float w = dot(hadamard(aw2, Ia), aw2) + dot(hadamard(aw2, Ib), aw2);
    const V3 ai = aw2 * __fdiv_rn(ae, w);
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
  const float ts = len(vt);
  const V3 rna = cross(ra, n), rnb = cross(rb, n);
  const float wn = (ima + dot(hadamard(rna, Ia), rna)) + (imb + dot(hadamard(rnb, Ib), rnb));
  if (wn < 1e-8f) return;
  const float excess = fmaxf(pen - slop, 0.0f);
  const float bias = __fdiv_rn(baumgarte * excess, dt);
  const float vrest = vn < -0.5f ? rest * vn : 0.0f;
  const float jn = fmaxf(__fdiv_rn(-(vn + vrest) + bias, wn), 0.0f);
  const V3 in_ = n * jn;
  const float pcorr = baumgarte * excess;
  if (ima > 1e-8f) {
    s.vel(ia) = with_w(madd(in_, ima, v3(s.vel(ia))), s.vel(ia).w);
    s.ang(ia) = with_w(v3(s.ang(ia)) + hadamard(cross(ra, in_), Ia), s.ang(ia).w);
    s.pos(ia) = with_w(madd(n, pcorr * __fdiv_rn(ima, isum), v3(s.pos(ia))), s.pos(ia).w);
  }
  if (imb > 1e-8f) {
    s.vel(ib) = with_w(msub(in_, imb, v3(s.vel(ib))), s.vel(ib).w);
    s.ang(ib) = with_w(v3(s.ang(ib)) - hadamard(cross(rb, in_), Ib), s.ang(ib).w);
    s.pos(ib) = with_w(msub(n, pcorr * __fdiv_rn(imb, isum), v3(s.pos(ib))), s.pos(ib).w);
  }
  const float jacc = jx + jn;
  if (ts > 1e-6f && jacc > 1e-6f) {
    const V3 t = vt * rcp_(ts);
    const V3 rta = cross(ra, t), rtb = cross(rb, t);
    const float wt = (ima + dot(hadamard(rta, Ia), rta)) + (imb + dot(hadamard(rtb, Ib), rtb));
    if (wt > 1e-8f) {
      const float jt = fminf(__fdiv_rn(ts, wt), fr * jacc);
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
__device__ __forceinline__ bool narrow_core(uint32_t ta, uint32_t tb, V3 pa, V3 pb, float ra, float rb, float hl,
                                            float4 cq, V3& point, V3& normal, float& pen) {
  if (ta == 0 && tb == 0) {
    const V3 d = pb - pa;
    const float dist = len(d);
    const float md = ra + rb;
    if (dist < md && dist > 1e-6f) {
      normal = d * rcp_(dist);
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
    const V3 cpos = ta == 1 ? pa : pb;
    const float cr = ta == 1 ? ra : rb;
    const V3 axis = rotate(v3(0.0f, 0.0f, 1.0f), cq);
    const V3 p1 = msub(axis, hl, cpos), p2 = madd(axis, hl, cpos);
    const float d1 = p1.z - cr, d2 = p2.z - cr;
    if (d1 < 0.0f || d2 < 0.0f) {
      point = d1 < d2 ? p1 : p2;
      point.z = 0.0f;
      pen = -fminf(d1, d2);
      normal = ta == 1 ? v3(0.0f, 0.0f, 1.0f) : v3(0.0f, 0.0f, -1.0f);
      return true;
    }
  }
  return false;
}

// True for the type pairs narrow_core can report a contact for.
__host__ __device__ inline bool narrow_supported(uint32_t ta, uint32_t tb) {
  return (ta == 0 && tb == 0) || (ta == 0 && tb == 3) || (ta == 3 && tb == 0) || (ta == 1 && tb == 3) ||
         (ta == 3 && tb == 1);
}

}  // namespace zb
