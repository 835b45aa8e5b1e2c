// Environment-per-lane step kernel for sm_100a.
//
// One launch runs every substep of one World.step (src/world/world.zig:694-792).  Each
// lane owns one environment and runs the whole step for it serially, in exactly the
// order the reference's dispatch sequence defines (world.zig:934-1293), so no lane ever
// waits for another: the warp executes one instruction stream for 32 environments of the
// same model, and every model load is warp-uniform (served by the constant cache from
// the __grid_constant__ FModel).
//
// Shared memory holds the environment's bodies, joint torques/states and a compressed
// contact list, laid out [item][lane] so that the 32 lanes of a warp touch 32
// consecutive words.  The contact list is compressed by two facts of the reference
// pipeline:
//  * the narrow phase result of a slot depends only on its geom pair and the body poses
//    (narrow_phase, all_shaders.metal:751-894), so point/normal/penetration are kept once
//    per "hittable" candidate pair (a pair whose geom types the narrow phase handles);
//  * warm starting (match_cached_contacts, 1483-1544) depends only on the slot's body
//    pair and point, so it is evaluated once per hittable pair as well.
// Per slot only the candidate index, the slot's original position (for the in-place
// write-back of slots that never made contact), and the accumulated normal impulse are
// kept.  Slot order, the unbounded counter, the frozen 64-slot list, the stable sort by
// body-pair key and the first-strict-minimum match rule are those of the reference.
//
// Environments whose contact buffer the fast path cannot represent (slot indices that
// are not broad-phase candidates, an unsorted list, non-zero tangent impulses on a
// matched slot -- none of which this library ever writes) are left untouched here and
// appended to a list that the general kernel (step_kernel.cu) then steps.
#include <cuda_runtime.h>

#include <algorithm>

#include "devmath.cuh"
#include "fast_model.h"
#include "model_access.cuh"
#include "physics.cuh"
#include "step_kernel.h"
#include "zeno_types.h"

namespace zb {

// ------------------------------------------------------------------------------------
// Shared-memory plan: per-environment byte offsets, each section 16-byte aligned.  The
// block region of a section is (per-env offset) * envs_per_block; element (item, lane)
// sits at (item * envs_per_block + lane) * element size inside it.
// ------------------------------------------------------------------------------------
struct FPlan {
  uint32_t pos, quat, vel, ang;               // float4 [B]
  uint32_t jt, jp, jv;                        // float [J]
  uint32_t imp;                               // float [M]   normal impulse per slot
  uint32_t meta;                              // u32 [M]     slot word (below)
  uint32_t aux;                               // u8 [M]      prev key ranks (substep 0), then hit slots
  uint32_t pp, nt;                            // float4 [H]  (point, pen), (normal, warm start)
  uint32_t nlh;                               // u8 [H]      list length at the pair's last hit
  uint32_t hdr;                               // u32 [4]     count, prev count, prev-separate, unusable
  uint32_t flags;                             // u32
  uint32_t bytes;
};

__host__ __device__ inline uint32_t fa16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline FPlan fast_plan(uint32_t B, uint32_t J, uint32_t M, uint32_t H) {
  FPlan p;
  uint32_t o = 0;
  const uint32_t b4 = fa16(16u * B), j1 = fa16(4u * J), m4 = fa16(4u * M), m1 = fa16(M), h4 = fa16(16u * H),
                 h1 = fa16(H);
  p.pos = o, o += b4;
  p.quat = o, o += b4;
  p.vel = o, o += b4;
  p.ang = o, o += b4;
  p.jt = o, o += j1;
  p.jp = o, o += j1;
  p.jv = o, o += j1;
  p.imp = o, o += m4;
  p.meta = o, o += m4;
  p.aux = o, o += m1;
  p.pp = o, o += h4;
  p.nt = o, o += h4;
  p.nlh = o, o += h1;
  p.hdr = o, o += 16;
  p.flags = o, o += 16;
  p.bytes = o;
  return p;
}

uint32_t fast_env_smem_bytes(uint32_t B, uint32_t J, uint32_t M, uint32_t H) { return fast_plan(B, J, M, H).bytes; }

// Slot word: candidate | origin << 8 | hittable index << 16 (7 bits) | visited << 23 | key rank << 24
__device__ __forceinline__ uint32_t sw_pair(uint32_t w) { return w & 0xFFu; }
__device__ __forceinline__ uint32_t sw_origin(uint32_t w) { return (w >> 8) & 0xFFu; }
__device__ __forceinline__ uint32_t sw_hit(uint32_t w) { return (w >> 16) & 0x7Fu; }
__device__ __forceinline__ uint32_t sw_rank(uint32_t w) { return w >> 24; }
constexpr uint32_t kVisited = 1u << 23;

__device__ __forceinline__ uint32_t slot_word(const ModelS& m, uint32_t p, uint32_t origin) {
  const uint32_t pi = m.pinfo(p);
  return p | (origin << 8) | (((pi >> 16) & 0x7Fu) << 16) | (pi & 0xFF000000u);
}

// Candidate index of a stored (body a, body b, geom a, geom b) tuple, kNoPair when the
// tuple is not one the broad phase emits.
__device__ __forceinline__ uint32_t lookup_pair(const ModelS& m, uint4 ix) {
  if (ix.z >= m.f.G || ix.w >= m.f.G) return fm::kNoPair;
  const uint32_t p = m.ggpair(ix.z, ix.w);
  if (p == fm::kNoPair) return fm::kNoPair;
  if (ix.x != m.gbody(ix.z) || ix.y != m.gbody(ix.w)) return fm::kNoPair;
  return p;
}

// Body state of this lane's environment.
struct LaneBodies {
  float4 *p, *q, *v, *w;
  uint32_t st;
  __device__ __forceinline__ float4& pos(uint32_t b) { return p[b * st]; }
  __device__ __forceinline__ float4& quat(uint32_t b) { return q[b * st]; }
  __device__ __forceinline__ float4& vel(uint32_t b) { return v[b * st]; }
  __device__ __forceinline__ float4& ang(uint32_t b) { return w[b * st]; }
};

// Narrow phase of hittable pair h on the current poses.
__device__ __forceinline__ bool narrow_h(const ModelS& m, uint32_t h, LaneBodies& S, V3& point, V3& normal,
                                         float& pen) {
  const uint32_t hi = m.hinfo(h);
  const float4 ga = m.hga(h), gb = m.hgb(h);
  const V3 pa = v3(S.pos((hi >> 16) & 0xFFu)) + v3(ga);
  const V3 pb = v3(S.pos(hi >> 24)) + v3(gb);
  return narrow_core(hi & 0xFFu, (hi >> 8) & 0xFFu, pa, pb, ga.w, gb.w, m.hhl(h), m.hcq(h), point, normal, pen);
}

enum : uint32_t {
  kSkipState = 1u,        // leave body / joint state untouched (handed over, or outside the step mask)
  kWriteJointState = 2u,  // publish joint positions / velocities
  kAccWritten = 4u,       // accelerations already written (auto-reset replaced the velocities)
};

// Everything one lane does for its environment between the cooperative load and store.
// Returns false when the environment must go to the general kernel (nothing written).
__device__ __forceinline__ bool run_env(const StepArgs& a, const FModel& f, const FPlan& pl, const unsigned char* hot,
                                        unsigned char* blk, uint32_t epb, uint32_t l, uint32_t e, uint32_t& flags_out) {
  const ModelS m{hot, f};
  const uint32_t B = a.B, J = a.J, A = a.A, M = a.M, H = f.H, P = f.P;
  LaneBodies S{reinterpret_cast<float4*>(blk + pl.pos * epb) + l, reinterpret_cast<float4*>(blk + pl.quat * epb) + l,
               reinterpret_cast<float4*>(blk + pl.vel * epb) + l, reinterpret_cast<float4*>(blk + pl.ang * epb) + l,
               epb};
  // pose before integration, read back by the velocity update: an L2-resident scratch,
  // [body][pos, quat][env] so that a warp's accesses are contiguous
  const size_t E = a.num_envs;
  float4* ppos = a.pose_scratch + e;
  float4* pquat = a.pose_scratch + E + e;
  const size_t pst = 2 * E;
  float* jt = reinterpret_cast<float*>(blk + pl.jt * epb) + l;
  float* jp = reinterpret_cast<float*>(blk + pl.jp * epb) + l;
  float* jv = reinterpret_cast<float*>(blk + pl.jv * epb) + l;
  float* imp = reinterpret_cast<float*>(blk + pl.imp * epb) + l;
  uint32_t* meta = reinterpret_cast<uint32_t*>(blk + pl.meta * epb) + l;
  uint8_t* aux = blk + pl.aux * epb + l;
  float4* pp = reinterpret_cast<float4*>(blk + pl.pp * epb) + l;
  float4* nt = reinterpret_cast<float4*>(blk + pl.nt * epb) + l;
  uint8_t* nlh = blk + pl.nlh * epb + l;

  uint32_t* hdr = reinterpret_cast<uint32_t*>(blk + pl.hdr * epb) + l;

  // ---------------- contact list of the previous step ----------------
  // The block loaded the slots (slot words, impulses, previous-list key ranks) and marked
  // lists whose tuples are not broad-phase candidates.  Both lists are sorted by key
  // whenever this library wrote them; anything else goes to the general kernel.
  if (hdr[3 * epb]) return false;
  uint32_t count = hdr[0];
  const uint32_t prev_count0 = hdr[epb];
  const bool sep = hdr[2 * epb] != 0;
  const uint32_t n0 = count < M ? count : M;
  Contact* gc = a.contacts + size_t(e) * M;
  const Contact* gprev = sep ? a.prev_contacts + size_t(e) * M : gc;
  const uint32_t n_prev0 = prev_count0 < M ? prev_count0 : M;
  uint32_t last = 0;
  for (uint32_t i = 0; i < n0; ++i) {
    const uint32_t r = sw_rank(meta[i * epb]);
    if (r < last) return false;
    last = r;
  }
  last = 0;
  for (uint32_t j = 0; j < n_prev0; ++j) {  // previous-substep list (cache_contacts, 1454-1478)
    const uint32_t r = aux[j * epb];
    if (r < last) return false;
    last = r;
  }
  for (uint32_t h = 0; h < H; ++h) nlh[h * epb] = 0;

  const float dt = a.dt, inv_dt = a.inv_dt;
  const V3 grav{a.gravity[0], a.gravity[1], a.gravity[2]};
  const float* act = a.actions + size_t(e) * A;
  // apply_actions (196-229): the torques are the same in every substep
  if (a.substeps > 0)
    for (uint32_t k = 0; k < A; ++k) {
      const float tq = clampf(act[k], f.a_cmin[k], f.a_cmax[k]) * f.a_gear[k];
      jt[f.a_joint[k] * epb] = clampf(tq, f.a_fmin[k], f.a_fmax[k]);
    }

  uint64_t prev_hit = 0;
  uint32_t n_prev = n_prev0;
  for (uint32_t s = 0; s < a.substeps; ++s) {
    // ---- kinematic bodies (update_kinematic 304-339; massless, so no gravity wrench) ----
    for (uint32_t b = 0; b < B; ++b) {
      if ((m.body(b) & 0xFFu) != 1u) continue;
      S.pos(b) = with_w(madd(v3(S.vel(b)), dt, v3(S.pos(b))), 0.0f);
      const float4 q = S.quat(b);
      S.quat(b) = qnormalize(qmadd(qmul_v((v3(S.ang(b)) * dt) * 0.5f, q), 1.0f, q));
    }
    // ---- wrench (compute_forces 345-388, apply_joint_forces 122-190) and semi-implicit
    //      Euler (save_prev_state 1900-1913, integrate 394-462), children first: a body's
    //      wrench reads only its own and its parent's orientation, neither yet integrated.
    //      Four bodies at a time: all their wrenches first, then their integration, so
    //      the four dependency chains overlap.
    for (uint32_t hi_b = B; hi_b > 0;) {
      constexpr int kC = 4;
      const uint32_t nc = hi_b < kC ? hi_b : kC;
      V3 F[kC], T[kC];
      float4 q[kC], x[kC], v0[kC], w0[kC];
#pragma unroll
      for (int c = 0; c < kC; ++c) {
        if (uint32_t(c) >= nc) continue;
        const uint32_t b = hi_b - 1 - c;
        const float4 mi = m.imi(b);
        q[c] = S.quat(b);
        x[c] = S.pos(b);
        v0[c] = S.vel(b);
        w0[c] = S.ang(b);
        F[c] = v3(m.gforce(b));
        T[c] = V3{0.0f, 0.0f, 0.0f};
        if (!(mi.x < 1e-8f)) T[c] = cross(rotate(v3(m.com(b)), q[c]), F[c]);
        const uint32_t bi = m.body(b);
        const uint32_t k0 = (bi >> 8) & 0xFFu, k1 = (bi >> 16) & 0xFFu;
        for (uint32_t k = k0; k < k1; ++k) {
          const uint32_t ent = m.jf(k);
          const uint32_t j = ent & 0x7Fu;
          const float tau = jt[j * epb];
          if (fabsf(tau) < 1e-6f) continue;
          const uint32_t ji = m.jinfo(j);
          const V3 fj = rotate(v3(m.jaxis(j)), S.quat((ji >> 8) & 0xFFu)) * tau;
          if ((ji & 0xFFu) == 2u) F[c] = (ent & 0x80u) ? F[c] - fj : F[c] + fj;
          else T[c] = (ent & 0x80u) ? T[c] - fj : T[c] + fj;
        }
      }
#pragma unroll
      for (int c = 0; c < kC; ++c) {
        if (uint32_t(c) >= nc) continue;
        const uint32_t b = hi_b - 1 - c;
        const float4 mi = m.imi(b);
        ppos[b * pst] = x[c];
        pquat[b * pst] = q[c];
        if (mi.x < 1e-8f) continue;
        const V3 v = madd(F[c] * mi.x, dt, v3(v0[c])) * 0.999f;
        S.vel(b) = with_w(v, 0.0f);
        S.pos(b) = with_w(madd(v, dt, v3(x[c])), 0.0f);
        const V3 w = madd(hadamard(v3(mi.y, mi.z, mi.w), T[c]), dt, v3(w0[c])) * 0.999f;
        S.ang(b) = with_w(w, 0.0f);
        S.quat(b) = qnormalize(qmadd(qmul_v((w * dt) * 0.5f, q[c]), 1.0f, q[c]));
      }
      hi_b -= nc;
    }
    // ---- broad phase (broad_phase 468-533): candidates in emission order ----
    const uint32_t n_old = count < M ? count : M;
    for (uint32_t p0 = 0; p0 < P; p0 += 64) {
      const uint32_t pn = P - p0 < 64u ? P - p0 : 64u;
      uint64_t pass = 0;
#pragma unroll 4
      for (uint32_t i = 0; i < pn; ++i) {
        const uint32_t p = p0 + i;
        const uint32_t pb = m.pbody(p);
        bool ok = true;
        if (!(pb >> 16)) {
          const uint32_t pi = m.pinfo(p);
          const V3 pa = v3(S.pos(pb & 0xFFu)) + v3(m.gps(pi & 0xFFu));
          const V3 pc = v3(S.pos((pb >> 8) & 0xFFu)) + v3(m.gps((pi >> 8) & 0xFFu));
          const V3 d = pc - pa;
          ok = !(dot(d, d) >= m.pmd2(p));
        }
        pass |= uint64_t(ok) << i;
      }
      if (count >= M) {  // the list is frozen: only the counter advances
        count += uint32_t(__popcll(pass));
        continue;
      }
      while (pass) {
        const uint32_t i = uint32_t(__ffsll(pass)) - 1u;
        pass &= pass - 1;
        if (count < M) meta[count * epb] = slot_word(m, p0 + i, count);
        ++count;
      }
    }
    const uint32_t n = count < M ? count : M;
    // ---- stable sort by key (sort_contacts 711-745): insert the new slots in order ----
    for (uint32_t q = n_old; q < n; ++q) {
      const uint32_t w = meta[q * epb];
      const float x = imp[q * epb];
      uint32_t r = q;
      while (r > 0 && sw_rank(meta[(r - 1) * epb]) > sw_rank(w)) {
        meta[r * epb] = meta[(r - 1) * epb];
        imp[r * epb] = imp[(r - 1) * epb];
        --r;
      }
      meta[r * epb] = w;
      imp[r * epb] = x;
    }
    // ---- narrow phase + warm start (narrow_phase 751-894, match_cached_contacts
    //      1483-1544), once per hittable pair.  First pass: the match, against the
    //      previous substep's points, which the second pass then overwrites.
    for (uint32_t h = 0; h < H; ++h) {
      V3 point, normal;
      float pen;
      if (!narrow_h(m, h, S, point, normal, pen)) continue;
      const uint32_t rank = m.pinfo(m.hpair(h)) >> 24;
      float best = 0.04f;
      int js = -1;
      float val = 0.0f;
      if (s == 0) {
        uint32_t lo = 0, hi = n_prev;  // first previous slot with key >= this key
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (aux[mid * epb] < rank) lo = mid + 1;
          else hi = mid;
        }
        for (uint32_t j = lo; j < n_prev && aux[j * epb] == rank; ++j) {
          const float4 q = *reinterpret_cast<const float4*>(gprev[j].position_pen);
          if (q.w < 0.0f) continue;
          const V3 d = xyz(q) - point;
          const float dsq = dot(d, d);
          if (dsq < best) {
            best = dsq;
            js = int(j);
          }
        }
        if (js >= 0) {
          const float4 pi = *reinterpret_cast<const float4*>(gprev[js].impulses);
          // tangent impulses are never written by the solver; a stored non-zero value
          // would have to be carried per slot, which only the general kernel does
          if ((__float_as_uint(pi.y) | __float_as_uint(pi.z)) != 0u) return false;
          val = pi.x * 0.8f;
        }
      } else {
        uint32_t lo = 0, hi = n;
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (sw_rank(meta[mid * epb]) < rank) lo = mid + 1;
          else hi = mid;
        }
        for (uint32_t j = lo; j < n; ++j) {
          const uint32_t w = meta[j * epb];
          if (sw_rank(w) != rank) break;
          if (sw_origin(w) >= n_prev) continue;  // appended in this substep
          const uint32_t hj = sw_hit(w);
          if (hj == fm::kNoHit || !((prev_hit >> hj) & 1ull)) continue;
          const V3 d = xyz(pp[hj * epb]) - point;
          const float dsq = dot(d, d);
          if (dsq < best) {
            best = dsq;
            js = int(j);
          }
        }
        if (js >= 0) val = imp[uint32_t(js) * epb] * 0.8f;
      }
      reinterpret_cast<float*>(&nt[h * epb])[3] = val;
    }
    uint64_t hit_now = 0;
    for (uint32_t h = 0; h < H; ++h) {
      V3 point, normal;
      float pen;
      if (narrow_h(m, h, S, point, normal, pen)) {
        pp[h * epb] = with_w(point, pen);
        const float warm = nt[h * epb].w;
        nt[h * epb] = with_w(normal, warm);
        nlh[h * epb] = uint8_t(n);
        hit_now |= 1ull << h;
      } else {
        reinterpret_cast<float*>(&pp[h * epb])[3] = -1.0f;
      }
    }
    // slot impulses (narrow zeroes them, a match warm-starts them) and the hit-slot list
    uint32_t nh = 0;
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t hh = sw_hit(meta[i * epb]);
      if (hh != fm::kNoHit && ((hit_now >> hh) & 1ull)) {
        imp[i * epb] = nt[hh * epb].w;
        aux[nh * epb] = uint8_t(i);
        ++nh;
      }
    }
    // ---- XPBD joints (solve_joints 909-1399), colour by colour in batches ----
    for (uint32_t it = 0; it < a.iterations; ++it)
      for (uint32_t q = 0; q < a.K; ++q) solve_constraint(m, m.constraint(q), S);
    // ---- contacts in slot order (solve_contacts 1644-1793) ----
    for (uint32_t it = 0; it < a.iterations; ++it)
      for (uint32_t v = 0; v < nh; ++v) {
        const uint32_t i = aux[v * epb];
        const uint32_t hh = sw_hit(meta[i * epb]);
        const uint32_t hi = m.hinfo(hh);
        const float4 nn = nt[hh * epb];
        float jx = imp[i * epb];
        solve_contact(m, pp[hh * epb], make_float4(nn.x, nn.y, nn.z, m.hfr(hh)), jx, a.restitution, (hi >> 16) & 0xFFu,
                      hi >> 24, S, dt, a.baumgarte, a.slop);
        imp[i * epb] = jx;
      }
    // ---- velocities from the position change (xpbd_update_velocities 1922-1961) ----
    for (uint32_t b = 0; b < B; ++b) {
      if (m.imi(b).x < 1e-8f) continue;
      S.vel(b) = with_w((v3(S.pos(b)) - v3(ppos[b * pst])) * inv_dt, 0.0f);
      float4 dq = qmul(S.quat(b), qconj(pquat[b * pst]));
      if (dq.w < 0.0f) dq = qneg(dq);
      S.ang(b) = with_w((xyz(dq) * 2.0f) * inv_dt, 0.0f);
    }
    prev_hit = hit_now;
    n_prev = n;
  }

  // ---------------- joint states and sensors from the final substep ----------------
  uint32_t flags = 0;
  const bool stepped = a.substeps > 0;
  const bool publish = a.step_mask == nullptr || a.step_mask[e] != 0;
  if (stepped) {
    for (uint32_t j = 0; j < J; ++j) {  // update_joint_states 1550-1638
      const uint32_t ji = m.jinfo(j);
      const uint32_t ty = ji & 0xFFu, ia = (ji >> 8) & 0xFFu, ib = (ji >> 16) & 0xFFu;
      float p = 0.0f, v = 0.0f;
      const float4 qa = S.quat(ia), qb = S.quat(ib);
      const V3 axl = v3(m.jaxis(j));
      if (ty == 1) {
        const V3 aw = rotate(axl, qa);
        const float4 qrel = qmul(qconj(qa), qb);
        p = 2.0f * atan2r(dot(xyz(qrel), axl), qrel.w);
        v = dot(v3(S.ang(ib)) - v3(S.ang(ia)), aw);
      } else if (ty == 2) {
        const V3 aw = rotate(axl, qa);
        const V3 ra = rotate(v3(f.j_ap[j]), qa);
        const V3 rb = rotate(v3(f.j_ac[j]), qb);
        p = dot((v3(S.pos(ib)) + rb) - (v3(S.pos(ia)) + ra), aw);
        const V3 vpa = v3(S.vel(ia)) + cross(v3(S.ang(ia)), ra), vpb = v3(S.vel(ib)) + cross(v3(S.ang(ib)), rb);
        v = dot(vpb - vpa, aw);
      }
      jp[j * epb] = p;
      jv[j * epb] = v;
    }
    if (publish) {  // read_sensors 1799-1893
      float* gobs = a.obs + size_t(e) * a.obs_dim;
      for (uint32_t si = 0; si < a.S; ++si) {
        const uint32_t sinfo = f.s_info[si];
        const uint32_t o = (sinfo >> 8) & 0xFFu;
        float* out = gobs + (sinfo >> 16);
        switch (sinfo & 0xFFu) {
          case 0: out[0] = jp[o * epb]; break;
          case 1: out[0] = jv[o * epb]; break;
          case 2: {
            const V3 lg = rotate(grav, qconj(S.quat(o)));
            out[0] = lg.x, out[1] = lg.y, out[2] = lg.z;
            break;
          }
          case 3:
          case 10: {
            const float4 w = S.ang(o);
            out[0] = w.x, out[1] = w.y, out[2] = w.z;
            break;
          }
          case 7: {
            const float4 x = S.pos(o);
            out[0] = x.x, out[1] = x.y, out[2] = x.z;
            break;
          }
          case 8: {
            const float4 x = S.quat(o);
            out[0] = x.x, out[1] = x.y, out[2] = x.z, out[3] = x.w;
            break;
          }
          case 9: {
            const float4 x = S.vel(o);
            out[0] = x.x, out[1] = x.y, out[2] = x.z;
            break;
          }
          default: break;
        }
      }
    }

    // ---------------- contact slots back to memory ----------------
    // A slot whose pair made contact while the slot was in the list carries that pair's
    // last contact; any other slot keeps the record stored at its original position,
    // marked invalid.  Sorting may have moved slots, so the in-place write follows the
    // permutation's cycles.
    const uint32_t n_fin = count < M ? count : M;
    Contact* dst = publish ? gc : a.prev_contacts + size_t(e) * M;
    const bool inplace = publish;
    for (uint32_t i = 0; i < n_fin; ++i) {
      if (meta[i * epb] & kVisited) continue;
      uint4 saved[4];
      const uint32_t oi = sw_origin(meta[i * epb]);
      const bool cycle = inplace && oi != i;
      if (cycle)
        for (int c = 0; c < 4; ++c) saved[c] = reinterpret_cast<const uint4*>(gc + i)[c];
      uint32_t j = i;
      for (uint32_t guard = 0; guard < n_fin; ++guard) {
        const uint32_t w = meta[j * epb];
        meta[j * epb] = w | kVisited;
        const uint32_t p = sw_pair(w), o = sw_origin(w), hh = sw_hit(w);
        const uint32_t pi = m.pinfo(p), pbody = m.pbody(p);
        const uint4 idx = make_uint4(pbody & 0xFFu, (pbody >> 8) & 0xFFu, pi & 0xFFu, (pi >> 8) & 0xFFu);
        uint4* out = reinterpret_cast<uint4*>(dst + j);
        if (hh != fm::kNoHit && o < nlh[hh * epb]) {
          const float4 nn = nt[hh * epb];
          out[0] = *reinterpret_cast<const uint4*>(&pp[hh * epb]);
          const float4 nf = make_float4(nn.x, nn.y, nn.z, m.hfr(hh));
          out[1] = *reinterpret_cast<const uint4*>(&nf);
          out[2] = idx;
          const float4 im = make_float4(imp[j * epb], 0.0f, 0.0f, a.restitution);
          out[3] = *reinterpret_cast<const uint4*>(&im);
        } else if (inplace && o == j) {
          reinterpret_cast<float*>(out)[3] = -1.0f;
          out[2] = idx;
        } else {
          uint4 r[4];
          if (cycle && o == i) {
            for (int c = 0; c < 4; ++c) r[c] = saved[c];
          } else {
            for (int c = 0; c < 4; ++c) r[c] = reinterpret_cast<const uint4*>(gc + o)[c];
          }
          r[0].w = __float_as_uint(-1.0f);
          r[2] = idx;
          for (int c = 0; c < 4; ++c) out[c] = r[c];
        }
        if (!cycle || o == i) break;
        j = o;
      }
    }
  }

  // ---------------- caches, counters, task extension ----------------
  if (!publish) {
    // step_subset: an env outside the mask keeps its public state, but the reference
    // still advanced its contact cache (world.zig:833-929 restores only public buffers).
    if (stepped) {
      a.prev_counts[e] = count;
      a.prev_sep[e] = 1;
    }
    flags_out = flags | kSkipState;
    return true;
  }
  uint32_t count_out = count;
  if (stepped) flags |= kWriteJointState;
  if (a.task.enabled) {
    const DTask& tk = a.task;
    const uint32_t tb = tk.body;
    const float z = S.pos(tb).z;
    const bool done = !(z >= tk.z_min && z <= tk.z_max);
    float ctrl = 0.0f;
    for (uint32_t k = 0; k < A; ++k) ctrl = fma_(act[k], act[k], ctrl);
    float r = fma_(tk.forward_weight, S.vel(tb).x, tk.alive_bonus);
    r = fma_(-tk.ctrl_cost, ctrl, r);
    a.rewards[e] = r;
    a.dones[e] = done ? 1 : 0;
    if (done && tk.auto_reset) {
      // accelerations of the step just taken, before the state is replaced
      const float4* gv0 = reinterpret_cast<const float4*>(a.vel) + size_t(e) * B;
      float4* gacc = reinterpret_cast<float4*>(a.acc) + size_t(e) * B;
      for (uint32_t b = 0; b < B; ++b) {
        const float4 v0 = gv0[b], v1 = S.vel(b);
        gacc[b] = make_float4((v1.x - v0.x) * a.inv_step, (v1.y - v0.y) * a.inv_step, (v1.z - v0.z) * a.inv_step, 0.0f);
      }
      flags |= kAccWritten | kWriteJointState;
      // FK-consistent noisy reset from the initial template
      const uint32_t ep = a.episode[e];
      const float* t = a.init_state;
      for (uint32_t b = 0; b < B; ++b) {
        S.pos(b) = reinterpret_cast<const float4*>(t)[b];
        S.quat(b) = reinterpret_cast<const float4*>(t)[B + b];
        S.vel(b) = reinterpret_cast<const float4*>(t)[2 * B + b];
        S.ang(b) = reinterpret_cast<const float4*>(t)[3 * B + b];
      }
      for (uint32_t j = 0; j < J; ++j) {
        jp[j * epb] = t[16 * B + j];
        jv[j * epb] = t[16 * B + J + j];
      }
      if (tk.noise != 0.0f) {
        const uint64_t genv = uint64_t(e) + tk.env_offset;
        const uint32_t rb = tk.body;
        float4 x = S.pos(rb);
        x.x = x.x + tk.noise * uniform_pm1(tk.seed, genv, ep, 0u);
        x.y = x.y + tk.noise * uniform_pm1(tk.seed, genv, ep, 1u);
        x.z = x.z + tk.noise * uniform_pm1(tk.seed, genv, ep, 2u);
        S.pos(rb) = x;
        for (uint32_t j = 0; j < J; ++j) {
          const uint32_t ji = m.jinfo(j);
          if ((ji & 0xFFu) != 1u) continue;
          const float th = tk.noise * uniform_pm1(tk.seed, genv, ep, 3u + j);
          const uint32_t pa = (ji >> 8) & 0xFFu, ch = (ji >> 16) & 0xFFu;
          const float4 qp = S.quat(pa);
          const V3 anchor = v3(S.pos(pa)) + rotate(v3(f.j_ap[j]), qp);
          const V3 ax = rotate(v3(m.jaxis(j)), qp);
          const float al = len(ax);
          if (!(al > 1e-8f)) continue;
          const V3 hv = ax * __fdiv_rn(0.5f * th, al);
          const float4 qr = qnormalize(make_float4(hv.x, hv.y, hv.z, 1.0f));
          const uint32_t end = ch + (m.body(ch) >> 24);
          for (uint32_t d = ch; d < end; ++d) {
            const V3 rel = v3(S.pos(d)) - anchor;
            S.pos(d) = with_w(anchor + rotate(rel, qr), S.pos(d).w);
            S.quat(d) = qnormalize(qmul(qr, S.quat(d)));
          }
        }
      }
      a.episode[e] = ep + 1;
      count_out = 0;
    }
  }
  a.counts[e] = count_out;
  if (stepped) {
    a.prev_counts[e] = count;
    a.prev_sep[e] = 0;
  }
  flags_out = flags;
  return true;
}

__global__ void __launch_bounds__(32) fast_step_kernel(const __grid_constant__ StepArgs a,
                                                       const __grid_constant__ FModel f) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t epb = blockDim.x, l = threadIdx.x;
  const uint32_t e0 = blockIdx.x * epb;
  if (e0 >= a.num_envs) return;
  const uint32_t nb = min(epb, a.num_envs - e0);
  const unsigned wmask = epb == 32 ? 0xFFFFFFFFu : ((1u << epb) - 1u);
  const uint32_t B = a.B, J = a.J, M = a.M;
  const FPlan pl = fast_plan(B, J, M, f.H);
  // shared memory: the model's hot image, then the per-environment sections
  unsigned char* hot = smem_raw;
  unsigned char* blk = smem_raw + f.hot_bytes;
  for (uint32_t t = l; t < f.hot_bytes / 16u; t += epb) reinterpret_cast<uint4*>(hot)[t] = f.hot[t];
  __syncwarp(wmask);
  // gravity force per body for this step (compute_forces 345-388): g / (1/m), zero when massless
  for (uint32_t b = l; b < B; b += epb) {
    const float4 mi = reinterpret_cast<const float4*>(hot + f.o_imi)[b];
    const V3 g{a.gravity[0], a.gravity[1], a.gravity[2]};
    reinterpret_cast<float4*>(hot + f.o_gforce)[b] =
        mi.x < 1e-8f ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : with_w(g * rcp_(mi.x), 0.0f);
  }
  float4* s_pos = reinterpret_cast<float4*>(blk + pl.pos * epb);
  float4* s_quat = reinterpret_cast<float4*>(blk + pl.quat * epb);
  float4* s_vel = reinterpret_cast<float4*>(blk + pl.vel * epb);
  float4* s_ang = reinterpret_cast<float4*>(blk + pl.ang * epb);
  float* s_jt = reinterpret_cast<float*>(blk + pl.jt * epb);
  float* s_jp = reinterpret_cast<float*>(blk + pl.jp * epb);
  float* s_jv = reinterpret_cast<float*>(blk + pl.jv * epb);
  uint32_t* s_flags = reinterpret_cast<uint32_t*>(blk + pl.flags * epb);

  // ---- coalesced load of the block's body state and joint torques ----
  const size_t eb = size_t(e0) * B;
  float4* gpos = reinterpret_cast<float4*>(a.pos) + eb;
  float4* gquat = reinterpret_cast<float4*>(a.quat) + eb;
  float4* gvel = reinterpret_cast<float4*>(a.vel) + eb;
  float4* gang = reinterpret_cast<float4*>(a.angvel) + eb;
  float4* gacc = reinterpret_cast<float4*>(a.acc) + eb;
  for (uint32_t t = l; t < nb * B; t += epb) {
    const uint32_t el = t / B, b = t - el * B, si = b * epb + el;
    s_pos[si] = gpos[t];
    s_quat[si] = gquat[t];
    s_vel[si] = gvel[t];
    s_ang[si] = gang[t];
  }
  float* gjt = a.jtorque + size_t(e0) * J;
  float* gjp = a.jpos + size_t(e0) * J;
  float* gjv = a.jvel + size_t(e0) * J;
  for (uint32_t t = l; t < nb * J; t += epb) {
    const uint32_t el = t / J, j = t - el * J;
    s_jt[j * epb + el] = gjt[t];
  }
  // ---- contact list headers, then the slots: slot words, impulses, previous-list ranks ----
  uint32_t* s_hdr = reinterpret_cast<uint32_t*>(blk + pl.hdr * epb);
  float* s_imp = reinterpret_cast<float*>(blk + pl.imp * epb);
  uint32_t* s_meta = reinterpret_cast<uint32_t*>(blk + pl.meta * epb);
  uint8_t* s_aux = blk + pl.aux * epb;
  if (l < nb) {
    const uint32_t e = e0 + l;
    s_hdr[l] = a.counts[e];
    s_hdr[epb + l] = a.prev_counts[e];
    s_hdr[2 * epb + l] = a.prev_sep[e];
    s_hdr[3 * epb + l] = 0;
  }
  __syncwarp(wmask);
  const ModelS m{hot, f};
  const Contact* gcb = a.contacts + size_t(e0) * M;
  constexpr uint32_t kU = 4;  // slots per thread per round: their loads are in flight together
  for (uint32_t t0 = l; t0 < nb * M; t0 += kU * epb) {
    uint4 ix[kU], px[kU];
    float im[kU];
#pragma unroll
    for (uint32_t u = 0; u < kU; ++u) {
      const uint32_t t = t0 + u * epb;
      if (t >= nb * M) continue;
      const uint32_t el = t / M, i = t - el * M;
      ix[u] = *reinterpret_cast<const uint4*>(gcb[t].indices);
      im[u] = gcb[t].impulses[0];
      if (s_hdr[2 * epb + el] != 0 && i < s_hdr[epb + el])
        px[u] = *reinterpret_cast<const uint4*>(a.prev_contacts[size_t(e0 + el) * M + i].indices);
      else
        px[u] = ix[u];
    }
#pragma unroll
    for (uint32_t u = 0; u < kU; ++u) {
      const uint32_t t = t0 + u * epb;
      if (t >= nb * M) continue;
      const uint32_t el = t / M, i = t - el * M;
      s_imp[i * epb + el] = im[u];
      if (i < s_hdr[el]) {  // i < min(count, M)
        const uint32_t p = lookup_pair(m, ix[u]);
        if (p == fm::kNoPair) s_hdr[3 * epb + el] = 1;
        else s_meta[i * epb + el] = slot_word(m, p, i);
      }
      if (i < s_hdr[epb + el]) {  // previous list
        const uint32_t p = lookup_pair(m, px[u]);
        if (p == fm::kNoPair) s_hdr[3 * epb + el] = 1;
        else s_aux[i * epb + el] = uint8_t(m.pinfo(p) >> 24);
      }
    }
  }
  __syncwarp(wmask);

  if (l < nb) {
    uint32_t flags = kSkipState;
    const uint32_t e = e0 + l;
    if (!run_env(a, f, pl, hot, blk, epb, l, e, flags)) {
      flags = kSkipState;
      a.odd_list[atomicAdd(a.odd_count, 1u)] = e;
    }
    s_flags[l] = flags;
  }
  __syncwarp(wmask);

  // ---- coalesced store: state, accelerations, joint torques and states ----
  for (uint32_t t = l; t < nb * B; t += epb) {
    const uint32_t el = t / B, b = t - el * B, si = b * epb + el;
    const uint32_t fl = s_flags[el];
    if (fl & kSkipState) continue;
    const float4 v1 = s_vel[si];
    if (!(fl & kAccWritten)) {
      const float4 v0 = gvel[t];
      gacc[t] = make_float4((v1.x - v0.x) * a.inv_step, (v1.y - v0.y) * a.inv_step, (v1.z - v0.z) * a.inv_step, 0.0f);
    }
    gpos[t] = s_pos[si];
    gquat[t] = s_quat[si];
    gvel[t] = v1;
    gang[t] = s_ang[si];
  }
  for (uint32_t t = l; t < nb * J; t += epb) {
    const uint32_t el = t / J, j = t - el * J;
    const uint32_t fl = s_flags[el];
    if (fl & kSkipState) continue;
    gjt[t] = s_jt[j * epb + el];
    if (fl & kWriteJointState) {
      gjp[t] = s_jp[j * epb + el];
      gjv[t] = s_jv[j * epb + el];
    }
  }
}

static size_t fast_smem(const StepArgs& args, const FModel& model, int envs_per_block) {
  return size_t(model.hot_bytes) + size_t(fast_plan(args.B, args.J, args.M, model.H).bytes) * envs_per_block;
}

cudaError_t launch_fast_step(const StepArgs& args, const FModel& model, int envs_per_block, cudaStream_t stream) {
  if (args.num_envs == 0) return cudaSuccess;
  if (envs_per_block < 1 || envs_per_block > 32) return cudaErrorInvalidValue;
  const size_t smem = fast_smem(args, model, envs_per_block);
  cudaError_t err = cudaFuncSetAttribute(fast_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  const uint32_t blocks = (args.num_envs + envs_per_block - 1) / envs_per_block;
  fast_step_kernel<<<blocks, envs_per_block, smem, stream>>>(args, model);
  return cudaGetLastError();
}

int fast_max_active_blocks(const StepArgs& args, const FModel& model, int envs_per_block) {
  const size_t smem = fast_smem(args, model, envs_per_block);
  if (cudaFuncSetAttribute(fast_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fast_step_kernel, envs_per_block, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace zb
