// Step kernel with compressed per-environment state, for sm_100a.
//
// One launch runs every substep of one World.step (src/world/world.zig:694-792).  Each
// environment is owned by a group of L lanes (L = 1 or 2) that runs the whole step for
// it in the order the reference's dispatch sequence defines (world.zig:934-1293).  All
// environments of a launch share one model, so a warp executes one coherent instruction
// stream, and the model is read from a per-block shared-memory copy with warp-uniform
// addresses.  With L = 1 a lane steps its environment alone; with L > 1 the lanes split
// the constraints of a colour, the contacts of a level, and the per-body / per-pair loops,
// and meet at __syncwarp on the group mask.
//
// Shared memory holds the environment's bodies, joint torques/states and a compressed
// contact list, laid out [item][environment] so that the groups of a warp touch
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
#include "stage_clock.cuh"
#include "step_kernel.h"
#include "zeno_types.h"

namespace zb {

// ------------------------------------------------------------------------------------
// Shared-memory plan: per-environment byte offsets, each section 16-byte aligned.  The
// block region of a section is (per-env offset) * envs_per_block; element (item, env)
// sits at (item * envs_per_block + env) * element size inside it.
// ------------------------------------------------------------------------------------
struct FPlan {
  uint32_t pos, quat, vel, ang;  // float4 [B]
  uint32_t jt, jp, jv;           // float [J]
  uint32_t imp;                  // float [M]   normal impulse per slot
  uint32_t meta;                 // u32 [M]     slot word (below)
  uint32_t aux;                  // u8 [M]      prev key ranks (substep 0), then the contact schedule
  uint32_t pp, nt;               // float4 [H]  (point, pen), (normal, warm start)
  uint32_t nlh;                  // u8 [H]      list length at the pair's last hit
  uint32_t blev;                 // u8 [B]      (L > 1) contact level per body
  uint32_t lofs;                 // u8 [M + 1]  (L > 1) contact level offsets into the schedule
  uint32_t hdr;                  // u32 [4]     count, prev count, prev-separate, unusable
  uint32_t flags;                // u32
  uint32_t bytes;
};

__host__ __device__ inline uint32_t fa16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline FPlan fast_plan(uint32_t B, uint32_t J, uint32_t M, uint32_t H, uint32_t L) {
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
  p.blev = o, o += L > 1 ? fa16(B) : 0u;
  p.lofs = o, o += L > 1 ? fa16(M + 1) : 0u;
  p.hdr = o, o += 16;
  p.flags = o, o += 16;
  p.bytes = o;
  return p;
}

uint32_t fast_env_smem_bytes(uint32_t B, uint32_t J, uint32_t M, uint32_t H, uint32_t L) {
  return fast_plan(B, J, M, H, L).bytes;
}

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

// 32 bytes (two 16-byte parts) to a 32-byte aligned global address in one 256-bit store.
__device__ __forceinline__ void store32(void* p, uint4 a, uint4 b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// Body state of one environment (stride: environments per block).
struct EnvBodies {
  float4 *p, *q, *v, *w;
  uint32_t st;
  __device__ __forceinline__ float4& pos(uint32_t b) { return p[b * st]; }
  __device__ __forceinline__ float4& quat(uint32_t b) { return q[b * st]; }
  __device__ __forceinline__ float4& vel(uint32_t b) { return v[b * st]; }
  __device__ __forceinline__ float4& ang(uint32_t b) { return w[b * st]; }
};

// The L lanes that own one environment.  Every group of a warp runs the same sequence
// of synchronisations (the model fixes the loop bounds; data-dependent ones run to the
// warp's maximum), so all of them sync and shuffle on one warp-wide mask: __syncwarp with
// a different mask per group costs about 200 cycles on sm_100a, with one mask a few.
template <int L>
struct Group {
  uint32_t lane;  // 0 .. L-1
  unsigned mask;  // the lanes of the warp's active groups
  int src;        // warp lane of the group's lane 0
  __device__ __forceinline__ void sync() const {
    if constexpr (L > 1) __syncwarp(mask);
  }
  __device__ __forceinline__ uint32_t bcast(uint32_t v) const {
    if constexpr (L > 1) return __shfl_sync(mask, v, src);
    return v;
  }
  __device__ __forceinline__ uint64_t or_all(uint64_t v) const {
    if constexpr (L > 1) {
#pragma unroll
      for (int o = 1; o < L; o <<= 1) v |= __shfl_xor_sync(mask, v, o);
    }
    return v;
  }
  __device__ __forceinline__ uint32_t warp_max(uint32_t v) const {
    if constexpr (L > 1) return __reduce_max_sync(mask, v);
    return v;
  }
};

// Narrow phase of hittable pair h on the current poses (the world's narrow-phase mode is
// uniform across the launch; models with GJK pairs, mode 2, never reach this kernel, so
// mode 2 is mode 1 here).
__device__ __forceinline__ bool narrow_h(const ModelS& m, uint32_t h, EnvBodies& S, V3& point, V3& normal,
                                         float& pen) {
  const uint32_t hi = m.hinfo(h);
  const float4 ga = m.hga(h), gb = m.hgb(h);
  const uint32_t ba = (hi >> 16) & 0xFFu, bb = hi >> 24;
  if (m.f.narrow_mode >= 1) {
    const float4 sz = m.hsz(h);
    return narrow_cpu(hi & 0xFFu, (hi >> 8) & 0xFFu, ga, make_float2(sz.x, sz.y), gb, make_float2(sz.z, sz.w),
                      S.pos(ba), S.quat(ba), S.pos(bb), S.quat(bb), point, normal, pen);
  }
  const V3 pa = v3(S.pos(ba)) + v3(ga);
  const V3 pb = v3(S.pos(bb)) + v3(gb);
  return narrow_core(hi & 0xFFu, (hi >> 8) & 0xFFu, pa, pb, ga.w, gb.w, m.hhl(h), v3(m.hcax(h)), point, normal, pen);
}

enum : uint32_t {
  kSkipState = 1u,        // leave body / joint state untouched (handed over, or outside the step mask)
  kWriteJointState = 2u,  // publish joint positions / velocities
  kAccWritten = 4u,       // accelerations already written (auto-reset replaced the velocities)
};
// Deferred write-back of an environment whose sort moved slots (header word 2 after the
// step: n_fin | n0 << 8 | these bits); the block writes its records once every group is done.
enum : uint32_t {
  kWbDeferred = 1u << 16,
  kWbPublish = 1u << 17,  // into the contacts buffer (else into the step_subset cache)
};
constexpr uint32_t kWbParts = 12;  // 16-byte record parts staged per thread

// Everything a group does for its environment between the cooperative load and store.
// The block has already handed over the environments this kernel cannot represent.
template <int L, bool C>
__device__ __forceinline__ void run_env(const StepArgs& a, const FModel& f, const FPlan& pl, const unsigned char* hot,
                                        unsigned char* blk, uint32_t ne, uint32_t g, const Group<L>& G, uint32_t e,
                                        uint32_t& flags_out, StageClock<C>& clk) {
  clk.mark(kStPrologue);
  const ModelS m{hot, f};
  const uint32_t B = a.B, J = a.J, A = a.A, M = a.M, H = f.H, P = f.P;
  const uint32_t lane = G.lane;
  EnvBodies S{reinterpret_cast<float4*>(blk + pl.pos * ne) + g, reinterpret_cast<float4*>(blk + pl.quat * ne) + g,
              reinterpret_cast<float4*>(blk + pl.vel * ne) + g, reinterpret_cast<float4*>(blk + pl.ang * ne) + g, ne};
  // pose before integration, read back by the velocity update: an L2-resident scratch,
  // [body][pos, quat][env] so that a warp's accesses are contiguous
  const size_t E = a.num_envs;
  float4* ppos = a.pose_scratch + e;
  float4* pquat = a.pose_scratch + E + e;
  const size_t pst = 2 * E;
  float* jt = reinterpret_cast<float*>(blk + pl.jt * ne) + g;
  float* jp = reinterpret_cast<float*>(blk + pl.jp * ne) + g;
  float* jv = reinterpret_cast<float*>(blk + pl.jv * ne) + g;
  float* imp = reinterpret_cast<float*>(blk + pl.imp * ne) + g;
  uint32_t* meta = reinterpret_cast<uint32_t*>(blk + pl.meta * ne) + g;
  uint8_t* aux = blk + pl.aux * ne + g;
  float4* pp = reinterpret_cast<float4*>(blk + pl.pp * ne) + g;
  float4* nt = reinterpret_cast<float4*>(blk + pl.nt * ne) + g;
  uint8_t* nlh = blk + pl.nlh * ne + g;
  uint8_t* blev = blk + pl.blev * ne + g;
  uint8_t* lofs = blk + pl.lofs * ne + g;
  uint32_t* hdr = reinterpret_cast<uint32_t*>(blk + pl.hdr * ne) + g;

  // ---------------- contact list of the previous step ----------------
  // loaded by the block: slot words, impulses, previous-list key ranks
  uint32_t count = hdr[0];
  const uint32_t prev_count0 = hdr[ne];
  const bool sep = hdr[2 * ne] != 0;
  const uint32_t n0 = count < M ? count : M;
  Contact* gc = a.contacts + size_t(e) * M;
  const Contact* gprev = sep ? a.prev_contacts + size_t(e) * M : gc;
  const uint32_t n_prev0 = prev_count0 < M ? prev_count0 : M;
  for (uint32_t h = lane; h < H; h += L) nlh[h * ne] = 0;

  const float dt = a.dt, inv_dt = a.inv_dt;
  const V3 grav{a.gravity[0], a.gravity[1], a.gravity[2]};
  const float* act = a.actions + size_t(e) * A;
  // apply_actions (196-229): the torques are the same in every substep; actuators that
  // share a joint are applied in index order by one lane
  if (a.substeps > 0) {
    const uint32_t k0 = a.actuators_unique ? lane : (lane == 0 ? 0u : A);
    const uint32_t ks = a.actuators_unique ? uint32_t(L) : 1u;
    for (uint32_t k = k0; k < A; k += ks) {
      const float tq = clampf(act[k], f.a_cmin[k], f.a_cmax[k]) * f.a_gear[k];
      jt[f.a_joint[k] * ne] = clampf(tq, f.a_fmin[k], f.a_fmax[k]);
    }
  }
  G.sync();

  uint64_t prev_hit = 0;
  uint32_t n_prev = n_prev0;
  uint32_t nh = 0, nlev = 0, nlev_w = 0;  // contact schedule: hit slots, levels (L > 1), warp max
  bool moved = false;  // (lane 0) did sorting move a slot away from its original position
  for (uint32_t s = 0; s < a.substeps; ++s) {
    // ---- kinematic bodies (update_kinematic 304-339; massless, so no gravity wrench) ----
    for (uint32_t b = lane; b < B; b += L) {
      if ((m.body(b) & 0xFFu) != 1u) continue;
      S.pos(b) = with_w(madd(v3(S.vel(b)), dt, v3(S.pos(b))), 0.0f);
      const float4 q = S.quat(b);
      S.quat(b) = qnormalize(qmadd(qmul_v((v3(S.ang(b)) * dt) * 0.5f, q), 1.0f, q));
    }
    G.sync();
    clk.mark(kStActions);
    // ---- wrench (compute_forces 345-388, apply_joint_forces 122-190) and semi-implicit
    //      Euler (save_prev_state 1900-1913, integrate 394-462), children first: a body's
    //      wrench reads only its own and its parent's orientation, neither yet integrated.
    //      Four bodies per round: all their wrenches first, then their integration.
    for (uint32_t hi_b = B; hi_b > 0;) {
      constexpr int kC = 4 / L;  // bodies per lane per round
      const uint32_t nc = hi_b < 4u ? hi_b : 4u;
      V3 F[kC], T[kC];
      float4 q[kC], x[kC], v0[kC], w0[kC];
#pragma unroll
      for (int c = 0; c < kC; ++c) {
        const uint32_t idx = uint32_t(c) * L + lane;
        if (idx >= nc) continue;
        const uint32_t b = hi_b - 1 - idx;
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
          const float tau = jt[j * ne];
          if (fabsf(tau) < 1e-6f) continue;
          const uint32_t ji = m.jinfo(j);
          const V3 fj = rotate(v3(m.jaxis(j)), S.quat((ji >> 8) & 0xFFu)) * tau;
          if ((ji & 0xFFu) == 2u) F[c] = (ent & 0x80u) ? F[c] - fj : F[c] + fj;
          else T[c] = (ent & 0x80u) ? T[c] - fj : T[c] + fj;
        }
      }
      G.sync();
#pragma unroll
      for (int c = 0; c < kC; ++c) {
        const uint32_t idx = uint32_t(c) * L + lane;
        if (idx >= nc) continue;
        const uint32_t b = hi_b - 1 - idx;
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
      G.sync();
      hi_b -= nc;
    }
    clk.mark(kStIntegrate);
    // ---- broad phase (broad_phase 468-533): candidates in emission order ----
    const uint32_t n_old = count < M ? count : M;
    uint32_t run_first = 0, run_last = 0;  // key ranks of the first and last appended slots
    bool run_sorted = true;  // the appended slots are in key order (as emission order gives
                             // when geoms are numbered in body order)
    for (uint32_t p0 = 0; p0 < P; p0 += 64) {
      const uint32_t pn = P - p0 < 64u ? P - p0 : 64u;
      uint64_t pass = 0;
      // branch-free, so that the loads of several candidates are in flight together: the
      // distance test is evaluated for plane pairs too and discarded (they always pass)
#pragma unroll 4
      for (uint32_t i = lane; i < pn; i += L) {
        const uint32_t p = p0 + i;
        const uint32_t pb = m.pbody(p);
        const uint32_t pi = m.pinfo(p);
        const V3 pa = v3(S.pos(pb & 0xFFu)) + v3(m.gps(pi & 0xFFu));
        const V3 pc = v3(S.pos((pb >> 8) & 0xFFu)) + v3(m.gps((pi >> 8) & 0xFFu));
        const V3 d = pc - pa;
        const bool ok = ((pb >> 16) != 0u) | !(dot(d, d) >= m.pmd2(p));
        pass |= uint64_t(ok) << i;
      }
      pass = G.or_all(pass);
      if (count >= M) {  // the list is frozen: only the counter advances
        count += uint32_t(__popcll(pass));
        continue;
      }
      while (pass) {
        const uint32_t i = uint32_t(__ffsll(pass)) - 1u;
        pass &= pass - 1;
        if (count < M) {
          const uint32_t w = slot_word(m, p0 + i, count);
          if (count == n_old) run_first = sw_rank(w);
          run_sorted &= sw_rank(w) >= run_last;
          run_last = sw_rank(w);
          if (lane == 0) meta[count * ne] = w;
        }
        ++count;
      }
    }
    const uint32_t n = count < M ? count : M;
    clk.mark(kStBroad);
    // ---- stable sort by key (sort_contacts 711-745) ----
    // The stored slots [0, n_old) are sorted.  When the appended run [n_old, n) is sorted
    // too, the stable sort is a merge: an old slot i lands at i + #(appended with a
    // smaller key), an appended slot q at #(old with a key <= its key) + (q - n_old).
    // Nothing moves when the run starts at or above the last old key (the first substep
    // after a reset, a list that only grows at its end).  Lists that do move are merged
    // by the whole warp, one list at a time: each active lane takes up to three slots,
    // finds their places by binary search in the other run, and all lanes scatter after a
    // warp barrier (so the list needs no scratch).  Unsorted runs, and warps with too few
    // active lanes for the list, take the serial insertion sort below.
    bool need_merge = false;
    if (run_sorted && n > n_old && n_old > 0) need_merge = run_first < sw_rank(meta[(n_old - 1) * ne]);
    const uint32_t nact = __popc(G.mask);
    const bool coop = need_merge && 3u * nact >= M;
    uint32_t todo = __ballot_sync(G.mask, coop && lane == 0);
    if (todo) {  // warp-uniform
      const uint32_t wl = threadIdx.x & 31u;
      const uint32_t idx = __popc(G.mask & ((1u << wl) - 1u));
      const uint32_t nbits = 32u - __clz(M);  // binary-search rounds for ranges of up to M slots
      __syncwarp(G.mask);  // the appended slot words of every group are in place
      do {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const uint32_t gs = ((threadIdx.x & ~31u) + uint32_t(src)) / L;
        const uint32_t so = __shfl_sync(G.mask, n_old, src), sn = __shfl_sync(G.mask, n, src);
        uint32_t* mt = reinterpret_cast<uint32_t*>(blk + pl.meta * ne) + gs;
        float* ip = reinterpret_cast<float*>(blk + pl.imp * ne) + gs;
        uint32_t w[3], lo[3], hi[3], thr[3];
        float x[3];
#pragma unroll
        for (uint32_t u = 0; u < 3; ++u) {
          const uint32_t sl = idx + u * nact;
          const bool have = sl < sn;
          w[u] = have ? mt[sl * ne] : 0u;
          x[u] = have ? ip[sl * ne] : 0.0f;
          // old slot: count appended slots with rank < its rank; appended slot: count
          // old slots with rank <= its rank (rank < rank + 1)
          const bool old_slot = sl < so;
          lo[u] = have ? (old_slot ? so : 0u) : 0u;
          hi[u] = have ? (old_slot ? sn : so) : 0u;
          thr[u] = sw_rank(w[u]) + (old_slot ? 0u : 1u);
        }
        for (uint32_t it = 0; it < nbits; ++it) {
#pragma unroll
          for (uint32_t u = 0; u < 3; ++u) {
            const uint32_t mid = (lo[u] + hi[u]) >> 1;
            const uint32_t r = sw_rank(mt[(mid < M ? mid : M - 1u) * ne]);
            if (lo[u] < hi[u]) {
              if (r < thr[u]) lo[u] = mid + 1u;
              else hi[u] = mid;
            }
          }
        }
        __syncwarp(G.mask);
#pragma unroll
        for (uint32_t u = 0; u < 3; ++u) {
          const uint32_t sl = idx + u * nact;
          if (sl >= sn) continue;
          const uint32_t pos = sl < so ? sl + (lo[u] - so) : lo[u] + (sl - so);
          mt[pos * ne] = w[u];
          ip[pos * ne] = x[u];
        }
        __syncwarp(G.mask);
      } while (todo);
    }
    moved |= coop;
    // Serial insertion: each insertion shifts the larger-keyed slots up by one; the slot
    // words and impulses are read four at a time ahead of the comparisons, so four shifts
    // share one shared-memory latency.
    if (lane == 0 && !coop && n > n_old && (need_merge || !run_sorted)) {
      for (uint32_t q = n_old; q < n; ++q) {
        const uint32_t w = meta[q * ne];
        const float x = imp[q * ne];
        const uint32_t rk = sw_rank(w);
        uint32_t r = q;
        while (r > 0) {
          uint32_t mw[4];
          float mi[4];
#pragma unroll
          for (uint32_t u = 0; u < 4; ++u) {
            const uint32_t k = r > u ? r - 1 - u : 0u;
            mw[u] = meta[k * ne];
            mi[u] = imp[k * ne];
          }
          uint32_t shifted = 0;
          bool stop = false;
#pragma unroll
          for (uint32_t u = 0; u < 4; ++u) {
            if (stop || u >= r || sw_rank(mw[u]) <= rk) {
              stop = true;
              continue;
            }
            meta[(r - u) * ne] = mw[u];
            imp[(r - u) * ne] = mi[u];
            ++shifted;
          }
          r -= shifted;
          if (stop) break;
        }
        moved |= r != q;
        meta[r * ne] = w;
        imp[r * ne] = x;
      }
    }
    G.sync();
    clk.mark(kStSort);
    // ---- narrow phase + warm start (narrow_phase 751-894, match_cached_contacts
    //      1483-1544), once per hittable pair.  The match reads the previous substep's
    //      points of the pairs with this pair's key.  When no two hittable pairs share a
    //      key, that is only this pair's own point, so one pass matches and then stores;
    //      otherwise this pass only matches and a second one stores.
    const bool one_pass = m.f.hit_keys_unique != 0;
    uint64_t hit_now = 0;
    // the warm-start match and the stores of hittable pair h, given its narrow-phase result
    auto narrow_finish = [&](uint32_t h, bool hit, V3 point, V3 normal, float pen) {
      if (!hit) {
        if (one_pass) reinterpret_cast<float*>(&pp[h * ne])[3] = -1.0f;
        return;
      }
      const uint32_t rank = m.pinfo(m.hpair(h)) >> 24;
      float best = 0.04f;
      int js = -1;
      float val = 0.0f;
      if (s == 0) {
        uint32_t lo = 0, hi = n_prev;  // first previous slot with key >= this key
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (aux[mid * ne] < rank) lo = mid + 1;
          else hi = mid;
        }
        for (uint32_t j = lo; j < n_prev && aux[j * ne] == rank; ++j) {
          const float4 q = *reinterpret_cast<const float4*>(gprev[j].position_pen);
          if (q.w < 0.0f) continue;
          const V3 d = xyz(q) - point;
          const float dsq = dot(d, d);
          if (dsq < best) {
            best = dsq;
            js = int(j);
          }
        }
        // (tangent impulses of valid previous slots are zero: the block checked)
        if (js >= 0) val = gprev[js].impulses[0] * 0.8f;
      } else {
        uint32_t lo = 0, hi = n;
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (sw_rank(meta[mid * ne]) < rank) lo = mid + 1;
          else hi = mid;
        }
        for (uint32_t j = lo; j < n; ++j) {
          const uint32_t w = meta[j * ne];
          if (sw_rank(w) != rank) break;
          if (sw_origin(w) >= n_prev) continue;  // appended in this substep
          const uint32_t hj = sw_hit(w);
          if (hj == fm::kNoHit || !((prev_hit >> hj) & 1ull)) continue;
          const V3 d = xyz(pp[hj * ne]) - point;
          const float dsq = dot(d, d);
          if (dsq < best) {
            best = dsq;
            js = int(j);
          }
        }
        if (js >= 0) val = imp[uint32_t(js) * ne] * 0.8f;
      }
      if (one_pass) {
        pp[h * ne] = with_w(point, pen);
        nt[h * ne] = with_w(normal, val);
        nlh[h * ne] = uint8_t(n);
        hit_now |= 1ull << h;
      } else {
        reinterpret_cast<float*>(&nt[h * ne])[3] = val;
      }
    };
    // Capsule-plane pairs (the first n_capsule_plane hittables; the reference GPU narrow
    // phase only): four per lane and round, their tests first -- independent and
    // branch-free, so the loads and arithmetic of the four overlap -- then each one's match
    // and stores in turn (one copy of that code; the results move down the registers).
    uint32_t hc = 0;
    if (m.f.narrow_mode == 0) {
      hc = m.f.n_capsule_plane;
      for (uint32_t h0 = lane; h0 < hc; h0 += 4 * L) {
        bool hit[4];
        V3 pt[4], nm[4];
        float pe[4];
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) {
          const uint32_t h = h0 + u * L < hc ? h0 + u * L : h0;  // (clamped: a valid pair, result unused)
          const uint32_t hi = m.hinfo(h);
          const bool ca = (hi & 0xFFu) == 1u;  // the capsule is geom A
          const float4 g = ca ? m.hga(h) : m.hgb(h);
          const V3 cpos = v3(S.pos(ca ? (hi >> 16) & 0xFFu : hi >> 24)) + v3(g);
          hit[u] = capsule_plane(cpos, g.w, m.hhl(h), v3(m.hcax(h)), ca, pt[u], nm[u], pe[u]);
        }
#pragma unroll 1
        for (uint32_t u = 0; u < 4 && h0 + u * L < hc; ++u) {
          narrow_finish(h0 + u * L, hit[0], pt[0], nm[0], pe[0]);
          hit[0] = hit[1], pt[0] = pt[1], nm[0] = nm[1], pe[0] = pe[1];
          hit[1] = hit[2], pt[1] = pt[2], nm[1] = nm[2], pe[1] = pe[2];
          hit[2] = hit[3], pt[2] = pt[3], nm[2] = nm[3], pe[2] = pe[3];
        }
      }
    }
    for (uint32_t h = hc + lane; h < H; h += L) {
      V3 point, normal;
      float pen;
      const bool hit = narrow_h(m, h, S, point, normal, pen);
      narrow_finish(h, hit, point, normal, pen);
    }
    G.sync();
    for (uint32_t h = lane; h < H && !one_pass; h += L) {
      V3 point, normal;
      float pen;
      if (narrow_h(m, h, S, point, normal, pen)) {
        pp[h * ne] = with_w(point, pen);
        const float warm = nt[h * ne].w;
        nt[h * ne] = with_w(normal, warm);
        nlh[h * ne] = uint8_t(n);
        hit_now |= 1ull << h;
      } else {
        reinterpret_cast<float*>(&pp[h * ne])[3] = -1.0f;
      }
    }
    hit_now = G.or_all(hit_now);
    G.sync();
    clk.mark(kStNarrow);
    // contact schedule.  L = 1: the hit slots in slot order.  L > 1: the hit slots by
    // level -- a slot's level is one more than the highest level of an earlier hit slot
    // sharing a dynamic body -- stable within a level; solving level by level, a level's
    // slots in parallel, equals solving the slots one after another in slot order.  The
    // schedule depends only on the slot list and the set of hit pairs, so it is kept from
    // the previous substep when neither changed (aux holds it from substep 1 on).
    const bool reuse = s > 0 && n == n_prev && hit_now == prev_hit;
    if constexpr (L == 1) {
      if (!reuse) {  // eight slot words per shared-memory round trip
        nh = 0;
        for (uint32_t i0 = 0; i0 < n; i0 += 8) {
          uint32_t w8[8];
#pragma unroll
          for (uint32_t u = 0; u < 8; ++u) w8[u] = i0 + u < n ? meta[(i0 + u) * ne] : (fm::kNoHit << 16);
#pragma unroll
          for (uint32_t u = 0; u < 8; ++u) {
            const uint32_t hh = sw_hit(w8[u]);
            if (hh != fm::kNoHit && ((hit_now >> hh) & 1ull)) aux[nh++ * ne] = uint8_t(i0 + u);
          }
        }
      }
    } else {
      if (lane == 0 && !reuse) {
        nlev = 0;
        // the hit slots as a bit mask (eight slot words per shared-memory round trip), so
        // that the two passes below visit only them (lists of up to 64 slots)
        uint64_t hs = ~0ull;
        if (n <= 64) {
          hs = 0;
          for (uint32_t i0 = 0; i0 < n; i0 += 8) {
            uint32_t w8[8];
#pragma unroll
            for (uint32_t u = 0; u < 8; ++u) w8[u] = i0 + u < n ? meta[(i0 + u) * ne] : (fm::kNoHit << 16);
#pragma unroll
            for (uint32_t u = 0; u < 8; ++u) {
              const uint32_t hh = sw_hit(w8[u]);
              if (hh != fm::kNoHit && ((hit_now >> hh) & 1ull)) hs |= 1ull << (i0 + u);
            }
          }
        }
        for (int pass = 0; pass < 2; ++pass) {  // pass 0 counts per level, pass 1 places
          for (uint32_t b = 0; b < B; ++b) blev[b * ne] = 0;
          if (pass == 1) {
            uint32_t acc = 0;
            for (uint32_t v = 0; v <= nlev; ++v) {
              const uint32_t c = lofs[v * ne];
              lofs[v * ne] = uint8_t(acc);
              acc += c;
            }
          } else {
            for (uint32_t v = 0; v <= n; ++v) lofs[v * ne] = 0;
          }
          uint64_t todo = hs;
          for (uint32_t i = 0; i < n; ++i) {
            if (n <= 64) {  // next hit slot from the mask
              if (!todo) break;
              i = uint32_t(__ffsll(todo)) - 1u;
              todo &= todo - 1;
            }
            const uint32_t hh = sw_hit(meta[i * ne]);
            if (hh == fm::kNoHit || !((hit_now >> hh) & 1ull)) continue;
            const uint32_t hi = m.hinfo(hh);
            const uint32_t ba = (hi >> 16) & 0xFFu, bb = hi >> 24;
            const bool da = m.imi(ba).x > 1e-8f, db = m.imi(bb).x > 1e-8f;
            uint32_t lv = 0;
            if (da && blev[ba * ne] > lv) lv = blev[ba * ne];
            if (db && blev[bb * ne] > lv) lv = blev[bb * ne];
            if (da) blev[ba * ne] = uint8_t(lv + 1);
            if (db) blev[bb * ne] = uint8_t(lv + 1);
            if (pass == 0) {
              lofs[lv * ne] = uint8_t(lofs[lv * ne] + 1);
              if (lv + 1 > nlev) nlev = lv + 1;
            } else {
              aux[lofs[lv * ne] * ne] = uint8_t(i);
              lofs[lv * ne] = uint8_t(lofs[lv * ne] + 1);
            }
          }
        }
        // lofs[v] now holds the end of level v: shift to starts with lofs[nlev] = end
        for (uint32_t v = nlev; v > 0; --v) lofs[v * ne] = lofs[(v - 1) * ne];
        lofs[0] = 0;
      }
      nlev = G.bcast(nlev);
      nlev_w = G.warp_max(nlev);  // every group of the warp runs as many levels (and syncs)
      G.sync();
      nh = lofs[nlev * ne];
    }
    // slot impulses of the hit slots (narrow zeroes them, a match warm-starts them); four
    // slots' dependent loads (schedule -> slot word -> pair impulse) per round
    for (uint32_t v0 = lane; v0 < nh; v0 += 4 * L) {
      uint32_t i4[4];
      float w4[4];
#pragma unroll
      for (uint32_t u = 0; u < 4; ++u) i4[u] = v0 + u * L < nh ? aux[(v0 + u * L) * ne] : 0u;
#pragma unroll
      for (uint32_t u = 0; u < 4; ++u) {  // (listed slots are hit, so their pair index is valid)
        const uint32_t hh = v0 + u * L < nh ? sw_hit(meta[i4[u] * ne]) : 0u;
        w4[u] = nt[hh * ne].w;
      }
#pragma unroll
      for (uint32_t u = 0; u < 4; ++u)
        if (v0 + u * L < nh) imp[i4[u] * ne] = w4[u];
    }
    clk.mark(kStSchedule);
    // ---- XPBD joints (solve_joints 909-1399): with one lane as the model's hinge groups;
    //      with two as the groups by dependency level, or (models whose constraint indices
    //      do not fit the group words) colour by colour, as runs of one type, a run's
    //      constraints (one colour: disjoint bodies) split across the lanes.
    if constexpr (L == 1) {  // one lane: the sweep as hinge groups (hinge_groups, model.cpp)
      for (uint32_t it = 0; it < a.iterations; ++it)
        for (uint32_t g = 0; g < f.num_groups; ++g) {
          const uint32_t gw = m.group(g);
          const uint32_t k0 = gw & 0xFFu, kind = gw >> 24;
          if (kind != 0u) {
            const uint32_t k2 = kind == 2u ? (gw >> 16) & 0xFFu : k0;
            solve_hinge(m, m.constraint(k0), m.constraint((gw >> 8) & 0xFFu), m.constraint(k2), kind == 2u, S);
            continue;
          }
          const ConstraintV c = m.constraint(k0);
          switch (c.type) {
            case 2: solve_typed<2>(m, c, S); break;
            case 3: solve_typed<3>(m, c, S); break;
            case 4: solve_typed<4>(m, c, S); break;
            case 5: solve_typed<5>(m, c, S); break;
            case 7: solve_typed<7>(m, c, S); break;
            case 10: solve_typed<10>(m, c, S); break;
            default: break;
          }
        }
    } else if (f.num_glv > 0) {  // several lanes: hinge groups level by level, split across the lanes
      for (uint32_t it = 0; it < a.iterations; ++it)
        for (uint32_t v = 0; v < f.num_glv; ++v) {
          const uint32_t g1 = m.glv(v + 1);
          for (uint32_t g = m.glv(v) + lane; g < g1; g += L) {
            const uint32_t gw = m.gword(g);
            const uint32_t k0 = gw & 0xFFu, kind = gw >> 24;
            if (kind != 0u) {
              const uint32_t k2 = kind == 2u ? (gw >> 16) & 0xFFu : k0;
              solve_hinge(m, m.constraint(k0), m.constraint((gw >> 8) & 0xFFu), m.constraint(k2), kind == 2u, S);
              continue;
            }
            const ConstraintV c = m.constraint(k0);
            switch (c.type) {
              case 2: solve_typed<2>(m, c, S); break;
              case 3: solve_typed<3>(m, c, S); break;
              case 4: solve_typed<4>(m, c, S); break;
              case 5: solve_typed<5>(m, c, S); break;
              case 7: solve_typed<7>(m, c, S); break;
              case 10: solve_typed<10>(m, c, S); break;
              default: break;
            }
          }
          G.sync();
        }
    } else
    for (uint32_t it = 0; it < a.iterations; ++it)
      for (uint32_t r = 0; r < f.num_runs; ++r) {
        const uint32_t rw = m.run(r);
        const uint32_t k0 = (rw & 0xFFFu) + lane, k1 = (rw & 0xFFFu) + ((rw >> 12) & 0xFFFu);
        switch (rw >> 24) {
          case 2: for (uint32_t k = k0; k < k1; k += L) solve_typed<2>(m, m.constraint(k), S); break;
          case 3: for (uint32_t k = k0; k < k1; k += L) solve_typed<3>(m, m.constraint(k), S); break;
          case 4: for (uint32_t k = k0; k < k1; k += L) solve_typed<4>(m, m.constraint(k), S); break;
          case 5: for (uint32_t k = k0; k < k1; k += L) solve_typed<5>(m, m.constraint(k), S); break;
          case 7: for (uint32_t k = k0; k < k1; k += L) solve_typed<7>(m, m.constraint(k), S); break;
          case 10: for (uint32_t k = k0; k < k1; k += L) solve_typed<10>(m, m.constraint(k), S); break;
          default: break;
        }
        G.sync();
      }
    clk.mark(kStJoints);
    // ---- contacts (solve_contacts 1644-1793) ----
    auto contact = [&](uint32_t i) {
      const uint32_t hh = sw_hit(meta[i * ne]);
      const uint32_t hi = m.hinfo(hh);
      const float4 nn = nt[hh * ne];
      float jx = imp[i * ne];
      solve_contact(m, pp[hh * ne], make_float4(nn.x, nn.y, nn.z, m.hfr(hh)), jx, a.restitution, (hi >> 16) & 0xFFu,
                    hi >> 24, S, dt, a.baumgarte, a.slop);
      imp[i * ne] = jx;
    };
    if constexpr (L == 1) {
      for (uint32_t it = 0; it < a.iterations; ++it)
        for (uint32_t v = 0; v < nh; ++v) contact(aux[v * ne]);
    } else {
      for (uint32_t it = 0; it < a.iterations; ++it)
        for (uint32_t lv = 0; lv < nlev_w; ++lv) {
          const uint32_t v0 = lv < nlev ? lofs[lv * ne] : 0u, v1 = lv < nlev ? lofs[(lv + 1) * ne] : 0u;
          for (uint32_t v = v0 + lane; v < v1; v += L) contact(aux[v * ne]);
          G.sync();
        }
    }
    clk.mark(kStContacts);
    // ---- velocities from the position change (xpbd_update_velocities 1922-1961); the
    //      saved poses (L2 scratch) of four bodies per round are loaded before any is used ----
    constexpr uint32_t kV = 4 / L;  // bodies per lane per round
    for (uint32_t b0 = lane; b0 < B; b0 += kV * L) {
      float4 p0[kV], q0[kV];
#pragma unroll
      for (uint32_t u = 0; u < kV; ++u) {
        const uint32_t b = b0 + u * L;
        if (b < B) p0[u] = ppos[b * pst], q0[u] = pquat[b * pst];
      }
#pragma unroll
      for (uint32_t u = 0; u < kV; ++u) {
        const uint32_t b = b0 + u * L;
        if (b >= B || m.imi(b).x < 1e-8f) continue;
        S.vel(b) = with_w((v3(S.pos(b)) - v3(p0[u])) * inv_dt, 0.0f);
        float4 dq = qmul(S.quat(b), qconj(q0[u]));
        if (dq.w < 0.0f) dq = qneg(dq);
        S.ang(b) = with_w((xyz(dq) * 2.0f) * inv_dt, 0.0f);
      }
    }
    G.sync();
    clk.mark(kStVelocities);
    prev_hit = hit_now;
    n_prev = n;
  }
  moved = G.bcast(moved ? 1u : 0u) != 0;

  // ---------------- joint states and sensors from the final substep ----------------
  uint32_t flags = 0;
  const bool stepped = a.substeps > 0;
  const bool publish = a.step_mask == nullptr || a.step_mask[e] != 0;
  if (stepped) {
    for (uint32_t j = lane; j < J; j += L) {  // update_joint_states 1550-1638
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
      jp[j * ne] = p;
      jv[j * ne] = v;
    }
    G.sync();
    if (publish) {  // read_sensors 1799-1893
      float* gobs = a.obs + size_t(e) * a.obs_dim;
      for (uint32_t si = lane; si < a.S; si += L) {
        const uint32_t sinfo = f.s_info[si];
        const uint32_t o = (sinfo >> 8) & 0xFFu;
        float* out = gobs + (sinfo >> 16);
        switch (sinfo & 0xFFu) {
          case 0: out[0] = jp[o * ne]; break;
          case 1: out[0] = jv[o * ne]; break;
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

    clk.mark(kStJointState);
    // ---------------- contact slots back to memory ----------------
    // A slot whose pair made contact while the slot was in the list carries that pair's
    // last contact; any other slot keeps the record stored at its original position,
    // marked invalid.  When sorting moved slots, the in-place write follows the
    // permutation's cycles (one lane) so that no record is overwritten before it is read.
    // Environments whose sort moved slots and whose records fit the block's staging
    // registers are written by the whole block after every group is done
    // (write_back_moved: all reads first, then all writes); the rest here.
    const uint32_t n_fin = count < M ? count : M;
    Contact* dst = publish ? gc : a.prev_contacts + size_t(e) * M;
    const bool inplace = publish;
    const bool defer = moved && 4u * n_fin <= kWbParts * ne * uint32_t(L);
    if (defer && lane == 0) hdr[2 * ne] = n_fin | (n0 << 8) | kWbDeferred | (publish ? kWbPublish : 0u);
    if (inplace && !moved) {
      // every slot is at its original position: the records are independent, so four
      // slots' shared-memory reads are in flight together (no visited marks needed)
      for (uint32_t j0 = lane; j0 < n_fin; j0 += 4 * L) {
        uint32_t w4[4], pi4[4], pb4[4];
        bool hit4[4];
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) w4[u] = j0 + u * L < n_fin ? meta[(j0 + u * L) * ne] : (fm::kNoHit << 16);
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) {
          const uint32_t hh = sw_hit(w4[u]);
          pi4[u] = m.pinfo(sw_pair(w4[u]));
          pb4[u] = m.pbody(sw_pair(w4[u]));
          hit4[u] = hh != fm::kNoHit && sw_origin(w4[u]) < nlh[(hh != fm::kNoHit ? hh : 0u) * ne];
        }
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) {
          const uint32_t j = j0 + u * L;
          if (j >= n_fin) continue;
          const uint32_t o = sw_origin(w4[u]), hh = sw_hit(w4[u]);
          const uint4 idx = make_uint4(pb4[u] & 0xFFu, (pb4[u] >> 8) & 0xFFu, pi4[u] & 0xFFu, (pi4[u] >> 8) & 0xFFu);
          uint4* out = reinterpret_cast<uint4*>(dst + j);
          if (hit4[u]) {
            const float4 nn = nt[hh * ne];
            const float4 nf = make_float4(nn.x, nn.y, nn.z, m.hfr(hh));
            const uint4 p0 = *reinterpret_cast<const uint4*>(&pp[hh * ne]), p1 = *reinterpret_cast<const uint4*>(&nf);
            const float4 im = make_float4(imp[j * ne], 0.0f, 0.0f, a.restitution);
            const uint4 p3 = *reinterpret_cast<const uint4*>(&im);
            if constexpr (L == 1) {
              store32(out, p0, p1);
              if (o < n0) out[3] = p3;
              else store32(out + 2, idx, p3);
            } else {
              out[0] = p0;
              out[1] = p1;
              if (o >= n0) out[2] = idx;
              out[3] = p3;
            }
          } else {
            reinterpret_cast<float*>(out)[3] = -1.0f;
            if (o >= n0) out[2] = idx;  // a slot loaded at this position keeps its stored tuple
          }
        }
      }
    }
    const uint32_t i0 = (defer || (inplace && !moved)) ? n_fin : (moved ? (lane == 0 ? 0u : n_fin) : lane);
    const uint32_t istep = moved ? 1u : uint32_t(L);
    for (uint32_t i = i0; i < n_fin; i += istep) {
      if (meta[i * ne] & kVisited) continue;
      uint4 saved[4];
      const uint32_t oi = sw_origin(meta[i * ne]);
      const bool cycle = inplace && oi != i;
      if (cycle)
        for (int c = 0; c < 4; ++c) saved[c] = reinterpret_cast<const uint4*>(gc + i)[c];
      uint32_t j = i;
      for (uint32_t guard = 0; guard < n_fin; ++guard) {
        const uint32_t w = meta[j * ne];
        meta[j * ne] = w | kVisited;
        const uint32_t p = sw_pair(w), o = sw_origin(w), hh = sw_hit(w);
        const uint32_t pi = m.pinfo(p), pbody = m.pbody(p);
        const uint4 idx = make_uint4(pbody & 0xFFu, (pbody >> 8) & 0xFFu, pi & 0xFFu, (pi >> 8) & 0xFFu);
        uint4* out = reinterpret_cast<uint4*>(dst + j);
        if (hh != fm::kNoHit && o < nlh[hh * ne]) {
          // a slot loaded at this position keeps its stored tuple (the loader matched it
          // exactly), so then only the impulses follow the point and normal.  One lane:
          // 256-bit stores (with two lanes their operands spill registers).
          const float4 nn = nt[hh * ne];
          const float4 nf = make_float4(nn.x, nn.y, nn.z, m.hfr(hh));
          const uint4 p0 = *reinterpret_cast<const uint4*>(&pp[hh * ne]), p1 = *reinterpret_cast<const uint4*>(&nf);
          const float4 im = make_float4(imp[j * ne], 0.0f, 0.0f, a.restitution);
          const uint4 p3 = *reinterpret_cast<const uint4*>(&im);
          const bool same_tuple = inplace && o == j && o < n0;
          if constexpr (L == 1) {
            store32(out, p0, p1);
            if (same_tuple) out[3] = p3;
            else store32(out + 2, idx, p3);
          } else {
            out[0] = p0;
            out[1] = p1;
            if (!same_tuple) out[2] = idx;
            out[3] = p3;
          }
        } else if (inplace && o == j) {
          reinterpret_cast<float*>(out)[3] = -1.0f;
          if (o >= n0) out[2] = idx;  // a slot loaded at this position keeps its stored tuple
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

  // ---------------- caches, counters, task extension (one lane) ----------------
  G.sync();
  clk.mark(kStWriteBack);
  if (!publish) {
    // step_subset: an env outside the mask keeps its public state, but the reference
    // still advanced its contact cache (world.zig:833-929 restores only public buffers).
    if (stepped && lane == 0) {
      a.prev_counts[e] = count;
      a.prev_sep[e] = 1;
    }
    flags_out = flags | kSkipState;
    clk.mark(kStTask);
    return;
  }
  if (stepped) flags |= kWriteJointState;
  if (lane == 0) {
    uint32_t count_out = count;
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
          jp[j * ne] = t[16 * B + j];
          jv[j * ne] = t[16 * B + J + j];
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
            const V3 hv = ax * div_(0.5f * th, al);
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
  }
  flags_out = flags;
  clk.mark(kStTask);
}

// The second half of a 64-byte contact record (indices, impulses: one 32-byte sector) in
// one 256-bit load; records are 64-byte aligned, so the address is 32-byte aligned.
__device__ __forceinline__ void load_idx_imp(const Contact* c, uint4& ix, uint4& iq) {
  uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
  asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
               : "l"(reinterpret_cast<const unsigned char*>(c) + 32));
  ix = make_uint4(r0, r1, r2, r3);
  iq = make_uint4(r4, r5, r6, r7);
}

// Asynchronous global -> shared copies (cp.async, completion tracked per thread in commit
// groups; wait_group N returns once at most N of the thread's groups are still pending).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uint32_t(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(uint32_t(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Contact records of the block's deferred environments (their sort moved slots), one
// environment at a time by the whole block: thread t stages parts t, t + nt, ... (part =
// 16 bytes of a 64-byte record) that copy a stored record, the block synchronises, then
// every part is written.  A slot whose pair made contact while in the list carries that
// pair's last contact; any other slot gets the record stored at its original position,
// marked invalid, with its own indices.  Since all reads precede all writes, the in-place
// permutation needs no cycle walk.  run_env defers only environments with
// 4 * n_fin <= kWbParts * nt, so every part has a staging register.
__device__ __forceinline__ void write_back_moved(const StepArgs& a, const ModelS& m, const FPlan& pl,
                                                 unsigned char* blk, uint32_t ne, uint32_t nb, uint32_t e0,
                                                 uint32_t tid, uint32_t nt) {
  const uint32_t* s_hdr = reinterpret_cast<const uint32_t*>(blk + pl.hdr * ne);
  const uint32_t* s_meta = reinterpret_cast<const uint32_t*>(blk + pl.meta * ne);
  const float* s_imp = reinterpret_cast<const float*>(blk + pl.imp * ne);
  const float4* s_pp = reinterpret_cast<const float4*>(blk + pl.pp * ne);
  const float4* s_nt = reinterpret_cast<const float4*>(blk + pl.nt * ne);
  const uint8_t* s_nlh = blk + pl.nlh * ne;
  const uint32_t M = a.M;
  for (uint32_t el = 0; el < nb; ++el) {
    const uint32_t d = s_hdr[2 * ne + el];  // the same for every thread
    if (!(d & kWbDeferred)) continue;
    const uint32_t n_fin = d & 0xFFu, n0 = (d >> 8) & 0xFFu, total = 4u * n_fin;
    const bool pub = (d & kWbPublish) != 0;
    const Contact* gc = a.contacts + size_t(e0 + el) * M;
    Contact* dst = pub ? a.contacts + size_t(e0 + el) * M : a.prev_contacts + size_t(e0 + el) * M;
    uint4 stash[kWbParts];
#pragma unroll
    for (uint32_t r = 0; r < kWbParts; ++r) {
      const uint32_t t = tid + r * nt;
      if (t >= total) continue;
      const uint32_t j = t >> 2, w = s_meta[j * ne + el];
      const uint32_t o = sw_origin(w), hh = sw_hit(w);
      const bool hit = hh != fm::kNoHit && o < s_nlh[hh * ne + el];
      if (!hit && !(pub && o == j)) stash[r] = reinterpret_cast<const uint4*>(gc + o)[t & 3u];
    }
    __syncthreads();
#pragma unroll
    for (uint32_t r = 0; r < kWbParts; ++r) {
      const uint32_t t = tid + r * nt;
      if (t >= total) continue;
      const uint32_t j = t >> 2, part = t & 3u, w = s_meta[j * ne + el];
      const uint32_t p = sw_pair(w), o = sw_origin(w), hh = sw_hit(w);
      const bool hit = hh != fm::kNoHit && o < s_nlh[hh * ne + el];
      uint4* out = reinterpret_cast<uint4*>(dst + j) + part;
      uint4 idx = make_uint4(0u, 0u, 0u, 0u);
      if (part == 2) {
        const uint32_t pi = m.pinfo(p), pbody = m.pbody(p);
        idx = make_uint4(pbody & 0xFFu, (pbody >> 8) & 0xFFu, pi & 0xFFu, (pi >> 8) & 0xFFu);
      }
      if (hit) {
        uint4 v;
        if (part == 0) {
          v = *reinterpret_cast<const uint4*>(&s_pp[hh * ne + el]);
        } else if (part == 1) {
          const float4 nn = s_nt[hh * ne + el];
          const float4 nf = make_float4(nn.x, nn.y, nn.z, m.hfr(hh));
          v = *reinterpret_cast<const uint4*>(&nf);
        } else if (part == 2) {
          v = idx;
        } else {
          const float4 im = make_float4(s_imp[j * ne + el], 0.0f, 0.0f, a.restitution);
          v = *reinterpret_cast<const uint4*>(&im);
        }
        *out = v;
      } else if (pub && o == j) {
        if (part == 0) reinterpret_cast<float*>(out)[3] = -1.0f;
        else if (part == 2 && o >= n0) *out = idx;
      } else {
        uint4 v = stash[r];
        if (part == 0) v.w = __float_as_uint(-1.0f);
        if (part == 2) v = idx;
        *out = v;
      }
    }
  }
}

// blockDim.x = envs_per_block * L threads (envs_per_block <= 32); group g (= threadIdx.x / L)
// owns env e0 + g.
template <int L, bool C>
__global__ void __launch_bounds__(32 * L, 1) fast_step_kernel(const __grid_constant__ StepArgs a,
                                                        const __grid_constant__ FModel f) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t nt = blockDim.x, tid = threadIdx.x;
  StageClock<C> clk;
  if constexpr (C) {
    __shared__ unsigned long long s_clk[kStageCount];
    clk.start(s_clk, tid == 0);
    __syncthreads();
  }
  const uint32_t ne = nt / L;  // environments per block
  const uint32_t e0 = blockIdx.x * ne;
  if (e0 >= a.num_envs) return;
  const uint32_t nb = min(ne, a.num_envs - e0);
  const uint32_t B = a.B, J = a.J, M = a.M;
  const FPlan pl = fast_plan(B, J, M, f.H, L);
  // shared memory: the model's hot image, then the per-environment sections
  unsigned char* hot = smem_raw;
  unsigned char* blk = smem_raw + f.hot_bytes;
  // With one lane per environment the slot loader's first round (below) is issued before
  // anything else: its addresses need neither the image nor the list headers, which take
  // two memory round trips.  (With two lanes the held registers would spill.)
  // With the slot cache (the kernel's own copy of the lists it wrote last step) the lists
  // arrive by cp.async with the state instead, and only environments whose cache entry is
  // not current read the records.
  const bool cached = a.slot_cache_w != nullptr;
  const Contact* gcb = a.contacts + size_t(e0) * M;
  constexpr uint32_t kU = 8;  // slots per thread per round: their loads are in flight together
  uint4 ix[kU], iq[kU];
  if constexpr (L == 1) {
    if (!cached) {
#pragma unroll
      for (uint32_t u = 0; u < kU; ++u) {
        const uint32_t t = tid + u * nt;
        if (t < nb * M) load_idx_imp(gcb + t, ix[u], iq[u]);
      }
    }
  }
  // the hot image and (below) the block's state arrive by cp.async, all copies in flight at once
  for (uint32_t t = tid; t < f.hot_bytes / 16u; t += nt) cp_async16(reinterpret_cast<uint4*>(hot) + t, f.hot + t);
  cp_async_commit();
  float4* s_pos = reinterpret_cast<float4*>(blk + pl.pos * ne);
  float4* s_quat = reinterpret_cast<float4*>(blk + pl.quat * ne);
  float4* s_vel = reinterpret_cast<float4*>(blk + pl.vel * ne);
  float4* s_ang = reinterpret_cast<float4*>(blk + pl.ang * ne);
  float* s_jt = reinterpret_cast<float*>(blk + pl.jt * ne);
  float* s_jp = reinterpret_cast<float*>(blk + pl.jp * ne);
  float* s_jv = reinterpret_cast<float*>(blk + pl.jv * ne);
  uint32_t* s_flags = reinterpret_cast<uint32_t*>(blk + pl.flags * ne);

  // ---- coalesced load of the block's body state and joint torques ----
  const size_t eb = size_t(e0) * B;
  float4* gpos = reinterpret_cast<float4*>(a.pos) + eb;
  float4* gquat = reinterpret_cast<float4*>(a.quat) + eb;
  float4* gvel = reinterpret_cast<float4*>(a.vel) + eb;
  float4* gang = reinterpret_cast<float4*>(a.angvel) + eb;
  float4* gacc = reinterpret_cast<float4*>(a.acc) + eb;
  for (uint32_t t = tid; t < nb * B; t += nt) {
    const uint32_t el = t / B, b = t - el * B, si = b * ne + el;
    cp_async16(s_pos + si, gpos + t);
    cp_async16(s_quat + si, gquat + t);
    cp_async16(s_vel + si, gvel + t);
    cp_async16(s_ang + si, gang + t);
  }
  float* gjt = a.jtorque + size_t(e0) * J;
  float* gjp = a.jpos + size_t(e0) * J;
  float* gjv = a.jvel + size_t(e0) * J;
  for (uint32_t t = tid; t < nb * J; t += nt) {
    const uint32_t el = t / J, j = t - el * J;
    cp_async4(s_jt + j * ne + el, gjt + t);
  }
  uint32_t* s_hdr = reinterpret_cast<uint32_t*>(blk + pl.hdr * ne);
  float* s_imp = reinterpret_cast<float*>(blk + pl.imp * ne);
  uint32_t* s_meta = reinterpret_cast<uint32_t*>(blk + pl.meta * ne);
  uint8_t* s_aux = blk + pl.aux * ne;
  const size_t E = a.num_envs;
  // slot loops of the cache: thread tid serves environment tid % ne, slots tid / ne + k L
  const uint32_t sc_el = tid % ne, sc_i0 = tid / ne;
  if (cached && sc_el < nb) {  // slot words and impulses from the cache, straight into their places
    for (uint32_t i = sc_i0; i < M; i += L) {
      cp_async4(s_meta + i * ne + sc_el, a.slot_cache_w + size_t(i) * E + e0 + sc_el);
      cp_async4(s_imp + i * ne + sc_el, a.slot_cache_imp + size_t(i) * E + e0 + sc_el);
    }
  }
  cp_async_commit();
  cp_async_wait<1>();  // this thread's part of the hot image
  __syncthreads();
  // gravity force per body for this step (compute_forces 345-388): g / (1/m), zero when massless
  for (uint32_t b = tid; b < B; b += nt) {
    const float4 mi = reinterpret_cast<const float4*>(hot + f.o_imi)[b];
    const V3 gv{a.gravity[0], a.gravity[1], a.gravity[2]};
    reinterpret_cast<float4*>(hot + f.o_gforce)[b] =
        mi.x < 1e-8f ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : with_w(gv * rcp_(mi.x), 0.0f);
  }
  // ---- contact list headers, then the slots: slot words, impulses, previous-list ranks ----
  for (uint32_t el = tid; el < nb; el += nt) {
    const uint32_t e = e0 + el;
    const uint32_t c = a.counts[e], pc = a.prev_counts[e], sep = a.prev_sep[e];
    s_hdr[el] = c;
    s_hdr[ne + el] = pc;
    s_hdr[2 * ne + el] = sep;
    s_hdr[3 * ne + el] = 0;
    // (cached launches) 1: read this environment's records.  The cache holds the list the
    // last step left, so it serves when that step wrote it, the previous list was not
    // separated by a subset step, and the counter has not grown since (it only shrinks,
    // by a reset)
    if (cached) s_flags[el] = (a.slot_cache_ok[e] != 0 && sep == 0 && c <= pc) ? 0u : 1u;
  }
  bool need_records = true;
  if (cached) need_records = __syncthreads_or(tid < nb && s_flags[tid] != 0) != 0;
  else __syncthreads();
  if (cached && need_records) {  // the cache copies land before any record overwrites them
    cp_async_wait<0>();
    __syncthreads();
  }
  const ModelS m{hot, f};
  // An environment is handed over (s_hdr[3] set) when a slot tuple of either list is not
  // a broad-phase candidate, when a list is not sorted by key, or when a slot of the
  // previous list carries non-zero tangent impulses (a warm start would copy them; this
  // kernel keeps only normal impulses).  This library never writes any of these.  Only
  // the second half of each 64-byte record (indices, impulses) is read.
  for (uint32_t t0 = tid; need_records && t0 < nb * M; t0 += kU * nt) {
    if (L != 1 || t0 != tid || cached) {
#pragma unroll
      for (uint32_t u = 0; u < kU; ++u) {
        const uint32_t t = t0 + u * nt;
        if (t < nb * M && !(cached && s_flags[t / M] == 0)) load_idx_imp(gcb + t, ix[u], iq[u]);
      }
    }
#pragma unroll
    for (uint32_t u = 0; u < kU; ++u) {
      const uint32_t t = t0 + u * nt;
      if (t >= nb * M) continue;
      const uint32_t el = t / M, i = t - el * M;
      if (cached && s_flags[el] == 0) continue;
      s_imp[i * ne + el] = __uint_as_float(iq[u].x);
      if (i < s_hdr[el]) {  // i < min(count, M)
        const uint32_t p = lookup_pair(m, ix[u]);
        if (p == fm::kNoPair) s_hdr[3 * ne + el] = 1;
        else s_meta[i * ne + el] = slot_word(m, p, i);
      }
      if (i < s_hdr[ne + el]) {  // previous list: the same records unless a subset step separated it
        uint4 px = ix[u], pq = iq[u];
        if (s_hdr[2 * ne + el] != 0) {
          const Contact& pr = a.prev_contacts[size_t(e0 + el) * M + i];
          px = *reinterpret_cast<const uint4*>(pr.indices);
          pq = *reinterpret_cast<const uint4*>(pr.impulses);
        }
        const uint32_t p = lookup_pair(m, px);
        if (p == fm::kNoPair || (pq.y | pq.z) != 0u) s_hdr[3 * ne + el] = 1;
        else s_aux[i * ne + el] = uint8_t(m.pinfo(p) >> 24);
      }
    }
  }
  __syncthreads();
  // both lists sorted by key: one thread per environment walks its slots (at each slot
  // index the threads read consecutive words)
  for (uint32_t el = tid; need_records && el < nb; el += nt) {
    if (s_hdr[3 * ne + el] || (cached && s_flags[el] == 0)) continue;
    const uint32_t nc = min(s_hdr[el], M), np = min(s_hdr[ne + el], M);
    bool bad = false;
    uint32_t r0 = nc > 0 ? sw_rank(s_meta[el]) : 0u;
#pragma unroll 8
    for (uint32_t i = 1; i < nc; ++i) {
      const uint32_t r1 = sw_rank(s_meta[i * ne + el]);
      bad |= r0 > r1;
      r0 = r1;
    }
    uint32_t a0 = np > 0 ? s_aux[el] : 0u;
#pragma unroll 8
    for (uint32_t i = 1; i < np; ++i) {
      const uint32_t a1 = s_aux[i * ne + el];
      bad |= a0 > a1;
      a0 = a1;
    }
    if (bad) s_hdr[3 * ne + el] = 1;
  }
  cp_async_wait<0>();  // this thread's part of the body state and joint torques (and cache)
  __syncthreads();
  if (cached) {
    // cached lists: each slot word gets its slot as origin (the cache holds the words as
    // the last step left them), and the previous-list key ranks are the stored list's
    if (sc_el < nb && s_flags[sc_el] == 0) {
      const uint32_t np = min(s_hdr[ne + sc_el], M);
#pragma unroll 4
      for (uint32_t i = sc_i0; i < np; i += L) {
        const uint32_t w = s_meta[i * ne + sc_el];
        s_meta[i * ne + sc_el] = (w & ~(0xFFu << 8 | kVisited)) | (i << 8);
        s_aux[i * ne + sc_el] = uint8_t(sw_rank(w));
      }
    }
    __syncthreads();
    for (uint32_t el = tid; el < nb; el += nt) s_flags[el] = 0;
  }
  for (uint32_t el = tid; el < nb; el += nt)
    if (s_hdr[3 * ne + el]) {
      a.odd_list[atomicAdd(a.odd_count, 1u)] = e0 + el;
      s_flags[el] = kSkipState;
    }

  const uint32_t g = tid / L;
  const bool active = g < nb && s_hdr[3 * ne + g] == 0;
  const unsigned wmask = __ballot_sync(__activemask(), active);
  if (active) {
    Group<L> G;
    G.lane = tid % L;
    G.src = int((tid & 31u) - G.lane);
    G.mask = wmask;
    uint32_t flags = kSkipState;
    run_env<L, C>(a, f, pl, hot, blk, ne, g, G, e0 + g, flags, clk);
    if (G.lane == 0) s_flags[g] = flags;
  }
  __syncthreads();
  write_back_moved(a, m, pl, blk, ne, nb, e0, tid, nt);

  // ---- coalesced store: state, accelerations, joint torques and states; the step-start
  //      velocities (for the accelerations) of four elements are loaded before any store ----
  for (uint32_t t0 = tid; t0 < nb * B; t0 += 4 * nt) {
    uint32_t fl[4], si[4];
    float4 v0[4];
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      const uint32_t t = t0 + u * nt;
      fl[u] = kSkipState;
      if (t >= nb * B) continue;
      const uint32_t el = t / B, b = t - el * B;
      si[u] = b * ne + el;
      fl[u] = s_flags[el];
      if (!(fl[u] & (kSkipState | kAccWritten))) v0[u] = gvel[t];
    }
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      const uint32_t t = t0 + u * nt;
      if (fl[u] & kSkipState) continue;
      const float4 v1 = s_vel[si[u]];
      if (!(fl[u] & kAccWritten))
        gacc[t] = make_float4((v1.x - v0[u].x) * a.inv_step, (v1.y - v0[u].y) * a.inv_step,
                              (v1.z - v0[u].z) * a.inv_step, 0.0f);
      gpos[t] = s_pos[si[u]];
      gquat[t] = s_quat[si[u]];
      gvel[t] = v1;
      gang[t] = s_ang[si[u]];
    }
  }
  for (uint32_t t = tid; t < nb * J; t += nt) {
    const uint32_t el = t / J, j = t - el * J;
    const uint32_t fl = s_flags[el];
    if (fl & kSkipState) continue;
    gjt[t] = s_jt[j * ne + el];
    if (fl & kWriteJointState) {
      gjp[t] = s_jp[j * ne + el];
      gjv[t] = s_jv[j * ne + el];
    }
  }
  if (a.slot_cache_w != nullptr) {  // the lists as this step left them, for the next step's slot cache
    // (slot words as they stand; the next step's prologue re-sets their origin fields)
    const size_t En = a.num_envs;  // (re-read from the parameters: nothing stays live across the step)
    const uint32_t el = tid % ne;
    if (el < nb && !(s_flags[el] & kSkipState)) {
#pragma unroll 4
      for (uint32_t i = tid / ne; i < M; i += L) {
        a.slot_cache_w[size_t(i) * En + e0 + el] = s_meta[i * ne + el];
        a.slot_cache_imp[size_t(i) * En + e0 + el] = s_imp[i * ne + el];
      }
    }
    for (uint32_t el = tid; el < nb; el += nt) a.slot_cache_ok[e0 + el] = (s_flags[el] & kSkipState) ? 0 : 1;
  }
  if constexpr (C) {  // (the first thread's own stores are issued; the block's others may still drain)
    clk.mark(kStEpilogue);
    clk.publish(a.stage_clk);
  }
}

static size_t fast_smem(const StepArgs& args, const FModel& model, int lanes, int envs_per_block) {
  return size_t(model.hot_bytes) +
         size_t(fast_plan(args.B, args.J, args.M, model.H, uint32_t(lanes)).bytes) * envs_per_block;
}

template <int L, bool C>
static cudaError_t launch_lc(const StepArgs& args, const FModel& model, int envs_per_block, cudaStream_t stream) {
  const size_t smem = fast_smem(args, model, L, envs_per_block);
  cudaError_t err =
      cudaFuncSetAttribute(fast_step_kernel<L, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  const uint32_t blocks = (args.num_envs + envs_per_block - 1) / envs_per_block;
  fast_step_kernel<L, C><<<blocks, envs_per_block * L, smem, stream>>>(args, model);
  return cudaGetLastError();
}

// the stage-profiling instantiation runs when args.stage_clk is set
template <int L>
static cudaError_t launch_l(const StepArgs& args, const FModel& model, int envs_per_block, cudaStream_t stream) {
  return args.stage_clk ? launch_lc<L, true>(args, model, envs_per_block, stream)
                        : launch_lc<L, false>(args, model, envs_per_block, stream);
}

bool fast_lanes_supported(int lanes) { return lanes == 1 || lanes == 2; }

cudaError_t launch_fast_step(const StepArgs& args, const FModel& model, int lanes, int envs_per_block,
                             cudaStream_t stream) {
  if (args.num_envs == 0) return cudaSuccess;
  if (envs_per_block < 1 || envs_per_block > 32) return cudaErrorInvalidValue;
  switch (lanes) {
    case 1: return launch_l<1>(args, model, envs_per_block, stream);
    case 2: return launch_l<2>(args, model, envs_per_block, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int L>
static int max_active_l(const StepArgs& args, const FModel& model, int envs_per_block) {
  const size_t smem = fast_smem(args, model, L, envs_per_block);
  if (cudaFuncSetAttribute(fast_step_kernel<L, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fast_step_kernel<L, false>, envs_per_block * L, smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int fast_max_active_blocks(const StepArgs& args, const FModel& model, int lanes, int envs_per_block) {
  if (envs_per_block < 1 || envs_per_block > 32) return 0;
  switch (lanes) {
    case 1: return max_active_l<1>(args, model, envs_per_block);
    case 2: return max_active_l<2>(args, model, envs_per_block);
    default: return 0;
  }
}

}  // namespace zb
