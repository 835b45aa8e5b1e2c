// Packs a HostModel into the constant-bank FModel of the environment-per-lane kernel.
#include "fast_model.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "model.h"
#include "zeno_types.h"

namespace zb {
namespace {
// The type pairs the selected narrow phase can report a contact for: narrow_core (mode 0)
// or narrow_cpu (modes 1 and 2; box-capsule pairs of mode 2 are rejected before this),
// physics.cuh.
inline bool narrow_pair_supported(uint32_t mode, uint32_t ta, uint32_t tb) {
  if (mode >= 1) {
    if (ta > 3 || tb > 3) return false;
    if ((ta == 1 && tb == 2) || (ta == 2 && tb == 1)) return false;
    return !(ta == 3 && tb == 3);
  }
  return (ta == 0 && tb == 0) || (ta == 0 && tb == 3) || (ta == 3 && tb == 0) || (ta == 1 && tb == 3) ||
         (ta == 3 && tb == 1);
}
inline float4 f4(const float* v) { return make_float4(v[0], v[1], v[2], v[3]); }
// +z rotated by q, evaluated exactly as the kernels' capsule_axis / rotate (physics.cuh,
// devmath.cuh): the same products and fused multiply-adds in the same order.
inline float4 capsule_axis_host(const float* q) {
  const float v[3] = {0.0f, 0.0f, 1.0f};
  auto cross = [](const float* a, const float* b, float* o) {
    o[0] = std::fmaf(a[1], b[2], -(a[2] * b[1]));
    o[1] = std::fmaf(a[2], b[0], -(a[0] * b[2]));
    o[2] = std::fmaf(a[0], b[1], -(a[1] * b[0]));
  };
  float uv[3], uuv[3];
  cross(q, v, uv);
  cross(q, uv, uuv);
  return make_float4(std::fmaf(2.0f, std::fmaf(q[3], uv[0], uuv[0]), v[0]),
                     std::fmaf(2.0f, std::fmaf(q[3], uv[1], uuv[1]), v[1]),
                     std::fmaf(2.0f, std::fmaf(q[3], uv[2], uuv[2]), v[2]), 0.0f);
}
}  // namespace

bool pack_fast_model(const HostModel& h, uint32_t max_contacts, uint32_t narrow_mode, FModel* out,
                     std::vector<uint8_t>* hot, std::string* why) {
  auto fail = [&](const char* msg) {
    if (why) *why = msg;
    return false;
  };
  const uint32_t P = uint32_t(h.pairs.size());
  if (h.B > fm::kB) return fail("more bodies than the constant-bank model holds");
  if (h.J > fm::kJ || h.jf_list.size() > fm::kJF) return fail("more joints than the constant-bank model holds");
  if (h.K > fm::kK) return fail("more constraints than the constant-bank model holds");
  if (h.G > fm::kG) return fail("more geoms than the constant-bank model holds");
  if (P > fm::kP) return fail("more broad-phase candidates than the constant-bank model holds");
  if (h.A > fm::kA) return fail("more actuators than the constant-bank model holds");
  if (h.S > fm::kS || h.obs_dim > 0xFFFFu) return fail("more sensors than the constant-bank model holds");
  if (max_contacts > fm::kMaxSlots) return fail("more contact slots per env than the per-slot byte fields index");

  FModel& m = *out;
  std::memset(&m, 0, sizeof(m));
  for (uint32_t b = 0; b < h.B; ++b) {
    const DBody& d = h.bodies[b];
    if (d.type == 1 && d.inv_mass_inertia[0] >= 1e-8f) return fail("kinematic body with mass");
    m.imi[b] = f4(d.inv_mass_inertia);
    m.com[b] = f4(d.com);
    m.body[b] = (d.type & 0xFFu) | (d.jf_begin << 8) | (d.jf_end << 16) | (std::min<uint32_t>(h.subtree[b], 255u) << 24);
  }
  for (size_t k = 0; k < h.jf_list.size(); ++k) {
    const uint32_t ent = h.jf_list[k];
    m.jf[k] = uint8_t((ent & 0x7Fu) | ((ent >> 31) ? 0x80u : 0u));
  }
  for (uint32_t j = 0; j < h.J; ++j) {
    const DJoint& d = h.joints[j];
    // The fused force + integration pass visits bodies children first; it needs every
    // joint's parent body to precede its child (MJCF tree order guarantees it).
    if (d.parent >= d.child) return fail("joint parent does not precede its child");
    m.j_ap[j] = f4(d.anchor_parent);
    m.j_ac[j] = f4(d.anchor_child);
    m.j_axis[j] = f4(d.axis);
    m.j_info[j] = (d.type & 0xFFu) | (d.parent << 8) | (d.child << 16);
  }
  for (uint32_t k = 0; k < h.K; ++k) {
    const DConstraint& c = h.constraints[k];
    m.c_aa[k] = f4(c.anchor_a);
    m.c_ab[k] = f4(c.anchor_b);
    m.c_at[k] = f4(c.axis_target);
    m.c_lim[k] = f4(c.limits);
    m.c_info[k] = (c.body_a & 0xFFu) | ((c.body_b & 0xFFu) << 8) | ((c.type & 0xFFu) << 16);
  }
  for (uint32_t g = 0; g < h.G; ++g) {
    m.g_ps[g] = f4(h.geoms[g].pos_size0);
    m.g_body[g] = h.geoms[g].body;
  }
  std::memset(m.gg_pair, int(fm::kNoPair), sizeof(m.gg_pair));

  // sort_contacts key (min body << 16 | max body in the reference); only its order is
  // used, so the kernel carries the dense rank of each candidate's key.
  if (h.corrected) return fail("corrected semantics run on the general kernel");
  std::vector<uint32_t> keys(P);
  for (uint32_t p = 0; p < P; ++p) {
    const uint32_t ta = h.geoms[h.pairs[p].ga].type, tb = h.geoms[h.pairs[p].gb].type;
    if (narrow_mode == 2 && ((ta == 1 && tb == 2) || (ta == 2 && tb == 1)))
      return fail("box-capsule candidates need GJK + EPA (general kernel)");
    const uint32_t ba = h.geoms[h.pairs[p].ga].body, bb = h.geoms[h.pairs[p].gb].body;
    keys[p] = (std::min(ba, bb) << 16) | std::max(ba, bb);
  }
  std::vector<uint32_t> distinct = keys;
  std::sort(distinct.begin(), distinct.end());
  distinct.erase(std::unique(distinct.begin(), distinct.end()), distinct.end());

  // Hittable candidates are numbered with the capsule-plane pairs first (reference GPU
  // narrow phase), which the kernel tests four at a time; the numbering is internal (slot
  // words, pair tables, hit masks) and does not change results.
  std::vector<uint32_t> hit_index(P, fm::kNoHit);
  uint32_t H = 0, n_cp = 0;
  for (int pass = 0; pass < 2; ++pass)
    for (uint32_t p = 0; p < P; ++p) {
      const DGeom &ga = h.geoms[h.pairs[p].ga], &gb = h.geoms[h.pairs[p].gb];
      if (!narrow_pair_supported(narrow_mode, ga.type, gb.type)) continue;
      const bool cp = narrow_mode == 0 && ((ga.type == 1 && gb.type == 3) || (ga.type == 3 && gb.type == 1));
      if (cp != (pass == 0)) continue;
      if (H >= fm::kH) return fail("more hittable candidates than the constant-bank model holds");
      hit_index[p] = H++;
      n_cp += cp ? 1u : 0u;
    }
  for (uint32_t p = 0; p < P; ++p) {
    const DPair& pr = h.pairs[p];
    const DGeom &ga = h.geoms[pr.ga], &gb = h.geoms[pr.gb];
    const uint32_t rank = uint32_t(std::lower_bound(distinct.begin(), distinct.end(), keys[p]) - distinct.begin());
    const uint32_t hidx = hit_index[p];
    if (hidx != fm::kNoHit) {
      m.h_pair[hidx] = p;
      m.h_info[hidx] = (ga.type & 0xFFu) | ((gb.type & 0xFFu) << 8) | (ga.body << 16) | (gb.body << 24);
      m.h_ga[hidx] = f4(ga.pos_size0);
      m.h_gb[hidx] = f4(gb.pos_size0);
      const DGeom& cap = ga.type == 1 ? ga : gb;
      m.h_cax[hidx] = capsule_axis_host(cap.quat);
      m.h_hl[hidx] = cap.size12_fr_rest[0];
      m.h_sz[hidx] = make_float4(ga.size12_fr_rest[0], ga.size12_fr_rest[1], gb.size12_fr_rest[0], gb.size12_fr_rest[1]);
      const float fp = ga.size12_fr_rest[2] * gb.size12_fr_rest[2];  // one IEEE product, then sqrt
      m.h_fr[hidx] = std::sqrt(fp);
    }
    m.p_info[p] = pr.ga | (pr.gb << 8) | (hidx << 16) | (rank << 24);
    m.p_body[p] = ga.body | (gb.body << 8) | ((pr.plane ? 1u : 0u) << 16);
    m.p_md2[p] = pr.min_dist_sq;
    m.gg_pair[pr.ga * fm::kG + pr.gb] = uint8_t(p);
  }
  for (uint32_t k = 0; k < h.A; ++k) {
    const DActuator& d = h.actuators[k];
    if (d.joint >= h.J) return fail("actuator on a joint index outside the model");
    m.a_joint[k] = d.joint;
    m.a_cmin[k] = d.ctrl_min, m.a_cmax[k] = d.ctrl_max, m.a_gear[k] = d.gear;
    m.a_fmin[k] = d.force_min, m.a_fmax[k] = d.force_max;
  }
  for (uint32_t s = 0; s < h.S; ++s) {
    const DSensor& d = h.sensors[s];
    const bool joint_sensor = d.type == 0 || d.type == 1;
    if (d.object >= (joint_sensor ? h.J : h.B)) return fail("sensor object index outside the model");
    m.s_info[s] = (d.type & 0xFFu) | ((d.object & 0xFFu) << 8) | (d.offset << 16);
  }
  m.P = P, m.H = H, m.G = h.G;
  m.n_capsule_plane = n_cp;
  m.narrow_mode = narrow_mode;
  {
    std::vector<uint8_t> seen(256, 0);
    m.hit_keys_unique = 1;
    for (uint32_t hh = 0; hh < H; ++hh) {
      const uint32_t rank = m.p_info[m.h_pair[hh]] >> 24;
      if (seen[rank]++) m.hit_keys_unique = 0;
    }
  }

  // hot image
  std::vector<uint8_t>& img = *hot;
  img.clear();
  auto section = [&](uint32_t bytes) {
    const uint32_t off = uint32_t((img.size() + 15) & ~size_t(15));
    img.resize(off + ((bytes + 15) & ~15u), 0);
    return off;
  };
  auto put = [&](uint32_t off, const void* src, size_t bytes) {
    if (bytes) std::memcpy(img.data() + off, src, bytes);
  };
  const uint32_t B = h.B, J = h.J, K = h.K, G = h.G, JF = uint32_t(h.jf_list.size());
  m.o_imi = section(16 * B), put(m.o_imi, m.imi, 16 * B);
  m.o_com = section(16 * B), put(m.o_com, m.com, 16 * B);
  m.o_body = section(4 * B), put(m.o_body, m.body, 4 * B);
  m.o_jf = section(4 * JF);
  for (uint32_t k = 0; k < JF; ++k) {
    const uint32_t v = m.jf[k];
    put(m.o_jf + 4 * k, &v, 4);
  }
  m.o_jaxis = section(16 * J), put(m.o_jaxis, m.j_axis, 16 * J);
  m.o_jinfo = section(4 * J), put(m.o_jinfo, m.j_info, 4 * J);
  m.o_caa = section(16 * K), put(m.o_caa, m.c_aa, 16 * K);
  m.o_cab = section(16 * K), put(m.o_cab, m.c_ab, 16 * K);
  m.o_cat = section(16 * K), put(m.o_cat, m.c_at, 16 * K);
  m.o_clim = section(16 * K), put(m.o_clim, m.c_lim, 16 * K);
  m.o_cinfo = section(4 * K), put(m.o_cinfo, m.c_info, 4 * K);
  m.o_pbody = section(4 * P), put(m.o_pbody, m.p_body, 4 * P);
  m.o_pinfo = section(4 * P), put(m.o_pinfo, m.p_info, 4 * P);
  m.o_pmd2 = section(4 * P), put(m.o_pmd2, m.p_md2, 4 * P);
  m.o_gps = section(16 * G), put(m.o_gps, m.g_ps, 16 * G);
  m.o_hinfo = section(4 * H), put(m.o_hinfo, m.h_info, 4 * H);
  m.o_hga = section(16 * H), put(m.o_hga, m.h_ga, 16 * H);
  m.o_hgb = section(16 * H), put(m.o_hgb, m.h_gb, 16 * H);
  m.o_hcax = section(16 * H), put(m.o_hcax, m.h_cax, 16 * H);
  m.o_hhl = section(4 * H), put(m.o_hhl, m.h_hl, 4 * H);
  m.o_hfr = section(4 * H), put(m.o_hfr, m.h_fr, 4 * H);
  m.o_hpair = section(4 * H), put(m.o_hpair, m.h_pair, 4 * H);
  m.o_hsz = section(16 * H), put(m.o_hsz, m.h_sz, 16 * H);
  m.o_gbody = section(4 * G), put(m.o_gbody, m.g_body, 4 * G);
  m.o_ggpair = section(G * G);
  for (uint32_t ga = 0; ga < G; ++ga) put(m.o_ggpair + ga * G, &m.gg_pair[ga * fm::kG], G);
  m.o_gforce = section(16 * B);
  // The colour sweep as runs of one constraint type: each colour split into maximal runs
  // of equal type, in order.  A run's constraints belong to one colour (disjoint bodies),
  // and the type dispatch happens once per run instead of once per constraint.
  std::vector<uint32_t> runs;
  for (uint32_t col = 0; col < h.num_colors; ++col) {
    const uint32_t start = h.kcolor_ranges[2 * col], cnt = h.kcolor_ranges[2 * col + 1];
    for (uint32_t k = start; k < start + cnt;) {
      const uint32_t t = h.constraints[k].type & 0xFFu;
      uint32_t n = 1;
      while (k + n < start + cnt && (h.constraints[k + n].type & 0xFFu) == t) ++n;
      if (k > 0xFFFu || n > 0xFFFu) return fail("constraint run out of range");
      runs.push_back(k | (n << 12) | (t << 24));
      k += n;
    }
  }
  m.num_runs = uint32_t(runs.size());
  m.o_runs = section(4 * m.num_runs), put(m.o_runs, runs.data(), 4 * runs.size());
  // Hinge groups (model.cpp hinge_groups) for one lane per environment, in sweep order:
  // k0 | k1 << 8 | k2 << 16 | kind << 24 (unused members kNoGroup).
  {
    std::vector<uint32_t> groups;
    for (size_t g = 0; g + 3 < h.hinge_groups.size(); g += 4) {
      const uint32_t* q = &h.hinge_groups[g];
      if (q[0] >= fm::kNoGroup || q[1] >= fm::kNoGroup || q[2] >= fm::kNoGroup)
        return fail("constraint index out of the group word's range");
      const uint32_t k1 = q[3] >= 1 ? q[1] : fm::kNoGroup, k2 = q[3] == 2 ? q[2] : fm::kNoGroup;
      groups.push_back(q[0] | (k1 << 8) | (k2 << 16) | (q[3] << 24));
    }
    m.num_groups = uint32_t(groups.size());
    m.o_groups = section(4 * m.num_groups), put(m.o_groups, groups.data(), 4 * groups.size());
  }
  {
    std::vector<uint32_t> words;
    bool fits = !h.jgroup_levels.empty();
    for (size_t g = 0; fits && 2 * g + 1 < h.jgroup_words.size(); ++g) {
      const uint32_t w0 = h.jgroup_words[2 * g], w1 = h.jgroup_words[2 * g + 1];
      const uint32_t k0 = w0 & 0xFFFFu, k1 = w0 >> 16, k2 = w1 & 0xFFFFu, kind = w1 >> 16;
      if (k0 >= fm::kNoGroup || k1 >= fm::kNoGroup || k2 >= fm::kNoGroup) fits = false;
      words.push_back(k0 | ((kind >= 1 ? k1 : fm::kNoGroup) << 8) | ((kind == 2 ? k2 : fm::kNoGroup) << 16) |
                      (kind << 24));
    }
    m.num_glv = fits ? uint32_t(h.jgroup_levels.size() - 1) : 0u;
    if (m.num_glv) {
      m.o_glv = section(4 * (m.num_glv + 1)), put(m.o_glv, h.jgroup_levels.data(), 4 * (m.num_glv + 1));
      m.o_gwords = section(4 * words.size()), put(m.o_gwords, words.data(), 4 * words.size());
    }
  }
  section(0);
  m.hot_bytes = uint32_t(img.size());
  m.hot = nullptr;
  return true;
}

}  // namespace zb
