// MJCF loader for the host runtime.  Reproduces the token-stream semantics of the
// reference parser (src/mjcf/parser.zig) so the resulting model is identical:
//   tokenizer, self-closing detection, comments          parser.zig:1345-1457
//   attribute lookup (first match, quoted values)        parser.zig:1463-1503
//   number parsing (whole token, single-space fields)    parser.zig:1505-1587
//   <option>, <default>, <worldbody>, <actuator>, <sensor> parser.zig:184-822
//   element defaults                                     src/mjcf/schema.zig:100-199
//   Scene conversion, mass/inertia, geoms, sensors       parser.zig:826-1337
//   <include file=...> splicing                          parser.zig:55-171
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

#include "scene.h"

namespace zb {

uint32_t Scene::obs_dim() const {
  uint32_t d = 0;
  for (const SSensor& s : sensors) d += s.dim;
  return d;
}

namespace {

inline bool ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

enum class Kind { Open, Close, Text, Comment };
struct Tok {
  Kind kind;
  std::string name, attrs;
};

class Lexer {
 public:
  explicit Lexer(const std::string& s) : s_(s) {}
  bool next(Tok& t) {
    while (p_ < s_.size() && ws(s_[p_])) ++p_;
    if (p_ >= s_.size()) return false;
    if (s_[p_] != '<') {
      size_t b = p_;
      while (p_ < s_.size() && s_[p_] != '<') ++p_;
      t = Tok{Kind::Text, s_.substr(b, p_ - b), ""};
      return true;
    }
    ++p_;
    if (p_ >= s_.size()) return false;
    if (s_.compare(p_, 3, "!--") == 0 && s_.size() - p_ >= 3) {
      for (; p_ + 2 < s_.size(); ++p_)
        if (s_[p_] == '-' && s_[p_ + 1] == '-' && s_[p_ + 2] == '>') {
          p_ += 3;
          break;
        }
      t = Tok{Kind::Comment, "", ""};
      return true;
    }
    const bool closing = s_[p_] == '/';
    if (closing) ++p_;
    size_t nb = p_;
    while (p_ < s_.size() && !ws(s_[p_]) && s_[p_] != '>' && s_[p_] != '/') ++p_;
    std::string name = s_.substr(nb, p_ - nb);
    while (p_ < s_.size() && ws(s_[p_])) ++p_;
    size_t ab = p_;
    while (p_ < s_.size() && s_[p_] != '>') ++p_;
    size_t ae = p_;
    if (!closing) {  // "/" as the last non-space character before '>' marks self-closing
      size_t k = p_;
      while (k > ab && ws(s_[k - 1])) --k;
      if (k > ab && s_[k - 1] == '/') ae = k - 1;
    }
    std::string attrs = closing ? std::string() : s_.substr(ab, ae - ab);
    if (p_ < s_.size()) ++p_;
    t = Tok{closing ? Kind::Close : Kind::Open, std::move(name), std::move(attrs)};
    return true;
  }

 private:
  const std::string& s_;
  size_t p_ = 0;
};

// First attribute with the given name; values must be quoted.
bool attr(const std::string& a, const char* key, std::string& out) {
  size_t p = 0, n = a.size();
  while (p < n) {
    while (p < n && ws(a[p])) ++p;
    size_t kb = p;
    while (p < n && a[p] != '=' && !ws(a[p])) ++p;
    size_t ke = p;
    while (p < n && (ws(a[p]) || a[p] == '=')) ++p;
    if (p >= n) break;
    char q = a[p];
    if (q != '"' && q != '\'') continue;
    size_t vb = ++p;
    while (p < n && a[p] != q) ++p;
    size_t ve = p++;
    if (a.compare(kb, ke - kb, key) == 0 && std::strlen(key) == ke - kb) {
      out = a.substr(vb, ve - vb);
      return true;
    }
  }
  return false;
}

bool num(const std::string& s, float& out) {
  if (s.empty() || ws(s[0])) return false;
  char* end = nullptr;
  float v = std::strtof(s.c_str(), &end);
  if (end != s.c_str() + s.size()) return false;
  out = v;
  return true;
}

bool unum(const std::string& s, uint32_t& out) {
  size_t i = (!s.empty() && s[0] == '+') ? 1 : 0;
  if (i >= s.size()) return false;
  uint64_t v = 0;
  for (; i < s.size(); ++i) {
    if (s[i] < '0' || s[i] > '9') return false;
    v = v * 10 + uint64_t(s[i] - '0');
    if (v > 0xFFFFFFFFull) return false;
  }
  out = uint32_t(v);
  return true;
}

// Fields separated by single spaces (empty fields are kept, as splitScalar does).
std::vector<std::string> fields(const std::string& s) {
  std::vector<std::string> f;
  std::string cur;
  for (char c : s) {
    if (c == ' ') {
      f.push_back(cur);
      cur.clear();
    } else {
      cur.push_back(c);
    }
  }
  f.push_back(cur);
  return f;
}

// All of the first n fields must parse; otherwise `out` is left untouched.
bool vec(const std::string& s, size_t n, float* out) {
  std::vector<std::string> f = fields(s);
  if (f.size() < n) return false;
  float tmp[8];
  for (size_t i = 0; i < n; ++i)
    if (!num(f[i], tmp[i])) return false;
  std::memcpy(out, tmp, n * sizeof(float));
  return true;
}

struct XJoint {
  std::string name;
  int type = 3;  // schema JointType: 0 free, 1 ball, 2 slide, 3 hinge
  float pos[3] = {0, 0, 0}, axis[3] = {0, 0, 1};
  bool ranged = false;
  float range[2] = {0, 0};
  float damping = 0, stiffness = 0, armature = 0, ref = 0;
};
struct XGeom {
  std::string name;
  int type = 1;  // schema GeomType: 0 plane 1 sphere 2 capsule 3 cylinder 4 box 5 mesh 6 hfield
  float pos[3] = {0, 0, 0}, quat_wxyz[4] = {1, 0, 0, 0}, size[3] = {0.05f, 0, 0};
  bool has_euler = false;  // read only by the corrected loader
  float euler[3] = {0, 0, 0};
  bool has_fromto = false, has_mass = false;
  float fromto[6] = {0, 0, 0, 0, 0, 0}, mass = 0, density = 1000;
  float friction[3] = {1, 0.005f, 0.0001f};
  uint32_t contype = 1, conaffinity = 1;
};
struct XBody {
  std::string name;
  float pos[3] = {0, 0, 0}, quat_wxyz[4] = {1, 0, 0, 0};
  bool has_euler = false;
  float euler[3] = {0, 0, 0};
  bool has_inertial = false;
  float in_mass = 1.0f;
  bool in_diag = false, in_full = false;
  float in_diag_v[3] = {0, 0, 0}, in_full_v[6] = {0, 0, 0, 0, 0, 0};
  std::vector<XJoint> joints;
  std::vector<XGeom> geoms;
  std::vector<XBody> kids;
  std::vector<std::string> sites;  // site names (corrected sensor resolution)
};
struct XActuator {
  std::string joint;
  bool has_ctrl = false, has_force = false;
  float ctrl[2] = {0, 0}, force[2] = {0, 0}, gear = 1, kp = 0, kv = 0;
};
struct XSensor {
  int type = 0;  // jointpos .. subtreecom in schema order
  std::string joint, objtype, objname, site;
  float noise = 0;
};
struct XDefaults {
  XJoint joint;
  XGeom geom;
};
struct XModel {
  float timestep = 0.002f, gravity[3] = {0, 0, -9.81f};
  bool angle_degree = true;       // <compiler angle>, read only by the corrected loader
  std::string eulerseq = "xyz";   // <compiler eulerseq>
  std::map<std::string, XDefaults> defaults;
  XBody world;
  std::vector<XActuator> actuators;
  std::vector<XSensor> sensors;
};

int lookup(const std::string& s, std::initializer_list<const char*> names) {
  int i = 0;
  for (const char* n : names) {
    if (s == n) return i;
    ++i;
  }
  return -1;
}

void joint_attrs(XJoint& j, const std::string& a) {
  std::string v;
  float f;
  if (attr(a, "name", v)) j.name = v;
  if (attr(a, "type", v)) {
    int t = lookup(v, {"free", "ball", "slide", "hinge"});
    if (t >= 0) j.type = t;
  }
  if (attr(a, "pos", v)) vec(v, 3, j.pos);
  if (attr(a, "axis", v)) vec(v, 3, j.axis);
  if (attr(a, "range", v)) {
    float r[2];
    j.ranged = vec(v, 2, r);
    if (j.ranged) j.range[0] = r[0], j.range[1] = r[1];
  }
  if (attr(a, "damping", v) && num(v, f)) j.damping = f;
  if (attr(a, "stiffness", v) && num(v, f)) j.stiffness = f;
  if (attr(a, "armature", v) && num(v, f)) j.armature = f;
  if (attr(a, "ref", v) && num(v, f)) j.ref = f;
}

void geom_attrs(XGeom& g, const std::string& a) {
  std::string v;
  float f;
  uint32_t u;
  if (attr(a, "name", v)) g.name = v;
  if (attr(a, "type", v)) {
    int t = lookup(v, {"plane", "sphere", "capsule", "cylinder", "box", "mesh", "hfield"});
    if (t >= 0) g.type = t;
  }
  if (attr(a, "pos", v)) vec(v, 3, g.pos);
  if (attr(a, "quat", v)) vec(v, 4, g.quat_wxyz);
  if (attr(a, "euler", v)) g.has_euler = vec(v, 3, g.euler);
  if (attr(a, "size", v)) {  // up to three fields, unparsable ones read as 0
    std::vector<std::string> fs = fields(v);
    for (int i = 0; i < 3; ++i) g.size[i] = (i < int(fs.size()) && num(fs[i], f)) ? f : 0.0f;
  }
  if (attr(a, "fromto", v)) g.has_fromto = vec(v, 6, g.fromto);
  if (attr(a, "mass", v)) {
    g.has_mass = num(v, f);
    if (g.has_mass) g.mass = f;
  }
  if (attr(a, "density", v) && num(v, f)) g.density = f;
  if (attr(a, "friction", v)) vec(v, 3, g.friction);
  if (attr(a, "contype", v) && unum(v, u)) g.contype = u;
  if (attr(a, "conaffinity", v) && unum(v, u)) g.conaffinity = u;
  if (attr(a, "mesh", v)) g.type = 5;
}

class Reader {
 public:
  explicit Reader(const std::string& xml) : lx_(xml) {}

  void read(XModel& m) {
    Tok t;
    while (lx_.next(t))
      if (t.kind == Kind::Open && t.name == "mujoco") {
        top(m);
        return;
      }
  }

 private:
  Lexer lx_;

  void skip_until_close(const char* name) {
    Tok t;
    while (lx_.next(t))
      if (t.kind == Kind::Close && t.name == name) return;
  }

  void top(XModel& m) {
    Tok t;
    while (lx_.next(t)) {
      if (t.kind == Kind::Close && t.name == "mujoco") return;
      if (t.kind != Kind::Open) continue;
      if (t.name == "option") {
        std::string v;
        float f;
        m.timestep = 0.002f;
        m.gravity[0] = 0.0f, m.gravity[1] = 0.0f, m.gravity[2] = -9.81f;
        if (attr(t.attrs, "timestep", v)) m.timestep = num(v, f) ? f : 0.002f;
        if (attr(t.attrs, "gravity", v)) vec(v, 3, m.gravity);
      } else if (t.name == "compiler") {
        std::string v;
        if (attr(t.attrs, "angle", v)) m.angle_degree = v != "radian";
        if (attr(t.attrs, "eulerseq", v) && v.size() == 3) m.eulerseq = v;
      } else if (t.name == "default") {
        defaults(m);
      } else if (t.name == "worldbody") {
        body(m, m.world, "worldbody", "main");
      } else if (t.name == "actuator") {
        actuators(m);
      } else if (t.name == "sensor") {
        sensors(m);
      } else if (t.name == "asset" || t.name == "tendon" || t.name == "equality") {
        skip_until_close(t.name.c_str());
      }
    }
  }

  // A nested <default class=...> starts a fresh class; the first </default> ends the
  // whole section (what remains of an outer default is then ignored by the caller).
  void defaults(XModel& m) {
    std::string cls = "main";
    XDefaults cur;
    Tok t;
    while (lx_.next(t)) {
      if (t.kind == Kind::Close && t.name == "default") {
        if (!cls.empty()) m.defaults[cls] = cur;
        return;
      }
      if (t.kind != Kind::Open) continue;
      if (t.name == "default") {
        if (!cls.empty()) m.defaults[cls] = cur;
        std::string v;
        cls = attr(t.attrs, "class", v) ? v : std::string("main");
        cur = XDefaults{};
      } else if (t.name == "geom") {
        cur.geom = XGeom{};
        geom_attrs(cur.geom, t.attrs);
      } else if (t.name == "joint") {
        cur.joint = XJoint{};
        joint_attrs(cur.joint, t.attrs);
      }
    }
  }

  template <class T>
  T from_class(const XModel& m, const std::string& a, const std::string& cls, T XDefaults::*member) {
    std::string use = cls, v;
    if (attr(a, "class", v)) use = v;
    auto it = m.defaults.find(use);
    return it == m.defaults.end() ? T{} : it->second.*member;
  }

  void body(XModel& m, XBody& b, const char* end, const std::string& cls) {
    Tok t;
    std::string v;
    while (lx_.next(t)) {
      if (t.kind == Kind::Close && t.name == end) return;
      if (t.kind != Kind::Open) continue;
      if (t.name == "body") {
        XBody k;
        if (attr(t.attrs, "name", v)) k.name = v;
        if (attr(t.attrs, "pos", v)) vec(v, 3, k.pos);
        if (attr(t.attrs, "quat", v)) vec(v, 4, k.quat_wxyz);
        if (attr(t.attrs, "euler", v)) k.has_euler = vec(v, 3, k.euler);
        std::string kc = attr(t.attrs, "childclass", v) ? v : cls;
        body(m, k, "body", kc);
        b.kids.push_back(std::move(k));
      } else if (t.name == "joint") {
        XJoint j = from_class(m, t.attrs, cls, &XDefaults::joint);
        joint_attrs(j, t.attrs);
        b.joints.push_back(j);
      } else if (t.name == "geom") {
        XGeom g = from_class(m, t.attrs, cls, &XDefaults::geom);
        geom_attrs(g, t.attrs);
        b.geoms.push_back(g);
      } else if (t.name == "site") {
        b.sites.push_back(attr(t.attrs, "name", v) ? v : std::string());
      } else if (t.name == "inertial") {
        float f;
        b.has_inertial = true;
        b.in_mass = 1.0f;
        b.in_diag = b.in_full = false;
        if (attr(t.attrs, "mass", v)) b.in_mass = num(v, f) ? f : 1.0f;
        if (attr(t.attrs, "diaginertia", v)) b.in_diag = vec(v, 3, b.in_diag_v);
        if (attr(t.attrs, "fullinertia", v)) b.in_full = vec(v, 6, b.in_full_v);
      }
    }
  }

  void actuators(XModel& m) {
    Tok t;
    std::string v;
    while (lx_.next(t)) {
      if (t.kind == Kind::Close && t.name == "actuator") return;
      if (t.kind != Kind::Open || lookup(t.name, {"motor", "position", "velocity", "general"}) < 0) continue;
      XActuator a;
      float f;
      if (attr(t.attrs, "joint", v)) a.joint = v;
      if (attr(t.attrs, "ctrlrange", v)) a.has_ctrl = vec(v, 2, a.ctrl);
      if (attr(t.attrs, "forcerange", v)) a.has_force = vec(v, 2, a.force);
      if (attr(t.attrs, "gear", v)) a.gear = num(v, f) ? f : 1.0f;
      if (attr(t.attrs, "kp", v)) a.kp = num(v, f) ? f : 0.0f;
      if (attr(t.attrs, "kv", v)) a.kv = num(v, f) ? f : 0.0f;
      m.actuators.push_back(a);
    }
  }

  void sensors(XModel& m) {
    Tok t;
    std::string v;
    while (lx_.next(t)) {
      if (t.kind == Kind::Close && t.name == "sensor") return;
      if (t.kind != Kind::Open) continue;
      XSensor s;
      int ty = lookup(t.name, {"jointpos", "jointvel", "accelerometer", "gyro", "touch", "force", "torque",
                               "framepos", "framequat", "framelinvel", "frameangvel", "subtreecom"});
      s.type = ty < 0 ? 0 : ty;  // unknown sensor elements read as jointpos
      float f;
      if (attr(t.attrs, "joint", v)) s.joint = v;
      if (attr(t.attrs, "objtype", v)) s.objtype = v;
      if (attr(t.attrs, "objname", v)) s.objname = v;
      if (attr(t.attrs, "site", v)) s.site = v;
      if (attr(t.attrs, "noise", v)) s.noise = num(v, f) ? f : 0.0f;
      m.sensors.push_back(s);
    }
  }
};

// ---------------------------------------------------------------- Scene conversion
constexpr float kPi = 3.14159265358979323846f;

float fromto_half_length(const XGeom& g, float fallback) {
  if (!g.has_fromto) return fallback;
  float dx = g.fromto[3] - g.fromto[0], dy = g.fromto[4] - g.fromto[1], dz = g.fromto[5] - g.fromto[2];
  return std::sqrt(dx * dx + dy * dy + dz * dz) * 0.5f;
}

float volume(const XGeom& g) {
  const float k43 = 4.0f / 3.0f;
  const float r = g.size[0];
  switch (g.type) {
    case 1: return k43 * kPi * r * r * r;
    case 4: return 8.0f * g.size[0] * g.size[1] * g.size[2];
    case 2: {
      float hl = fromto_half_length(g, g.size[1]);
      return kPi * r * r * (2.0f * hl) + k43 * kPi * r * r * r;
    }
    case 3: return kPi * r * r * (2.0f * fromto_half_length(g, g.size[1]));
    case 5: return k43 * kPi * r * r * r;
    default: return 1.0f;  // plane, hfield
  }
}

void geom_inertia(const XGeom& g, float m, float I[3]) {
  const float r = g.size[0];
  switch (g.type) {
    case 1:
    case 5: I[0] = I[1] = I[2] = 0.4f * m * r * r; return;
    case 4: {
      float m12 = m / 12.0f, sx = g.size[0] * 2.0f, sy = g.size[1] * 2.0f, sz = g.size[2] * 2.0f;
      I[0] = m12 * (sy * sy + sz * sz);
      I[1] = m12 * (sx * sx + sz * sz);
      I[2] = m12 * (sx * sx + sy * sy);
      return;
    }
    case 2: {  // cylinder plus two hemispherical caps
      float r2 = r * r, h = 2.0f * fromto_half_length(g, g.size[1]), h2 = h * h;
      float total = h + (4.0f / 3.0f) * r;
      float mc = total > 0 ? m * h / total : m;
      float mh = (m - mc) * 0.5f;
      float axial = 0.5f * mc * r2, trans = mc * (3.0f * r2 + h2) / 12.0f;
      float ih = 0.4f * mh * r2, off = h * 0.5f + 0.375f * r;
      float iht = ih + mh * off * off;
      I[0] = trans + 2.0f * iht;
      I[1] = trans + 2.0f * iht;
      I[2] = axial + 2.0f * ih;
      return;
    }
    case 3: {
      float r2 = r * r, h = 2.0f * fromto_half_length(g, g.size[1]);
      I[0] = I[1] = m * (3.0f * r2 + h * h) / 12.0f;
      I[2] = 0.5f * m * r2;
      return;
    }
    default: I[0] = I[1] = I[2] = 0.0f; return;
  }
}

void mass_props(const XBody& b, SBody& out) {
  out.com[0] = out.com[1] = out.com[2] = 0.0f;
  if (b.has_inertial) {  // explicit <inertial>: com offset stays 0
    out.mass = b.in_mass;
    if (b.in_diag) std::memcpy(out.inertia, b.in_diag_v, 12);
    else if (b.in_full) std::memcpy(out.inertia, b.in_full_v, 12);
    else out.inertia[0] = out.inertia[1] = out.inertia[2] = 0.4f * b.in_mass * 0.05f * 0.05f;
    return;
  }
  if (b.geoms.empty()) {
    out.mass = 1.0f;
    out.inertia[0] = out.inertia[1] = out.inertia[2] = 0.0f;
    return;
  }
  float M = 0, I[3] = {0, 0, 0}, c[3] = {0, 0, 0};
  for (const XGeom& g : b.geoms) {
    float gm = g.has_mass ? g.mass : g.density * volume(g);
    float gi[3];
    geom_inertia(g, gm, gi);
    // parallel-axis shift by the geom's pos attribute (fromto midpoints are not used)
    float d2[3] = {g.pos[0] * g.pos[0], g.pos[1] * g.pos[1], g.pos[2] * g.pos[2]};
    I[0] += gi[0] + gm * (d2[1] + d2[2]);
    I[1] += gi[1] + gm * (d2[0] + d2[2]);
    I[2] += gi[2] + gm * (d2[0] + d2[1]);
    for (int k = 0; k < 3; ++k) c[k] += gm * g.pos[k];
    M += gm;
  }
  if (M <= 0) M = 1.0f;
  out.mass = M;
  std::memcpy(out.inertia, I, 12);
  for (int k = 0; k < 3; ++k) out.com[k] = c[k] / M;
}

SGeom to_geom(const XGeom& x, uint32_t body) {
  SGeom g;
  g.body = body;
  std::memcpy(g.pos, x.pos, 12);
  g.quat[0] = x.quat_wxyz[1], g.quat[1] = x.quat_wxyz[2], g.quat[2] = x.quat_wxyz[3], g.quat[3] = x.quat_wxyz[0];
  g.friction = x.friction[0];
  g.contype = x.contype;
  g.conaffinity = x.conaffinity;
  static const uint32_t kType[7] = {3, 0, 1, 4, 2, 5, 6};  // schema order -> primitives order
  g.type = kType[x.type];
  g.size[0] = g.size[1] = g.size[2] = 0.0f;
  switch (x.type) {
    case 1: g.size[0] = x.size[0]; break;
    case 2:
      if (x.has_fromto) {
        const float* f = x.fromto;
        float dx = f[3] - f[0], dy = f[4] - f[1], dz = f[5] - f[2];
        float len = std::sqrt(dx * dx + dy * dy + dz * dz);
        for (int k = 0; k < 3; ++k) g.pos[k] = (f[k] + f[k + 3]) * 0.5f;
        g.size[0] = x.size[0];
        g.size[1] = len * 0.5f;
      } else {
        g.size[0] = x.size[0];
        g.size[1] = x.size[1];
      }
      break;
    case 4: std::memcpy(g.size, x.size, 12); break;
    case 3: g.size[0] = x.size[0], g.size[1] = x.size[1]; break;
    case 5: g.size[0] = 0.1f; break;
    case 6: g.size[0] = g.size[1] = g.size[2] = 1.0f; break;
    default: break;  // plane: zero size
  }
  return g;
}

void euler_quat(const float e[3], float q[4]) {
  float cr = std::cos(e[0] * 0.5f), sr = std::sin(e[0] * 0.5f);
  float cp = std::cos(e[1] * 0.5f), sp = std::sin(e[1] * 0.5f);
  float cy = std::cos(e[2] * 0.5f), sy = std::sin(e[2] * 0.5f);
  q[0] = sr * cp * cy - cr * sp * sy;
  q[1] = cr * sp * cy + sr * cp * sy;
  q[2] = cr * cp * sy - sr * sp * cy;
  q[3] = cr * cp * cy + sr * sp * sy;
}

void add_children(Scene& sc, const XBody& parent, int32_t parent_id, const float parent_pos[3]) {
  for (const XBody& x : parent.kids) {
    SBody b;
    b.name = x.name;
    b.parent = parent_id;
    for (int k = 0; k < 3; ++k) b.pos[k] = x.pos[k] + parent_pos[k];
    if (x.has_euler) euler_quat(x.euler, b.quat);
    else b.quat[0] = x.quat_wxyz[1], b.quat[1] = x.quat_wxyz[2], b.quat[2] = x.quat_wxyz[3], b.quat[3] = x.quat_wxyz[0];
    mass_props(x, b);
    const uint32_t id = uint32_t(sc.bodies.size());
    sc.bodies.push_back(b);
    if (x.joints.empty() && parent_id >= 0) {  // implicit fixed joint
      SJoint j;
      j.type = 0;
      j.parent = uint32_t(parent_id);
      j.child = id;
      std::memcpy(j.anchor_parent, x.pos, 12);
      sc.joints.push_back(j);
    }
    for (const XJoint& xj : x.joints) {
      SJoint j;
      j.name = xj.name;
      j.parent = parent_id >= 0 ? uint32_t(parent_id) : 0u;
      j.child = id;
      for (int k = 0; k < 3; ++k) {
        j.anchor_parent[k] = x.pos[k] + xj.pos[k];
        j.anchor_child[k] = xj.pos[k];
        j.axis[k] = xj.axis[k];
      }
      static const uint32_t kJ[4] = {4, 3, 2, 1};  // free, ball, slide, hinge
      j.type = kJ[xj.type];
      j.damping = xj.damping, j.stiffness = xj.stiffness, j.armature = xj.armature, j.ref = xj.ref;
      if (xj.ranged) j.lower = xj.range[0], j.upper = xj.range[1], j.limited = true;
      if (!j.name.empty()) sc.joint_by_name[j.name] = uint32_t(sc.joints.size());
      sc.joints.push_back(j);
    }
    for (const XGeom& g : x.geoms) sc.geoms.push_back(to_geom(g, id));
    add_children(sc, x, int32_t(id), b.pos);
  }
}

// ---------------------------------------------------------------- corrected semantics
// Frame math of the corrected loader: plain IEEE single precision in written order (the
// file is compiled without contraction), quaternions xyzw.
constexpr float kDeg = 0.017453292519943295f;  // pi / 180

struct Q {
  float x, y, z, w;
};
// quatMultiply order (src/physics/body.zig:238-245)
Q qmul(Q a, Q b) {
  return Q{a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y, a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
           a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w, a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z};
}
// rotateByQuat (src/physics/body.zig:254-264): v + 2 (w (q x v) + q x (q x v))
void qrot(const float v[3], Q q, float o[3]) {
  const float u0 = q.y * v[2] - q.z * v[1], u1 = q.z * v[0] - q.x * v[2], u2 = q.x * v[1] - q.y * v[0];
  const float t0 = q.y * u2 - q.z * u1, t1 = q.z * u0 - q.x * u2, t2 = q.x * u1 - q.y * u0;
  o[0] = v[0] + 2.0f * (q.w * u0 + t0);
  o[1] = v[1] + 2.0f * (q.w * u1 + t1);
  o[2] = v[2] + 2.0f * (q.w * u2 + t2);
}
Q qunit(Q q) {
  const float n = std::sqrt(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
  if (!(n > 0.0f)) return Q{0, 0, 0, 1};
  return Q{q.x / n, q.y / n, q.z / n, q.w / n};
}
Q from_wxyz(const float* q) { return Q{q[1], q[2], q[3], q[0]}; }
// Euler angles in the compiler's sequence: lower-case letters rotate about the moving
// axes (q = q r), upper-case about the fixed axes (q = r q).
Q euler_seq(const float e[3], bool degree, const std::string& seq) {
  Q q{0, 0, 0, 1};
  for (int i = 0; i < 3; ++i) {
    const char c = seq[size_t(i)];
    const int ax = (c | 0x20) - 'x';
    if (ax < 0 || ax > 2) continue;
    const float a = degree ? e[i] * kDeg : e[i];
    const float h = a * 0.5f, s = std::sin(h);
    Q r{0, 0, 0, std::cos(h)};
    (ax == 0 ? r.x : ax == 1 ? r.y : r.z) = s;
    q = (c >= 'a') ? qmul(q, r) : qmul(r, q);
  }
  return q;
}
// Shortest-arc rotation taking local +z onto the direction of d.
Q z_onto(const float d[3]) {
  const float len = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (!(len > 1e-12f)) return Q{0, 0, 0, 1};
  const float ux = d[0] / len, uy = d[1] / len, uz = d[2] / len;
  if (uz < -1.0f + 1e-6f) return Q{1, 0, 0, 0};
  return qunit(Q{-uy, ux, 0.0f, 1.0f + uz});
}
bool fromto_oriented(const XGeom& g) { return g.has_fromto && (g.type == 2 || g.type == 3); }
// Local orientation of a geom: fromto segment, else euler, else the (normalised) quat.
Q geom_quat(const XGeom& g, const XModel& m) {
  if (fromto_oriented(g)) {
    const float d[3] = {g.fromto[3] - g.fromto[0], g.fromto[4] - g.fromto[1], g.fromto[5] - g.fromto[2]};
    return z_onto(d);
  }
  if (g.has_euler) return euler_seq(g.euler, m.angle_degree, m.eulerseq);
  return qunit(from_wxyz(g.quat_wxyz));
}
void geom_centre(const XGeom& g, float c[3]) {
  for (int k = 0; k < 3; ++k) c[k] = fromto_oriented(g) ? (g.fromto[k] + g.fromto[k + 3]) * 0.5f : g.pos[k];
}

SGeom to_geom_corrected(const XGeom& x, uint32_t body, const XModel& m) {
  SGeom g = to_geom(x, body);
  geom_centre(x, g.pos);
  if (x.type == 3 && x.has_fromto) g.size[1] = fromto_half_length(x, x.size[1]);
  const Q q = geom_quat(x, m);
  g.quat[0] = q.x, g.quat[1] = q.y, g.quat[2] = q.z, g.quat[3] = q.w;
  return g;
}

void mass_props_corrected(const XBody& b, SBody& out, const XModel& m) {
  if (b.has_inertial || b.geoms.empty()) {
    mass_props(b, out);
    return;
  }
  out.com[0] = out.com[1] = out.com[2] = 0.0f;
  float M = 0, I[3] = {0, 0, 0}, c[3] = {0, 0, 0};
  for (const XGeom& g : b.geoms) {
    const float gm = g.has_mass ? g.mass : g.density * volume(g);
    float gi[3];
    geom_inertia(g, gm, gi);
    const Q q = geom_quat(g, m);
    const float e0[3] = {1, 0, 0}, e1[3] = {0, 1, 0}, e2[3] = {0, 0, 1};
    float c0[3], c1[3], c2[3];  // columns of the geom's rotation
    qrot(e0, q, c0), qrot(e1, q, c1), qrot(e2, q, c2);
    float d[3];
    geom_centre(g, d);
    const float d2[3] = {d[0] * d[0], d[1] * d[1], d[2] * d[2]};
    for (int k = 0; k < 3; ++k) {
      const float rk = c0[k] * c0[k] * gi[0] + c1[k] * c1[k] * gi[1] + c2[k] * c2[k] * gi[2];
      const float off = k == 0 ? d2[1] + d2[2] : k == 1 ? d2[0] + d2[2] : d2[0] + d2[1];
      I[k] += rk + gm * off;
    }
    for (int k = 0; k < 3; ++k) c[k] += gm * d[k];
    M += gm;
  }
  if (M <= 0) M = 1.0f;
  out.mass = M;
  std::memcpy(out.inertia, I, 12);
  for (int k = 0; k < 3; ++k) out.com[k] = c[k] / M;
}

void add_children_corrected(Scene& sc, const XBody& parent, int32_t parent_id, const float parent_pos[3], Q pq,
                            const XModel& m, std::unordered_map<std::string, uint32_t>& site_body) {
  for (const XBody& x : parent.kids) {
    SBody b;
    b.name = x.name;
    b.parent = parent_id;
    const Q ql = x.has_euler ? euler_seq(x.euler, m.angle_degree, m.eulerseq) : qunit(from_wxyz(x.quat_wxyz));
    float r[3];
    qrot(x.pos, pq, r);
    for (int k = 0; k < 3; ++k) b.pos[k] = parent_pos[k] + r[k];
    const Q qw = qmul(pq, ql);
    b.quat[0] = qw.x, b.quat[1] = qw.y, b.quat[2] = qw.z, b.quat[3] = qw.w;
    mass_props_corrected(x, b, m);
    const uint32_t id = uint32_t(sc.bodies.size());
    sc.bodies.push_back(b);
    if (x.joints.empty() && parent_id >= 0) {  // implicit fixed joint
      SJoint j;
      j.type = 0;
      j.parent = uint32_t(parent_id);
      j.child = id;
      std::memcpy(j.anchor_parent, x.pos, 12);
      sc.joints.push_back(j);
    }
    for (const XJoint& xj : x.joints) {
      SJoint j;
      j.name = xj.name;
      j.parent = parent_id >= 0 ? uint32_t(parent_id) : 0u;
      j.child = id;
      float t[3], a[3];
      qrot(xj.pos, ql, t);
      qrot(xj.axis, ql, a);
      const float n = std::sqrt(a[0] * a[0] + a[1] * a[1] + a[2] * a[2]);
      for (int k = 0; k < 3; ++k) {
        j.anchor_parent[k] = x.pos[k] + t[k];
        j.anchor_child[k] = xj.pos[k];
        j.axis[k] = n > 0.0f ? a[k] / n : xj.axis[k];
      }
      static const uint32_t kJ[4] = {4, 3, 2, 1};  // free, ball, slide, hinge
      j.type = kJ[xj.type];
      j.damping = xj.damping, j.stiffness = xj.stiffness, j.armature = xj.armature, j.ref = xj.ref;
      if (xj.ranged) {
        const bool angular = xj.type == 1 || xj.type == 3;
        const float s = (angular && m.angle_degree) ? kDeg : 1.0f;
        j.lower = angular && m.angle_degree ? xj.range[0] * s : xj.range[0];
        j.upper = angular && m.angle_degree ? xj.range[1] * s : xj.range[1];
        j.limited = true;
      }
      if (!j.name.empty()) sc.joint_by_name[j.name] = uint32_t(sc.joints.size());
      sc.joints.push_back(j);
    }
    for (const XGeom& g : x.geoms) sc.geoms.push_back(to_geom_corrected(g, id, m));
    for (const std::string& s : x.sites)
      if (!s.empty()) site_body.emplace(s, id);
    add_children_corrected(sc, x, int32_t(id), b.pos, qw, m, site_body);
  }
}

// <include file="..."/>: splice the included file's content between its <mujoco> tags.
std::string splice_includes(const std::string& xml, const std::string& dir) {
  if (xml.find("<include") == std::string::npos) return xml;
  std::string out;
  size_t p = 0;
  while (p < xml.size()) {
    size_t at = xml.find("<include", p);
    if (at == std::string::npos) {
      out.append(xml, p, std::string::npos);
      break;
    }
    out.append(xml, p, at - p);
    size_t rel = xml.find("/>", at);
    if (rel == std::string::npos) rel = xml.find('>', at);
    if (rel == std::string::npos) {
      p = at + 8;
      continue;
    }
    size_t tag_end = std::min(rel + 2, xml.size());
    std::string tag = xml.substr(at, tag_end - at);
    size_t fpos = tag.find("file");
    while (fpos != std::string::npos) {
      size_t q = fpos + 4;
      while (q < tag.size() && (tag[q] == ' ' || tag[q] == '=' || tag[q] == '\t')) ++q;
      if (q < tag.size() && (tag[q] == '"' || tag[q] == '\'')) {
        char qc = tag[q];
        size_t e = tag.find(qc, q + 1);
        std::string file = tag.substr(q + 1, (e == std::string::npos ? tag.size() : e) - q - 1);
        std::string path = dir.empty() ? file : dir + "/" + file;
        std::ifstream in(path);
        if (in) {
          std::stringstream ss;
          ss << in.rdbuf();
          size_t slash = path.find_last_of('/');
          std::string sub = splice_includes(ss.str(), slash == std::string::npos ? dir : path.substr(0, slash));
          size_t mb = sub.find("<mujoco"), me = sub.rfind("</mujoco>");
          if (mb != std::string::npos && me != std::string::npos) {
            size_t gt = sub.find('>', mb);
            if (gt != std::string::npos && gt + 1 <= me) sub = sub.substr(gt + 1, me - gt - 1);
          }
          out += sub;
        }
        break;
      }
      fpos = tag.find("file", q);
    }
    p = tag_end;
  }
  return out.empty() ? xml : out;
}

}  // namespace

bool load_mjcf(const std::string& text, const std::string& base_dir, Scene* out, std::string* err,
               bool corrected) {
  XModel m;
  std::string xml = splice_includes(text, base_dir);
  Reader(xml).read(m);
  Scene sc;
  sc.corrected = corrected;
  sc.timestep = m.timestep;
  std::memcpy(sc.gravity, m.gravity, 12);
  SBody world;
  world.name = "world";
  world.type = 0;
  sc.bodies.push_back(world);
  const float origin[3] = {0, 0, 0};
  std::unordered_map<std::string, uint32_t> site_body;
  if (corrected) {
    for (const XGeom& g : m.world.geoms) sc.geoms.push_back(to_geom_corrected(g, 0, m));
    for (const std::string& s : m.world.sites)
      if (!s.empty()) site_body.emplace(s, 0u);
    add_children_corrected(sc, m.world, 0, origin, Q{0, 0, 0, 1}, m, site_body);
  } else {
    for (const XGeom& g : m.world.geoms) sc.geoms.push_back(to_geom(g, 0));
    add_children(sc, m.world, 0, origin);
  }
  for (const XActuator& xa : m.actuators) {
    auto it = xa.joint.empty() ? sc.joint_by_name.end() : sc.joint_by_name.find(xa.joint);
    if (it == sc.joint_by_name.end()) continue;
    SActuator a;
    a.joint = it->second;
    a.gear = xa.gear, a.kp = xa.kp, a.kv = xa.kv;
    if (xa.has_ctrl) a.ctrl_min = xa.ctrl[0], a.ctrl_max = xa.ctrl[1];
    if (xa.has_force) a.force_min = xa.force[0], a.force_max = xa.force[1];
    sc.actuators.push_back(a);
  }
  static const uint32_t kDim[12] = {1, 1, 3, 3, 1, 3, 3, 3, 4, 3, 3, 3};
  for (const XSensor& xs : m.sensors) {
    SSensor s;
    s.type = uint32_t(xs.type);  // schema order equals SensorType values 0..11
    s.dim = kDim[xs.type];
    s.noise = xs.noise;
    if (xs.type <= 1) {
      auto it = xs.joint.empty() ? sc.joint_by_name.end() : sc.joint_by_name.find(xs.joint);
      s.object = it == sc.joint_by_name.end() ? 0u : it->second;
    } else if (corrected) {  // body named by objname (objtype body / xbody), else the site's body
      const bool body_obj = xs.objtype.empty() || xs.objtype == "body" || xs.objtype == "xbody";
      uint32_t obj = 0;
      if (body_obj && !xs.objname.empty()) {
        for (uint32_t i = 0; i < sc.bodies.size(); ++i)
          if (sc.bodies[i].name == xs.objname) {
            obj = i;
            break;
          }
      } else {
        const std::string& site = xs.objtype == "site" ? xs.objname : xs.site;
        auto it = site.empty() ? site_body.end() : site_body.find(site);
        if (it != site_body.end()) obj = it->second;
      }
      s.object = obj;
    }
    sc.sensors.push_back(s);
  }
  if (sc.sensors.empty()) {  // root-body frame sensors plus pos/vel per joint
    uint32_t root = 0;
    for (uint32_t i = 0; i < sc.bodies.size(); ++i)
      if (sc.bodies[i].type == 2 && (corrected ? sc.bodies[i].parent == 0 : sc.bodies[i].parent < 0)) {
        root = i;
        break;
      }
    const uint32_t ft[4] = {7, 8, 9, 10}, fd[4] = {3, 4, 3, 3};
    for (int k = 0; k < 4; ++k) sc.sensors.push_back(SSensor{ft[k], root, fd[k], 0.0f, 0.0f});
    for (uint32_t j = 0; j < sc.joints.size(); ++j) {
      sc.sensors.push_back(SSensor{0, j, 1, 0.0f, 0.0f});
      sc.sensors.push_back(SSensor{1, j, 1, 0.0f, 0.0f});
    }
  }
  *out = std::move(sc);
  (void)err;
  return true;
}

bool load_mjcf_file(const std::string& path, Scene* out, std::string* err, bool corrected) {
  std::ifstream in(path);
  if (!in) {
    if (err) *err = "file not found: " + path;
    return false;
  }
  std::stringstream ss;
  ss << in.rdbuf();
  size_t slash = path.find_last_of('/');
  return load_mjcf(ss.str(), slash == std::string::npos ? "." : path.substr(0, slash), out, err, corrected);
}

}  // namespace zb
