// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle for the batched physics step.
// Nothing in the product (zeno_b200/, include/) may include or link this file.
//
// Serial restatement of the reference MJCF loader: XmlTokenizer / getAttr / number
// parsing (src/mjcf/parser.zig:1340-1587), element parsing (parser.zig:184-822), schema
// defaults (src/mjcf/schema.zig:100-199), and the Scene conversion
// (parser.zig:826-1337: convertToScene, processBody, computeBodyMassInertia, geomMass,
// geomVolume, geomInertia, convertGeom, convertSensor, eulerToQuat).
// Include directives (parser.zig:55-171) are not restated: the oracle is fed complete
// MJCF text.
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "oracle_model.h"

namespace zo {
namespace {

const float kPiF = 3.14159265358979323846f;  // std.math.pi as f32

bool is_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

struct Token {
  enum Kind { Start, End, Text, Comment } kind;
  std::string name;
  std::string attrs;
};

// parser.zig:1353-1457 XmlTokenizer
struct Tokenizer {
  const std::string& s;
  size_t pos = 0;
  explicit Tokenizer(const std::string& src) : s(src) {}
  void skip_ws() {
    while (pos < s.size() && is_ws(s[pos])) pos++;
  }
  bool next(Token* t) {
    skip_ws();
    if (pos >= s.size()) return false;
    if (s[pos] == '<') return tag(t);
    size_t st = pos;
    while (pos < s.size() && s[pos] != '<') pos++;
    t->kind = Token::Text;
    t->name = s.substr(st, pos - st);
    t->attrs.clear();
    return true;
  }
  bool tag(Token* t) {
    pos++;
    if (pos >= s.size()) return false;
    if (s.size() - pos >= 3 && s.compare(pos, 3, "!--") == 0) {
      while (pos + 2 < s.size()) {
        if (s[pos] == '-' && s[pos + 1] == '-' && s[pos + 2] == '>') {
          pos += 3;
          break;
        }
        pos++;
      }
      t->kind = Token::Comment;
      t->name.clear();
      t->attrs.clear();
      return true;
    }
    bool is_end = s[pos] == '/';
    if (is_end) pos++;
    size_t ns = pos;
    while (pos < s.size() && !is_ws(s[pos]) && s[pos] != '>' && s[pos] != '/') pos++;
    t->name = s.substr(ns, pos - ns);
    skip_ws();
    size_t as = pos;
    while (pos < s.size() && s[pos] != '>') pos++;
    size_t ae = pos;
    if (!is_end) {
      size_t chk = pos;
      while (chk > as && is_ws(s[chk - 1])) chk--;
      if (chk > as && s[chk - 1] == '/') ae = chk - 1;
    }
    t->attrs = s.substr(as, ae - as);
    if (pos < s.size()) pos++;
    t->kind = is_end ? Token::End : Token::Start;
    if (is_end) t->attrs.clear();
    return true;
  }
};

// parser.zig:1463-1503 getAttr: first attribute with that exact name
bool get_attr(const std::string& a, const char* name, std::string* out) {
  size_t pos = 0;
  while (pos < a.size()) {
    while (pos < a.size() && is_ws(a[pos])) pos++;
    size_t ns = pos;
    while (pos < a.size() && a[pos] != '=' && !is_ws(a[pos])) pos++;
    std::string an = a.substr(ns, pos - ns);
    while (pos < a.size() && (is_ws(a[pos]) || a[pos] == '=')) pos++;
    if (pos >= a.size()) break;
    char q = a[pos];
    if (q != '"' && q != '\'') continue;
    pos++;
    size_t vs = pos;
    while (pos < a.size() && a[pos] != q) pos++;
    std::string v = a.substr(vs, pos - vs);
    pos++;
    if (an == name) {
      *out = v;
      return true;
    }
  }
  return false;
}

// std.fmt.parseFloat(f32): whole string must be a number (no surrounding whitespace)
bool parse_float(const std::string& s, float* out) {
  if (s.empty() || is_ws(s[0])) return false;
  errno = 0;
  char* end = nullptr;
  float v = std::strtof(s.c_str(), &end);
  if (end != s.c_str() + s.size()) return false;
  *out = v;
  return true;
}

// std.fmt.parseInt(u32, s, 10)
bool parse_u32(const std::string& s, uint32_t* out) {
  size_t i = 0;
  if (!s.empty() && s[0] == '+') i = 1;
  if (i >= s.size()) return false;
  uint64_t v = 0;
  for (; i < s.size(); i++) {
    if (s[i] < '0' || s[i] > '9') return false;
    v = v * 10 + uint64_t(s[i] - '0');
    if (v > 0xFFFFFFFFull) return false;
  }
  *out = uint32_t(v);
  return true;
}

// std.mem.splitScalar(u8, s, ' '): empty fields are kept
std::vector<std::string> split_space(const std::string& s) {
  std::vector<std::string> r;
  size_t st = 0;
  for (size_t i = 0; i <= s.size(); i++) {
    if (i == s.size() || s[i] == ' ') {
      r.push_back(s.substr(st, i - st));
      st = i + 1;
    }
  }
  return r;
}

bool parse_vecn(const std::string& s, int n, float* out) {
  auto parts = split_space(s);
  float tmp[8];
  for (int i = 0; i < n; i++) {
    if (i >= int(parts.size())) return false;
    if (!parse_float(parts[i], &tmp[i])) return false;
  }
  for (int i = 0; i < n; i++) out[i] = tmp[i];
  return true;
}

// parseSize: up to three fields, unparsable fields become 0
void parse_size(const std::string& s, float out[3]) {
  out[0] = out[1] = out[2] = 0;
  auto parts = split_space(s);
  for (size_t i = 0; i < parts.size() && i < 3; i++) {
    float v;
    out[i] = parse_float(parts[i], &v) ? v : 0.0f;
  }
}

// ----- schema.zig structures -----
enum MGeomType { GPlane, GSphere, GCapsule, GCylinder, GBox, GMesh, GHfield };
enum MJointType { JFree, JBall, JSlide, JHinge };
enum MActType { AMotor, APosition, AVelocity, AGeneral };

struct MJoint {
  std::string name;
  MJointType type = JHinge;
  float pos[3] = {0, 0, 0};
  float axis[3] = {0, 0, 1};
  bool has_range = false;
  float range[2] = {0, 0};
  bool limited = false;
  float damping = 0, stiffness = 0, armature = 0, ref = 0;
};
struct MGeom {
  std::string name;
  MGeomType type = GSphere;
  float pos[3] = {0, 0, 0};
  float quat[4] = {1, 0, 0, 0};  // wxyz
  float size[3] = {0.05f, 0, 0};
  bool has_fromto = false;
  float fromto[6] = {0, 0, 0, 0, 0, 0};
  bool has_euler = false;  // corrected loader only
  float euler[3] = {0, 0, 0};
  bool has_mass = false;
  float mass = 0;
  float density = 1000;
  float friction[3] = {1, 0.005f, 0.0001f};
  uint32_t contype = 1, conaffinity = 1;
};
struct MInertial {
  float mass = 1.0f;
  bool has_diag = false, has_full = false;
  float diag[3] = {0, 0, 0};
  float full[6] = {0, 0, 0, 0, 0, 0};
};
struct MBody {
  std::string name;
  float pos[3] = {0, 0, 0};
  float quat[4] = {1, 0, 0, 0};
  bool has_euler = false;
  float euler[3] = {0, 0, 0};
  bool has_inertial = false;
  MInertial inertial;
  std::vector<MJoint> joints;
  std::vector<MGeom> geoms;
  std::vector<MBody> children;
  std::vector<std::string> sites;  // corrected loader only
};
struct MActuator {
  std::string joint;
  MActType type = AMotor;
  bool has_ctrl = false, has_force = false;
  float ctrl[2] = {0, 0}, force[2] = {0, 0};
  float gear = 1, kp = 0, kv = 0;
};
enum MSensType { SJointPos, SJointVel, SAccel, SGyro, STouch, SForce, STorque, SFramePos, SFrameQuat,
                 SFrameLinVel, SFrameAngVel, SSubtreeCom };
struct MSensor {
  MSensType type = SJointPos;
  std::string joint;
  std::string objtype, objname, site;  // corrected loader only
  float noise = 0;
};
struct MDefault {
  MJoint joint;
  MGeom geom;
};
struct MModel {
  float timestep = 0.002f;
  float gravity[3] = {0, 0, -9.81f};
  bool degree = true;            // <compiler angle> (corrected loader only)
  std::string eulerseq = "xyz";  // <compiler eulerseq> (corrected loader only)
  std::map<std::string, MDefault> defaults;
  MBody world;
  std::vector<MActuator> actuators;
  std::vector<MSensor> sensors;
};

bool geom_type_from(const std::string& s, MGeomType* t) {
  static const std::map<std::string, MGeomType> m = {{"plane", GPlane}, {"sphere", GSphere},
                                                     {"capsule", GCapsule}, {"cylinder", GCylinder},
                                                     {"box", GBox}, {"mesh", GMesh}, {"hfield", GHfield}};
  auto it = m.find(s);
  if (it == m.end()) return false;
  *t = it->second;
  return true;
}
bool joint_type_from(const std::string& s, MJointType* t) {
  static const std::map<std::string, MJointType> m = {
      {"free", JFree}, {"ball", JBall}, {"slide", JSlide}, {"hinge", JHinge}};
  auto it = m.find(s);
  if (it == m.end()) return false;
  *t = it->second;
  return true;
}
bool sensor_type_from(const std::string& s, MSensType* t) {
  static const std::map<std::string, MSensType> m = {
      {"jointpos", SJointPos},       {"jointvel", SJointVel},       {"accelerometer", SAccel},
      {"gyro", SGyro},               {"touch", STouch},             {"force", SForce},
      {"torque", STorque},           {"framepos", SFramePos},       {"framequat", SFrameQuat},
      {"framelinvel", SFrameLinVel}, {"frameangvel", SFrameAngVel}, {"subtreecom", SSubtreeCom}};
  auto it = m.find(s);
  if (it == m.end()) return false;
  *t = it->second;
  return true;
}

// parser.zig:424-462 applyJointAttrs
void apply_joint_attrs(MJoint* j, const std::string& a) {
  std::string v;
  if (get_attr(a, "name", &v)) j->name = v;
  if (get_attr(a, "type", &v)) joint_type_from(v, &j->type);
  if (get_attr(a, "pos", &v)) parse_vecn(v, 3, j->pos);
  if (get_attr(a, "axis", &v)) parse_vecn(v, 3, j->axis);
  if (get_attr(a, "range", &v)) {
    float r[2];
    j->has_range = parse_vecn(v, 2, r);
    if (j->has_range) {
      j->range[0] = r[0];
      j->range[1] = r[1];
    }
    j->limited = j->has_range;
  }
  float f;
  if (get_attr(a, "damping", &v) && parse_float(v, &f)) j->damping = f;
  if (get_attr(a, "stiffness", &v) && parse_float(v, &f)) j->stiffness = f;
  if (get_attr(a, "armature", &v) && parse_float(v, &f)) j->armature = f;
  if (get_attr(a, "ref", &v) && parse_float(v, &f)) j->ref = f;
}

// parser.zig:482-542 applyGeomAttrs
void apply_geom_attrs(MGeom* g, const std::string& a) {
  std::string v;
  if (get_attr(a, "name", &v)) g->name = v;
  if (get_attr(a, "type", &v)) geom_type_from(v, &g->type);
  if (get_attr(a, "pos", &v)) parse_vecn(v, 3, g->pos);
  if (get_attr(a, "quat", &v)) parse_vecn(v, 4, g->quat);
  if (get_attr(a, "size", &v)) parse_size(v, g->size);
  if (get_attr(a, "fromto", &v)) {
    float ft[6];
    g->has_fromto = parse_vecn(v, 6, ft);
    if (g->has_fromto) std::memcpy(g->fromto, ft, sizeof(ft));
  }
  float f;
  if (get_attr(a, "mass", &v)) {
    g->has_mass = parse_float(v, &f);
    if (g->has_mass) g->mass = f;
  }
  if (get_attr(a, "density", &v) && parse_float(v, &f)) g->density = f;
  if (get_attr(a, "friction", &v)) parse_vecn(v, 3, g->friction);
  uint32_t u;
  if (get_attr(a, "contype", &v) && parse_u32(v, &u)) g->contype = u;
  if (get_attr(a, "conaffinity", &v) && parse_u32(v, &u)) g->conaffinity = u;
  if (get_attr(a, "mesh", &v)) g->type = GMesh;
  if (get_attr(a, "euler", &v)) g->has_euler = parse_vecn(v, 3, g->euler);
}

MJoint joint_with_defaults(const std::string& a, const MModel& m, const std::string& cls) {
  std::string use = cls;
  std::string c;
  if (get_attr(a, "class", &c)) use = c;
  auto it = m.defaults.find(use);
  MJoint j = it != m.defaults.end() ? it->second.joint : MJoint{};
  apply_joint_attrs(&j, a);
  return j;
}
MGeom geom_with_defaults(const std::string& a, const MModel& m, const std::string& cls) {
  std::string use = cls;
  std::string c;
  if (get_attr(a, "class", &c)) use = c;
  auto it = m.defaults.find(use);
  MGeom g = it != m.defaults.end() ? it->second.geom : MGeom{};
  apply_geom_attrs(&g, a);
  return g;
}

// parser.zig:326-370 parseBodyContent
void parse_body_content(Tokenizer& tk, MModel& m, MBody* body, const std::string& end_tag,
                        const std::string& cls) {
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == end_tag) break;
    if (t.kind != Token::Start) continue;
    std::string v;
    if (t.name == "body") {
      MBody ch;
      if (get_attr(t.attrs, "name", &v)) ch.name = v;
      if (get_attr(t.attrs, "pos", &v) && !parse_vecn(v, 3, ch.pos)) ch.pos[0] = ch.pos[1] = ch.pos[2] = 0;
      if (get_attr(t.attrs, "quat", &v) && !parse_vecn(v, 4, ch.quat)) {
        ch.quat[0] = 1;
        ch.quat[1] = ch.quat[2] = ch.quat[3] = 0;
      }
      if (get_attr(t.attrs, "euler", &v)) ch.has_euler = parse_vecn(v, 3, ch.euler);
      std::string cc = cls;
      if (get_attr(t.attrs, "childclass", &v)) cc = v;
      parse_body_content(tk, m, &ch, "body", cc);
      body->children.push_back(ch);
    } else if (t.name == "joint") {
      body->joints.push_back(joint_with_defaults(t.attrs, m, cls));
    } else if (t.name == "geom") {
      body->geoms.push_back(geom_with_defaults(t.attrs, m, cls));
    } else if (t.name == "site") {
      body->sites.push_back(get_attr(t.attrs, "name", &v) ? v : std::string());
    } else if (t.name == "inertial") {
      MInertial in;
      float f;
      if (get_attr(t.attrs, "mass", &v)) in.mass = parse_float(v, &f) ? f : 1.0f;
      if (get_attr(t.attrs, "diaginertia", &v)) in.has_diag = parse_vecn(v, 3, in.diag);
      if (get_attr(t.attrs, "fullinertia", &v)) in.has_full = parse_vecn(v, 6, in.full);
      body->has_inertial = true;
      body->inertial = in;
    }
  }
}

// parser.zig:772-822 parseDefaults
void parse_defaults(Tokenizer& tk, MModel& m) {
  std::string cls = "main";
  MDefault cur;
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == "default") {
      if (!cls.empty()) m.defaults[cls] = cur;
      break;
    }
    if (t.kind != Token::Start) continue;
    std::string v;
    if (t.name == "default") {
      if (!cls.empty()) m.defaults[cls] = cur;
      cls = get_attr(t.attrs, "class", &v) ? v : std::string("main");
      cur = MDefault{};
    } else if (t.name == "geom") {
      cur.geom = MGeom{};
      apply_geom_attrs(&cur.geom, t.attrs);
    } else if (t.name == "joint") {
      cur.joint = MJoint{};
      apply_joint_attrs(&cur.joint, t.attrs);
    }
  }
}

void parse_actuators(Tokenizer& tk, MModel& m) {
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == "actuator") break;
    if (t.kind != Token::Start) continue;
    if (t.name != "motor" && t.name != "position" && t.name != "velocity" && t.name != "general") continue;
    MActuator a;
    a.type = t.name == "motor" ? AMotor : t.name == "position" ? APosition : t.name == "velocity" ? AVelocity : AGeneral;
    std::string v;
    if (get_attr(t.attrs, "joint", &v)) a.joint = v;
    if (get_attr(t.attrs, "ctrlrange", &v)) a.has_ctrl = parse_vecn(v, 2, a.ctrl);
    if (get_attr(t.attrs, "forcerange", &v)) a.has_force = parse_vecn(v, 2, a.force);
    float f;
    if (get_attr(t.attrs, "gear", &v)) a.gear = parse_float(v, &f) ? f : 1.0f;
    if (get_attr(t.attrs, "kp", &v)) a.kp = parse_float(v, &f) ? f : 0.0f;
    if (get_attr(t.attrs, "kv", &v)) a.kv = parse_float(v, &f) ? f : 0.0f;
    m.actuators.push_back(a);
  }
}

void parse_sensors(Tokenizer& tk, MModel& m) {
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == "sensor") break;
    if (t.kind != Token::Start) continue;
    MSensor s;
    if (!sensor_type_from(t.name, &s.type)) s.type = SJointPos;
    std::string v;
    if (get_attr(t.attrs, "joint", &v)) s.joint = v;
    if (get_attr(t.attrs, "objtype", &v)) s.objtype = v;
    if (get_attr(t.attrs, "objname", &v)) s.objname = v;
    if (get_attr(t.attrs, "site", &v)) s.site = v;
    float f;
    if (get_attr(t.attrs, "noise", &v)) s.noise = parse_float(v, &f) ? f : 0.0f;
    m.sensors.push_back(s);
  }
}

// Skip the content of an element that the reference parses but which does not reach
// the Scene (asset, tendon, equality): consume tokens to the matching end tag name.
void skip_to_end(Tokenizer& tk, const char* name) {
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == name) break;
  }
}

void parse_mujoco(Tokenizer& tk, MModel& m) {
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::End && t.name == "mujoco") break;
    if (t.kind != Token::Start) continue;
    std::string v;
    if (t.name == "option") {
      m.timestep = 0.002f;
      m.gravity[0] = 0;
      m.gravity[1] = 0;
      m.gravity[2] = -9.81f;
      float f;
      if (get_attr(t.attrs, "timestep", &v)) m.timestep = parse_float(v, &f) ? f : 0.002f;
      if (get_attr(t.attrs, "gravity", &v) && !parse_vecn(v, 3, m.gravity)) {
        m.gravity[0] = 0;
        m.gravity[1] = 0;
        m.gravity[2] = -9.81f;
      }
    } else if (t.name == "compiler") {
      if (get_attr(t.attrs, "angle", &v)) m.degree = !(v == "radian");
      if (get_attr(t.attrs, "eulerseq", &v) && v.size() == 3) m.eulerseq = v;
    } else if (t.name == "default") {
      parse_defaults(tk, m);
    } else if (t.name == "asset") {
      skip_to_end(tk, "asset");
    } else if (t.name == "worldbody") {
      parse_body_content(tk, m, &m.world, "worldbody", "main");
    } else if (t.name == "actuator") {
      parse_actuators(tk, m);
    } else if (t.name == "sensor") {
      parse_sensors(tk, m);
    } else if (t.name == "tendon") {
      skip_to_end(tk, "tendon");
    } else if (t.name == "equality") {
      skip_to_end(tk, "equality");
    }
  }
}

// ----- conversion (parser.zig:826-1337) -----
float geom_volume(const MGeom& g) {
  const float pi = kPiF;
  const float four_thirds = 4.0f / 3.0f;
  auto half_len_of = [&](float hl) {
    if (g.has_fromto) {
      float dx = g.fromto[3] - g.fromto[0];
      float dy = g.fromto[4] - g.fromto[1];
      float dz = g.fromto[5] - g.fromto[2];
      hl = std::sqrt(dx * dx + dy * dy + dz * dz) * 0.5f;
    }
    return hl;
  };
  switch (g.type) {
    case GSphere: return four_thirds * pi * g.size[0] * g.size[0] * g.size[0];
    case GBox: return 8.0f * g.size[0] * g.size[1] * g.size[2];
    case GCapsule: {
      float r = g.size[0];
      float hl = half_len_of(g.size[1]);
      float cyl = pi * r * r * (2.0f * hl);
      float sph = four_thirds * pi * r * r * r;
      return cyl + sph;
    }
    case GCylinder: {
      float r = g.size[0];
      float hl = half_len_of(g.size[1]);
      return pi * r * r * (2.0f * hl);
    }
    case GPlane: return 1.0f;
    case GMesh: {
      float r = g.size[0];
      return four_thirds * pi * r * r * r;
    }
    case GHfield: return 1.0f;
  }
  return 1.0f;
}

float geom_mass(const MGeom& g) {
  if (g.has_mass) return g.mass;
  return g.density * geom_volume(g);
}

void geom_inertia(const MGeom& g, float mass, float out[3]) {
  auto half_len_of = [&](float hl) {
    if (g.has_fromto) {
      float dx = g.fromto[3] - g.fromto[0];
      float dy = g.fromto[4] - g.fromto[1];
      float dz = g.fromto[5] - g.fromto[2];
      hl = std::sqrt(dx * dx + dy * dy + dz * dz) * 0.5f;
    }
    return hl;
  };
  switch (g.type) {
    case GSphere: {
      float r = g.size[0];
      float i = 0.4f * mass * r * r;
      out[0] = out[1] = out[2] = i;
      return;
    }
    case GBox: {
      float m12 = mass / 12.0f;
      float sx = g.size[0] * 2.0f, sy = g.size[1] * 2.0f, sz = g.size[2] * 2.0f;
      out[0] = m12 * (sy * sy + sz * sz);
      out[1] = m12 * (sx * sx + sz * sz);
      out[2] = m12 * (sx * sx + sy * sy);
      return;
    }
    case GCapsule: {
      float r = g.size[0];
      float hl = half_len_of(g.size[1]);
      float r2 = r * r;
      float h = 2.0f * hl;
      float h2 = h * h;
      float total_h = h + (4.0f / 3.0f) * r;
      float m_cyl = total_h > 0 ? mass * h / total_h : mass;
      float m_hem = (mass - m_cyl) * 0.5f;
      float i_cyl_axial = 0.5f * m_cyl * r2;
      float i_cyl_trans = m_cyl * (3.0f * r2 + h2) / 12.0f;
      float i_hem = 0.4f * m_hem * r2;
      float offset = h * 0.5f + 0.375f * r;
      float i_hem_trans = i_hem + m_hem * offset * offset;
      out[0] = i_cyl_trans + 2.0f * i_hem_trans;
      out[1] = i_cyl_trans + 2.0f * i_hem_trans;
      out[2] = i_cyl_axial + 2.0f * i_hem;
      return;
    }
    case GCylinder: {
      float r = g.size[0];
      float hl = half_len_of(g.size[1]);
      float r2 = r * r;
      float h = 2.0f * hl;
      out[0] = mass * (3.0f * r2 + h * h) / 12.0f;
      out[1] = mass * (3.0f * r2 + h * h) / 12.0f;
      out[2] = 0.5f * mass * r2;
      return;
    }
    case GMesh: {
      float r = g.size[0];
      float i = 0.4f * mass * r * r;
      out[0] = out[1] = out[2] = i;
      return;
    }
    case GPlane:
    case GHfield: out[0] = out[1] = out[2] = 0; return;
  }
}

void body_mass_inertia(const MBody& b, float* mass, float inertia[3], float com[3]) {
  com[0] = com[1] = com[2] = 0;
  if (b.has_inertial) {
    *mass = b.inertial.mass;
    if (b.inertial.has_diag) {
      std::memcpy(inertia, b.inertial.diag, 12);
    } else if (b.inertial.has_full) {
      std::memcpy(inertia, b.inertial.full, 12);
    } else {
      float r = 0.05f;
      float i = 0.4f * b.inertial.mass * r * r;
      inertia[0] = inertia[1] = inertia[2] = i;
    }
    return;
  }
  if (b.geoms.empty()) {
    *mass = 1.0f;
    inertia[0] = inertia[1] = inertia[2] = 0;
    return;
  }
  float tm = 0, ti[3] = {0, 0, 0}, c[3] = {0, 0, 0};
  for (const MGeom& g : b.geoms) {
    float gm = geom_mass(g);
    float gi[3] = {0, 0, 0};
    geom_inertia(g, gm, gi);
    const float* d = g.pos;
    float dsq[3] = {d[0] * d[0], d[1] * d[1], d[2] * d[2]};
    ti[0] += gi[0] + gm * (dsq[1] + dsq[2]);
    ti[1] += gi[1] + gm * (dsq[0] + dsq[2]);
    ti[2] += gi[2] + gm * (dsq[0] + dsq[1]);
    c[0] += gm * d[0];
    c[1] += gm * d[1];
    c[2] += gm * d[2];
    tm += gm;
  }
  if (tm <= 0) tm = 1.0f;
  *mass = tm;
  std::memcpy(inertia, ti, 12);
  com[0] = c[0] / tm;
  com[1] = c[1] / tm;
  com[2] = c[2] / tm;
}

GeomDef convert_geom(const MGeom& mg) {
  GeomDef g;
  std::memcpy(g.pos, mg.pos, 12);
  g.quat[0] = mg.quat[1];
  g.quat[1] = mg.quat[2];
  g.quat[2] = mg.quat[3];
  g.quat[3] = mg.quat[0];
  g.friction = mg.friction[0];
  g.contype = mg.contype;
  g.conaffinity = mg.conaffinity;
  switch (mg.type) {
    case GSphere: g.type = kSphere; g.size[0] = mg.size[0]; g.size[1] = 0; g.size[2] = 0; break;
    case GCapsule:
      g.type = kCapsule;
      if (mg.has_fromto) {
        const float* f = mg.fromto;
        float dx = f[3] - f[0], dy = f[4] - f[1], dz = f[5] - f[2];
        float len = std::sqrt(dx * dx + dy * dy + dz * dz);
        g.pos[0] = (f[0] + f[3]) * 0.5f;
        g.pos[1] = (f[1] + f[4]) * 0.5f;
        g.pos[2] = (f[2] + f[5]) * 0.5f;
        g.size[0] = mg.size[0];
        g.size[1] = len * 0.5f;
        g.size[2] = 0;
      } else {
        g.size[0] = mg.size[0];
        g.size[1] = mg.size[1];
        g.size[2] = 0;
      }
      break;
    case GBox: g.type = kBox; std::memcpy(g.size, mg.size, 12); break;
    case GCylinder: g.type = kCylinder; g.size[0] = mg.size[0]; g.size[1] = mg.size[1]; g.size[2] = 0; break;
    case GPlane: g.type = kPlane; g.size[0] = g.size[1] = g.size[2] = 0; break;
    case GMesh: g.type = kMesh; g.size[0] = 0.1f; g.size[1] = 0; g.size[2] = 0; break;
    case GHfield: g.type = kHeightfield; g.size[0] = g.size[1] = g.size[2] = 1; break;
  }
  return g;
}

void euler_to_quat(const float e[3], float q[4]) {
  float cr = std::cos(e[0] * 0.5f), sr = std::sin(e[0] * 0.5f);
  float cp = std::cos(e[1] * 0.5f), sp = std::sin(e[1] * 0.5f);
  float cy = std::cos(e[2] * 0.5f), sy = std::sin(e[2] * 0.5f);
  q[0] = sr * cp * cy - cr * sp * sy;
  q[1] = cr * sp * cy + sr * cp * sy;
  q[2] = cr * cp * sy - sr * sp * cy;
  q[3] = cr * cp * cy + sr * sp * sy;
}

void process_body(Scene* sc, const MBody& mb, int32_t parent_id, const float ppos[3]) {
  for (const MBody& ch : mb.children) {
    float pos[3] = {ch.pos[0] + ppos[0], ch.pos[1] + ppos[1], ch.pos[2] + ppos[2]};
    float q[4];
    if (ch.has_euler) {
      euler_to_quat(ch.euler, q);
    } else {
      q[0] = ch.quat[1];
      q[1] = ch.quat[2];
      q[2] = ch.quat[3];
      q[3] = ch.quat[0];
    }
    bool has_joints = !ch.joints.empty();
    BodyDef bd;
    bd.name = ch.name;
    bd.parent = parent_id;
    bd.type = kDynamic;
    std::memcpy(bd.pos, pos, 12);
    std::memcpy(bd.quat, q, 16);
    body_mass_inertia(ch, &bd.mass, bd.inertia, bd.com);
    uint32_t bid = uint32_t(sc->bodies.size());
    sc->bodies.push_back(bd);
    if (!ch.name.empty()) sc->body_names[ch.name] = bid;
    if (!has_joints && parent_id >= 0) {
      JointDef jd;
      jd.type = kFixed;
      jd.parent = uint32_t(parent_id);
      jd.child = bid;
      std::memcpy(jd.anchor_parent, ch.pos, 12);
      sc->joints.push_back(jd);
    }
    for (const MJoint& mj : ch.joints) {
      JointDef jd;
      jd.name = mj.name;
      jd.parent = parent_id >= 0 ? uint32_t(parent_id) : 0u;
      jd.child = bid;
      for (int k = 0; k < 3; k++) {
        jd.anchor_parent[k] = ch.pos[k] + mj.pos[k];
        jd.anchor_child[k] = mj.pos[k];
        jd.axis[k] = mj.axis[k];
      }
      jd.damping = mj.damping;
      jd.stiffness = mj.stiffness;
      jd.armature = mj.armature;
      jd.ref = mj.ref;
      jd.type = mj.type == JFree ? kFree : mj.type == JBall ? kBall : mj.type == JSlide ? kPrismatic : kRevolute;
      if (mj.has_range) {
        jd.lower = mj.range[0];
        jd.upper = mj.range[1];
        jd.limited = true;
      }
      uint32_t jid = uint32_t(sc->joints.size());
      sc->joints.push_back(jd);
      if (!mj.name.empty()) sc->joint_names[mj.name] = jid;
    }
    for (const MGeom& mg : ch.geoms) {
      GeomDef g = convert_geom(mg);
      g.body = bid;
      sc->geoms.push_back(g);
    }
    process_body(sc, ch, int32_t(bid), pos);
  }
}

// ----- corrected semantics (not the reference's behaviour) -----
// The MJCF compiler rules of MuJoCo's documentation that the reference loader skips:
// angle units (<compiler angle>, default degree) for hinge/ball ranges and euler angles;
// euler sequences (<compiler eulerseq>, default "xyz", lower case = moving axes); body
// frames composed with the parent's rotation; joint pos/axis given in the child frame
// (moved into the parent frame, where the constraints read them; axes normalised); geom
// orientation (quat, euler, fromto segment for capsules and cylinders) and fromto centres;
// body inertia from rotated geom inertia (the diagonal is kept); frame/site sensors
// resolved to their body; automatic sensors on the world's first child.  Plain IEEE
// single precision in written order.
constexpr float kDegF = 0.017453292519943295f;  // pi / 180

struct Qt {
  float x, y, z, w;
};
Qt qt_mul(Qt a, Qt b) {  // quatMultiply (body.zig:238-245)
  Qt r;
  r.x = a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y;
  r.y = a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x;
  r.z = a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w;
  r.w = a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z;
  return r;
}
void qt_rot(const float v[3], Qt q, float o[3]) {  // rotateByQuat (body.zig:254-264)
  float uv[3] = {q.y * v[2] - q.z * v[1], q.z * v[0] - q.x * v[2], q.x * v[1] - q.y * v[0]};
  float uuv[3] = {q.y * uv[2] - q.z * uv[1], q.z * uv[0] - q.x * uv[2], q.x * uv[1] - q.y * uv[0]};
  for (int k = 0; k < 3; k++) o[k] = v[k] + 2.0f * (q.w * uv[k] + uuv[k]);
}
Qt qt_unit(Qt q) {
  float n = std::sqrt(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
  if (!(n > 0.0f)) return Qt{0, 0, 0, 1};
  return Qt{q.x / n, q.y / n, q.z / n, q.w / n};
}
Qt qt_from_wxyz(const float* q) { return Qt{q[1], q[2], q[3], q[0]}; }
Qt euler_rotation(const float e[3], bool degree, const std::string& seq) {
  Qt q{0, 0, 0, 1};
  for (int i = 0; i < 3; i++) {
    char c = seq[size_t(i)];
    int axis = (c | 0x20) - 'x';
    if (axis < 0 || axis > 2) continue;
    float ang = degree ? e[i] * kDegF : e[i];
    float half = ang * 0.5f;
    Qt r{0, 0, 0, std::cos(half)};
    float s = std::sin(half);
    if (axis == 0) r.x = s;
    else if (axis == 1) r.y = s;
    else r.z = s;
    bool moving_axes = c >= 'a';
    q = moving_axes ? qt_mul(q, r) : qt_mul(r, q);
  }
  return q;
}
Qt z_to_dir(const float d[3]) {  // shortest arc from local +z onto d
  float len = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (!(len > 1e-12f)) return Qt{0, 0, 0, 1};
  float ux = d[0] / len, uy = d[1] / len, uz = d[2] / len;
  if (uz < -1.0f + 1e-6f) return Qt{1, 0, 0, 0};
  return qt_unit(Qt{-uy, ux, 0.0f, 1.0f + uz});
}
bool oriented_by_fromto(const MGeom& g) { return g.has_fromto && (g.type == GCapsule || g.type == GCylinder); }
Qt geom_local_quat(const MGeom& g, const MModel& m) {
  if (oriented_by_fromto(g)) {
    float d[3] = {g.fromto[3] - g.fromto[0], g.fromto[4] - g.fromto[1], g.fromto[5] - g.fromto[2]};
    return z_to_dir(d);
  }
  if (g.has_euler) return euler_rotation(g.euler, m.degree, m.eulerseq);
  return qt_unit(qt_from_wxyz(g.quat));
}
void geom_local_centre(const MGeom& g, float c[3]) {
  for (int k = 0; k < 3; k++) c[k] = oriented_by_fromto(g) ? (g.fromto[k] + g.fromto[k + 3]) * 0.5f : g.pos[k];
}

GeomDef convert_geom_corrected(const MGeom& mg, const MModel& m) {
  GeomDef g = convert_geom(mg);
  geom_local_centre(mg, g.pos);
  if (mg.type == GCylinder && mg.has_fromto) {
    const float* f = mg.fromto;
    float dx = f[3] - f[0], dy = f[4] - f[1], dz = f[5] - f[2];
    g.size[1] = std::sqrt(dx * dx + dy * dy + dz * dz) * 0.5f;
  }
  Qt q = geom_local_quat(mg, m);
  g.quat[0] = q.x;
  g.quat[1] = q.y;
  g.quat[2] = q.z;
  g.quat[3] = q.w;
  return g;
}

void body_mass_inertia_corrected(const MBody& b, const MModel& m, float* mass, float inertia[3], float com[3]) {
  if (b.has_inertial || b.geoms.empty()) {
    body_mass_inertia(b, mass, inertia, com);
    return;
  }
  float tm = 0, ti[3] = {0, 0, 0}, c[3] = {0, 0, 0};
  for (const MGeom& g : b.geoms) {
    float gm = geom_mass(g);
    float gi[3] = {0, 0, 0};
    geom_inertia(g, gm, gi);
    Qt q = geom_local_quat(g, m);
    const float ex[3] = {1, 0, 0}, ey[3] = {0, 1, 0}, ez[3] = {0, 0, 1};
    float rx[3], ry[3], rz[3];  // rotated geom axes = columns of the rotation
    qt_rot(ex, q, rx);
    qt_rot(ey, q, ry);
    qt_rot(ez, q, rz);
    float d[3];
    geom_local_centre(g, d);
    float dsq[3] = {d[0] * d[0], d[1] * d[1], d[2] * d[2]};
    for (int k = 0; k < 3; k++) {
      float diag = rx[k] * rx[k] * gi[0] + ry[k] * ry[k] * gi[1] + rz[k] * rz[k] * gi[2];
      float perp = k == 0 ? dsq[1] + dsq[2] : (k == 1 ? dsq[0] + dsq[2] : dsq[0] + dsq[1]);
      ti[k] += diag + gm * perp;
    }
    for (int k = 0; k < 3; k++) c[k] += gm * d[k];
    tm += gm;
  }
  if (tm <= 0) tm = 1.0f;
  *mass = tm;
  std::memcpy(inertia, ti, 12);
  for (int k = 0; k < 3; k++) com[k] = c[k] / tm;
}

void process_body_corrected(Scene* sc, const MBody& mb, int32_t parent_id, const float ppos[3], Qt pq,
                            const MModel& m, std::map<std::string, uint32_t>* site_body) {
  for (const MBody& ch : mb.children) {
    Qt ql = ch.has_euler ? euler_rotation(ch.euler, m.degree, m.eulerseq) : qt_unit(qt_from_wxyz(ch.quat));
    float off[3];
    qt_rot(ch.pos, pq, off);
    float pos[3] = {ppos[0] + off[0], ppos[1] + off[1], ppos[2] + off[2]};
    Qt qw = qt_mul(pq, ql);
    BodyDef bd;
    bd.name = ch.name;
    bd.parent = parent_id;
    bd.type = kDynamic;
    std::memcpy(bd.pos, pos, 12);
    bd.quat[0] = qw.x;
    bd.quat[1] = qw.y;
    bd.quat[2] = qw.z;
    bd.quat[3] = qw.w;
    body_mass_inertia_corrected(ch, m, &bd.mass, bd.inertia, bd.com);
    uint32_t bid = uint32_t(sc->bodies.size());
    sc->bodies.push_back(bd);
    if (!ch.name.empty()) sc->body_names[ch.name] = bid;
    if (ch.joints.empty() && parent_id >= 0) {
      JointDef jd;
      jd.type = kFixed;
      jd.parent = uint32_t(parent_id);
      jd.child = bid;
      std::memcpy(jd.anchor_parent, ch.pos, 12);
      sc->joints.push_back(jd);
    }
    for (const MJoint& mj : ch.joints) {
      JointDef jd;
      jd.name = mj.name;
      jd.parent = parent_id >= 0 ? uint32_t(parent_id) : 0u;
      jd.child = bid;
      float jp[3], ax[3];
      qt_rot(mj.pos, ql, jp);
      qt_rot(mj.axis, ql, ax);
      float n = std::sqrt(ax[0] * ax[0] + ax[1] * ax[1] + ax[2] * ax[2]);
      for (int k = 0; k < 3; k++) {
        jd.anchor_parent[k] = ch.pos[k] + jp[k];
        jd.anchor_child[k] = mj.pos[k];
        jd.axis[k] = n > 0.0f ? ax[k] / n : mj.axis[k];
      }
      jd.damping = mj.damping;
      jd.stiffness = mj.stiffness;
      jd.armature = mj.armature;
      jd.ref = mj.ref;
      jd.type = mj.type == JFree ? kFree : mj.type == JBall ? kBall : mj.type == JSlide ? kPrismatic : kRevolute;
      if (mj.has_range) {
        bool angular = mj.type == JHinge || mj.type == JBall;
        jd.lower = (angular && m.degree) ? mj.range[0] * kDegF : mj.range[0];
        jd.upper = (angular && m.degree) ? mj.range[1] * kDegF : mj.range[1];
        jd.limited = true;
      }
      uint32_t jid = uint32_t(sc->joints.size());
      sc->joints.push_back(jd);
      if (!mj.name.empty()) sc->joint_names[mj.name] = jid;
    }
    for (const MGeom& mg : ch.geoms) {
      GeomDef g = convert_geom_corrected(mg, m);
      g.body = bid;
      sc->geoms.push_back(g);
    }
    for (const std::string& s : ch.sites)
      if (!s.empty()) site_body->emplace(s, bid);
    process_body_corrected(sc, ch, int32_t(bid), pos, qw, m, site_body);
  }
}

}  // namespace

float BodyDef::inv_mass() const {
  if (type == kStatic || type == kKinematic || mass <= 0.0f) return 0.0f;
  return 1.0f / mass;
}
void BodyDef::inv_inertia(float o[3]) const {
  if (type == kStatic || type == kKinematic) {
    o[0] = o[1] = o[2] = 0;
    return;
  }
  for (int i = 0; i < 3; i++) o[i] = inertia[i] > 1e-6f ? 1.0f / inertia[i] : 0.0f;
}

bool parse_mjcf(const std::string& xml, Scene* sc, bool corrected) {
  MModel m;
  Tokenizer tk(xml);
  Token t;
  while (tk.next(&t)) {
    if (t.kind == Token::Start && t.name == "mujoco") {
      parse_mujoco(tk, m);
      break;
    }
  }
  *sc = Scene{};
  sc->corrected = corrected;
  sc->timestep = m.timestep;
  std::memcpy(sc->gravity, m.gravity, 12);
  BodyDef world;
  world.name = "world";
  world.type = kStatic;
  sc->bodies.push_back(world);
  sc->body_names["world"] = 0;
  std::map<std::string, uint32_t> site_body;
  for (const MGeom& mg : m.world.geoms) {
    GeomDef g = corrected ? convert_geom_corrected(mg, m) : convert_geom(mg);
    g.body = 0;
    sc->geoms.push_back(g);
  }
  float zero[3] = {0, 0, 0};
  if (corrected) {
    for (const std::string& s : m.world.sites)
      if (!s.empty()) site_body.emplace(s, 0u);
    process_body_corrected(sc, m.world, 0, zero, Qt{0, 0, 0, 1}, m, &site_body);
  } else {
    process_body(sc, m.world, 0, zero);
  }
  for (const MActuator& ma : m.actuators) {
    auto it = sc->joint_names.find(ma.joint);
    if (ma.joint.empty() || it == sc->joint_names.end()) continue;
    ActuatorDef a;
    a.joint = it->second;
    a.gear = ma.gear;
    a.kp = ma.kp;
    a.kv = ma.kv;
    if (ma.has_ctrl) {
      a.ctrl_min = ma.ctrl[0];
      a.ctrl_max = ma.ctrl[1];
    }
    if (ma.has_force) {
      a.force_min = ma.force[0];
      a.force_max = ma.force[1];
    }
    sc->actuators.push_back(a);
  }
  for (const MSensor& ms : m.sensors) {
    SensorDef s;
    s.noise = ms.noise;
    auto joint_id = [&]() -> uint32_t {
      auto it = sc->joint_names.find(ms.joint);
      return (ms.joint.empty() || it == sc->joint_names.end()) ? 0u : it->second;
    };
    // corrected: non-joint sensors observe the body named by objname (objtype body /
    // xbody), else the body holding the site
    auto body_id = [&]() -> uint32_t {
      if (!corrected) return 0u;
      bool body_obj = ms.objtype.empty() || ms.objtype == "body" || ms.objtype == "xbody";
      if (body_obj && !ms.objname.empty()) {
        for (uint32_t i = 0; i < sc->bodies.size(); i++)
          if (sc->bodies[i].name == ms.objname) return i;
        return 0u;
      }
      const std::string& site = ms.objtype == "site" ? ms.objname : ms.site;
      auto it = site.empty() ? site_body.end() : site_body.find(site);
      return it == site_body.end() ? 0u : it->second;
    };
    s.object = body_id();
    switch (ms.type) {
      case SJointPos: s.type = kJointPos; s.object = joint_id(); s.dim = 1; break;
      case SJointVel: s.type = kJointVel; s.object = joint_id(); s.dim = 1; break;
      case SAccel: s.type = kAccelerometer; s.dim = 3; break;
      case SGyro: s.type = kGyro; s.dim = 3; break;
      case STouch: s.type = kTouch; s.dim = 1; break;
      case SForce: s.type = kForce; s.dim = 3; break;
      case STorque: s.type = kTorque; s.dim = 3; break;
      case SFramePos: s.type = kFramePos; s.dim = 3; break;
      case SFrameQuat: s.type = kFrameQuat; s.dim = 4; break;
      case SFrameLinVel: s.type = kFrameLinVel; s.dim = 3; break;
      case SFrameAngVel: s.type = kFrameAngVel; s.dim = 3; break;
      case SSubtreeCom: s.type = kSubtreeCom; s.dim = 3; break;
    }
    sc->sensors.push_back(s);
  }
  if (sc->sensors.empty()) {  // scene.zig:211-226 autoAddSensors -> sensors.zig:191-207
    uint32_t root = 0;
    for (size_t i = 0; i < sc->bodies.size(); i++) {
      if (sc->bodies[i].type == kDynamic && (corrected ? sc->bodies[i].parent == 0 : sc->bodies[i].parent < 0)) {
        root = uint32_t(i);
        break;
      }
    }
    SensorType ft[4] = {kFramePos, kFrameQuat, kFrameLinVel, kFrameAngVel};
    uint32_t fd[4] = {3, 4, 3, 3};
    for (int k = 0; k < 4; k++) {
      SensorDef s;
      s.type = ft[k];
      s.object = root;
      s.dim = fd[k];
      sc->sensors.push_back(s);
    }
    for (uint32_t j = 0; j < sc->joints.size(); j++) {
      SensorDef a, b;
      a.type = kJointPos;
      a.object = j;
      b.type = kJointVel;
      b.object = j;
      sc->sensors.push_back(a);
      sc->sensors.push_back(b);
    }
  }
  return true;
}

}  // namespace zo
