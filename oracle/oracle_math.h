// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle for the batched physics step.
// Nothing in the product (zeno_b200/, include/) may include or link this file.
//
// Canonical single-precision arithmetic for the oracle.  The reference step runs as
// Metal compute kernels compiled with the Metal compiler's default (fast-math) options
// (src/metal/device.zig:51-56 passes no compile options), so its exact rounding is
// unspecified.  The oracle therefore fixes ONE evaluation order: every vector helper
// below is written with explicit fused multiply-adds, IEEE-754 correctly rounded +,-,*,
// and reciprocals / reciprocal square roots built from those by Newton-Raphson (rsq_r,
// rcp_r).  The CUDA kernel evaluates the same expressions in the same order (built with
// -fmad=false, so nvcc adds no contractions of its own), which makes the oracle and the
// GPU bit-identical.  This file is built with -ffp-contract=off.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

namespace zo {

struct F3 { float x, y, z; };
struct F4 { float x, y, z, w; };

// Reciprocal square root and reciprocal by Newton-Raphson from a bit-pattern initial
// guess, residual form, three iterations each (within 1 ulp), from fused multiply-adds and
// products only:
//   rsq_r: y0 from 0x5f375a86 - (bits(x) >> 1) (Lomont, "Fast inverse square root",
//          2003); e = 1 - (x y) y, y = y + (y/2) e; for finite x > 0 (rsq_r(0) is a large
//          finite value, so |v| = d rsq_r(d) is exactly 0 for d = 0);
//   rcp_r: y0 = +-float(0x7ef311c3 - bits(|x|)) (exponent negation); e = 1 - x y,
//          y = y + y e; for finite x != 0 with |x| < 2^125.
// Outside those domains the results are unspecified but deterministic; the step discards
// them through its guards.
static inline uint32_t bits_of(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
}
static inline float float_of(uint32_t u) {
  float x;
  std::memcpy(&x, &u, 4);
  return x;
}
static inline float rsq_r(float x) {
  float y = float_of(0x5f375a86u - (bits_of(x) >> 1));
  y = std::fmaf(0.5f * y, std::fmaf(-(x * y), y, 1.0f), y);
  y = std::fmaf(0.5f * y, std::fmaf(-(x * y), y, 1.0f), y);
  y = std::fmaf(0.5f * y, std::fmaf(-(x * y), y, 1.0f), y);
  return y;
}
static inline float rcp_r(float x) {
  const uint32_t sign = bits_of(x) & 0x80000000u, ax = bits_of(x) & 0x7fffffffu;
  float y = float_of((0x7ef311c3u - ax) | sign);
  y = std::fmaf(y, std::fmaf(-x, y, 1.0f), y);
  y = std::fmaf(y, std::fmaf(-x, y, 1.0f), y);
  y = std::fmaf(y, std::fmaf(-x, y, 1.0f), y);
  return y;
}
static inline float div_r(float a, float b) { return a * rcp_r(b); }

static inline F3 f3(float x, float y, float z) { return F3{x, y, z}; }
static inline F4 f4(float x, float y, float z, float w) { return F4{x, y, z, w}; }
static inline F3 xyz(const F4& q) { return F3{q.x, q.y, q.z}; }

static inline F3 add(F3 a, F3 b) { return F3{a.x + b.x, a.y + b.y, a.z + b.z}; }
static inline F3 sub(F3 a, F3 b) { return F3{a.x - b.x, a.y - b.y, a.z - b.z}; }
static inline F3 mul(F3 a, float s) { return F3{a.x * s, a.y * s, a.z * s}; }
static inline F3 mulv(F3 a, F3 b) { return F3{a.x * b.x, a.y * b.y, a.z * b.z}; }
static inline F3 neg(F3 a) { return F3{-a.x, -a.y, -a.z}; }
// a + b*s with one rounding per component
static inline F3 madd(F3 b, float s, F3 a) {
  return F3{std::fmaf(b.x, s, a.x), std::fmaf(b.y, s, a.y), std::fmaf(b.z, s, a.z)};
}
// a - b*s with one rounding per component
static inline F3 msub(F3 b, float s, F3 a) {
  return F3{std::fmaf(-b.x, s, a.x), std::fmaf(-b.y, s, a.y), std::fmaf(-b.z, s, a.z)};
}
static inline float dot(F3 a, F3 b) {
  return std::fmaf(a.x, b.x, std::fmaf(a.y, b.y, a.z * b.z));
}
static inline F3 cross(F3 a, F3 b) {
  return F3{std::fmaf(a.y, b.z, -(a.z * b.y)), std::fmaf(a.z, b.x, -(a.x * b.z)),
            std::fmaf(a.x, b.y, -(a.y * b.x))};
}
// |a| = d rsq(d) with d = a.a; unit() also returns a / |a| as a * rsq(d)
static inline float length(F3 a) {
  const float d = dot(a, a);
  return d * rsq_r(d);
}
static inline F3 unit(F3 a, float* l) {
  const float d = dot(a, a);
  const float inv = rsq_r(d);
  *l = d * inv;
  return F3{a.x * inv, a.y * inv, a.z * inv};
}

static inline F4 qmul(F4 a, F4 b) {
  return F4{std::fmaf(a.w, b.x, std::fmaf(a.x, b.w, std::fmaf(a.y, b.z, -(a.z * b.y)))),
            std::fmaf(a.w, b.y, std::fmaf(-a.x, b.z, std::fmaf(a.y, b.w, a.z * b.x))),
            std::fmaf(a.w, b.z, std::fmaf(a.x, b.y, std::fmaf(-a.y, b.x, a.z * b.w))),
            std::fmaf(a.w, b.w, -std::fmaf(a.x, b.x, std::fmaf(a.y, b.y, a.z * b.z)))};
}
static inline F4 qconj(F4 q) { return F4{-q.x, -q.y, -q.z, q.w}; }
static inline F4 qneg(F4 q) { return F4{-q.x, -q.y, -q.z, -q.w}; }
// q + d*s
static inline F4 qmadd(F4 d, float s, F4 q) {
  return F4{std::fmaf(d.x, s, q.x), std::fmaf(d.y, s, q.y), std::fmaf(d.z, s, q.z),
            std::fmaf(d.w, s, q.w)};
}
// q - d*s
static inline F4 qmsub(F4 d, float s, F4 q) {
  return F4{std::fmaf(-d.x, s, q.x), std::fmaf(-d.y, s, q.y), std::fmaf(-d.z, s, q.z),
            std::fmaf(-d.w, s, q.w)};
}
// all_shaders.metal:99-102 quat_normalize: len > 1e-8 ? q/len : identity.
// Canonical form: inv = rsq(|q|^2), len = |q|^2 inv, four products.
static inline F4 qnormalize(F4 q) {
  const float d = std::fmaf(q.x, q.x, std::fmaf(q.y, q.y, std::fmaf(q.z, q.z, q.w * q.w)));
  const float inv = rsq_r(d);
  if (d * inv > 1e-8f) return F4{q.x * inv, q.y * inv, q.z * inv, q.w * inv};
  return F4{0.f, 0.f, 0.f, 1.f};
}
// all_shaders.metal:92-97 rotate_by_quat: v + 2*(w*(qv x v) + qv x (qv x v))
static inline F3 rotate(F3 v, F4 q) {
  F3 qv{q.x, q.y, q.z};
  F3 uv = cross(qv, v);
  F3 uuv = cross(qv, uv);
  return F3{std::fmaf(2.0f, std::fmaf(q.w, uv.x, uuv.x), v.x),
            std::fmaf(2.0f, std::fmaf(q.w, uv.y, uuv.y), v.y),
            std::fmaf(2.0f, std::fmaf(q.w, uv.z, uuv.z), v.z)};
}

// ---------------------------------------------------------------------------------
// Reproducible arctangent.  atan(a) on [0,1] is a * P(a^2) with a degree-8 polynomial
// fitted (weighted least squares towards minimax relative error, see
// zeno_b200/csrc/fit_atan_poly.py) to 1.5e-8 relative error; evaluated by Horner with
// fused multiply-adds it is within 1.5 ulp of the true value.  atan2 reduces to that
// interval with one reciprocal (rcp_r) and the usual octant identities.  Special values: a zero
// denominator and numerator give +0 (or pi for x<0); a NaN operand returns NaN.  The CUDA kernel carries an identical restatement.
// ---------------------------------------------------------------------------------
static const float kAtanC[9] = {1.0f,
                                -0.33333075046539307f,
                                0.1999262422323227f,
                                -0.14203670620918274f,
                                0.1064101979136467f,
                                -0.07504455000162125f,
                                0.04269323870539665f,
                                -0.016069602221250534f,
                                0.002850116929039359f};
static const float kPi = 3.14159265358979f;
static const float kHalfPi = 1.57079632679490f;

static inline float atan_unit(float a) {  // a in [0,1]
  float s = a * a;
  float p = kAtanC[8];
  p = std::fmaf(p, s, kAtanC[7]);
  p = std::fmaf(p, s, kAtanC[6]);
  p = std::fmaf(p, s, kAtanC[5]);
  p = std::fmaf(p, s, kAtanC[4]);
  p = std::fmaf(p, s, kAtanC[3]);
  p = std::fmaf(p, s, kAtanC[2]);
  p = std::fmaf(p, s, kAtanC[1]);
  p = std::fmaf(p, s, kAtanC[0]);
  return a * p;
}

static inline float atan2_r(float y, float x) {
  if (x != x || y != y) return x + y;  // NaN in, NaN out
  float ax = std::fabs(x), ay = std::fabs(y);
  float mx = ax > ay ? ax : ay;
  float mn = ax > ay ? ay : ax;
  float a = (mx == 0.0f) ? 0.0f : mn * rcp_r(mx);
  float r = atan_unit(a);
  if (ay > ax) r = kHalfPi - r;
  if (x < 0.0f) r = kPi - r;
  if (y < 0.0f) r = -r;
  return r;
}

// asin(x) for x in [-1, 1] by the classic range reduction (Cody & Waite): |x| <= 1/2:
// a + a z P(z) with z = a^2; above: pi/2 - 2 (s + s z P(z)) with z = (1 - a)/2 and
// s = sqrt(z) = z rsq(z).  P: degree 4 on [0, 1/4] (zeno_b200/csrc/fit_asin_poly.py),
// Horner with fused multiply-adds; within 2.4 ulp.  The CUDA kernel carries an identical
// restatement.
static inline float asin_r(float x) {
  const float a = std::fabs(x);
  const bool small = a <= 0.5f;
  float z, s;
  if (small) {
    z = a * a;
    s = a;
  } else {
    z = 0.5f * (1.0f - a);
    s = z * rsq_r(z);
  }
  float p = 0.0421663373708725f;
  p = std::fmaf(p, z, 0.024179499596357346f);
  p = std::fmaf(p, z, 0.045470379292964935f);
  p = std::fmaf(p, z, 0.07495297491550446f);
  p = std::fmaf(p, z, 0.16666752099990845f);
  const float t = std::fmaf(s * z, p, s);
  const float r = small ? t : std::fmaf(-2.0f, t, kHalfPi);
  return x < 0.0f ? -r : r;
}

static inline float clampf(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }

}  // namespace zo
