// Reproducible single-precision vector math for the step kernel.
//
// The reference evaluates these expressions in Metal with the compiler's default
// fast-math settings, so its rounding is unspecified.  This build fixes one canonical
// evaluation order -- explicit fused multiply-adds (__fmaf_rn), correctly rounded +, -, *,
// and reciprocals / reciprocal square roots built from those (rsq_, rcp_) -- and compiles
// with -fmad=false so nvcc adds no contractions of its own.  Every operation is then
// IEEE-754 deterministic, and the results are bit-identical to any other implementation
// that evaluates the same expressions in the same order (the CPU oracle does).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace zb {

struct V3 {
  float x, y, z;
};

__device__ __forceinline__ V3 v3(float x, float y, float z) { return V3{x, y, z}; }
__device__ __forceinline__ V3 v3(float4 a) { return V3{a.x, a.y, a.z}; }
__device__ __forceinline__ float fma_(float a, float b, float c) { return __fmaf_rn(a, b, c); }
// Reciprocal square root and reciprocal from multiplies and fused multiply-adds only
// (Newton-Raphson from a bit-pattern initial guess, residual form), three iterations
// each: within 1 ulp, deterministic, and reproducible by any implementation that runs the
// same steps.
//   rsq_: y0 from the bit trick 0x5f375a86 - (bits(x) >> 1) (Lomont, "Fast inverse square
//         root", 2003); e = 1 - (x y) y, y = y + (y/2) e.  For finite x > 0; rsq_(0) is a
//         large finite value, so |v| = d rsq_(d) is exactly 0 for d = 0.
//   rcp_: y0 = +-float(0x7ef311c3 - bits(|x|)) (exponent negation, relative error < 13 %);
//         e = 1 - x y, y = y + y e.  For finite x != 0 with |x| < 2^125.
// Outside those domains the results are unspecified (but still deterministic); every use
// in the step kernels sits behind a guard that discards such a result.
__device__ __forceinline__ float rsq_(float x) {
  float y = __uint_as_float(0x5f375a86u - (__float_as_uint(x) >> 1));
  y = fma_(0.5f * y, fma_(-(x * y), y, 1.0f), y);
  y = fma_(0.5f * y, fma_(-(x * y), y, 1.0f), y);
  y = fma_(0.5f * y, fma_(-(x * y), y, 1.0f), y);
  return y;
}
__device__ __forceinline__ float rcp_(float x) {
  const uint32_t sign = __float_as_uint(x) & 0x80000000u, ax = __float_as_uint(x) & 0x7fffffffu;
  float y = __uint_as_float((0x7ef311c3u - ax) | sign);
  y = fma_(y, fma_(-x, y, 1.0f), y);
  y = fma_(y, fma_(-x, y, 1.0f), y);
  y = fma_(y, fma_(-x, y, 1.0f), y);
  return y;
}
__device__ __forceinline__ float div_(float a, float b) { return a * rcp_(b); }

__device__ __forceinline__ V3 operator+(V3 a, V3 b) { return V3{a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ V3 operator-(V3 a, V3 b) { return V3{a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ V3 operator-(V3 a) { return V3{-a.x, -a.y, -a.z}; }
__device__ __forceinline__ V3 operator*(V3 a, float s) { return V3{a.x * s, a.y * s, a.z * s}; }
__device__ __forceinline__ V3 hadamard(V3 a, V3 b) { return V3{a.x * b.x, a.y * b.y, a.z * b.z}; }
// a + b*s, a - b*s (one rounding per component)
__device__ __forceinline__ V3 madd(V3 b, float s, V3 a) {
  return V3{fma_(b.x, s, a.x), fma_(b.y, s, a.y), fma_(b.z, s, a.z)};
}
__device__ __forceinline__ V3 msub(V3 b, float s, V3 a) {
  return V3{fma_(-b.x, s, a.x), fma_(-b.y, s, a.y), fma_(-b.z, s, a.z)};
}
__device__ __forceinline__ float dot(V3 a, V3 b) { return fma_(a.x, b.x, fma_(a.y, b.y, a.z * b.z)); }
__device__ __forceinline__ V3 cross(V3 a, V3 b) {
  return V3{fma_(a.y, b.z, -(a.z * b.y)), fma_(a.z, b.x, -(a.x * b.z)), fma_(a.x, b.y, -(a.y * b.x))};
}
// |a| = d rsq(d), d = a.a; unit(a, l) also returns a / |a| as a * rsq(d).
__device__ __forceinline__ float len(V3 a) {
  const float d = dot(a, a);
  return d * rsq_(d);
}
__device__ __forceinline__ V3 unit(V3 a, float& l) {
  const float d = dot(a, a);
  const float inv = rsq_(d);
  l = d * inv;
  return a * inv;
}

__device__ __forceinline__ float4 qmul(float4 a, float4 b) {
  return make_float4(fma_(a.w, b.x, fma_(a.x, b.w, fma_(a.y, b.z, -(a.z * b.y)))),
                     fma_(a.w, b.y, fma_(-a.x, b.z, fma_(a.y, b.w, a.z * b.x))),
                     fma_(a.w, b.z, fma_(a.x, b.y, fma_(-a.y, b.x, a.z * b.w))),
                     fma_(a.w, b.w, -fma_(a.x, b.x, fma_(a.y, b.y, a.z * b.z))));
}
// (v, 0) (x) q
__device__ __forceinline__ float4 qmul_v(V3 v, float4 b) { return qmul(make_float4(v.x, v.y, v.z, 0.0f), b); }
__device__ __forceinline__ float4 qconj(float4 q) { return make_float4(-q.x, -q.y, -q.z, q.w); }
__device__ __forceinline__ float4 qneg(float4 q) { return make_float4(-q.x, -q.y, -q.z, -q.w); }
__device__ __forceinline__ float4 qmadd(float4 d, float s, float4 q) {
  return make_float4(fma_(d.x, s, q.x), fma_(d.y, s, q.y), fma_(d.z, s, q.z), fma_(d.w, s, q.w));
}
__device__ __forceinline__ float4 qmsub(float4 d, float s, float4 q) {
  return make_float4(fma_(-d.x, s, q.x), fma_(-d.y, s, q.y), fma_(-d.z, s, q.z), fma_(-d.w, s, q.w));
}
// quat_normalize (all_shaders.metal:99-102): len > 1e-8 ? q * (1/len) : identity.
// Written as a select (the reciprocal is computed either way): no branch on the chain.
__device__ __forceinline__ float4 qnormalize(float4 q) {
  const float d = fma_(q.x, q.x, fma_(q.y, q.y, fma_(q.z, q.z, q.w * q.w)));
  const float inv = rsq_(d);
  const bool ok = d * inv > 1e-8f;
  return make_float4(ok ? q.x * inv : 0.0f, ok ? q.y * inv : 0.0f, ok ? q.z * inv : 0.0f, ok ? q.w * inv : 1.0f);
}
// c ? a : b per component
__device__ __forceinline__ float4 sel4(bool c, float4 a, float4 b) {
  return make_float4(c ? a.x : b.x, c ? a.y : b.y, c ? a.z : b.z, c ? a.w : b.w);
}
// rotate_by_quat (all_shaders.metal:92-97): v + 2*(w*(qv x v) + qv x (qv x v))
__device__ __forceinline__ V3 rotate(V3 v, float4 q) {
  V3 qv{q.x, q.y, q.z};
  V3 uv = cross(qv, v);
  V3 uuv = cross(qv, uv);
  return V3{fma_(2.0f, fma_(q.w, uv.x, uuv.x), v.x), fma_(2.0f, fma_(q.w, uv.y, uuv.y), v.y),
            fma_(2.0f, fma_(q.w, uv.z, uuv.z), v.z)};
}
__device__ __forceinline__ V3 xyz(float4 q) { return V3{q.x, q.y, q.z}; }
__device__ __forceinline__ float4 with_w(V3 v, float w) { return make_float4(v.x, v.y, v.z, w); }
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

// Arctangent from IEEE operations only.  atan(a) on [0,1] = a * P(a^2), P of degree 8
// fitted towards minimax relative error (zeno_b200/csrc/fit_atan_poly.py; 1.5e-8
// relative, <= 1.5 ulp in float with Horner FMAs).  atan2 reduces by octant with one
// division.  Zero/zero gives +0 (pi for x < 0); NaN in gives NaN out.
__device__ __forceinline__ float atan_unit(float a) {
  float s = a * a;
  float p = 0.002850116929039359f;
  p = fma_(p, s, -0.016069602221250534f);
  p = fma_(p, s, 0.04269323870539665f);
  p = fma_(p, s, -0.07504455000162125f);
  p = fma_(p, s, 0.1064101979136467f);
  p = fma_(p, s, -0.14203670620918274f);
  p = fma_(p, s, 0.1999262422323227f);
  p = fma_(p, s, -0.33333075046539307f);
  p = fma_(p, s, 1.0f);
  return a * p;
}
__device__ __forceinline__ float atan2r(float y, float x) {
  if (x != x || y != y) return x + y;
  float ax = fabsf(x), ay = fabsf(y);
  float mx = ax > ay ? ax : ay;
  float mn = ax > ay ? ay : ax;
  float a = (mx == 0.0f) ? 0.0f : mn * rcp_(mx);
  float r = atan_unit(a);
  if (ay > ax) r = 1.57079632679490f - r;
  if (x < 0.0f) r = 3.14159265358979f - r;
  if (y < 0.0f) r = -r;
  return r;
}
// Arcsine with the classic range reduction (Cody & Waite): |x| <= 1/2: a + a z P(z),
// z = a^2; above: pi/2 - 2 (s + s z P(z)), z = (1 - a)/2, s = sqrt(z) = z rsq(z).  P of
// degree 4 on [0, 1/4] fitted by zeno_b200/csrc/fit_asin_poly.py; within 2.4 ulp.  The
// branch skips the square root where the joint solver's small angles fall.
__device__ __forceinline__ float asinr(float x) {
  const float a = fabsf(x);
  const bool small = a <= 0.5f;
  float z, s;
  if (small) {
    z = a * a;
    s = a;
  } else {
    z = 0.5f * (1.0f - a);
    s = z * rsq_(z);
  }
  float p = 0.0421663373708725f;
  p = fma_(p, z, 0.024179499596357346f);
  p = fma_(p, z, 0.045470379292964935f);
  p = fma_(p, z, 0.07495297491550446f);
  p = fma_(p, z, 0.16666752099990845f);
  const float t = fma_(s * z, p, s);
  const float r = small ? t : fma_(-2.0f, t, 1.57079632679490f);
  return x < 0.0f ? -r : r;
}

// splitmix64 finalizer (counter-based random numbers for the episode-reset extension)
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float uniform_pm1(uint64_t seed, uint64_t env, uint32_t episode, uint32_t k) {
  uint64_t h = mix64(mix64(mix64(seed) ^ env) ^ ((uint64_t(episode) << 32) | k));
  float u = float(uint32_t(h >> 40)) * (1.0f / 16777216.0f);
  return 2.0f * u - 1.0f;
}

}  // namespace zb
