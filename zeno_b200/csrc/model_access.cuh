// Model accessors for the physics templates of physics.cuh.
//   ModelS reads the FModel hot image in shared memory (environment-per-lane kernel).
//   ModelG reads the device tables (general kernel).
#pragma once
#include <stdint.h>

#include "fast_model.h"
#include "physics.cuh"
#include "zeno_types.h"

namespace zb {

// The hot image of an FModel, copied into shared memory by each block; every read is a
// warp-uniform broadcast.  Offsets come from the FModel kernel parameter.
struct ModelS {
  const unsigned char* h;
  const FModel& f;
  template <class T>
  __device__ __forceinline__ T at(uint32_t off, uint32_t i) const {
    return reinterpret_cast<const T*>(h + off)[i];
  }
  __device__ __forceinline__ float4 imi(uint32_t b) const { return at<float4>(f.o_imi, b); }
  __device__ __forceinline__ float4 com(uint32_t b) const { return at<float4>(f.o_com, b); }
  __device__ __forceinline__ uint32_t body(uint32_t b) const { return at<uint32_t>(f.o_body, b); }
  __device__ __forceinline__ uint32_t jf(uint32_t k) const { return at<uint32_t>(f.o_jf, k); }
  __device__ __forceinline__ float4 jaxis(uint32_t j) const { return at<float4>(f.o_jaxis, j); }
  __device__ __forceinline__ uint32_t jinfo(uint32_t j) const { return at<uint32_t>(f.o_jinfo, j); }
  __device__ __forceinline__ ConstraintV constraint(uint32_t k) const {
    const uint32_t i = at<uint32_t>(f.o_cinfo, k);
    return ConstraintV{i & 0xFFu, (i >> 8) & 0xFFu, (i >> 16) & 0xFFu, at<float4>(f.o_caa, k), at<float4>(f.o_cab, k),
                       at<float4>(f.o_cat, k), at<float4>(f.o_clim, k)};
  }
  __device__ __forceinline__ uint32_t pbody(uint32_t p) const { return at<uint32_t>(f.o_pbody, p); }
  __device__ __forceinline__ uint32_t pinfo(uint32_t p) const { return at<uint32_t>(f.o_pinfo, p); }
  __device__ __forceinline__ float pmd2(uint32_t p) const { return at<float>(f.o_pmd2, p); }
  __device__ __forceinline__ float4 gps(uint32_t g) const { return at<float4>(f.o_gps, g); }
  __device__ __forceinline__ uint32_t hinfo(uint32_t x) const { return at<uint32_t>(f.o_hinfo, x); }
  __device__ __forceinline__ float4 hga(uint32_t x) const { return at<float4>(f.o_hga, x); }
  __device__ __forceinline__ float4 hgb(uint32_t x) const { return at<float4>(f.o_hgb, x); }
  __device__ __forceinline__ float4 hcax(uint32_t x) const { return at<float4>(f.o_hcax, x); }
  __device__ __forceinline__ float hhl(uint32_t x) const { return at<float>(f.o_hhl, x); }
  __device__ __forceinline__ float hfr(uint32_t x) const { return at<float>(f.o_hfr, x); }
  __device__ __forceinline__ uint32_t hpair(uint32_t x) const { return at<uint32_t>(f.o_hpair, x); }
  __device__ __forceinline__ float4 hsz(uint32_t x) const { return at<float4>(f.o_hsz, x); }
  __device__ __forceinline__ uint32_t gbody(uint32_t g) const { return at<uint32_t>(f.o_gbody, g); }
  __device__ __forceinline__ uint32_t ggpair(uint32_t ga, uint32_t gb) const { return h[f.o_ggpair + ga * f.G + gb]; }
  __device__ __forceinline__ float4 gforce(uint32_t b) const { return at<float4>(f.o_gforce, b); }
  __device__ __forceinline__ uint32_t run(uint32_t r) const { return at<uint32_t>(f.o_runs, r); }
  __device__ __forceinline__ uint32_t group(uint32_t g) const { return at<uint32_t>(f.o_groups, g); }
  __device__ __forceinline__ uint32_t glv(uint32_t v) const { return at<uint32_t>(f.o_glv, v); }
  __device__ __forceinline__ uint32_t gword(uint32_t g) const { return at<uint32_t>(f.o_gwords, g); }
};

struct ModelG {
  const DBody* bodies;
  const DConstraint* constraints;
  __device__ __forceinline__ float4 imi(uint32_t b) const {
    return __ldg(reinterpret_cast<const float4*>(bodies[b].inv_mass_inertia));
  }
  __device__ __forceinline__ float4 com(uint32_t b) const { return __ldg(reinterpret_cast<const float4*>(bodies[b].com)); }
  __device__ __forceinline__ ConstraintV constraint(uint32_t k) const {
    const DConstraint& d = constraints[k];
    return ConstraintV{__ldg(&d.body_a), __ldg(&d.body_b), __ldg(&d.type) & 0xFFu,
                       __ldg(reinterpret_cast<const float4*>(d.anchor_a)),
                       __ldg(reinterpret_cast<const float4*>(d.anchor_b)),
                       __ldg(reinterpret_cast<const float4*>(d.axis_target)),
                       __ldg(reinterpret_cast<const float4*>(d.limits))};
  }
};

}  // namespace zb
