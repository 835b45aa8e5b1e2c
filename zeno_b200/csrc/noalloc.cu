// zeno_world_reset_to_state_noalloc: the reset_to_state operation without any device
// allocation.
//
// zeno_world_reset_to_state stages the caller's host arrays in device memory before the
// masked copy kernel scatters them into the world; that staging buffer comes from
// cudaMallocAsync on every call.  Some callers cannot allocate device memory at that
// point: a process whose remaining HBM is already reserved by another allocator (for
// example a training framework's caching allocator), or a control loop that must not
// risk an allocation blocking or failing in the middle of an episode.  This entry point
// stages through a fixed array in the library's own static device memory instead and
// calls no cudaMalloc / cudaFree / allocating library routine.
//
// Limits and sharing:
//  * capacity: kStagingFloat4 float4 = 16 MiB, so num_envs * num_bodies must be at most
//    1,048,576; larger worlds are rejected with ZENO_INVALID_ARGUMENT and a message in
//    zeno_last_error().
//  * every GPU that loads libzeno.so holds this array until the process exits.
//  * one array per device, shared by every call and every world on that device; it keeps
//    the last call's contents.  Nothing needs clearing: each call writes every element it
//    later reads.  Calls that overlap on the GPU (different worlds on one device stepping
//    on different streams at the same time) race on the array; serialize them.
//  * the first call on a device resolves the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call before any
//    stream capture.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/zeno.h"
#include "world.h"

namespace {

constexpr size_t kStagingFloat4 = size_t(1) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float4 g_noalloc_staging[kStagingFloat4];

std::mutex g_setup_mu;
float* g_staging_ptr[kMaxDevices] = {};

// Device address of the staging array on `dev` (resolved once per device, with `dev`
// current).  Returns nullptr and fills *err on failure.
float* staging_for(int dev, std::string* err) {
  if (dev < 0 || dev >= kMaxDevices) {
    *err = "device ordinal out of range";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_staging_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_staging);
    if (e != cudaSuccess) {
      *err = std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
      return nullptr;
    }
    g_staging_ptr[dev] = static_cast<float*>(p);
  }
  return g_staging_ptr[dev];
}

}  // namespace

namespace zb {
// Defined in capi.cpp: records the message returned by zeno_last_error().
void set_last_error(const std::string& msg);
}  // namespace zb

extern "C" int zeno_world_reset_to_state_noalloc(ZenoWorldHandle world, const float* positions,
                                                 const float* quaternions, const float* velocities,
                                                 const float* angular_velocities, const uint8_t* env_mask) {
  if (!world) return ZENO_INVALID_HANDLE;
  if (!positions || !quaternions) return ZENO_INVALID_ARGUMENT;
  zb::World* w = static_cast<zb::World*>(world);
  const size_t need = size_t(w->config().num_envs) * w->model().B;
  if (need > kStagingFloat4) {
    zb::set_last_error("zeno_world_reset_to_state_noalloc: num_envs * num_bodies = " + std::to_string(need) +
                       " exceeds the static staging capacity of " + std::to_string(kStagingFloat4) + " bodies");
    return ZENO_INVALID_ARGUMENT;
  }
  int prev_dev = -1;
  cudaGetDevice(&prev_dev);
  const int dev = w->device();
  if (prev_dev != dev) {
    const cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) {
      zb::set_last_error(std::string("zeno_world_reset_to_state_noalloc: cudaSetDevice: ") + cudaGetErrorString(e));
      return ZENO_METAL_ERROR;
    }
  }
  std::string err;
  float* staging = staging_for(dev, &err);
  int rc = ZENO_METAL_ERROR;
  if (staging) {
    rc = w->reset_to_state_staged(positions, quaternions, velocities, angular_velocities, env_mask, staging);
  } else {
    zb::set_last_error("zeno_world_reset_to_state_noalloc: " + err);
  }
  if (prev_dev >= 0 && prev_dev != dev) cudaSetDevice(prev_dev);
  return rc;
}
