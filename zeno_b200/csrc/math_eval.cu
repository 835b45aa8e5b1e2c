// zeno_eval_math: the step kernels' canonical scalar functions (devmath.cuh) evaluated on
// the GPU over an array, so their bits can be compared with another implementation's.
#include <cuda_runtime.h>

#include <cstdint>

#include "devmath.cuh"

namespace zb {
namespace {

__global__ void eval_math_kernel(uint32_t fn, const float* x, const float* y, float* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
    const float a = x[i];
    float r = 0.0f;
    switch (fn) {
      case 0: r = rsq_(a); break;
      case 1: r = rcp_(a); break;
      case 2: r = atan2r(a, y[i]); break;
      case 3: r = asinr(a); break;
      case 4: r = len(V3{a, y[i], 0.5f * a}); break;
      default: break;
    }
    out[i] = r;
  }
}

}  // namespace
}  // namespace zb

extern "C" int zeno_eval_math(uint32_t fn, const float* x, const float* y, float* out, uint64_t n) {
  if (fn > 4 || !x || !out || ((fn == 2 || fn == 4) && !y)) return -6;
  if (n == 0) return 0;
  float *dx = nullptr, *dy = nullptr, *dout = nullptr;
  const size_t bytes = size_t(n) * sizeof(float);
  cudaError_t e = cudaMalloc(&dx, bytes);
  if (e == cudaSuccess && y) e = cudaMalloc(&dy, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&dout, bytes);
  if (e == cudaSuccess) e = cudaMemcpy(dx, x, bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && y) e = cudaMemcpy(dy, y, bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    const uint64_t blocks = (n + 255) / 256;
    zb::eval_math_kernel<<<unsigned(blocks < 148 * 32 ? blocks : 148 * 32), 256>>>(fn, dx, dy, dout, n);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(out, dout, bytes, cudaMemcpyDeviceToHost);
  cudaFree(dx);
  cudaFree(dy);
  cudaFree(dout);
  return e == cudaSuccess ? 0 : -4;
}
