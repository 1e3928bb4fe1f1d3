// FP32 throughput probe for the roofline of the FMA-bound kernels: packed
// f32x2 FMA (FFMA2) and scalar FFMA issue rates with many independent chains.
// Built into libholysht_b200_probe.so by holysht_b200/build.py and driven by
// `python -m holysht_b200.tools.fp32_peak`.
#include <cuda_runtime.h>

namespace {

constexpr int kChains = 8;

__global__ void ffma2_loop(float2* out, int iters, float2 a) {
  float2 acc[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) acc[c] = make_float2(threadIdx.x * 1e-7f + c, blockIdx.x * 1e-7f);
  const float2 b = make_float2(0.999999f, 1.000001f);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) acc[c] = __ffma2_rn(acc[c], b, a);
  }
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    s.x += acc[c].x;
    s.y += acc[c].y;
  }
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void ffma_loop(float* out, int iters, float a) {
  float acc[2 * kChains];
#pragma unroll
  for (int c = 0; c < 2 * kChains; ++c) acc[c] = threadIdx.x * 1e-7f + c;
  const float b = 0.999999f;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < 2 * kChains; ++c) acc[c] = fmaf(acc[c], b, a);
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < 2 * kChains; ++c) s += acc[c];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace

extern "C" {

// Runs one probe (packed = 1: FFMA2, 0: FFMA) and returns FLOP/s, or a
// negative value on a CUDA error.  Every thread performs 2*kChains FMAs
// (2 FLOP each) per iteration in both variants.
double holysht_probe_fp32_flops(int packed, int blocks, int threads, int iters) {
  void* buf = nullptr;
  if (cudaMalloc(&buf, (size_t)blocks * threads * sizeof(float2)) != cudaSuccess) return -1.0;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int rep = 0; rep < 2; ++rep) {  // first round warms up
    cudaEventRecord(e0);
    if (packed)
      ffma2_loop<<<blocks, threads>>>(static_cast<float2*>(buf), iters, make_float2(1e-6f, 1e-6f));
    else
      ffma_loop<<<blocks, threads>>>(static_cast<float*>(buf), iters, 1e-6f);
    cudaEventRecord(e1);
  }
  cudaError_t err = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(buf);
  if (err != cudaSuccess || cudaGetLastError() != cudaSuccess || ms <= 0.f) return -1.0;
  const double flops = 2.0 * 2.0 * kChains * (double)iters * blocks * threads;
  return flops / (ms * 1e-3);
}

}  // extern "C"
