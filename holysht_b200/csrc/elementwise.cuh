// Small element-wise kernels on the boundary of the hot path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hsb {

// In-place irfft preparation of a [rows, width] complex buffer:
// columns m >= mmax are zeroed, Im(m = 0) and (even nlon) Im(m = nlon/2) are
// dropped.  Same effect as the reference's prepare_irfft_inplace
// (cuda/fused_sht.cu:36-67), written as a grid-stride loop over float2.
__global__ void prepare_irfft_kernel(float2* __restrict__ data, long long rows, int width,
                                     int mmax, int nyquist) {
  const long long total = rows * (long long)width;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = static_cast<int>(i % width);
    float2 v = m < mmax ? data[i] : make_float2(0.f, 0.f);
    if (m == 0 || m == nyquist) v.y = 0.f;
    data[i] = v;
  }
}

// Stacked-real packing of a [B, 2, K, M] complex vector spectrum
// (reference fused_vector_forward_pack_real, cuda/fused_legendre.cu:3065-3108):
//   s0 = [c0.re; c0.im; c1.re; c1.im]   s1 = [c1.im; c1.re; c0.im; c0.re]
// each block of B planes of shape [K, M].
__global__ void vector_pack_real_kernel(float* __restrict__ s0, float* __restrict__ s1,
                                        const float2* __restrict__ in, int B, long long plane) {
  const long long total = (long long)B * plane;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / plane;
    const long long e = i % plane;
    const float2 c0 = in[(2 * b) * plane + e];
    const float2 c1 = in[(2 * b + 1) * plane + e];
    const long long q = (long long)B * plane;
    s0[0 * q + i] = c0.x;
    s0[1 * q + i] = c0.y;
    s0[2 * q + i] = c1.x;
    s0[3 * q + i] = c1.y;
    s1[0 * q + i] = c1.y;
    s1[1 * q + i] = c1.x;
    s1[2 * q + i] = c0.y;
    s1[3 * q + i] = c0.x;
  }
}

// Inverse of the packing above applied to the two real Legendre outputs
// (reference fused_vector_forward_recompose_real, cuda/fused_legendre.cu:3110-3155):
//   sph = (r00 - s11) + i (r01 + s10),  tor = (-s01 - r10) + i (s00 - r11)
__global__ void vector_recompose_real_kernel(float2* __restrict__ out, const float* __restrict__ o0,
                                             const float* __restrict__ o1, int B, long long plane) {
  const long long total = (long long)B * plane;
  const long long q = total;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / plane;
    const long long e = i % plane;
    const float r00 = o0[0 * q + i], r01 = o0[1 * q + i], r10 = o0[2 * q + i], r11 = o0[3 * q + i];
    const float s11 = o1[0 * q + i], s10 = o1[1 * q + i], s01 = o1[2 * q + i], s00 = o1[3 * q + i];
    out[(2 * b) * plane + e] = make_float2(r00 - s11, r01 + s10);
    out[(2 * b + 1) * plane + e] = make_float2(-s01 - r10, s00 - r11);
  }
}

}  // namespace hsb
