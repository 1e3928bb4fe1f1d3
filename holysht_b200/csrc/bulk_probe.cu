// Achievable read bandwidth of the streaming kernel's access pattern, for the
// roofline: 8 warps per CTA, every warp streams its own contiguous run of
// bytes into a private ring of shared-memory stages with cp.async.bulk and
// reads each stage once (no arithmetic).  Built into libholysht_b200_probe.so
// (a diagnostic library, not the product).
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr unsigned kProbeWaitLimit = 1u << 22;
__device__ unsigned g_probe_error = 0;

__device__ __forceinline__ unsigned su32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool probe_wait(unsigned bar, unsigned parity) {
  for (unsigned it = 0; it < kProbeWaitLimit; ++it) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (it > 32) __nanosleep(32);
  }
  atomicOr(&g_probe_error, 1u);
  return false;
}

template <int NS, int STKB>
__global__ void __launch_bounds__(256, 1) bulk_stream(const char* __restrict__ src, long long per_warp, float* sink) {
  constexpr int kStage = STKB * 1024;
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) unsigned long long bars[8][NS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const char* g = src + (blockIdx.x * 8LL + warp) * per_warp;
  unsigned char* my = sm + warp * NS * kStage;
  const unsigned bar0 = su32(&bars[warp][0]);
  if (lane == 0) {
    for (int i = 0; i < NS; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * i));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const long long n = per_warp / kStage;
  auto issue = [&](long long c) {
    const int slot = (int)(c % NS);
    const unsigned b = bar0 + 8 * slot;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(kStage) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(my + slot * kStage)),
                 "l"(g + c * kStage), "r"(kStage), "r"(b)
                 : "memory");
  };
  if (lane == 0)
    for (long long c = 0; c < NS && c < n; ++c) issue(c);
  float acc = 0.f;
  long long c = 0;
  for (; c < n; ++c) {
    const int slot = (int)(c % NS);
    if (!probe_wait(bar0 + 8 * slot, (unsigned)((c / NS) & 1))) break;
    const float4* s4 = reinterpret_cast<const float4*>(my + slot * kStage);
#pragma unroll 4
    for (int q = lane; q < kStage / 16; q += 32) {
      const float4 v = s4[q];
      acc += v.x + v.y + v.z + v.w;
    }
    __syncwarp();
    if (lane == 0 && c + NS < n) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(c + NS);
    }
  }
  if (c < n && lane == 0) {
    // a wait gave up: let the copies still in flight land before exiting
    for (long long d = c + 1; d < c + NS && d < n; ++d) probe_wait(bar0 + 8 * (int)(d % NS), (unsigned)((d / NS) & 1));
  }
  if (acc == 1.2345f) sink[0] = acc;  // keeps the reads
}

template <int NS, int STKB>
double run(const char* src, long long bytes, int ctas, int cluster, int reps, float* sink) {
  auto k = bulk_stream<NS, STKB>;
  const int smem = 8 * NS * STKB * 1024;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -2.0;
  const long long per_warp = (bytes / (ctas * 8LL)) / (STKB * 1024) * (STKB * 1024);
  if (per_warp <= 0) return -3.0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  for (int i = 0; i < 3; ++i)
    if (cudaLaunchKernelEx(&cfg, k, src, per_warp, sink) != cudaSuccess) return -4.0;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  for (int i = 0; i < reps; ++i) cudaLaunchKernelEx(&cfg, k, src, per_warp, sink);
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  unsigned err = 0;
  cudaMemcpyFromSymbol(&err, g_probe_error, sizeof(err));
  if (cudaGetLastError() != cudaSuccess || err) return -5.0;
  return (double)per_warp * ctas * 8 / (ms / reps * 1e-3) / 1e9;
}

}  // namespace

// GB/s of `reps` back-to-back launches streaming `bytes` of `src` (device
// memory) with `ctas` CTAs in clusters of `cluster`, `stages` ring stages of
// `stage_kb` KiB per warp.  Negative on error.  Supported (stages, stage_kb):
// (4, 4), (3, 4), (3, 8), (2, 8).
extern "C" double holysht_probe_bulk_stream(const void* src, long long bytes, int ctas, int cluster, int stages,
                                            int stage_kb, int reps, float* sink) {
  const char* s = static_cast<const char*>(src);
  if (stages == 4 && stage_kb == 4) return run<4, 4>(s, bytes, ctas, cluster, reps, sink);
  if (stages == 3 && stage_kb == 4) return run<3, 4>(s, bytes, ctas, cluster, reps, sink);
  if (stages == 3 && stage_kb == 8) return run<3, 8>(s, bytes, ctas, cluster, reps, sink);
  if (stages == 2 && stage_kb == 8) return run<2, 8>(s, bytes, ctas, cluster, reps, sink);
  return -1.0;
}
