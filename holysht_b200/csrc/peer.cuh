// Cross-GPU barrier over NVLink peer memory for the order-partitioned transforms.
//
// Every rank owns a signal array of n_ranks 32-bit words in memory that all
// ranks can address (symmetric memory: the peers' arrays are mapped into this
// GPU's address space).  Barrier number `epoch` (increasing from 1):
//   1. one thread per peer q stores `epoch` into word `rank` of q's array with
//      release semantics at system scope (after a system-scope fence), which
//      orders every store this GPU made before the barrier (the contraction's
//      peer stores of an earlier kernel on the same stream) before the flag;
//   2. the same thread then waits, with acquire semantics, until word q of
//      this rank's own array holds at least `epoch` (peer q has arrived).
// The wait is bounded: after kLimit polls it sets bit 0 of *error and returns,
// so a peer that never arrives cannot hang the GPU; the host reads the error
// word.  One CTA of 32 threads (n_ranks <= 8).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hsb {
namespace peer {

constexpr unsigned kLimit = 1u << 24;

__device__ unsigned g_peer_error = 0;

struct BarrierParams {
  unsigned* signal[8];  // signal[q]: peer q's array, as mapped on this GPU
  int n_ranks;
  int rank;
  unsigned epoch;
};

__device__ __forceinline__ void store_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) barrier_kernel(const BarrierParams p) {
  const int q = threadIdx.x;
  if (q >= p.n_ranks) return;
  asm volatile("fence.sc.sys;\n" ::: "memory");
  store_release_sys(p.signal[q] + p.rank, p.epoch);
  const unsigned* mine = p.signal[p.rank] + q;
  for (unsigned it = 0; it < kLimit; ++it) {
    // wrap-safe "at least epoch": the difference is small and non-negative once q arrived
    if ((int)(load_acquire_sys(mine) - p.epoch) >= 0) return;
    if (it > 64) __nanosleep(128);
  }
  atomicOr(&g_peer_error, 1u);
}

}  // namespace peer
}  // namespace hsb
