// Dense per-order Legendre GEMM on the 5th-generation tensor cores (tcgen05).
//
// For large batches (the 1024x2048, 16x64-slice configuration) the per-order
// contraction is a real GEMM:  D_m[l, n] = sum_k A_m[l, k] X_m[k, n]  with
// A_m = the order-m slice of the table in the torch-harmonics layout
// W[m][l][k] (k contiguous, the module's `weights` buffer) and X_m the
// spectrum of order m transposed to Xt[m][n][k] (n = 2*batch + re/im).
//
// FP32 accuracy from TF32 tensor cores: each operand is stored split in
// global memory, hi = rna_tf32(x) and lo = x - hi (the table once per module,
// the spectrum by the input transpose); the products hi*hi + hi*lo + lo*hi of
// one 32-wide k block go to a TMEM accumulator that starts from zero, and the
// block sums are added into fp32 registers with round-to-nearest (the tensor
// core's own accumulation truncates, an error that grows with the chain
// length; the lo*lo term is below fp32 resolution).  Two TMEM slots alternate
// so the warps drain one block while the tensor core runs the next.
//
// CTA: one order m, 128 output rows l (TMEM lanes), 256 columns n (TMEM
// columns), the full k range in 32-wide blocks.  Pipeline per k block: one
// thread issues four TMA copies (cp.async.bulk.tensor, SWIZZLE_128B, K-major:
// A hi, A lo, B hi, B lo) -> one thread issues 4 k-steps x 3 tcgen05.mma
// (kind::tf32, cta_group::1) -> tcgen05.commit frees the stage.  Two stages in
// flight; no thread rewrites a stage.
// Epilogue: tcgen05.ld 32x32b -> coalesced row stores of D[m][l][n].
// Every mbarrier wait is bounded; a timeout sets a device error word and the
// CTA drains and releases its TMEM instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hsb {
namespace tc {

constexpr int kBM = 128;       // rows (l) per CTA = TMEM lanes
constexpr int kBN = 256;       // columns (n) per CTA = TMEM columns
constexpr int kBK = 32;        // k per stage (one 128-byte swizzle row of fp32)
constexpr int kTmemCols = 2 * kBN;  // two accumulator slots (k blocks alternate)
constexpr int kStages = 2;
constexpr int kThreads = 256;
constexpr int kABytes = kBM * kBK * 4;   // 16 KiB
constexpr int kBBytes = kBN * kBK * 4;   // 32 KiB
constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;  // hi and lo of A and B
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
constexpr unsigned kWaitLimit = 1u << 26;

// device error word: bit 0 = an mbarrier wait timed out
__device__ unsigned g_tc_error = 0;

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait: returns false (and records the timeout) instead of hanging
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  for (unsigned it = 0; it < kWaitLimit; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (it > 64) __nanosleep(64);
  }
  atomicOr(&g_tc_error, 1u);
  return false;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B (8-row groups of
// 128-byte rows, 1024 bytes apart), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(unsigned smem_addr) {
  const uint64_t start = (smem_addr & 0x3FFFFu) >> 4;
  const uint64_t lbo = 1;             // unused for swizzled K-major layouts
  const uint64_t sbo = 1024u >> 4;    // 8 rows x 128 bytes
  return start | (lbo << 16) | (sbo << 32) | (1ull << 46) | (2ull << 61);
}

// instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = 256
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4)                      // D format f32
         | (2u << 7) | (2u << 10)       // A, B format tf32
         | ((uint32_t)(n >> 3) << 17)   // N / 8
         | ((uint32_t)(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_tf32(unsigned tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         unsigned accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ float rna_tf32(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

struct DenseParams {
  int R, S;        // output rows and reduction length (forward: lmax, nlat; inverse: nlat, lmax)
  int M, N;        // orders with work (< lmax), columns = 2 * batch
  int inverse;     // 0: rows l >= m, all k; 1: all rows k, reduction l >= m
  int n_nt;        // column tiles
  int n_bands;     // forward: ceil(lmax / 128); inverse: row tiles ceil(nlat / 128)
  float* D;        // [M][R][N]
};

// tile index -> (m, l-tile, n-tile); orders grouped in bands of equal row-tile
// count, the bands with most row tiles first (longest work first)
__device__ __forceinline__ bool decode(const DenseParams& p, int t, int& m, int& lt, int& nt) {
  if (p.inverse) {  // every order has all row tiles; low orders (longest reductions) first
    const int per_m = p.n_bands * p.n_nt;
    if (t >= p.M * per_m) return false;
    m = t / per_m;
    lt = (t % per_m) / p.n_nt;
    nt = t % p.n_nt;
    return true;
  }
  for (int q = p.n_bands - 1; q >= 0; --q) {
    const int m_hi = min(p.M, p.R - kBM * q);
    const int m_lo = max(0, p.R - kBM * (q + 1));
    if (m_hi <= m_lo) continue;
    const int per_m = (q + 1) * p.n_nt;
    const int cnt = (m_hi - m_lo) * per_m;
    if (t < cnt) {
      m = m_lo + t / per_m;
      const int r = t % per_m;
      lt = r / p.n_nt;
      nt = r % p.n_nt;
      return true;
    }
    t -= cnt;
  }
  return false;
}

__global__ void __launch_bounds__(kThreads, 1)
    dense_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_a_lo, const __grid_constant__ CUtensorMap map_b_lo,
                        const DenseParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* d1_full = empty + kStages;
  uint64_t* d1_free = d1_full + 2;
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(d1_free + 2);

  int m, lt, nt;
  if (!decode(p, blockIdx.x, m, lt, nt)) return;  // uniform per CTA
  const int l0 = (p.inverse ? 0 : m) + lt * kBM;  // first output row of the tile
  const int n0 = nt * kBN;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kb0 = p.inverse ? m / kBK : 0;  // inverse: the table is zero for l < m
  const int nk = (p.S + kBK - 1) / kBK - kb0;

  auto a_hi = [&](int s) { return smem + s * kStageBytes; };
  auto a_lo = [&](int s) { return smem + s * kStageBytes + kABytes; };
  auto b_hi = [&](int s) { return smem + s * kStageBytes + 2 * kABytes; };
  auto b_lo = [&](int s) { return smem + s * kStageBytes + 2 * kABytes + kBBytes; };

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&d1_full[q], 1);
      mbar_init(&d1_free[q], kThreads / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  const unsigned tmem = *tmem_slot;
  constexpr uint32_t idesc = idesc_tf32(kBM, kBN);

  // both operands arrive already split (tf32 hi and fp32 residual lo planes)
  auto issue_loads = [&](int kb, int s) {
    mbar_expect_tx(&full[s], 2 * (kABytes + kBBytes));
    tma_load_3d(a_hi(s), &map_a, &full[s], (kb0 + kb) * kBK, l0, m);
    tma_load_3d(a_lo(s), &map_a_lo, &full[s], (kb0 + kb) * kBK, l0, m);
    tma_load_3d(b_hi(s), &map_b, &full[s], (kb0 + kb) * kBK, n0, m);
    tma_load_3d(b_lo(s), &map_b_lo, &full[s], (kb0 + kb) * kBK, n0, m);
  };
  if (tid == 0) issue_loads(0, 0);

  // TMEM: two accumulator slots of 256 columns; k block kb accumulates all its
  // products (hi*hi + hi*lo + lo*hi) into slot kb & 1 from zero, and the warps
  // drain it into fp32 registers (round to nearest) while the tensor core works
  // on the next block in the other slot.
  const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31 (the rows this warp may read)
  const int col_half = warp >> 2;   // warps 4-7 take the upper 128 columns
  const unsigned trow = tmem + ((unsigned)(quarter * 32) << 16) + (unsigned)(col_half * (kBN / 2));
  float acc[kBN / 2];
#pragma unroll
  for (int c = 0; c < kBN / 2; ++c) acc[c] = 0.f;

  auto tmem_ld32 = [&](unsigned taddr, unsigned (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  };
  // add TMEM columns [base, base + 128) of this thread's row into acc (round to nearest)
  auto drain_into_acc = [&](unsigned base) {
#pragma unroll
    for (int cc = 0; cc < kBN / 2; cc += 32) {
      unsigned r[32];
      tmem_ld32(base + (unsigned)cc, r);
      asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
      for (int q = 0; q < 32; ++q) acc[cc + q] += __uint_as_float(r[q]);
    }
  };
  auto drain_block = [&](int kb) {
    const int slot = kb & 1;
    mbar_wait(&d1_full[slot], (kb >> 1) & 1);
    __syncwarp();  // tcgen05.ld is warp-aligned: reconverge after the per-lane wait
    asm volatile("tcgen05.fence::after_thread_sync;\n");
    drain_into_acc(trow + (unsigned)(slot * kBN));
    asm volatile("tcgen05.fence::before_thread_sync;\n");
    __syncwarp();
    if (lane == 0) mbar_arrive(&d1_free[slot]);
  };

  for (int kb = 0; kb < nk; ++kb) {
    const int s = kb & 1;
    const unsigned ph = (kb >> 1) & 1;
    if (tid == 0 && kb + 1 < nk) {
      const int s2 = s ^ 1;
      if (kb + 1 >= kStages) mbar_wait(&empty[s2], ((kb + 1) / kStages - 1) & 1);  // MMAs of kb-1 done
      issue_loads(kb + 1, s2);
    }
    if (warp == 1 && lane == 0) {
      mbar_wait(&full[s], ph);  // the stage's four operand tiles have landed
      const int slot = kb & 1;
      if (kb >= 2) mbar_wait(&d1_free[slot], ((kb >> 1) - 1) & 1);  // block kb-2 drained
      asm volatile("tcgen05.fence::after_thread_sync;\n");
      const unsigned d = tmem + (unsigned)(slot * kBN);
      const unsigned ahi = smem_u32(a_hi(s)), alo = smem_u32(a_lo(s));
      const unsigned bhi = smem_u32(b_hi(s)), blo = smem_u32(b_lo(s));
#pragma unroll
      for (int j = 0; j < kBK / 8; ++j) {  // 8 tf32 = 32 bytes per k-step
        const unsigned off = j * 32;
        mma_tf32(d, sw128_desc(ahi + off), sw128_desc(bhi + off), idesc, j > 0 ? 1u : 0u);
        mma_tf32(d, sw128_desc(ahi + off), sw128_desc(blo + off), idesc, 1u);
        mma_tf32(d, sw128_desc(alo + off), sw128_desc(bhi + off), idesc, 1u);
      }
      mma_commit(&empty[s]);
      mma_commit(&d1_full[slot]);
    }
    __syncwarp();
    if (kb > 0) drain_block(kb - 1);
  }

  // ---- epilogue: the last block, then D[m][l][n] from the registers ----
  drain_block(nk - 1);
  {
    const int row = l0 + quarter * 32 + lane;
    const int nb = n0 + col_half * (kBN / 2);
    if (row < p.R) {
      float* dst = p.D + ((size_t)m * p.R + row) * p.N + nb;
      if (nb + kBN / 2 <= p.N && (p.N & 3) == 0) {
#pragma unroll
        for (int q = 0; q < kBN / 8; ++q)
          reinterpret_cast<float4*>(dst)[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      } else {
#pragma unroll
        for (int q = 0; q < kBN / 2; ++q)
          if (nb + q < p.N) dst[q] = acc[q];
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised variant (the one the library launches).  Same tile, same
// split-TF32 products and per-block draining, with the pipeline roles on
// separate warps so no role waits for another's unrelated work:
//   warp 0      TMA producer: four copies per stage into a 4-deep ring;
//   warp 1      MMA issuer: 2 k-steps x 3 tcgen05.mma per stage, commits;
//   warps 2..9  drain: each owns 32 TMEM lanes x 128 columns of the
//               accumulator and adds every finished block into registers.
// A stage is 16 k-values (64-byte rows, SWIZZLE_64B), 48 KiB for A hi/lo and
// B hi/lo, so four stages (192 KiB) keep three stages of loads in flight while
// the tensor core works on the fourth.
constexpr int kBK2 = 16;
constexpr int kStages2 = 4;
constexpr int kWsThreads = 320;
constexpr int kA2 = kBM * kBK2 * 4;   // 8 KiB
constexpr int kB2 = kBN * kBK2 * 4;   // 16 KiB
constexpr int kStage2 = 2 * kA2 + 2 * kB2;
constexpr int kWsSmemBytes = kStages2 * kStage2 + 1024 + 256;

// UMMA shared-memory descriptor: K-major, SWIZZLE_64B (8-row groups of
// 64-byte rows, 512 bytes apart), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw64_desc(unsigned smem_addr) {
  const uint64_t start = (smem_addr & 0x3FFFFu) >> 4;
  const uint64_t lbo = 1;
  const uint64_t sbo = 512u >> 4;
  return start | (lbo << 16) | (sbo << 32) | (1ull << 46) | (4ull << 61);
}

__global__ void __launch_bounds__(kWsThreads, 1)
    dense_ws_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_a_lo, const __grid_constant__ CUtensorMap map_b_lo,
                    const DenseParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages2 * kStage2);
  uint64_t* empty = full + kStages2;
  uint64_t* d_full = empty + kStages2;
  uint64_t* d_free = d_full + 2;
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(d_free + 2);

  int m, lt, nt;
  if (!decode(p, blockIdx.x, m, lt, nt)) return;  // uniform per CTA
  const int l0 = (p.inverse ? 0 : m) + lt * kBM;
  const int n0 = nt * kBN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb0 = p.inverse ? m / kBK2 : 0;  // inverse: the table is zero for l < m
  const int nk = (p.S + kBK2 - 1) / kBK2 - kb0;

  auto a_hi = [&](int s) { return smem + s * kStage2; };
  auto a_lo = [&](int s) { return smem + s * kStage2 + kA2; };
  auto b_hi = [&](int s) { return smem + s * kStage2 + 2 * kA2; };
  auto b_lo = [&](int s) { return smem + s * kStage2 + 2 * kA2 + kB2; };

  if (tid == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&d_full[q], 1);
      mbar_init(&d_free[q], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  const unsigned tmem = *tmem_slot;
  constexpr uint32_t idesc = idesc_tf32(kBM, kBN);

  if (warp == 0) {
    if (lane == 0) {  // producer
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages2;
        if (kb >= kStages2 && !mbar_wait(&empty[s], ((kb / kStages2) - 1) & 1)) break;
        mbar_expect_tx(&full[s], kStage2);
        const int kc = (kb0 + kb) * kBK2;
        tma_load_3d(a_hi(s), &map_a, &full[s], kc, l0, m);
        tma_load_3d(a_lo(s), &map_a_lo, &full[s], kc, l0, m);
        tma_load_3d(b_hi(s), &map_b, &full[s], kc, n0, m);
        tma_load_3d(b_lo(s), &map_b_lo, &full[s], kc, n0, m);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages2;
        const int slot = kb & 1;
        if (!mbar_wait(&full[s], (kb / kStages2) & 1)) break;
        if (kb >= 2 && !mbar_wait(&d_free[slot], ((kb >> 1) - 1) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n");
        const unsigned d = tmem + (unsigned)(slot * kBN);
        const unsigned ahi = smem_u32(a_hi(s)), alo = smem_u32(a_lo(s));
        const unsigned bhi = smem_u32(b_hi(s)), blo = smem_u32(b_lo(s));
#pragma unroll
        for (int j = 0; j < kBK2 / 8; ++j) {  // 8 tf32 = 32 bytes per k-step
          const unsigned off = j * 32;
          mma_tf32(d, sw64_desc(ahi + off), sw64_desc(bhi + off), idesc, j > 0 ? 1u : 0u);
          mma_tf32(d, sw64_desc(ahi + off), sw64_desc(blo + off), idesc, 1u);
          mma_tf32(d, sw64_desc(alo + off), sw64_desc(bhi + off), idesc, 1u);
        }
        mma_commit(&empty[s]);
        mma_commit(&d_full[slot]);
      }
    }
  } else {  // drain warps 2..9
    const int dw = warp - 2;
    const int quarter = warp & 3;  // the TMEM lanes this warp may read
    const int col_half = dw >> 2;
    const unsigned trow = tmem + ((unsigned)(quarter * 32) << 16) + (unsigned)(col_half * (kBN / 2));
    float acc[kBN / 2];
#pragma unroll
    for (int c = 0; c < kBN / 2; ++c) acc[c] = 0.f;
    for (int kb = 0; kb < nk; ++kb) {
      const int slot = kb & 1;
      const bool okw = mbar_wait(&d_full[slot], (kb >> 1) & 1);
      __syncwarp();
      if (!__all_sync(0xffffffffu, okw)) break;
      asm volatile("tcgen05.fence::after_thread_sync;\n");
#pragma unroll
      for (int cc = 0; cc < kBN / 2; cc += 32) {
        unsigned r[32];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
              "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
              "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
              "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(trow + (unsigned)(slot * kBN + cc)));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
        for (int q = 0; q < 32; ++q) acc[cc + q] += __uint_as_float(r[q]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;\n");
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[slot]);
    }
    const int row = l0 + quarter * 32 + lane;
    const int nb = n0 + col_half * (kBN / 2);
    if (row < p.R) {
      float* dst = p.D + ((size_t)m * p.R + row) * p.N + nb;
      if (nb + kBN / 2 <= p.N && (p.N & 3) == 0) {
#pragma unroll
        for (int q = 0; q < kBN / 8; ++q)
          reinterpret_cast<float4*>(dst)[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      } else {
#pragma unroll
        for (int q = 0; q < kBN / 2; ++q)
          if (nb + q < p.N) dst[q] = acc[q];
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Variant with the spectrum tile split in shared memory (the library's
// default): the input transpose writes one fp32 plane (half the bytes of a
// split plane pair) and the drain warps split each raw B tile into tf32 hi and
// residual lo, two stages ahead of the MMA (they convert stage kb + 2 before
// draining block kb).  Stage = A hi, A lo, B raw, B hi, B lo = 64 KiB; three
// stages.
constexpr int kStages3 = 3;
constexpr int kStage3 = 2 * kA2 + 3 * kB2;
constexpr int kWs3SmemBytes = kStages3 * kStage3 + 1024 + 256;

__global__ void __launch_bounds__(kWsThreads, 1)
    dense_ws3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_a_lo, const __grid_constant__ CUtensorMap map_b_lo,
                    const DenseParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages3 * kStage3);
  uint64_t* empty = full + kStages3;
  uint64_t* conv = empty + kStages3;
  uint64_t* d_full = conv + kStages3;
  uint64_t* d_free = d_full + 2;
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(d_free + 2);

  int m, lt, nt;
  if (!decode(p, blockIdx.x, m, lt, nt)) return;  // uniform per CTA
  const int l0 = (p.inverse ? 0 : m) + lt * kBM;
  const int n0 = nt * kBN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb0 = p.inverse ? m / kBK2 : 0;  // inverse: the table is zero for l < m
  const int nk = (p.S + kBK2 - 1) / kBK2 - kb0;

  auto a_hi = [&](int s) { return smem + s * kStage3; };
  auto a_lo = [&](int s) { return smem + s * kStage3 + kA2; };
  auto b_hi = [&](int s) { return smem + s * kStage3 + 2 * kA2; };
  auto b_lo = [&](int s) { return smem + s * kStage3 + 2 * kA2 + kB2; };
  auto b_raw = [&](int s) { return smem + s * kStage3 + 2 * kA2 + 2 * kB2; };

  if (tid == 0) {
    for (int s = 0; s < kStages3; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 8);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&d_full[q], 1);
      mbar_init(&d_free[q], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  const unsigned tmem = *tmem_slot;
  constexpr uint32_t idesc = idesc_tf32(kBM, kBN);

  if (warp == 0) {
    if (lane == 0) {  // producer
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages3;
        if (kb >= kStages3 && !mbar_wait(&empty[s], ((kb / kStages3) - 1) & 1)) break;
        mbar_expect_tx(&full[s], 2 * kA2 + kB2);
        const int kc = (kb0 + kb) * kBK2;
        tma_load_3d(a_hi(s), &map_a, &full[s], kc, l0, m);
        tma_load_3d(a_lo(s), &map_a_lo, &full[s], kc, l0, m);
        tma_load_3d(b_raw(s), &map_b, &full[s], kc, n0, m);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages3;
        const int slot = kb & 1;
        if (!mbar_wait(&full[s], (kb / kStages3) & 1)) break;
        if (!mbar_wait(&conv[s], (kb / kStages3) & 1)) break;  // B split by the drain warps
        if (kb >= 2 && !mbar_wait(&d_free[slot], ((kb >> 1) - 1) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n");
        const unsigned d = tmem + (unsigned)(slot * kBN);
        const unsigned ahi = smem_u32(a_hi(s)), alo = smem_u32(a_lo(s));
        const unsigned bhi = smem_u32(b_hi(s)), blo = smem_u32(b_lo(s));
#pragma unroll
        for (int j = 0; j < kBK2 / 8; ++j) {  // 8 tf32 = 32 bytes per k-step
          const unsigned off = j * 32;
          mma_tf32(d, sw64_desc(ahi + off), sw64_desc(bhi + off), idesc, j > 0 ? 1u : 0u);
          mma_tf32(d, sw64_desc(ahi + off), sw64_desc(blo + off), idesc, 1u);
          mma_tf32(d, sw64_desc(alo + off), sw64_desc(bhi + off), idesc, 1u);
        }
        mma_commit(&empty[s]);
        mma_commit(&d_full[slot]);
      }
    }
  } else {  // drain warps 2..9
    const int dw = warp - 2;
    const int quarter = warp & 3;  // the TMEM lanes this warp may read
    const int col_half = dw >> 2;
    const unsigned trow = tmem + ((unsigned)(quarter * 32) << 16) + (unsigned)(col_half * (kBN / 2));
    float acc[kBN / 2];
#pragma unroll
    for (int c = 0; c < kBN / 2; ++c) acc[c] = 0.f;
    // split the raw B tile of stage kb into tf32 hi and fp32 residual lo, in the
    // same (swizzled) positions, for the tensor core
    const int dtid = tid - 64;
    auto convert = [&](int kb) -> bool {
      const int s = kb % kStages3;
      const bool ok = mbar_wait(&full[s], (kb / kStages3) & 1);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ok)) return false;
      const float4* raw = reinterpret_cast<const float4*>(b_raw(s));
      float4* hi = reinterpret_cast<float4*>(b_hi(s));
      float4* lo = reinterpret_cast<float4*>(b_lo(s));
#pragma unroll
      for (int i = dtid; i < kB2 / 16; i += 256) {
        const float4 v = raw[i];
        const float4 h = make_float4(rna_tf32(v.x), rna_tf32(v.y), rna_tf32(v.z), rna_tf32(v.w));
        hi[i] = h;
        lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
      return true;
    };
    bool alive = convert(0) && (nk < 2 || convert(1));
    for (int kb = 0; kb < nk && alive; ++kb) {
      if (kb + 2 < nk && !convert(kb + 2)) break;
      const int slot = kb & 1;
      const bool okw = mbar_wait(&d_full[slot], (kb >> 1) & 1);
      __syncwarp();
      if (!__all_sync(0xffffffffu, okw)) break;
      asm volatile("tcgen05.fence::after_thread_sync;\n");
#pragma unroll
      for (int cc = 0; cc < kBN / 2; cc += 32) {
        unsigned r[32];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
              "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
              "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
              "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(trow + (unsigned)(slot * kBN + cc)));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
        for (int q = 0; q < 32; ++q) acc[cc + q] += __uint_as_float(r[q]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;\n");
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[slot]);
    }
    const int row = l0 + quarter * 32 + lane;
    const int nb = n0 + col_half * (kBN / 2);
    if (row < p.R) {
      float* dst = p.D + ((size_t)m * p.R + row) * p.N + nb;
      if (nb + kBN / 2 <= p.N && (p.N & 3) == 0) {
#pragma unroll
        for (int q = 0; q < kBN / 8; ++q)
          reinterpret_cast<float4*>(dst)[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      } else {
#pragma unroll
        for (int q = 0; q < kBN / 2; ++q)
          if (nb + q < p.N) dst[q] = acc[q];
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// input [B][S][W] complex (orders < M used) -> Xt [M][2B][S] fp32 * scale,
// optionally rounded to bf16 (after scaling), stored split: xt = rna_tf32(x),
// xt_lo = x - xt (the residual is exact in fp32)
__global__ void transpose_in_kernel(const float2* __restrict__ in, float* __restrict__ xt, float* __restrict__ xt_lo,
                                    int B, int S, int M, long long in_bs, long long in_rs, float scale,
                                    int round_bf16) {
  __shared__ float2 tile[32][33];
  const int b = blockIdx.z;
  const int m0 = blockIdx.x * 32, s0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int sidx = s0 + i, m = m0 + tx;
    tile[i][tx] = (sidx < S && m < M) ? in[(long long)b * in_bs + (long long)sidx * in_rs + m] : make_float2(0.f, 0.f);
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int m = m0 + i, sidx = s0 + tx;
    if (m < M && sidx < S) {
      const float2 v = tile[tx][i];
      float re = v.x * scale, im = v.y * scale;
      if (round_bf16) {
        re = __bfloat162float(__float2bfloat16_rn(re));
        im = __bfloat162float(__float2bfloat16_rn(im));
      }
      const long long off = ((long long)m * (2LL * B) + 2LL * b) * S;
      if (xt_lo == nullptr) {  // one fp32 plane: the GEMM kernel splits it
        xt[off + sidx] = re;
        xt[off + S + sidx] = im;
      } else {
        const float hre = rna_tf32(re), him = rna_tf32(im);
        xt[off + sidx] = hre;
        xt[off + S + sidx] = him;
        xt_lo[off + sidx] = re - hre;
        xt_lo[off + S + sidx] = im - him;
      }
    }
  }
}

// D [Mrows][R][2B] -> out [B][R][cols] complex.  Forward: exact zeros for m > r
// (r = l).  Columns m >= Mrows are zero.  irfft preparation: Im = 0 at m = 0
// and m = nyquist (-1: none).
__global__ void transpose_out_kernel(const float* __restrict__ D, float2* __restrict__ out, int B, int R, int cols,
                                     int Mrows, long long out_bs, long long out_rs, int forward, int zero_im0,
                                     int nyquist) {
  __shared__ float2 tile[32][33];
  const int r = blockIdx.z;
  const int m0 = blockIdx.x * 32, b0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int i = ty; i < 32; i += 8) {
    const int m = m0 + i, b = b0 + tx;
    float2 v = make_float2(0.f, 0.f);
    if (m < Mrows && (!forward || m <= r) && b < B) {
      const float* src = D + ((long long)m * R + r) * (2LL * B) + 2LL * b;
      v = make_float2(src[0], src[1]);
    }
    tile[i][tx] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int b = b0 + i, m = m0 + tx;
    if (b < B && m < cols) {
      float2 v = tile[tx][i];
      if ((zero_im0 && m == 0) || m == nyquist) v.y = 0.f;
      out[(long long)b * out_bs + (long long)r * out_rs + m] = v;
    }
  }
}

// table [n] -> hi [n] = rna_tf32(x), lo [n] = x - hi
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float h = rna_tf32(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

}  // namespace tc
}  // namespace hsb
