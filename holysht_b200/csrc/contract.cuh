// Per-order Legendre contraction for sm_100a.
//
// One kernel template covers every contraction on the HOLYSHT hot path:
//
//   forward  (DIR_FWD): out[b,p,l,m] = sum_k  W[l,k,m] * in[b,p,k,m]   (l >= m)
//   inverse  (DIR_INV): out[b,p,k,m] = sum_l  W[l,k,m] * in[b,p,l,m]   (l >= m)
//
// for three element kinds:
//   KIND_SCALAR  complex input/output, one table             (fused_legendre_*)
//   KIND_VECTOR  complex, two tables W0/W1, two components   (fused_vector_legendre_*)
//                sph = W0 c0 + i s W1 c1,  tor = i s W1 c0 - W0 c1,  s = w1_sign
//   KIND_REAL    real input/output, one table                (fused_legendre_*_real)
//
// The tables stay in the reference operator layout W[l][k][m] (m contiguous,
// torch-ext/torch_binding.cpp:12-24; zero above the diagonal m > l).  Lanes
// of a warp own 32 consecutive orders m, so every table load is one coalesced
// 128-byte row segment and each table element is read from HBM exactly once
// per batch group; only the l >= m triangle is ever loaded.
//
// Work decomposition:
//   * a CTA owns a 32-order m-tile x 32 output rows (8 warps x 4 rows) x a
//     batch group of NB batches;
//   * the reduction axis is split across a thread-block cluster of KS CTAs;
//     each CTA streams its slice of the input spectrum through a cp.async
//     double buffer in shared memory (all 8 warps reuse it) and its table
//     rows straight into registers (a 4-deep register ring), and the partial
//     sums are reduced through distributed shared memory at the end, in a
//     fixed rank order (deterministic);
//   * the inner product is FP32 FMA issued as packed f32x2 FMAs.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace hsb {

namespace cg = cooperative_groups;

enum Kind : int { KIND_SCALAR = 0, KIND_VECTOR = 1, KIND_REAL = 2 };
enum Dir : int { DIR_FWD = 0, DIR_INV = 1 };

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerWarp = 4;
constexpr int kRows = kWarps * kRowsPerWarp;  // output rows per CTA
constexpr int kMTile = 32;                     // orders per CTA (one per lane)
#ifndef HSB_CHUNK
#define HSB_CHUNK 16
#endif
#ifndef HSB_CHUNK_SMALL
#define HSB_CHUNK_SMALL 8
#endif
// reduction steps per shared-memory stage (vector kind / the others)
constexpr int kChunkVector = HSB_CHUNK;
constexpr int kChunkSmall = HSB_CHUNK_SMALL;
constexpr int kChunk = kChunkSmall;  // host-side minimum granularity
#ifndef HSB_RING
#define HSB_RING 16
#endif
#ifndef HSB_RING_SMALL
#define HSB_RING_SMALL 8
#endif
#ifndef HSB_VECTOR_MIN_BLOCKS
#define HSB_VECTOR_MIN_BLOCKS 1
#endif
// register ring for table rows (steps in flight + 1): deep for the vector kind
// (one CTA per SM, registers to spare), shallower for the two-CTA kinds
constexpr int kRingVector = HSB_RING;
constexpr int kRingSmall = HSB_RING_SMALL;
#ifndef HSB_PREFETCH_CHUNKS
#define HSB_PREFETCH_CHUNKS 2
#endif
constexpr int kPrefetchChunks = HSB_PREFETCH_CHUNKS;  // L2 prefetch distance of the table (chunks)
constexpr int kSmemBytes = 64 * 1024;

struct ContractParams {
  const void* in;
  void* out;
  const float* w0;
  const float* w1;
  long long in_bs, in_ps, in_rs;     // input strides (elements): batch, component, row
  long long out_bs, out_ps, out_rs;  // output strides (elements)
  long long w_ls, w_ks;              // table strides (floats) of l and k
  long long w_mt;                    // table stride (floats) of a 32-order m tile (32 = dense m)
  int B, K, L, M;                    // batch, nlat, lmax, mmax (table extents)
  int out_cols;                      // output columns written (>= M; extra are zero)
  int R, S;                          // output rows, reduction extent
  float scale;                       // applied to every output
  float w1_sign;                     // +1 (A) or -1 (conjugate transpose)
  int zero_imag_col0;                // irfft preparation: Im(m=0) = 0
  int nyquist;                       // irfft preparation: Im(m=nyquist) = 0, -1 = off
  int round_bf16;                    // round inputs to bf16 before use
  int n_rt, n_mt, j_act, n_bg;       // row tiles, m tiles, active m tiles, batch groups
  int n_compute, n_zero;             // tiles per batch group
  int ks;                            // cluster size (reduction split)
  int m_off, mt_off;                 // global order of local column 0 (multiple of 32), /32
};

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  return __ffma2_rn(a, b, c);
}

__device__ __forceinline__ void cp_async_bytes(void* smem_dst, const void* gsrc, int bytes_valid,
                                               int size) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  if (size == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gsrc),
                 "r"(bytes_valid));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gsrc),
                 "r"(bytes_valid));
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;\n" ::); }

// streaming table load: read once, no L1 allocation, evict-first in L2 so the
// table stream does not push the (re-read) input spectrum out of L2
__device__ __forceinline__ unsigned long long evict_first_policy() {
  unsigned long long pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
// Predicated streaming load: the destination is zeroed and the load issued
// under a predicate inside one asm block, so no instruction consumes the
// result until the FMA that needs it several steps later (a select or a
// multiply right after the load would stall the warp for the full latency).
__device__ __forceinline__ float ld_stream(const float* p, bool ok, unsigned long long pol) {
  float v;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %2, 0;\n\t"
      "mov.b32 %0, 0;\n\t"
      "@q ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %3;\n\t}"
      : "=f"(v)
      : "l"(p), "r"((int)ok), "l"(pol));
  return v;
}

__device__ __forceinline__ float4 ld_stream4(const float* p, bool ok, unsigned long long pol) {
  float4 v;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %4, 0;\n\t"
      "mov.b32 %0, 0;\n\tmov.b32 %1, 0;\n\tmov.b32 %2, 0;\n\tmov.b32 %3, 0;\n\t"
      "@q ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%5], %6;\n\t}"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "r"((int)ok), "l"(p), "l"(pol));
  return v;
}

// bulk L2 prefetch of a contiguous range (16-byte aligned, multiple of 16 bytes)
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const float* p) {
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p));
}

__device__ __forceinline__ float round_to_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Decode a tile index into (m tile j, row tile rt).  Compute tiles come first,
// ordered by m tile (longest reductions first for the inverse direction),
// then tiles that are entirely zero (rows above the diagonal, or orders with
// no l >= m inside the table).
template <int DIR>
__device__ __forceinline__ bool decode_tile(const ContractParams& p, int t, int& j, int& rt) {
  if (t < p.n_compute) {
    int rem = t;
    for (j = 0; j < p.j_act; ++j) {
      const int first = (DIR == DIR_FWD) ? j + p.mt_off : 0;
      const int cnt = p.n_rt > first ? p.n_rt - first : 0;
      if (rem < cnt) {
        rt = first + rem;
        return true;
      }
      rem -= cnt;
    }
    rt = 0;
    return true;  // unreachable for consistent host parameters
  }
  int rem = t - p.n_compute;
  for (j = 0; j < p.n_mt; ++j) {
    int cnt;
    if (j < p.j_act)
      cnt = (DIR == DIR_FWD) ? (j + p.mt_off < p.n_rt ? j + p.mt_off : p.n_rt) : 0;
    else
      cnt = p.n_rt;
    if (rem < cnt) {
      rt = rem;
      return false;
    }
    rem -= cnt;
  }
  rt = 0;
  j = p.n_mt;  // out of range: nothing to write
  return false;
}

template <int KIND>
struct KindTraits;
template <>
struct KindTraits<KIND_SCALAR> {
  static constexpr int P = 1;  // components per batch
  using SE = float2;           // staged element
};
template <>
struct KindTraits<KIND_VECTOR> {
  static constexpr int P = 2;
  using SE = float2;
};
template <>
struct KindTraits<KIND_REAL> {
  static constexpr int P = 1;
  using SE = float;
};

template <int KIND, int NB>
struct Acc {
  // number of packed (float2) accumulators per output row
  static constexpr int NA = KIND == KIND_VECTOR ? 2 * NB : (KIND == KIND_SCALAR ? NB : NB / 2);
};

template <int KIND, int DIR, int NB, typename TIN>
__device__ __forceinline__ void write_zero_tile(const ContractParams& p, int j, int rt, int bg,
                                                int rank) {
  constexpr int P = KindTraits<KIND>::P;
  constexpr int NA = Acc<KIND, NB>::NA;
  const int rpr = kRows / p.ks;
  const int total = rpr * NA * 32;
  for (int e = threadIdx.x; e < total; e += kThreads) {
    const int col = e & 31;
    const int a = (e >> 5) % NA;
    const int rl = e / (NA * 32);
    const int row = rt * kRows + rank * rpr + rl;
    const int mm = j * kMTile + col;
    if (row >= p.R || mm >= p.out_cols) continue;
    if (KIND == KIND_REAL) {
      float* out = static_cast<float*>(p.out);
      const int b = bg * NB + 2 * a;
      const long long off = (long long)row * p.out_rs + mm;
      if (b < p.B) out[(long long)b * p.out_bs + off] = 0.f;
      if (b + 1 < p.B) out[(long long)(b + 1) * p.out_bs + off] = 0.f;
    } else {
      float2* out = static_cast<float2*>(p.out);
      const int b = bg * NB + a / P;
      const int pl = a % P;
      if (b < p.B)
        out[(long long)b * p.out_bs + (long long)pl * p.out_ps + (long long)row * p.out_rs + mm] =
            make_float2(0.f, 0.f);
    }
  }
}

// GROUPED: the table is in the row-grouped layout built by the host
// (holysht_b200.ops.group_table): for every group of kRowsPerWarp output
// rows, every 32-order m tile and every reduction step, the 32 lanes' values
// of all rows and tables are contiguous ([rows][tables] per lane), so a lane
// fetches its whole step with one or two 16-byte loads and a warp's step is
// one contiguous 512-byte / 1-KB block.  Strides: w_ls = group, w_mt = m tile,
// w_ks = step (floats).  Otherwise the table is strided [l][k][m-tile][32].
template <int KIND, int DIR, int NB, typename TIN, bool GROUPED>
__global__ void __launch_bounds__(kThreads, KIND == KIND_VECTOR ? HSB_VECTOR_MIN_BLOCKS : 2)
    contract_kernel(const ContractParams p) {
  constexpr int P = KindTraits<KIND>::P;
  constexpr int PB = NB * P;  // staged planes per reduction step
  constexpr int kRing = (KIND == KIND_VECTOR) ? kRingVector : kRingSmall;
  constexpr int kChunk = (KIND == KIND_VECTOR) ? kChunkVector : kChunkSmall;
  constexpr int NA = Acc<KIND, NB>::NA;
  using SE = typename KindTraits<KIND>::SE;
  constexpr bool kAsyncStage = !std::is_same<TIN, __nv_bfloat16>::value;
  static_assert(kRows * NA * 32 * 8 <= kSmemBytes, "partial sums exceed shared memory");
  static_assert(2 * kChunk * PB * 32 * sizeof(SE) <= kSmemBytes, "stage exceeds shared memory");
  static_assert(KIND != KIND_REAL || NB % 2 == 0, "real kind pairs batches");
  static_assert(kChunk % kRing == 0, "ring slots are compile-time within a chunk");

  extern __shared__ __align__(16) unsigned char smem_raw[];
  SE* stage = reinterpret_cast<SE*>(smem_raw);  // [2][kChunk][PB][32]
  float2* part = reinterpret_cast<float2*>(smem_raw);  // [kRows][NA][32], after the loop

  cg::cluster_group cluster = cg::this_cluster();
  const int ks = p.ks;
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile = blockIdx.x / ks;
  const int bg = tile % p.n_bg;
  const int t = tile / p.n_bg;
  int j, rt;
  const bool compute = decode_tile<DIR>(p, t, j, rt);
  if (!compute) {
    // uniform across the cluster: no cluster barrier is reached on this path
    write_zero_tile<KIND, DIR, NB, TIN>(p, j, rt, bg, rank);
    return;
  }

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int m0 = j * kMTile;
  const int m = m0 + lane;
  const int mg = m + p.m_off;    // global order (triangle l >= m)
  const int m0g = m0 + p.m_off;
  const int row0 = rt * kRows;
  const int b0 = bg * NB;

  // reduction range of this cluster rank (chunk aligned)
  const int s_begin = (DIR == DIR_FWD) ? 0 : m0g;
  const int s_end = p.S;
  const int nsteps = s_end > s_begin ? s_end - s_begin : 0;
  const int per = ((nsteps + ks * kChunk - 1) / (ks * kChunk)) * kChunk;
  const int r_begin = min(s_end, s_begin + rank * per);
  const int r_end = min(s_end, r_begin + per);
  const int nchunks = (r_end - r_begin + kChunk - 1) / kChunk;

  // table offsets of this lane (32-bit: a table holds < 2^32 floats)
  constexpr int NT = (KIND == KIND_VECTOR) ? 2 : 1;        // tables
  constexpr int GF = kRowsPerWarp * NT;                     // grouped floats per lane-step
  const unsigned sstride = GROUPED ? (unsigned)p.w_ks : (unsigned)((DIR == DIR_FWD) ? p.w_ks : p.w_ls);
  const unsigned rstride = (unsigned)((DIR == DIR_FWD) ? p.w_ls : p.w_ks);
  unsigned roff[kRowsPerWarp];
  unsigned vmask = 0;
  unsigned gbase = 0;  // grouped: this lane's offset at step 0
  unsigned gwarp = 0;  // grouped: lane 0's offset at step 0 (prefetch)
  bool gvalid = false;
  if constexpr (GROUPED) {
    const int rg = (row0 / kRowsPerWarp) + warp;
    const int r_first = rg * kRowsPerWarp;
    gvalid = r_first < p.R && m < p.M && (DIR == DIR_INV || r_first + kRowsPerWarp - 1 >= mg);
    gwarp = (unsigned)rg * (unsigned)p.w_ls + (unsigned)j * (unsigned)p.w_mt;
    gbase = gwarp + (unsigned)lane * GF;
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) roff[i] = 0u;
  } else {
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int row = row0 + warp * kRowsPerWarp + i;
      bool ok = row < p.R && m < p.M;
      if (DIR == DIR_FWD) ok = ok && row >= mg;  // l >= m
      vmask |= ok ? (1u << i) : 0u;
      roff[i] = ok ? (unsigned)row * rstride + (unsigned)(j * p.w_mt) + (unsigned)lane : 0u;
    }
  }
  // warp-uniform row validity and lane-0 offsets for the L2 prefetch (strided layout)
  unsigned pf_off[kRowsPerWarp];
  unsigned pf_mask = 0;
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int row = row0 + warp * kRowsPerWarp + i;
    const bool ok = row < p.R && m0 < p.M && (DIR == DIR_INV || row >= m0g);
    pf_mask |= ok ? (1u << i) : 0u;
    pf_off[i] = ok ? (unsigned)row * rstride + (unsigned)(j * p.w_mt) : 0u;
  }
  const bool pf_any = pf_mask != 0;
  const int m_last = min(kMTile, p.M - m0) - 1;  // last valid lane of this tile
  const float* __restrict__ w0 = p.w0;
  const float* __restrict__ w1 = p.w1;
  const float w1s = p.w1_sign;

  float2 acc[kRowsPerWarp][NA];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int a = 0; a < NA; ++a) acc[i][a] = make_float2(0.f, 0.f);
  // vector kind: the four products per (row, batch), see the inner loop
  constexpr int NQ = (KIND == KIND_VECTOR) ? 2 * NB : 1;
  float2 vq[kRowsPerWarp][NQ];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int a = 0; a < NQ; ++a) vq[i][a] = make_float2(0.f, 0.f);

  // ---- staging of the input spectrum: [buf][step][plane][lane] ----
  constexpr int kStageElems = kChunk * PB * 32;
  auto stage_one = [&](SE* dst, int e, int ls, int bl, int pl, int col, int c0) {
    const int b = b0 + bl;
    const int s = c0 + ls;
    const int mm = m0 + col;
    const bool ok = s < r_end && b < p.B && mm < p.M;
    const long long off = ok ? (long long)b * p.in_bs + (long long)pl * p.in_ps + (long long)s * p.in_rs + mm : 0;
    if constexpr (kAsyncStage) {
      const SE* src = static_cast<const SE*>(p.in) + off;
      cp_async_bytes(dst + e, src, ok ? (int)sizeof(SE) : 0, (int)sizeof(SE));
    } else {
      const TIN* src = static_cast<const TIN*>(p.in) + off;
      dst[e] = ok ? static_cast<float>(*src) : 0.f;
    }
  };
  // vector kind: one thread stages both components of a (step, batch, order)
  // so it can combine them into u = c0 + i c1, v = c0 - i c1 without a barrier
  constexpr int kStageUnits = (KIND == KIND_VECTOR) ? kStageElems / 2 : kStageElems;
  auto stage_chunk = [&](int chunk, int buf) {
    const int c0 = r_begin + chunk * kChunk;
    SE* dst = stage + buf * kStageElems;
    for (int e = threadIdx.x; e < kStageUnits; e += kThreads) {
      const int col = e & 31;
      if constexpr (KIND == KIND_VECTOR) {
        const int bl = (e >> 5) % NB;
        const int ls = e / (NB * 32);
        const int i0 = (ls * PB + 2 * bl) * 32 + col;
        stage_one(dst, i0, ls, bl, 0, col, c0);
        stage_one(dst, i0 + 32, ls, bl, 1, col, c0);
      } else {
        const int pb = (e >> 5) % PB;
        const int ls = e / (PB * 32);
        stage_one(dst, e, ls, pb / P, pb % P, col, c0);
      }
    }
  };
  auto round_own = [&](int buf) {
    // each thread rounds the elements it staged itself (visible after its own wait)
    if constexpr (KIND == KIND_SCALAR) {
      float2* d = reinterpret_cast<float2*>(stage + buf * kStageElems);
      for (int e = threadIdx.x; e < kStageElems; e += kThreads) {
        float2 v = d[e];
        d[e] = make_float2(round_to_bf16(v.x), round_to_bf16(v.y));
      }
    } else if constexpr (KIND == KIND_REAL) {
      float* d = reinterpret_cast<float*>(stage + buf * kStageElems);
      for (int e = threadIdx.x; e < kStageElems; e += kThreads) d[e] = round_to_bf16(d[e]);
    }
  };
  auto combine_own = [&](int buf, bool round) {
    // vector kind: (c0, c1) -> (u, v) in place, on this thread's own pairs
    if constexpr (KIND == KIND_VECTOR) {
      float2* d = reinterpret_cast<float2*>(stage + buf * kStageElems);
      for (int e = threadIdx.x; e < kStageUnits; e += kThreads) {
        const int col = e & 31;
        const int bl = (e >> 5) % NB;
        const int ls = e / (NB * 32);
        const int i0 = (ls * PB + 2 * bl) * 32 + col;
        float2 a = d[i0], b = d[i0 + 32];
        if (round) {
          a = make_float2(round_to_bf16(a.x), round_to_bf16(a.y));
          b = make_float2(round_to_bf16(b.x), round_to_bf16(b.y));
        }
        d[i0] = make_float2(a.x - b.y, a.y + b.x);
        d[i0 + 32] = make_float2(a.x + b.y, a.y - b.x);
      }
    }
  };

  // ---- table register ring ----
  const unsigned long long pol = evict_first_policy();
  float wr0[kRing][kRowsPerWarp];
  float wr1[kRing][kRowsPerWarp];
  auto load_step = [&](int slot_s, float (&d0)[kRowsPerWarp], float (&d1)[kRowsPerWarp]) {
    const unsigned so = (unsigned)slot_s * sstride;
    bool sok = slot_s < r_end;
    if (DIR == DIR_INV) sok = sok && slot_s >= mg;  // l >= m
    if constexpr (GROUPED) {
      const bool ok = sok && gvalid;
      const float* a = w0 + gbase + so;
      if constexpr (KIND == KIND_VECTOR) {
        const float4 u = ld_stream4(a, ok, pol);      // rows 0,1 x (W0, W1)
        const float4 v = ld_stream4(a + 4, ok, pol);  // rows 2,3 x (W0, W1)
        d0[0] = u.x; d1[0] = u.y; d0[1] = u.z; d1[1] = u.w;
        d0[2] = v.x; d1[2] = v.y; d0[3] = v.z; d1[3] = v.w;
      } else {
        const float4 u = ld_stream4(a, ok, pol);
        d0[0] = u.x; d0[1] = u.y; d0[2] = u.z; d0[3] = u.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i) {
        const bool ok = sok && ((vmask >> i) & 1u);
        const unsigned off = roff[i] + so;
        d0[i] = ld_stream(w0 + off, ok, pol);
        if (KIND == KIND_VECTOR) d1[i] = ld_stream(w1 + off, ok, pol);
      }
    }
  };

  // L2 prefetch of the table lines of one future chunk: lane q < kChunk takes
  // step q, every valid row and table, first and last line of the 32 orders
  auto prefetch_chunk = [&](int chunk) {
    if constexpr (GROUPED) {
      // the warp's chunk is one contiguous block: one bulk prefetch by lane 0
      const int s0 = r_begin + chunk * kChunk;
      if (lane != 0 || s0 >= r_end || !pf_any) return;
      const int n = min(kChunk, r_end - s0);
      prefetch_l2_bulk(w0 + gwarp + (unsigned)s0 * sstride, (unsigned)(n * 32 * GF * 4));
      return;
    }
    if (lane >= kChunk) return;
    const int s = r_begin + chunk * kChunk + lane;
    if (s >= r_end) return;
    const unsigned so = (unsigned)s * sstride;
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      if (!((pf_mask >> i) & 1u)) continue;
      const float* a0 = w0 + pf_off[i] + so;
      prefetch_l2(a0);
      const bool two = ((reinterpret_cast<uintptr_t>(a0) >> 7) !=
                        (reinterpret_cast<uintptr_t>(a0 + m_last) >> 7));
      if (two) prefetch_l2(a0 + m_last);
      if (KIND == KIND_VECTOR) {
        const float* a1 = w1 + pf_off[i] + so;
        prefetch_l2(a1);
        if (two) prefetch_l2(a1 + m_last);
      }
    }
  };

  if (nchunks > 0) {
#pragma unroll
    for (int q = 0; q < kPrefetchChunks; ++q) prefetch_chunk(q);
    if constexpr (kAsyncStage) {
      stage_chunk(0, 0);
      cp_async_commit();
    }
#pragma unroll
    for (int q = 0; q < kRing - 1; ++q) load_step(r_begin + q, wr0[q], wr1[q]);

    for (int c = 0; c < nchunks; ++c) {
      const int buf = c & 1;
      if (c + kPrefetchChunks < nchunks) prefetch_chunk(c + kPrefetchChunks);
      if constexpr (kAsyncStage) {
        if (c + 1 < nchunks) stage_chunk(c + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait_1();
        if (KIND == KIND_VECTOR)
          combine_own(buf, p.round_bf16 != 0);
        else if (p.round_bf16)
          round_own(buf);
      } else {
        stage_chunk(c, buf);
      }
      __syncthreads();
      const SE* xs = stage + buf * kStageElems;
      const int c0 = r_begin + c * kChunk;
#pragma unroll 1
      for (int sh = 0; sh < kChunk; sh += kRing) {
#pragma unroll
      for (int sq = 0; sq < kRing; ++sq) {
        const int si = sh + sq;
        const int cur = sq;
        const int nxt = (sq + kRing - 1) % kRing;
        load_step(c0 + si + kRing - 1, wr0[nxt], wr1[nxt]);
        const SE* xrow = xs + si * PB * 32 + lane;
        if constexpr (KIND == KIND_SCALAR) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const float2 x = xrow[b * 32];
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) {
              const float w = wr0[cur][i];
              acc[i][b] = ffma2(make_float2(w, w), x, acc[i][b]);
            }
          }
        } else if constexpr (KIND == KIND_VECTOR) {
          // sph - i tor = Wp u and sph + i tor = Wm v with Wp = W0 + s W1,
          // Wm = W0 - s W1, u = c0 + i c1, v = c0 - i c1: two complex products
          // per (row, batch) instead of four real-table products
#pragma unroll
          for (int i = 0; i < kRowsPerWarp; ++i) {
            float wp, wm;
            if constexpr (GROUPED) {
              wp = wr0[cur][i];  // the grouped table already holds Wp, Wm
              wm = wr1[cur][i];
            } else {
              wp = fmaf(w1s, wr1[cur][i], wr0[cur][i]);
              wm = fmaf(-w1s, wr1[cur][i], wr0[cur][i]);
            }
            const float2 pwp = make_float2(wp, wp);
            const float2 pwm = make_float2(wm, wm);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              vq[i][2 * b] = ffma2(pwp, xrow[(2 * b) * 32], vq[i][2 * b]);
              vq[i][2 * b + 1] = ffma2(pwm, xrow[(2 * b + 1) * 32], vq[i][2 * b + 1]);
            }
          }
        } else {
#pragma unroll
          for (int bp = 0; bp < NB / 2; ++bp) {
            const float2 x = make_float2(xrow[(2 * bp) * 32], xrow[(2 * bp + 1) * 32]);
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) {
              const float w = wr0[cur][i];
              acc[i][bp] = ffma2(make_float2(w, w), x, acc[i][bp]);
            }
          }
        }
      }
      }
      __syncthreads();
    }
    if constexpr (kAsyncStage) cp_async_wait_0();
  }

  if constexpr (KIND == KIND_VECTOR) {
    // sph = (Wm v + Wp u) / 2,  tor = -i (Wm v - Wp u) / 2
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float2 pu = vq[i][2 * b], mv = vq[i][2 * b + 1];
        acc[i][2 * b] = make_float2(0.5f * (mv.x + pu.x), 0.5f * (mv.y + pu.y));
        acc[i][2 * b + 1] = make_float2(0.5f * (mv.y - pu.y), -0.5f * (mv.x - pu.x));
      }
  }
  // ---- cluster reduction: every warp stores its rows' partial sums into the
  // shared memory of the cluster rank that owns those rows (remote stores do not
  // stall the warp), one cluster barrier, then each owner adds the ks slices in
  // rank order (deterministic) from local shared memory.
  const int rpr = kRows / ks;  // rows per owner rank, a multiple of kRowsPerWarp
  cluster.sync();              // every CTA is done with its staging buffers (part aliases them)
  {
    const int row_local = warp * kRowsPerWarp;
    const int owner = row_local / rpr;
    const int rl0 = row_local - owner * rpr;
    float2* dst = cluster.map_shared_rank(part, owner) + ((rank * rpr + rl0) * NA) * 32 + lane;
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
      for (int a = 0; a < NA; ++a) dst[(i * NA + a) * 32] = acc[i][a];
  }
  cluster.sync();

  const int total = rpr * NA * 32;
  for (int e = threadIdx.x; e < total; e += kThreads) {
    const int col = e & 31;
    const int a = (e >> 5) % NA;
    const int rl = e / (NA * 32);
    const int rloc = rank * rpr + rl;
    float2 sum = make_float2(0.f, 0.f);
    for (int q = 0; q < ks; ++q) {
      const float2 v = part[((q * rpr + rl) * NA + a) * 32 + col];
      sum.x += v.x;
      sum.y += v.y;
    }
    const int row = row0 + rloc;
    const int mm = m0 + col;
    if (row >= p.R || mm >= p.out_cols) continue;
    sum.x *= p.scale;
    sum.y *= p.scale;
    if (KIND == KIND_REAL) {
      float* out = static_cast<float*>(p.out);
      const int b = b0 + 2 * a;
      const long long off = (long long)row * p.out_rs + mm;
      if (b < p.B) out[(long long)b * p.out_bs + off] = sum.x;
      if (b + 1 < p.B) out[(long long)(b + 1) * p.out_bs + off] = sum.y;
    } else {
      if ((p.zero_imag_col0 && mm == 0) || mm == p.nyquist) sum.y = 0.f;
      float2* out = static_cast<float2*>(p.out);
      const int b = b0 + a / P;
      const int pl = a % P;
      if (b < p.B)
        out[(long long)b * p.out_bs + (long long)pl * p.out_ps + (long long)row * p.out_rs + mm] =
            sum;
    }
  }
}

}  // namespace hsb
