// Warp-specialised streaming Legendre contraction for sm_100a (row groups of 8).
//
// Same contraction as contract.cuh (KIND_SCALAR / KIND_VECTOR, both
// directions), for the table layout HOLYSHT_TABLE_GROUPED8:
//
//   T[g][mt][s][q][lane][4]   g = row / 8, mt = m / 32, s = reduction step,
//                             lane = m % 32, q = quad of the lane's 8 rows x T tables
//   vector (T = 2): quad q holds (row 2q: T0, T1, row 2q+1: T0, T1), T0 = W0 + W1, T1 = W0 - W1
//   scalar (T = 1): quad q holds rows 4q .. 4q+3
//
// so one warp's step is one contiguous 1 KB (scalar) / 2 KB (vector) block in
// which every 16-byte read of the 32 lanes is a conflict-free 512-byte row.
//
// CTA = 8 warps x 8 rows (64 output rows) x 32 orders x NB batches, one CTA per
// SM; the reduction is split over a thread-block cluster of ks CTAs.
//   * every warp streams its own table block into a private ring of
//     shared-memory stages with cp.async.bulk (one elected lane, mbarrier
//     transaction counts), so the table never occupies registers and HBM
//     requests stay in flight without any per-load instruction;
//   * the input spectrum (shared by the 8 warps) goes through a 4-stage ring
//     staged 3 chunks ahead by all threads with cp.async.  Scalar: each
//     thread's copies arrive on the chunk's full mbarrier when they land
//     (cp.async.mbarrier.arrive.noinc).  Vector: the thread that staged a
//     (c0, c1) pair forms u = c0 + i c1, v = c0 - i c1 in place once its copies
//     have landed, then arrives.  An empty mbarrier per stage keeps a stage from
//     being refilled before every warp has read it: no __syncthreads in the
//     main loop;
//   * 8 rows per warp halve the spectrum reads per FMA relative to 4 rows; the
//     FMAs are packed f32x2 (FFMA2);
//   * persistent over work items (compute tile x batch group, longest
//     reduction first): cluster c takes items c, 2G-1-c, 2G+c, ... (snake
//     order), which balances the triangular inverse direction; ring positions
//     and mbarrier phases carry over from item to item;
//   * each item ends with a cluster reduction: every warp stores its partial
//     sums into the shared memory of the rank that owns its rows, one cluster
//     barrier, and the owner adds the ks slices in rank order (deterministic).
// Every mbarrier wait is bounded; a wait that gives up sets bit 0 of
// g_stream_error and the CTA skips the rest of its reduction: it waits for its
// outstanding cp.async copies (cp.async.wait_all) and, warp by warp, for the
// table bulk copies it issued but did not consume (bounded), issues no new
// copy, and still reaches every cluster barrier.  After bit 0 is set the
// output of that launch is undefined; the host reads the error word.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace hsb {
namespace stream {

namespace cg = cooperative_groups;

#ifndef HSB_STREAM_SPLIT
#define HSB_STREAM_SPLIT 1
#endif
constexpr int kCons = 8;                       // row groups of 8 (one table ring each) per CTA
// warps sharing one row group (1 or 2): each reads the group's whole table
// stage and accumulates all 8 rows for its share of the CTA's batches (twice
// the warps per SM to hide latency, half the registers per thread; the
// spectrum is not read twice)
constexpr int kSplit = HSB_STREAM_SPLIT;
constexpr int kWarps = kCons * kSplit;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 8;                // rows of a table group
constexpr int kWRows = kRowsPerWarp;           // rows one warp accumulates
constexpr int kRows = kCons * kRowsPerWarp;    // 64 output rows per CTA
constexpr int kMTile = 32;
#ifndef HSB_STREAM_CHUNK_V
#define HSB_STREAM_CHUNK_V 4
#endif
#ifndef HSB_STREAM_CHUNK_S
#define HSB_STREAM_CHUNK_S 8
#endif
#ifndef HSB_STREAM_TAB_STAGES_V
#define HSB_STREAM_TAB_STAGES_V 3
#endif
#ifndef HSB_STREAM_TAB_STAGES_S
#define HSB_STREAM_TAB_STAGES_S 3
#endif
// a chunk = the reduction steps of one spectrum stage and of one table stage
// per warp: 4 steps (8 KB of table per warp) for the vector kind, 8 steps
// (8 KB) for the scalar kind
constexpr int kMaxChunk = HSB_STREAM_CHUNK_V > HSB_STREAM_CHUNK_S ? HSB_STREAM_CHUNK_V : HSB_STREAM_CHUNK_S;
#ifndef HSB_STREAM_SPEC_STAGES
#define HSB_STREAM_SPEC_STAGES 4
#endif
#ifndef HSB_STREAM_SPEC_AHEAD
#define HSB_STREAM_SPEC_AHEAD 3
#endif
#ifndef HSB_STREAM_SPEC_STAGES_V
#define HSB_STREAM_SPEC_STAGES_V HSB_STREAM_SPEC_STAGES
#endif
#ifndef HSB_STREAM_SPEC_AHEAD_V
#define HSB_STREAM_SPEC_AHEAD_V HSB_STREAM_SPEC_AHEAD
#endif
// the parity-folded vector forward: 4 steps per chunk; its spectrum stage is
// twice the unfolded one, and the 4-stage spectrum ring (3 ahead) leaves room
// for 2 table stages.  Measured at 512 x 1024 b4: spectrum depth matters more
// than table depth (2 stages 1 ahead with 3 table stages: 114 vs 98 us)
#ifndef HSB_STREAM_PAR_CHUNK_V
#define HSB_STREAM_PAR_CHUNK_V 4
#endif
#ifndef HSB_STREAM_PAR_SPEC_STAGES_V
#define HSB_STREAM_PAR_SPEC_STAGES_V 4
#endif
#ifndef HSB_STREAM_PAR_SPEC_AHEAD_V
#define HSB_STREAM_PAR_SPEC_AHEAD_V 3
#endif
#ifndef HSB_STREAM_PAR_TAB_STAGES_V
#define HSB_STREAM_PAR_TAB_STAGES_V 2
#endif
// spectrum ring depth and chunks staged ahead of the one being read, per kind
template <int KIND, int FOLD = 0>
struct SpecRing {
  static constexpr bool kParV = KIND == 1 && FOLD == 1;
  static constexpr int kStages =
      kParV ? HSB_STREAM_PAR_SPEC_STAGES_V : KIND == 1 ? HSB_STREAM_SPEC_STAGES_V : HSB_STREAM_SPEC_STAGES;
  static constexpr int kAhead =
      kParV ? HSB_STREAM_PAR_SPEC_AHEAD_V : KIND == 1 ? HSB_STREAM_SPEC_AHEAD_V : HSB_STREAM_SPEC_AHEAD;
  static_assert(kStages >= kAhead + 1 && kAhead >= 1, "spectrum ring too shallow");
  static_assert((kStages & (kStages - 1)) == 0, "spectrum ring depth is a power of two");
};
constexpr int kSmemLimit = 227 * 1024 - 2048;  // dynamic shared memory per CTA, minus static and reserve
constexpr unsigned kWaitLimit = 1u << 22;

__device__ unsigned g_stream_error = 0;

struct Params {
  const float2* in;
  void* out;
  const float* table;
  long long in_bs, in_ps, in_rs;
  long long out_bs, out_ps, out_rs;
  long long t_group, t_mt;  // table strides (floats): row group of 8, m tile; a step is 256*T floats
  int B, M, R, S;           // batch, table orders, output rows, reduction extent
  int out_cols;
  float scale;
  int zero_imag_col0, nyquist;
  int n_mt, j_act, n_compute, n_zero, n_bg, ks;
  int m_off, mt_off;
  int stall_chunk;  // test hook, -1 = off: warp 0 of the first CTA never issues this table stage
  int round_bf16;   // round the staged spectrum to bfloat16 (after the caller's scaling)
  int kfull;        // PAR launches: the full latitude count K (S is ceil(K / 2))
  // Output to several GPUs (order-partitioned transforms): with n_peers > 0 every
  // output element is stored at column col_off + m of each peer[q] buffer (same
  // strides as out, plain peer stores over NVLink), or, when mc is set, once
  // through the NVLink multicast address mc (multimem.st: the switch delivers it
  // to every GPU's buffer).  n_peers == 0: the element goes to out.
  float2* peer[8];
  float2* mc;
  int n_peers;
  int col_off;
};

__device__ __forceinline__ void multimem_store(float2* addr, float2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};\n" ::"l"(addr), "f"(v.x), "f"(v.y)
               : "memory");
}

// Store one output element (offset in elements, strides of out).
__device__ __forceinline__ void store_out(const Params& p, long long off, float2 v) {
  if (p.n_peers == 0) {
    static_cast<float2*>(p.out)[off] = v;
    return;
  }
  off += p.col_off;
  if (p.mc != nullptr) {
    multimem_store(p.mc + off, v);
    return;
  }
#pragma unroll 1
  for (int q = 0; q < p.n_peers; ++q) p.peer[q][off] = v;
}

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
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
// bounded wait: false (and the error bit) instead of hanging
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  for (unsigned it = 0; it < kWaitLimit; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (it > 32) __nanosleep(32);
  }
  atomicOr(&g_stream_error, 1u);
  return false;
}
// one elected lane: expect `bytes` on `bar`, then bulk-copy them global -> shared
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "r"(ok ? 8 : 0));
}

// PAR (equatorial parity, forward direction): the reduction runs over the
// northern latitudes k < ceil(K/2) only, with the table's southern half
// folded in by symmetry, W(K-1-k) = s W(k) (W1 and the scalar table) and
// W0(K-1-k) = -s W0(k), s = (-1)^(l+m), which every grid here has.
//   scalar: the staged spectrum holds, per step, batch and lane, the
//     combinations X(k) + X(K-1-k) and X(k) - X(K-1-k) that even-l and odd-l
//     rows multiply (two sets);
//   vector: with Wp = W0 + W1, Wm = W0 - W1 (the unfolded kernel's tables),
//     Wp(K-1-k) = -s Wm(k) and Wm(K-1-k) = -s Wp(k).  The table stores
//     (Wp, Wn) with Wn = -(-1)^l Wm, and the staged spectrum holds
//     (u, t u') and (v, t v'), u = c0 + i c1, v = c0 - i c1 of row k, u', v'
//     of row K-1-k, t = (-1)^m; then, per row,
//       pu = sum_k Wp u + Wn (t u'),   mv = -(-1)^l sum_k Wn v + Wp (t v')
//     are the unfolded kernel's two sums, with no sign in the inner loop.
template <int KIND, int FOLD = 0>
struct Shape {
  static constexpr int P = KIND == 1 ? 2 : 1;  // components (KIND_VECTOR = 1)
  static constexpr int T = KIND == 1 ? 2 : 1;  // interleaved tables
  static constexpr int kStepFloats = 32 * kRowsPerWarp * T;  // one warp's step
  static constexpr int kQuads = kRowsPerWarp * T / 4;
  static constexpr int kChunk =
      FOLD == 1 ? (KIND == 1 ? HSB_STREAM_PAR_CHUNK_V : 4) : (KIND == 1 ? HSB_STREAM_CHUNK_V : HSB_STREAM_CHUNK_S);
};

// staged spectrum float2 per lane per step: the planes, or with PAR per
// batch (u, t u', v, t v') (vector) / two parity sets of one value (scalar)
template <int KIND, int NB, int FOLD>
constexpr int spec_per_step() {
  return FOLD == 1 ? (KIND == 1 ? 4 * NB : 2 * NB) : NB * Shape<KIND>::P;
}

// FOLD: 0 none, 1 forward parity fold, 2 inverse parity fold (scalar: every
// row accumulates its even-step and odd-step sums apart, NA = 2 NB)
template <int KIND, int NB, int FOLD = 0>
struct Smem {
  static constexpr int P = Shape<KIND>::P;
  static constexpr int PB = NB * P;
  static constexpr int SX = spec_per_step<KIND, NB, FOLD>();
  static constexpr int NA = (FOLD == 2 ? 2 : 1) * NB * P;  // complex accumulators per row
  static constexpr int kSpecBytes = SpecRing<KIND, FOLD>::kStages * Shape<KIND, FOLD>::kChunk * SX * 32 * 8;
  static constexpr int kStageBytes = kCons * Shape<KIND, FOLD>::kChunk * Shape<KIND>::kStepFloats * 4;  // all warps
  // table ring depth: the configured one, or as many as fit next to the spectrum ring
  static constexpr int kWant = FOLD == 1 ? (KIND == 1 ? HSB_STREAM_PAR_TAB_STAGES_V : 3)
                                         : (KIND == 1 ? HSB_STREAM_TAB_STAGES_V : HSB_STREAM_TAB_STAGES_S);
  static constexpr int kFit = (kSmemLimit - kSpecBytes) / kStageBytes;
  static constexpr int kTabStages = kWant < kFit ? kWant : kFit;
  static_assert(kTabStages >= 2, "table ring needs two stages");
  static constexpr int kTabBytes = kTabStages * kStageBytes;
  static constexpr int kPartBytes = kRows * NA * 32 * 8;
  static constexpr int kLoop = kSpecBytes + kTabBytes;
  static constexpr int kBytes = kLoop > kPartBytes ? kLoop : kPartBytes;
};

// Tile t -> m tile j and output rows [r0, r1); compute tiles first (by m
// tile), then tiles of exact zeros (rows above the diagonal, and m tiles
// with no l >= m inside the table).
template <int DIR>
__device__ __forceinline__ bool decode(const Params& p, int t, int& j, int& r0, int& r1) {
  if (t < p.n_compute) {
    int rem = t;
    for (j = 0; j < p.j_act; ++j) {
      const int first = DIR == 0 ? min(kMTile * (j + p.mt_off), p.R) : 0;
      const int cnt = (p.R - first + kRows - 1) / kRows;
      if (rem < cnt) {
        r0 = first + rem * kRows;
        r1 = min(r0 + kRows, p.R);
        return true;
      }
      rem -= cnt;
    }
  } else {
    int rem = t - p.n_compute;
    for (j = 0; j < p.n_mt; ++j) {
      const int zr = j < p.j_act ? (DIR == 0 ? min(kMTile * (j + p.mt_off), p.R) : 0) : p.R;
      const int cnt = (zr + kRows - 1) / kRows;
      if (rem < cnt) {
        r0 = rem * kRows;
        r1 = min(r0 + kRows, zr);
        return false;
      }
      rem -= cnt;
    }
  }
  j = p.n_mt;
  r0 = r1 = 0;
  return false;
}

// Exact zeros of the output outside the compute tiles (rows above the
// diagonal, and m tiles with no l >= m inside the table), spread over the
// grid's CTAs, written once the first tile's copies are in flight: the grid
// holds compute tiles only, so no SM is taken by a CTA that only writes zeros.
template <int DIR, int NB, int P>
__device__ __forceinline__ void write_zero_units(const Params& p) {
  const int nz = p.n_zero * p.n_bg;
  for (int z = blockIdx.x; z < nz; z += gridDim.x) {
    int j, r0, r1;
    decode<DIR>(p, p.n_compute + z / p.n_bg, j, r0, r1);
    const int b0 = (z % p.n_bg) * NB, m0 = j * kMTile;
    const int total = (r1 - r0) * NB * P * 32;
    for (int e = threadIdx.x; e < total; e += kThreads) {
      const int col = e & 31;
      const int a = (e >> 5) % (NB * P);
      const int row = r0 + e / (NB * P * 32);
      const int mm = m0 + col, b = b0 + a / P, pl = a % P;
      if (mm < p.out_cols && b < p.B) {
        store_out(p, (long long)b * p.out_bs + (long long)pl * p.out_ps + (long long)row * p.out_rs + mm,
                  make_float2(0.f, 0.f));
        // inverse fold: the tile's rows are the northern rows; zero their mirrors too
        if (DIR == 1 && p.kfull > 0 && p.kfull - 1 - row != row)
          store_out(p, (long long)b * p.out_bs + (long long)pl * p.out_ps +
                           (long long)(p.kfull - 1 - row) * p.out_rs + mm,
                    make_float2(0.f, 0.f));
      }
    }
  }
}

template <int KIND, int DIR, int NB, int FOLD = 0>
__global__ void __launch_bounds__(kThreads, 1) stream_kernel(const Params p) {
  constexpr bool PAR = FOLD == 1;   // forward fold
  constexpr bool IPAR = FOLD == 2;  // inverse fold
  static_assert(!PAR || DIR == 0, "the forward parity fold is for the forward direction");
  static_assert(!IPAR || (DIR == 1 && KIND == 0), "the inverse parity fold is for the scalar inverse direction");
  using S = Smem<KIND, NB, FOLD>;
  constexpr int P = S::P, PB = S::PB, NA = S::NA, SX = S::SX;
  // batches of this warp: NBW of the CTA's NB, from bh * NBW (a CTA of one
  // batch leaves its second warps idle)
  constexpr int NBW = NB >= kSplit ? NB / kSplit : NB;
  static_assert(NB % NBW == 0, "batch split");
  constexpr int NAW = (FOLD == 2 ? 2 : 1) * NBW * P;  // this warp's accumulators per row
  constexpr int T = Shape<KIND>::T;
  constexpr int kStepFloats = Shape<KIND>::kStepFloats;
  constexpr int kTabStages = S::kTabStages;
  constexpr int kChunk = Shape<KIND, FOLD>::kChunk;
  static_assert(!IPAR || kChunk % 2 == 0, "the inverse fold alternates accumulators by step");
  constexpr int kStageFloats = kChunk * kStepFloats;  // one warp's table stage
  constexpr int kSpecStageElems = kChunk * SX * 32;   // float2 per spectrum stage
  constexpr int kSpecStages = SpecRing<KIND, FOLD>::kStages;
  constexpr int kSpecAhead = SpecRing<KIND, FOLD>::kAhead;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  float2* spec = reinterpret_cast<float2*>(smem_raw);               // [stage][step][plane][lane]
  float* tab = reinterpret_cast<float*>(smem_raw + S::kSpecBytes);  // [warp][stage][step floats]
  float2* part = reinterpret_cast<float2*>(smem_raw);  // [source rank][owned row][NA][lane], after a tile
  __shared__ __align__(8) uint64_t full_bar[kSpecStages], empty_bar[kSpecStages];
  __shared__ __align__(8) uint64_t tab_bar[kCons][S::kTabStages];
  __shared__ __align__(8) uint64_t tab_free[kCons][S::kTabStages];  // kSplit > 1: both warps read

  cg::cluster_group cluster = cg::this_cluster();
  const int ks = p.ks;
  const int rank = static_cast<int>(cluster.block_rank());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_clusters = gridDim.x / ks;
  const int cid = blockIdx.x / ks;  // this CTA's cluster: every rank walks the same items
  const int n_items = p.n_compute * p.n_bg;

  if (cid >= n_items) {  // uniform across the cluster: this CTA only writes its share of the zeros
    write_zero_units<DIR, NB, P>(p);
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSpecStages; ++i) {
      mbar_init(&full_bar[i], kThreads);
      mbar_init(&empty_bar[i], kThreads);
    }
    for (int w = 0; w < kCons; ++w)
      for (int i = 0; i < kTabStages; ++i) {
        mbar_init(&tab_bar[w][i], 1);
        mbar_init(&tab_free[w][i], kSplit * 32);
      }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // ---- spectrum ring, staged by all threads ----
  // thread -> (batch, order) column and steps st_ls0, st_ls0 + kLsStep, ... of
  // each chunk; it copies every component of those entries.  Scalar: the
  // copies arrive on the chunk's full barrier when they land (no thread waits
  // for them).  Vector: the thread waits for its own copies one chunk later,
  // forms u = c0 + i c1, v = c0 - i c1 in place (once per CTA, not per warp)
  // and then arrives.
  constexpr int kLsStep = kThreads / (NB * 32);
  constexpr int kStageIters = (kChunk + kLsStep - 1) / kLsStep;
  static_assert(kThreads % (NB * 32) == 0, "spectrum staging map");
  const int st_b = (threadIdx.x >> 5) % NB;
  const int st_ls0 = threadIdx.x / (NB * 32);
  // PAR: the thread's raw copies (rows k and K-1-k) land in its own staged
  // positions and its combine pass overwrites them (no other thread reads them)
  float2* const st_dst = PAR ? spec + st_ls0 * SX * 32 + (KIND == 1 ? st_b * 128 + 2 * lane : st_b * 32 + lane)
                             : spec + (st_ls0 * PB + st_b * P) * 32 + lane;  // + slot * kSpecStageElems
  // the staged values need a pass by the thread that staged them (after its
  // own copies landed) for the vector kind (u, v) and for bfloat16 rounding;
  // otherwise the copies publish themselves
  const bool sync_stage = PAR || KIND == 1 || p.round_bf16 != 0;
  auto bf16 = [](float v) { return __bfloat162float(__float2bfloat16_rn(v)); };
  auto rnd = [&](float2 c) { return p.round_bf16 ? make_float2(bf16(c.x), bf16(c.y)) : c; };
  int m0g_cur = 0;  // first global order of the current item (parity of m)
  auto cadd = [](float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); };
  auto csub = [](float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); };
  auto ci = [](float2 a) { return make_float2(-a.y, a.x); };  // i * a
  auto combine = [&](int slot, int c_first_step) {
    float2* d = st_dst + slot * kSpecStageElems;
#pragma unroll
    for (int it = 0; it < kStageIters; ++it) {
      if (kChunk % kLsStep == 0 || st_ls0 + it * kLsStep < kChunk) {
        if constexpr (PAR) {
          // step s of the chunk; the equator row (odd K) pairs with itself
          const bool eq = (p.kfull & 1) && c_first_step + st_ls0 + it * kLsStep == p.S - 1;
          const bool odd_lane = ((m0g_cur + lane) & 1) != 0;  // odd order m
          if constexpr (KIND == 1) {
            float4* e = reinterpret_cast<float4*>(d + it * kLsStep * SX * 32);
            // raw: e[0] = (c0, c1) at row k, e[32] = (c0, c1) at row K-1-k
            const float4 r0 = e[0], r1 = e[32];
            const float2 c0 = rnd(make_float2(r0.x, r0.y)), c1 = rnd(make_float2(r0.z, r0.w));
            // t = (-1)^m on the mirror row, which the equator (odd K) does not have
            const float t = eq ? 0.f : (odd_lane ? -1.f : 1.f);
            const float2 d0 = rnd(make_float2(r1.x, r1.y)), d1 = rnd(make_float2(r1.z, r1.w));
            const float2 u = cadd(c0, ci(c1)), v = csub(c0, ci(c1));
            const float2 uq = cadd(d0, ci(d1)), vq = csub(d0, ci(d1));
            e[0] = make_float4(u.x, u.y, t * uq.x, t * uq.y);
            e[32] = make_float4(v.x, v.y, t * vq.x, t * vq.y);
          } else {
            float2* e = d + it * kLsStep * SX * 32;
            const float2 x = rnd(e[0]);
            const float2 y = eq ? make_float2(0.f, 0.f) : rnd(e[NB * 32]);
            const float2 pl = cadd(x, y), mi = csub(x, y);
            e[0] = odd_lane ? mi : pl;          // even rows: P where m is even
            e[NB * 32] = odd_lane ? pl : mi;    // odd rows
          }
          continue;
        }
        float2* e = d + it * kLsStep * PB * 32;
        if constexpr (KIND == 1) {
          float2 c0 = e[0], c1 = e[32];
          if (p.round_bf16) {
            c0 = make_float2(bf16(c0.x), bf16(c0.y));
            c1 = make_float2(bf16(c1.x), bf16(c1.y));
          }
          e[0] = make_float2(c0.x - c1.y, c0.y + c1.x);   // u = c0 + i c1
          e[32] = make_float2(c0.x + c1.y, c0.y - c1.x);  // v = c0 - i c1
        } else {
          const float2 c0 = e[0];
          e[0] = make_float2(bf16(c0.x), bf16(c0.y));
        }
      }
    }
  };
  auto publish_async = [&](int slot) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(&full_bar[slot]))
                 : "memory");
  };
  const int grp = warp / kSplit, bh = warp % kSplit;  // row group, and which batches of it this warp takes
  const bool bact = bh * NBW < NB;                    // the warp has batches
  const int bw0 = bh * NBW;                           // its first batch (CTA-local)
  float* my = tab + grp * kTabStages * kStageFloats;

  // running ring positions over all tiles of this CTA: spectrum chunks staged
  // and consumed (global chunk g lives in slot g % kSpecStages, phase
  // (g / kSpecStages) & 1), this warp's table stages (h: slot h % kTabStages)
  int gbase = 0, tbase = 0;
  bool alive = true;

  // Items (compute tile x batch group) are ordered by decreasing reduction
  // length; cluster c takes items c, 2G-1-c, 2G+c, ... (G clusters): long and
  // short items pair up, which balances the triangular inverse direction.
  for (int round = 0;; ++round) {
    const int idx = round * n_clusters + ((round & 1) ? n_clusters - 1 - cid : cid);
    if (idx >= n_items) break;
    const int bg = idx % p.n_bg;
    int j, r0, r1;
    decode<DIR>(p, idx / p.n_bg, j, r0, r1);
    const int b0 = bg * NB;
    const int m0 = j * kMTile;
    const int m0g = m0 + p.m_off;
    m0g_cur = m0g;
    const int s_begin = DIR == 0 ? 0 : min(m0g, p.S);
    const int nsteps = p.S - s_begin;
    const int per = ((nsteps + ks * kChunk - 1) / (ks * kChunk)) * kChunk;
    const int r_begin = min(p.S, s_begin + rank * per);
    const int r_end = min(p.S, r_begin + per);
    const int nchunks = (r_end - r_begin + kChunk - 1) / kChunk;
    const int n_valid = min(kCons, (r1 - r0 + kRowsPerWarp - 1) / kRowsPerWarp);  // row groups with rows

    float2 acc[kWRows][NAW];
#pragma unroll
    for (int i = 0; i < kWRows; ++i)
#pragma unroll
      for (int a = 0; a < NAW; ++a) acc[i][a] = make_float2(0.f, 0.f);

    const bool st_ok = m0 + lane < p.M && b0 + st_b < p.B;
    const float2* st_src = p.in + (st_ok ? (long long)(b0 + st_b) * p.in_bs + m0 + lane : 0);
    auto stage = [&](int c, int slot) {
      float2* dst = st_dst + slot * kSpecStageElems;
      const int s0 = r_begin + c * kChunk + st_ls0;
#pragma unroll
      for (int it = 0; it < kStageIters; ++it) {
        if (kChunk % kLsStep == 0 || st_ls0 + it * kLsStep < kChunk) {
          const int s = s0 + it * kLsStep;
          const bool ok = st_ok && s < r_end;
          const float2* src = ok ? st_src + (long long)s * p.in_rs : p.in;
          if constexpr (PAR) {
            const float2* src2 = ok ? st_src + (long long)(p.kfull - 1 - s) * p.in_rs : p.in;
            float2* e = dst + it * kLsStep * SX * 32;
            if constexpr (KIND == 1) {  // (c0, c1) of row k, then of row K-1-k, as float4s
              cp_async8(e, ok ? src : p.in, ok);
              cp_async8(e + 1, ok ? src + p.in_ps : p.in, ok);
              cp_async8(e + 64, ok ? src2 : p.in, ok);
              cp_async8(e + 65, ok ? src2 + p.in_ps : p.in, ok);
            } else {
              cp_async8(e, ok ? src : p.in, ok);
              cp_async8(e + NB * 32, ok ? src2 : p.in, ok);
            }
            continue;
          }
#pragma unroll
          for (int pl = 0; pl < P; ++pl)
            cp_async8(dst + (it * kLsStep * PB + pl) * 32, ok ? src + pl * p.in_ps : p.in, ok);
        }
      }
    };
    // stage chunk c of this tile (global chunk gbase + c), after the slot's previous reader is done
    auto stage_chunk = [&](int c) -> bool {
      const int g = gbase + c;
      const int slot = g & (kSpecStages - 1);
      if (g >= kSpecStages && !mbar_wait(&empty_bar[slot], ((g / kSpecStages) - 1) & 1)) return false;
      stage(c, slot);
      if (!sync_stage) publish_async(slot);
      return true;
    };

    // ---- this warp's table ring (one stage per chunk) ----
    const bool has_rows = grp < n_valid;
    const int g8 = (r0 >> 3) + grp;  // row group of 8 (r0 is a multiple of 8)
    const float* tsrc = p.table + (long long)(has_rows ? g8 : 0) * p.t_group + (long long)j * p.t_mt +
                        (long long)r_begin * kStepFloats;
    const int nst = has_rows ? nchunks : 0;
    auto issue_tab = [&](int q) {
      // test hook: the stage is never requested, so its wait runs out (bounded)
      if (q == p.stall_chunk && round == 0 && blockIdx.x == 0 && warp == 0) return;
      const int n = min(kChunk, r_end - (r_begin + q * kChunk));
      const int slot = (tbase + q) % kTabStages;
      bulk_load(my + slot * kStageFloats, tsrc + (long long)q * kChunk * kStepFloats,
                (unsigned)(n * kStepFloats * 4), &tab_bar[grp][slot]);
    };
    if (bh == 0 && lane == 0 && alive && nst > 0) {
      // the ring memory was last written by the generic proxy (partial sums)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      for (int q = 0; q < kTabStages && q < nst; ++q) issue_tab(q);
    }
    int issued = min(kTabStages, nst);

    auto step = [&](const float* ts, const float2* xs, auto hc) {
      // hc: step parity within the chunk (inverse fold: which accumulator half)
      constexpr int H = decltype(hc)::value;
      // ts: this step's table block; xs: this step's staged spectrum planes
      // (vector: planes 2b, 2b+1 hold u, v of batch b)
      constexpr int kQW = Shape<KIND>::kQuads;  // quads of this warp's rows
      float w[kWRows * T];
#pragma unroll
      for (int q = 0; q < kQW; ++q) {
        const float4 v = reinterpret_cast<const float4*>(ts)[q * 32 + lane];
        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
      }
      if constexpr (PAR && KIND == 1) {
        // per batch (u, t u') and (v, t v'); rows hold (Wp, Wn)
        const float4* xv = reinterpret_cast<const float4*>(xs) + bw0 * 64 + lane;
#pragma unroll
        for (int b = 0; b < NBW; ++b) {
          const float4 uu = xv[b * 64], vv = xv[b * 64 + 32];
#pragma unroll
          for (int i = 0; i < kWRows; ++i) {
            const float wp = w[2 * i], wn = w[2 * i + 1];
            acc[i][2 * b] = __ffma2_rn(make_float2(wp, wp), make_float2(uu.x, uu.y), acc[i][2 * b]);
            acc[i][2 * b] = __ffma2_rn(make_float2(wn, wn), make_float2(uu.z, uu.w), acc[i][2 * b]);
            acc[i][2 * b + 1] = __ffma2_rn(make_float2(wn, wn), make_float2(vv.x, vv.y), acc[i][2 * b + 1]);
            acc[i][2 * b + 1] = __ffma2_rn(make_float2(wp, wp), make_float2(vv.z, vv.w), acc[i][2 * b + 1]);
          }
        }
        return;
      }
      if constexpr (PAR) {
        // set 0 feeds the warp's even rows, set 1 its odd rows (kWRows == 8)
#pragma unroll
        for (int set = 0; set < 2; ++set) {
          float2 xv[NBW];
#pragma unroll
          for (int b = 0; b < NBW; ++b) xv[b] = xs[(set * NB + bw0 + b) * 32 + lane];
#pragma unroll
          for (int i = set; i < kWRows; i += 2) {
#pragma unroll
            for (int b = 0; b < NBW; ++b) acc[i][b] = __ffma2_rn(make_float2(w[i], w[i]), xv[b], acc[i][b]);
          }
        }
        return;
      }
      float2 x[NBW * P];
#pragma unroll
      for (int a = 0; a < NBW * P; ++a) x[a] = xs[(bw0 * P + a) * 32 + lane];
#pragma unroll
      for (int i = 0; i < kWRows; ++i) {
        if constexpr (KIND == 1) {
          const float wp = w[2 * i], wm = w[2 * i + 1];
#pragma unroll
          for (int b = 0; b < NBW; ++b) {
            acc[i][2 * b] = __ffma2_rn(make_float2(wp, wp), x[2 * b], acc[i][2 * b]);
            acc[i][2 * b + 1] = __ffma2_rn(make_float2(wm, wm), x[2 * b + 1], acc[i][2 * b + 1]);
          }
        } else {
          const float wv = w[i];
#pragma unroll
          for (int b = 0; b < NBW; ++b)
            acc[i][(IPAR ? H * NBW : 0) + b] =
                __ffma2_rn(make_float2(wv, wv), x[b], acc[i][(IPAR ? H * NBW : 0) + b]);
        }
      }
    };

    int consumed = 0;  // table stages of this tile this warp has consumed
    if (alive) {
#pragma unroll
      for (int q = 0; q < kSpecAhead; ++q) {
        if (q < nchunks && alive) alive = stage_chunk(q);
        if (sync_stage) cp_async_commit();
      }
      // the first item's copies are in flight: now the zeros (fire-and-forget
      // stores that drain while the table stream ramps up)
      if (round == 0) write_zero_units<DIR, NB, P>(p);
      if (sync_stage) {
        if (nchunks > 0 && alive) {
          cp_async_wait<kSpecAhead - 1>();  // this thread's copies of chunk 0 have landed
          combine(gbase & (kSpecStages - 1), r_begin);
          mbar_arrive(&full_bar[gbase & (kSpecStages - 1)]);
        }
      }
    }
    for (int c = 0; c < nchunks && alive; ++c) {
      const int cn = c + kSpecAhead;
      if (cn < nchunks && !stage_chunk(cn)) {
        alive = false;
        break;
      }
      if (sync_stage) {
        cp_async_commit();
        if (c + 1 < nchunks) {
          cp_async_wait<kSpecAhead - 1>();  // this thread's copies of chunk c + 1 have landed
          const int s1 = (gbase + c + 1) & (kSpecStages - 1);
          combine(s1, r_begin + (c + 1) * kChunk);
          mbar_arrive(&full_bar[s1]);
        }
      }
      const int g = gbase + c;
      const int cs = g & (kSpecStages - 1);
      if (!mbar_wait(&full_bar[cs], (g / kSpecStages) & 1)) {
        alive = false;
        break;
      }
      if (has_rows) {
        const int h = tbase + c;
        const int ts_ = h % kTabStages;
        if (!mbar_wait(&tab_bar[grp][ts_], (h / kTabStages) & 1)) {
          alive = false;
          break;
        }
        const float2* xs = spec + cs * kSpecStageElems;
        const float* tsb = my + ts_ * kStageFloats;
        const int s0 = r_begin + c * kChunk;
        if (!bact) {
          // no batches for this warp: it only releases the table stage below
        } else if (s0 + kChunk <= r_end) {
#pragma unroll
          for (int ls = 0; ls < kChunk; ls += 2) {
            step(tsb + ls * kStepFloats, xs + ls * SX * 32, std::integral_constant<int, 0>{});
            if (kChunk > 1)
              step(tsb + (ls + 1) * kStepFloats, xs + (ls + 1) * SX * 32, std::integral_constant<int, 1>{});
          }
        } else {
#pragma unroll 1
          for (int ls = 0; ls < r_end - s0; ++ls) {
            if (ls & 1)
              step(tsb + ls * kStepFloats, xs + ls * SX * 32, std::integral_constant<int, 1>{});
            else
              step(tsb + ls * kStepFloats, xs + ls * SX * 32, std::integral_constant<int, 0>{});
          }
        }
        ++consumed;
        // stage consumed by every lane (of both warps of the group): refill it
        // with chunk c + kTabStages
        __syncwarp();
        if constexpr (kSplit > 1) mbar_arrive(&tab_free[grp][ts_]);
        if (bh == 0 && lane == 0 && issued < nst) {
          if (kSplit == 1 || mbar_wait(&tab_free[grp][ts_], (h / kTabStages) & 1)) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            issue_tab(issued);
          } else {
            alive = false;
          }
        }
        ++issued;
      }
      mbar_arrive(&empty_bar[cs]);
    }
    // nothing may still be writing into the rings when they become the partial-sum buffer
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    if (!alive && bh == 0 && lane == 0 && has_rows) {
      // a wait gave up: let this warp's table copies still in flight land first
      const int done = min(issued, nst);
      for (int q = consumed; q < done; ++q) {
        const int h = tbase + q;
        mbar_wait(&tab_bar[grp][h % kTabStages], (h / kTabStages) & 1);
      }
    }
    __syncwarp();
    gbase += nchunks;
    tbase += nst;

    if constexpr (IPAR) {
      // accumulator halves: A = steps l with l = r_begin (mod 2), B = the others.
      // With e / o the sums over even / odd l + m (m = m0 + lane, m0 even), the
      // northern row k receives e + o and its mirror K-1-k receives e - o.
      const bool a_is_even = ((r_begin + lane) & 1) == 0;
#pragma unroll
      for (int i = 0; i < kWRows; ++i)
#pragma unroll
        for (int b = 0; b < NBW; ++b) {
          const float2 A = acc[i][b], Bv = acc[i][NBW + b];
          acc[i][b] = make_float2(A.x + Bv.x, A.y + Bv.y);
          acc[i][NBW + b] = a_is_even ? make_float2(A.x - Bv.x, A.y - Bv.y) : make_float2(Bv.x - A.x, Bv.y - A.y);
        }
    }
    if constexpr (KIND == 1) {
      // sph = (Wm v + Wp u) / 2,  tor = -i (Wm v - Wp u) / 2
      // (PAR: the mv sum carries the factor -(-1)^l; tile rows start even)
#pragma unroll
      for (int i = 0; i < kWRows; ++i)
#pragma unroll
        for (int b = 0; b < NBW; ++b) {
          const float2 pu = acc[i][2 * b];
          float2 mv = acc[i][2 * b + 1];
          if (PAR && ((r0 + grp * kRowsPerWarp + i) & 1) == 0) mv = make_float2(-mv.x, -mv.y);
          acc[i][2 * b] = make_float2(0.5f * (mv.x + pu.x), 0.5f * (mv.y + pu.y));
          acc[i][2 * b + 1] = make_float2(0.5f * (mv.y - pu.y), -0.5f * (mv.x - pu.x));
        }
    }

    // ---- cluster reduction: every warp stores its rows' partial sums straight
    // into the shared memory of the cluster rank that owns those rows (remote
    // stores do not stall the warp), one cluster barrier, then each owner adds
    // its ks slices in rank order (deterministic) from local shared memory.
    const int rpr = kRows / ks;  // rows per owner rank, a multiple of 8
    cluster.sync();              // every CTA of the cluster is done with its rings
    {
      const int row_local = grp * kRowsPerWarp;  // first row of this warp in the tile
      const int owner = row_local / rpr;
      const int rl0 = row_local - owner * rpr;
      float2* dst = cluster.map_shared_rank(part, owner) + ((rank * rpr + rl0) * NA) * 32 + lane;
      // local accumulator a -> the CTA's index: batch-major (b * P + plane), or
      // with the inverse fold half h of batch b at h * NB + b
      auto gidx = [&](int a) { return IPAR ? (a / NBW) * NB + bw0 + a % NBW : bw0 * P + a; };
      if (bact) {
#pragma unroll
        for (int i = 0; i < kWRows; ++i)
#pragma unroll
          for (int a = 0; a < NAW; ++a) dst[(i * NA + gidx(a)) * 32] = acc[i][a];
      }
    }
    cluster.sync();

    const int total = rpr * NA * 32;
    for (int e = threadIdx.x; e < total; e += kThreads) {
      const int col = e & 31;
      const int a = (e >> 5) % NA;
      const int rl = e / (NA * 32);
      const int row = r0 + rank * rpr + rl;
      const int mm = m0 + col;
      if (row >= r1 || mm >= p.out_cols) continue;
      float2 sum = make_float2(0.f, 0.f);
      for (int q = 0; q < ks; ++q) {
        const float2 v = part[((q * rpr + rl) * NA + a) * 32 + col];
        sum.x += v.x;
        sum.y += v.y;
      }
      sum.x *= p.scale;
      sum.y *= p.scale;
      // irfft preparation acts on global orders: column mm holds order m_off + mm
      // (an order slice of a partitioned transform starts at m_off)
      const int gcol = mm + p.m_off;
      if ((p.zero_imag_col0 && gcol == 0) || gcol == p.nyquist) sum.y = 0.f;
      if constexpr (IPAR) {  // a < NB: northern row; a >= NB: its mirror (not the equator twice)
        const int b = b0 + a % NB;
        const int orow = a < NB ? row : p.kfull - 1 - row;
        if (b < p.B && (a < NB || orow != row))
          store_out(p, (long long)b * p.out_bs + (long long)orow * p.out_rs + mm, sum);
        continue;
      }
      const int b = b0 + a / P, pl = a % P;
      if (b < p.B)
        store_out(p, (long long)b * p.out_bs + (long long)pl * p.out_ps + (long long)row * p.out_rs + mm, sum);
    }
    __syncthreads();  // partial sums read: the next tile's copies may reuse the memory
  }
}

}  // namespace stream
}  // namespace hsb
