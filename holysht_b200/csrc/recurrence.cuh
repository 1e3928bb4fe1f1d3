// Forward Legendre transforms with on-the-fly associated Legendre functions
// (the "recurrence" variant): no table stream.
//
//   out[b, l, m] = scale * sum_k X[b, k, m] * w_k P_l^m(x_k)        (l >= m)
//
// P is generated in registers by the three-term recurrence in l
//   P_l = a_lm x P_{l-1} - b_lm P_{l-2}
// in fp32, re-seeded every kSeg degrees from checkpoints (P_{l0}, P_{l0+1})
// computed in float64 on the host (quadrature weight folded in; values below
// fp32 range are exact zeros, which is what they contribute).  Re-seeding
// bounds the fp32 drift of the recurrence: with 16-degree segments the
// coefficients stay within ~6e-7 relative L2 of the float64 transform at
// lmax = 512.  The vector form runs the recurrences of orders m - 1 and m + 1
// and combines them by the ladder identities.
//
// Two kernel families: the segment-per-thread kernels (the default; one
// thread per order and checkpoint segment, partial sums in registers, see
// below) and the earlier paired-latitude kernels (threads over latitude with
// warp transpose-reductions every few degrees), kept for comparison.
#pragma once

#include <cuda_runtime.h>

#include <atomic>

namespace hsb {
namespace rec {

constexpr int kSeg = 16;      // degrees per checkpoint segment
constexpr int kNB = 4;        // batches per CTA
constexpr int kMaxWarps = 8;  // nlat <= 8 * 32 * 8 = 2048

struct RecParams {
  const float2* spec;  // [B][K][W] complex, element (b, k, m) at b*sbs + k*srs + m
  long long sbs, srs;
  const float* seeds;  // [M][nseg][K][2]
  const float* coef;   // [M][L][2]: a_lm, b_lm
  const float* x;      // [K] cos(theta_k)
  float2* out;         // [B][L][M]
  int B, K, L, M, nseg;
  float scale;
};

#ifndef HSB_REC_SEGS_PER_CTA
#define HSB_REC_SEGS_PER_CTA 4
#endif
constexpr int kSegPerCta = HSB_REC_SEGS_PER_CTA;  // checkpoint segments per CTA

// ---------------------------------------------------------------------------
// Paired-latitude scalar kernel (HSB_REC_PAIR=1, kept for comparison with the
// segment-per-thread kernel below, which the library launches by default):
//   * each thread holds KPT latitudes as KPT/2 pairs; the recurrence and the
//     contraction run on packed f32x2 operations whose two halves are the two
//     latitudes of a pair (fma.rn.f32x2 with no operand duplication: the
//     pair of Legendre values multiplies a pair of spectrum values directly);
//   * KPT = 16 latitudes per thread (one warp per 512 latitudes), so the
//     per-degree warp reduction (a transpose-reduce every 4 degrees) is
//     amortised over 4x the multiply-adds of the 4-latitude kernel;
//   * the CTA's recurrence coefficients (a, -b) sit in shared memory.
template <int KPT>
__global__ void __launch_bounds__(kMaxWarps * 32) recurrence_forward_pair_kernel(const RecParams p) {
  constexpr int NP = KPT / 2;
  __shared__ float red[kMaxWarps][32];
  __shared__ float2 cab[kSegPerCta * kSeg];
  const int m = blockIdx.x;
  const int b0 = blockIdx.z * kNB;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int lm = p.L - m;
  const int nseg = lm > 0 ? (lm + kSeg - 1) / kSeg : 0;
  const int c_begin = blockIdx.y * kSegPerCta;

  if (blockIdx.y == 0) {
    const int zrows = lm > 0 ? m : p.L;
    for (int e = tid; e < zrows * kNB; e += blockDim.x) {
      const int l = e / kNB, b = b0 + e % kNB;
      if (b < p.B) p.out[((long long)b * p.L + l) * p.M + m] = make_float2(0.f, 0.f);
    }
  }
  if (c_begin >= nseg) return;  // uniform per CTA
  const int c_end = min(nseg, c_begin + kSegPerCta);
  const int l_first = m + c_begin * kSeg;
  const int ndeg = min(p.L, m + c_end * kSeg) - l_first;
  for (int e = tid; e < kSegPerCta * kSeg; e += blockDim.x) {
    float2 ab = make_float2(0.f, 0.f);
    if (e < ndeg) {
      const float* c2 = p.coef + ((long long)m * p.L + l_first + e) * 2;
      ab = make_float2(c2[0], -c2[1]);
    }
    cab[e] = ab;
  }

  const int k0 = tid * KPT;
  float2 xp[NP];
  float2 Xr[NP][kNB], Xi[NP][kNB];  // (latitude 2i, 2i+1) pairs of the scaled spectrum
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int k = k0 + 2 * i;
    xp[i] = make_float2(k < p.K ? p.x[k] : 0.f, k + 1 < p.K ? p.x[k + 1] : 0.f);
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float2 s0 = make_float2(0.f, 0.f), s1 = s0;
      if (b0 + b < p.B) {
        const float2* row = p.spec + (long long)(b0 + b) * p.sbs + m;
        if (k < p.K) s0 = row[(long long)k * p.srs];
        if (k + 1 < p.K) s1 = row[(long long)(k + 1) * p.srs];
      }
      Xr[i][b] = make_float2(s0.x * p.scale, s1.x * p.scale);
      Xi[i][b] = make_float2(s0.y * p.scale, s1.y * p.scale);
    }
  }
  __syncthreads();  // coefficients staged

  // checkpoints of segment c: (P at lseg, P at lseg + 1) of latitudes 2i and 2i+1
  // (8-byte aligned pairs: a 16-byte load would be misaligned for odd nlat).
  // The next segment's are loaded while this one is computed.
  float2 sa[NP], sb[NP];
  auto load_seeds = [&](int c) {
    const float2* sd2 = reinterpret_cast<const float2*>(p.seeds + (((long long)m * p.nseg + c) * p.K + k0) * 2);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      sa[i] = k0 + 2 * i < p.K ? sd2[2 * i] : make_float2(0.f, 0.f);
      sb[i] = k0 + 2 * i + 1 < p.K ? sd2[2 * i + 1] : make_float2(0.f, 0.f);
    }
  };
  load_seeds(c_begin);
  for (int c = c_begin; c < c_end; ++c) {
    const int lseg = m + c * kSeg;
    float2 p1[NP], p2[NP];  // P at degrees l-1 and l-2 of each latitude pair
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      p2[i] = make_float2(sa[i].x, sb[i].x);  // degree lseg
      p1[i] = make_float2(sa[i].y, sb[i].y);  // degree lseg + 1
    }
    if (c + 1 < c_end) load_seeds(c + 1);
#pragma unroll
    for (int qb = 0; qb < kSeg; qb += 4) {
      float v[32];  // 4 degrees x (4 batches x re/im)
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int q = qb + q4;
        float2 pl[NP];
        if (q == 0) {
#pragma unroll
          for (int i = 0; i < NP; ++i) pl[i] = p2[i];
        } else if (q == 1) {
#pragma unroll
          for (int i = 0; i < NP; ++i) pl[i] = p1[i];
        } else {
          const float2 ab = cab[lseg + q - l_first];
          const float2 a2 = make_float2(ab.x, ab.x), nb2 = make_float2(ab.y, ab.y);
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            pl[i] = __ffma2_rn(a2, __fmul2_rn(xp[i], p1[i]), __fmul2_rn(nb2, p2[i]));
            p2[i] = p1[i];
            p1[i] = pl[i];
          }
        }
        float2 ar[kNB], ai[kNB];
#pragma unroll
        for (int b = 0; b < kNB; ++b) ar[b] = ai[b] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < NP; ++i)
#pragma unroll
          for (int b = 0; b < kNB; ++b) {
            ar[b] = __ffma2_rn(pl[i], Xr[i][b], ar[b]);
            ai[b] = __ffma2_rn(pl[i], Xi[i][b], ai[b]);
          }
#pragma unroll
        for (int b = 0; b < kNB; ++b) {
          v[q4 * 8 + 2 * b] = ar[b].x + ar[b].y;
          v[q4 * 8 + 2 * b + 1] = ai[b].x + ai[b].y;
        }
      }
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < d; ++i) {
          const float send = upper ? v[i] : v[i + d];
          const float keep = upper ? v[i + d] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
      float sum = v[0];
      if (nwarps > 1) {
        red[warp][lane] = sum;
        __syncthreads();
        sum = 0.f;
        if (warp == 0)
          for (int w = 0; w < nwarps; ++w) sum += red[w][lane];
      }
      if (warp == 0) {
        const int q4 = lane >> 3, b = (lane >> 1) & 3, ri = lane & 1;
        const int l = lseg + qb + q4;
        if (l < p.L && b0 + b < p.B)
          reinterpret_cast<float*>(p.out)[(((long long)(b0 + b) * p.L + l) * p.M + m) * 2 + ri] = sum;
      }
      if (nwarps > 1) __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Vector forward with on-the-fly tables.  The vector tables of order m are
// ladder combinations of the Legendre functions of orders m - 1 and m + 1:
//   W0[l, k] = alpha_l Q^{m-1}_l + beta_l Q^{m+1}_l
//   W1[l, k] = gamma_l Q^{m-1}_{l+1} + delta_l Q^{m+1}_{l+1},   Q^{m'}_l = w_k P_l^{m'}(x_k)
// Both recurrences run upwards in l in fp32 from float64 checkpoints every
// kSeg degrees (the state is (Q_l, Q_{l+1}) for each order), and the
// contraction is evaluated in the (W0 + W1, W0 - W1) form with u = c0 + i c1,
// v = c0 - i c1:  sph - i tor = sum_k (W0 + W1) u,  sph + i tor = sum_k (W0 - W1) v.
struct VecRecParams {
  const float2* spec;  // element (b, component, k, m) at b*sbs + p*sps + k*srs + m
  long long sbs, sps, srs;
  const float* seeds;  // [M][nseg][K][4]: Q^{m-1}_{l0}, Q^{m-1}_{l0+1}, Q^{m+1}_{l0}, Q^{m+1}_{l0+1}
  const float* coef;   // [M][L][8]: a, b (order m-1), a, b (order m+1) at degree l+2; alpha, beta, gamma, delta
  const float* x;      // [K] cos(theta_k)
  float2* out;         // [B][2][L][M]
  int B, K, L, M, nseg;
  float scale;
};

// Paired-latitude vector kernel (HSB_REC_PAIR=1, kept for comparison): both
// recurrences, the table combinations and the contraction on packed f32x2
// operations over latitude pairs (no operand duplication), KPT latitudes per
// thread, a transpose-reduce over the warp every 2 degrees.
template <int KPT>
__global__ void __launch_bounds__(kMaxWarps * 32) recurrence_vector_forward_pair_kernel(const VecRecParams p) {
  constexpr int NP = KPT / 2;
  __shared__ float red[kMaxWarps][32];
  __shared__ float cf[kSegPerCta * kSeg][8];  // am, -bm, ap, -bp, alpha, beta, gamma, delta
  const int m = blockIdx.x;
  const int b0 = blockIdx.z * kNB;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int lm = p.L - m;
  const int nseg = lm > 0 ? (lm + kSeg - 1) / kSeg : 0;
  const int c_begin = blockIdx.y * kSegPerCta;
  const long long plane = (long long)p.L * p.M;

  if (blockIdx.y == 0) {
    const int zrows = lm > 0 ? m : p.L;
    for (int e = tid; e < zrows * kNB * 2; e += blockDim.x) {
      const int l = e / (kNB * 2), r = e % (kNB * 2), b = b0 + r / 2, pc = r % 2;
      if (b < p.B) p.out[((long long)b * 2 + pc) * plane + (long long)l * p.M + m] = make_float2(0.f, 0.f);
    }
  }
  if (c_begin >= nseg) return;  // uniform per CTA
  const int c_end = min(nseg, c_begin + kSegPerCta);
  const int l_first = m + c_begin * kSeg;
  const int ndeg = min(p.L, m + c_end * kSeg) - l_first;
  for (int e = tid; e < kSegPerCta * kSeg * 8; e += blockDim.x) {
    const int dl = e / 8, f = e % 8;
    float v = dl < ndeg ? p.coef[((long long)m * p.L + l_first + dl) * 8 + f] : 0.f;
    cf[dl][f] = (f == 1 || f == 3) ? -v : v;
  }

  const int k0 = tid * KPT;
  float2 xp[NP];
  float2 ur[NP][kNB], ui[NP][kNB], vr[NP][kNB], vi[NP][kNB];  // latitude pairs of u = c0 + i c1, v = c0 - i c1
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int k = k0 + 2 * i;
    xp[i] = make_float2(k < p.K ? p.x[k] : 0.f, k + 1 < p.K ? p.x[k + 1] : 0.f);
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float2 c0a = make_float2(0.f, 0.f), c1a = c0a, c0b = c0a, c1b = c0a;
      if (b0 + b < p.B) {
        const float2* base = p.spec + (long long)(b0 + b) * p.sbs + m;
        if (k < p.K) {
          c0a = base[(long long)k * p.srs];
          c1a = base[(long long)k * p.srs + p.sps];
        }
        if (k + 1 < p.K) {
          c0b = base[(long long)(k + 1) * p.srs];
          c1b = base[(long long)(k + 1) * p.srs + p.sps];
        }
      }
      const float sc = p.scale;
      ur[i][b] = make_float2((c0a.x - c1a.y) * sc, (c0b.x - c1b.y) * sc);
      ui[i][b] = make_float2((c0a.y + c1a.x) * sc, (c0b.y + c1b.x) * sc);
      vr[i][b] = make_float2((c0a.x + c1a.y) * sc, (c0b.x + c1b.y) * sc);
      vi[i][b] = make_float2((c0a.y - c1a.x) * sc, (c0b.y - c1b.x) * sc);
    }
  }
  __syncthreads();  // coefficients staged

  for (int c = c_begin; c < c_end; ++c) {
    const int lseg = m + c * kSeg;
    const float4* sd = reinterpret_cast<const float4*>(p.seeds + (((long long)m * p.nseg + c) * p.K + k0) * 4);
    float2 qm0[NP], qm1[NP], qp0[NP], qp1[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const float4 a = k0 + 2 * i < p.K ? sd[2 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 bq = k0 + 2 * i + 1 < p.K ? sd[2 * i + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
      qm0[i] = make_float2(a.x, bq.x);
      qm1[i] = make_float2(a.y, bq.y);
      qp0[i] = make_float2(a.z, bq.z);
      qp1[i] = make_float2(a.w, bq.w);
    }
#pragma unroll
    for (int qb = 0; qb < kSeg; qb += 2) {
      float v[32];  // 2 degrees x (4 batches x (u, v) x re/im)
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        const float* k8 = cf[lseg + qb + q2 - l_first];
        const float2 am = make_float2(k8[0], k8[0]), nbm = make_float2(k8[1], k8[1]);
        const float2 ap = make_float2(k8[2], k8[2]), nbp = make_float2(k8[3], k8[3]);
        const float2 al = make_float2(k8[4], k8[4]), be = make_float2(k8[5], k8[5]);
        const float2 ga = make_float2(k8[6], k8[6]), de = make_float2(k8[7], k8[7]);
        float2 wp[NP], wm[NP];
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const float2 w0 = __ffma2_rn(al, qm0[i], __fmul2_rn(be, qp0[i]));
          const float2 w1 = __ffma2_rn(ga, qm1[i], __fmul2_rn(de, qp1[i]));
          wp[i] = __fadd2_rn(w0, w1);
          wm[i] = __fadd2_rn(w0, make_float2(-w1.x, -w1.y));
          // both recurrences to degree l + 2
          const float2 nm = __ffma2_rn(am, __fmul2_rn(xp[i], qm1[i]), __fmul2_rn(nbm, qm0[i]));
          const float2 np = __ffma2_rn(ap, __fmul2_rn(xp[i], qp1[i]), __fmul2_rn(nbp, qp0[i]));
          qm0[i] = qm1[i];
          qm1[i] = nm;
          qp0[i] = qp1[i];
          qp1[i] = np;
        }
#pragma unroll
        for (int b = 0; b < kNB; ++b) {
          float2 aur = make_float2(0.f, 0.f), aui = aur, avr = aur, avi = aur;
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            aur = __ffma2_rn(wp[i], ur[i][b], aur);
            aui = __ffma2_rn(wp[i], ui[i][b], aui);
            avr = __ffma2_rn(wm[i], vr[i][b], avr);
            avi = __ffma2_rn(wm[i], vi[i][b], avi);
          }
          v[q2 * 16 + b * 4 + 0] = aur.x + aur.y;
          v[q2 * 16 + b * 4 + 1] = aui.x + aui.y;
          v[q2 * 16 + b * 4 + 2] = avr.x + avr.y;
          v[q2 * 16 + b * 4 + 3] = avi.x + avi.y;
        }
      }
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < d; ++i) {
          const float send = upper ? v[i] : v[i + d];
          const float keep = upper ? v[i + d] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
      float sum = v[0];
      if (nwarps > 1) {
        red[warp][lane] = sum;
        __syncthreads();
        sum = 0.f;
        if (warp == 0)
          for (int w = 0; w < nwarps; ++w) sum += red[w][lane];
      }
      if (warp == 0) {
        const float other = __shfl_xor_sync(0xffffffffu, sum, 2);
        const int q2 = lane >> 4, b = (lane >> 2) & 3, which = (lane >> 1) & 1, ri = lane & 1;
        const int l = lseg + qb + q2;
        if (which == 0 && l < p.L && b0 + b < p.B) {
          const float pu = sum, mv = other;
          float* o = reinterpret_cast<float*>(p.out + (long long)(b0 + b) * 2 * plane + (long long)l * p.M + m);
          o[ri] = 0.5f * (mv + pu);
          o[2 * plane + (1 - ri)] = ri ? 0.5f * (mv - pu) : -0.5f * (mv - pu);
        }
      }
      if (nwarps > 1) __syncthreads();
    }
  }
}


// ---------------------------------------------------------------------------
// Segment-per-thread kernels: the default recurrence variant.
//
// A work item is one (order m, checkpoint segment c, degree block j): degrees
// l = m + 16c + j*DB .. m + 16c + (j+1)*DB - 1.  A thread owns one item for a
// group of kNB batches and walks its latitudes one at a time: it re-seeds the
// recurrence from the segment's float64-built checkpoints, runs it up the
// segment, and adds P * X for every degree of its block into DB x kNB complex
// partial sums held in registers.  The partial sums never cross lanes inside
// the latitude loop (the per-degree shuffle reductions of the pair kernels
// cost as many issue slots as their FMAs); the NKC warps of a CTA share the
// same 32 items, split the latitudes into NKC chunks, and meet once, in shared
// memory, at the end.  Items are uniform work (one segment x one latitude
// chunk), so the triangular l >= m structure needs no balancing.
//
// PAR (grids symmetric about the equator, x_{K-1-k} = -x_k and w_{K-1-k} =
// w_k): P_l^m(-x) = (-1)^(l+m) P_l^m(x), so only the northern latitudes are
// visited and they are contracted with E = X_k + X_{K-1-k} (l + m even) or
// O = X_k - X_{K-1-k} (l + m odd).  Since l - m = 16c + q, the parity is that
// of the degree's offset q inside the segment, known at compile time.  This
// halves both the recurrence and the contraction.  The equatorial row of an
// odd nlat is its own mirror and is used once (E = O = X).

// sum_{d=1}^{n} ceil(d / 16)
__host__ __device__ __forceinline__ long long seg_prefix(long long n) {
  const long long q = n / kSeg, r = n % kSeg;
  return (long long)kSeg * q * (q + 1) / 2 + r * (q + 1);
}
// number of (order, segment) pairs of the orders below m: order m' has
// ceil((L - m') / 16) segments.
__host__ __device__ __forceinline__ long long segs_before(int m, int L) {
  return seg_prefix(L) - seg_prefix((long long)L - m);
}

// the item's order and segment from its index among all (order, segment) pairs
__device__ __forceinline__ void decode_segment(int seg, int mlim, int L, int& m, int& c) {
  int lo = 0, hi = mlim - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (segs_before(mid, L) <= seg) lo = mid;
    else hi = mid - 1;
  }
  m = lo;
  c = (int)(seg - segs_before(lo, L));
}

// exact zeros of every row (b, l) of this CTA's batch group for m > l,
// rows spread over the grid's CTAs
__device__ __forceinline__ void zero_upper(float2* out, long long plane_stride, int planes, int B, int L,
                                           int M, int b0) {
  const int rows = kNB * planes * L;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int bp = r / L, l = r % L;
    const int b = b0 + bp / planes;
    if (b >= B) break;
    float2* row = out + ((long long)b * planes + bp % planes) * plane_stride + (long long)l * M;
    for (int mm = l + 1 + (int)threadIdx.x; mm < M; mm += blockDim.x) row[mm] = make_float2(0.f, 0.f);
  }
}

__device__ __forceinline__ void cp_async8(void* smem, const void* g, bool valid) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(sa), "l"(g), "r"(valid ? 8 : 0) : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* g) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* g) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Latitude ring: per warp and latitude, one stage holds the 32 lanes'
// checkpoints, cos theta, and the spectrum rows the latitude needs (each batch's
// row at k and, with PAR, at the mirror; c0 and c1 for the vector map) for the
// 32 consecutive orders m_lo .. m_lo + 31 starting at the warp's first item's
// order (32 consecutive segments span at most 32 orders).  Lane i copies order
// m_lo + i of every row and the checkpoint of its own item, so every cp.async
// reads and writes contiguous runs (copies in which many lanes read one address
// split into one shared-memory wavefront per lane); the checkpoints are
// contiguous across lanes in the latitude-major compact layout.  Stages are
// filled kDepth latitudes ahead of use: an iteration is a few hundred cycles and
// a first touch after the L2 is cold is on the order of a microsecond.  The ring
// is reused for the final reduction.
template <bool PAR, bool VEC, int NKC>
struct SegRing {
  static constexpr int kRows = (PAR ? 2 : 1) * (VEC ? 2 : 1) * kNB;  // spectrum rows per latitude
  static constexpr int kSeedBytes = VEC ? 16 : 8;
  static constexpr int kDepth = VEC ? 4 : 8;
  static constexpr int kWarpStage = 32 * kSeedBytes + 16 + kRows * 32 * 8;
  static constexpr int kBytes = kDepth * NKC * kWarpStage;
  static constexpr int kRedBytes = NKC * 32 * 33 * 4;
  static constexpr int kSmem = kBytes > kRedBytes ? kBytes : kRedBytes;
};

// dynamic shared memory of the scalar segment kernel
template <bool PAR, int NKC>
__host__ __device__ constexpr int seg_smem_bytes() {
  return SegRing<PAR, false, NKC>::kSmem;
}

template <int DB, bool PAR, int NKC, int J0>
__device__ __forceinline__ void seg_forward_body(const RecParams& p, int m, int c, int m_lo, bool live, int b0,
                                                 const float2* sdl, long long sd_kstride, unsigned char* smem) {
  using R = SegRing<PAR, false, NKC>;
  constexpr int Q0 = J0 * DB;  // first contracted offset inside the segment
  constexpr int QN = Q0 + DB;  // one past the last
  constexpr int D = R::kDepth;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lseg = m + c * kSeg;
  float ca[QN], cb[QN];  // a_l and -b_l of the steps q = 2 .. QN-1 (zero past lmax)
  const float* cm = p.coef + (long long)m * p.L * 2;
#pragma unroll
  for (int q = 2; q < QN; ++q) {
    const int l = lseg + q;
    const bool ok = l < p.L;
    ca[q] = ok ? cm[2 * l] : 0.f;
    cb[q] = ok ? -cm[2 * l + 1] : 0.f;
  }
  const int Kh = PAR ? (p.K + 1) / 2 : p.K;
  const int chunk = (Kh + NKC - 1) / NKC;
  const int kb = warp * chunk, ke = min(Kh, kb + chunk);
  const bool mok = m_lo + lane < p.M;
  bool bok[kNB];
  const float2* rows[kNB];  // this lane's column (order m_lo + lane) of each batch's spectrum
#pragma unroll
  for (int b = 0; b < kNB; ++b) {
    bok[b] = b0 + b < p.B && mok;
    rows[b] = p.spec + (long long)(b0 + b < p.B ? b0 + b : b0) * p.sbs + (mok ? m_lo + lane : m_lo);
  }
  const int mi = m - m_lo;  // this item's column in a stage

  // stage s of this warp: checkpoints [32] float2, cos theta, spectrum [kRows][32] float2
  auto stage = [&](int s) { return smem + (s * NKC + warp) * R::kWarpStage; };
  auto issue = [&](int k, int s) {
    unsigned char* st = stage(s);
    float2* sp = reinterpret_cast<float2*>(st + 32 * 8 + 16);
    const int km = p.K - 1 - k;
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      cp_async8(sp + b * 32 + lane, bok[b] ? rows[b] + (long long)k * p.srs : p.spec, bok[b]);
      if (PAR) {
        const bool v = bok[b] && km != k;
        cp_async8(sp + (kNB + b) * 32 + lane, v ? rows[b] + (long long)km * p.srs : p.spec, v);
      }
    }
    cp_async8(reinterpret_cast<float2*>(st) + lane, sdl + k * sd_kstride, true);
    if (lane == 0) cp_async4(st + 32 * 8, p.x + k);
  };

  float2 acc[DB][kNB];
#pragma unroll
  for (int q = 0; q < DB; ++q)
#pragma unroll
    for (int b = 0; b < kNB; ++b) acc[q][b] = make_float2(0.f, 0.f);

#pragma unroll
  for (int s = 0; s < D - 1; ++s) {
    if (kb + s < ke) issue(kb + s, s);
    cp_async_commit();
  }
  for (int k = kb, s = 0; k < ke; ++k, s = (s + 1 == D) ? 0 : s + 1) {
    __syncwarp();  // every lane is done reading the stage about to be refilled
    if (k + D - 1 < ke) issue(k + D - 1, (s == 0) ? D - 1 : s - 1);
    cp_async_commit();
    cp_async_wait<D - 1>();  // latitude k's copies have landed
    __syncwarp();            // and so have the other lanes' (each lane reads all columns)
    const unsigned char* st = stage(s);
    const float x = *reinterpret_cast<const float*>(st + 32 * 8);
    const float2 sk = reinterpret_cast<const float2*>(st)[lane];
    float p2 = sk.x, p1 = sk.y;  // degrees lseg and lseg + 1
    const float2* cur = reinterpret_cast<const float2*>(st + 32 * 8 + 16) + mi;
    float2 E[kNB], O[kNB];
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      const float2 X = cur[b * 32];
      if (PAR) {
        const float2 Xm = cur[(kNB + b) * 32];  // zero for the equatorial row of an odd nlat
        E[b] = make_float2(X.x + Xm.x, X.y + Xm.y);
        O[b] = make_float2(X.x - Xm.x, X.y - Xm.y);
      } else {
        E[b] = O[b] = X;
      }
    }
#pragma unroll
    for (int q = 0; q < QN; ++q) {
      float pl;
      if (q == 0) {
        pl = p2;
      } else if (q == 1) {
        pl = p1;
      } else {
        pl = fmaf(ca[q], __fmul_rn(x, p1), __fmul_rn(cb[q], p2));
        p2 = p1;
        p1 = pl;
      }
      if (q >= Q0) {
        const float2 pp = make_float2(pl, pl);
#pragma unroll
        for (int b = 0; b < kNB; ++b) acc[q - Q0][b] = __ffma2_rn(pp, (q & 1) ? O[b] : E[b], acc[q - Q0][b]);
      }
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();  // every warp is done with the ring the reduction reuses

  // the NKC latitude chunks meet in shared memory, 4 degrees at a time
  constexpr int NV = 32 / NKC;  // values summed and written per thread per round
  float* red = reinterpret_cast<float*>(smem);
  float* mine = red + tid * 33;
#pragma unroll
  for (int r = 0; r < DB / 4; ++r) {
#pragma unroll
    for (int qq = 0; qq < 4; ++qq)
#pragma unroll
      for (int b = 0; b < kNB; ++b) {
        mine[qq * 8 + b * 2] = acc[4 * r + qq][b].x;
        mine[qq * 8 + b * 2 + 1] = acc[4 * r + qq][b].y;
      }
    __syncthreads();
    const int v0 = warp * NV;
    float sum[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) sum[i] = 0.f;
#pragma unroll
    for (int w = 0; w < NKC; ++w)
#pragma unroll
      for (int i = 0; i < NV; ++i) sum[i] += red[(w * 32 + lane) * 33 + v0 + i];
    if (live) {
#pragma unroll
      for (int i = 0; i < NV; i += 2) {
        const int v = v0 + i, qq = v >> 3, b = (v >> 1) & 3;
        const int l = lseg + Q0 + 4 * r + qq;
        if (l < p.L && b0 + b < p.B)
          p.out[((long long)(b0 + b) * p.L + l) * p.M + m] = make_float2(sum[i] * p.scale, sum[i + 1] * p.scale);
      }
    }
    __syncthreads();
  }
}

// The item's order, segment and checkpoint pointer.  Lanes past the last
// segment take the last segment (they compute and write nothing), so every
// lane's order lies in m_lo .. m_lo + 31.  Checkpoints: compact layout
// [K][nsegs][S] (consecutive lanes contiguous) or [M][nseg][K][S].
template <int S>
__device__ __forceinline__ void seg_item(const float* seeds, bool compact, int nseg, int K, int mlim, int L,
                                         int nsegs, int seg, int& m, int& c, int& m_lo, const float*& sdl,
                                         long long& kstride) {
  const int sg = seg < nsegs ? seg : nsegs - 1;
  decode_segment(sg, mlim, L, m, c);
  m_lo = __shfl_sync(0xffffffffu, m, 0);
  if (compact) {
    sdl = seeds + (long long)sg * S;
    kstride = (long long)nsegs;
  } else {
    sdl = seeds + ((long long)m * nseg + c) * K * S;
    kstride = 1;
  }
}

// grid: x = J x ceil(nsegs / 32) (degree block j = x % J), y = batch group of kNB;
// dynamic shared memory seg_smem_bytes<PAR, NKC>()
template <int DB, bool PAR, int NKC>
__global__ void __launch_bounds__(NKC * 32) recurrence_forward_seg_kernel(const RecParams p, int mlim, int nsegs,
                                                                          int compact) {
  static_assert(DB == 8 || DB == 16, "degree block of 8 or 16");
  static_assert(NKC == 2 || NKC == 4 || NKC == 8, "2, 4 or 8 latitude chunks");
  constexpr int J = kSeg / DB;
  extern __shared__ __align__(16) unsigned char ssmem[];
  const int b0 = blockIdx.y * kNB;
  zero_upper(p.out, (long long)p.L * p.M, 1, p.B, p.L, p.M, b0);
  const int seg = (int)(blockIdx.x / J) * 32 + (int)(threadIdx.x & 31);
  int m, c, m_lo;
  const float* sdl;
  long long ks;
  seg_item<2>(p.seeds, compact != 0, p.nseg, p.K, mlim, p.L, nsegs, seg, m, c, m_lo, sdl, ks);
  const float2* sd2 = reinterpret_cast<const float2*>(sdl);
  const bool live = seg < nsegs;
  if constexpr (J == 2) {
    if (blockIdx.x % 2) seg_forward_body<DB, PAR, NKC, 1>(p, m, c, m_lo, live, b0, sd2, ks, ssmem);
    else seg_forward_body<DB, PAR, NKC, 0>(p, m, c, m_lo, live, b0, sd2, ks, ssmem);
  } else {
    seg_forward_body<DB, PAR, NKC, 0>(p, m, c, m_lo, live, b0, sd2, ks, ssmem);
  }
}

// Vector form.  Per degree the thread forms W0 = alpha Q^{m-1}_l + beta Q^{m+1}_l
// and W1 = gamma Q^{m-1}_{l+1} + delta Q^{m+1}_{l+1} from the two recurrences
// and accumulates S = sum (W0 + W1) u and D = sum (W0 - W1) v, u = c0 + i c1,
// v = c0 - i c1 (sph = (S + D) / 2, tor = i (S - D) / 2).  With PAR, W0 is odd
// and W1 even under the mirror times s = (-1)^(l+m) (Q^{m +/- 1}_l has parity
// (-1)^(l+m+1)), so a northern latitude k and its mirror k' give
//   S += (W0 + W1) u - s (W0 - W1) u',   D += (W0 - W1) v - s (W0 + W1) v'
// and the recurrences run for the northern half only.  Degree blocks of 8
// (J = 2 per segment) keep the 8 x 4 batches x (S, D) sums in 128 registers;
// the block j = 1 runs the recurrences through the segment's first 8 degrees
// without contracting them.  The per-degree coefficients of the CTA's 32 items
// sit in shared memory, lane-innermost (conflict-free 16-byte loads).
constexpr int kVDB = 8;
constexpr int kCoefBytes = 2 * kSeg * 32 * 16;  // [2 * 16 degrees][32 lanes] float4

// dynamic shared memory of the vector segment kernel: coefficients, then the ring
template <bool PAR, int NKC>
__host__ __device__ constexpr int vseg_smem_bytes() {
  return kCoefBytes + SegRing<PAR, true, NKC>::kSmem;
}

template <bool PAR, int NKC, int J0>
__device__ __forceinline__ void vseg_forward_body(const VecRecParams& p, int m, int c, int m_lo, bool live, int b0,
                                                  const float4* sdl, long long sd_kstride, unsigned char* smem) {
  using R = SegRing<PAR, true, NKC>;
  constexpr int Q0 = J0 * kVDB, QN = Q0 + kVDB;
  constexpr int D = R::kDepth;
  float4* cfs = reinterpret_cast<float4*>(smem);
  unsigned char* ring = smem + kCoefBytes;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lseg = m + c * kSeg;
  // coefficients of degrees lseg + q, q < QN: (am, -bm, ap, -bp), (alpha, beta, gamma, delta)
  for (int e = warp; e < QN * 2; e += NKC) {
    const int q = e >> 1, h = e & 1, l = lseg + q;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live && l < p.L) {
      const float4 raw = reinterpret_cast<const float4*>(p.coef + ((long long)m * p.L + l) * 8)[h];
      v = h ? raw : make_float4(raw.x, -raw.y, raw.z, -raw.w);
    }
    cfs[e * 32 + lane] = v;
  }
  __syncthreads();
  const int Kh = PAR ? (p.K + 1) / 2 : p.K;
  const int chunk = (Kh + NKC - 1) / NKC;
  const int kb = warp * chunk, ke = min(Kh, kb + chunk);
  const bool mok = m_lo + lane < p.M;
  bool bok[kNB];
  const float2* rows[kNB];  // this lane's column (order m_lo + lane) of each batch's c0 spectrum
#pragma unroll
  for (int b = 0; b < kNB; ++b) {
    bok[b] = b0 + b < p.B && mok;
    rows[b] = p.spec + (long long)(b0 + b < p.B ? b0 + b : b0) * p.sbs + (mok ? m_lo + lane : m_lo);
  }
  const int mi = m - m_lo;  // this item's column in a stage

  // stage s of this warp: checkpoints [32] float4, cos theta, spectrum [kRows][32] float2;
  // rows of batch b: c0, c1 at k (and c0, c1 at the mirror with PAR)
  constexpr int PB = PAR ? 4 : 2;
  auto stage = [&](int s) { return ring + (s * NKC + warp) * R::kWarpStage; };
  auto issue = [&](int k, int s) {
    unsigned char* st = stage(s);
    float2* sp = reinterpret_cast<float2*>(st + 32 * 16 + 16);
    const int km = p.K - 1 - k;
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      const float2* r0 = rows[b] + (long long)k * p.srs;
      cp_async8(sp + (PB * b + 0) * 32 + lane, bok[b] ? r0 : p.spec, bok[b]);
      cp_async8(sp + (PB * b + 1) * 32 + lane, bok[b] ? r0 + p.sps : p.spec, bok[b]);
      if (PAR) {
        const bool v = bok[b] && km != k;
        const float2* r1 = rows[b] + (long long)km * p.srs;
        cp_async8(sp + (PB * b + 2) * 32 + lane, v ? r1 : p.spec, v);
        cp_async8(sp + (PB * b + 3) * 32 + lane, v ? r1 + p.sps : p.spec, v);
      }
    }
    cp_async16(reinterpret_cast<float4*>(st) + lane, sdl + k * sd_kstride);
    if (lane == 0) cp_async4(st + 32 * 16, p.x + k);
  };

  float2 S[kVDB][kNB], Dd[kVDB][kNB];
#pragma unroll
  for (int q = 0; q < kVDB; ++q)
#pragma unroll
    for (int b = 0; b < kNB; ++b) S[q][b] = Dd[q][b] = make_float2(0.f, 0.f);

#pragma unroll
  for (int s = 0; s < D - 1; ++s) {
    if (kb + s < ke) issue(kb + s, s);
    cp_async_commit();
  }
  for (int k = kb, s = 0; k < ke; ++k, s = (s + 1 == D) ? 0 : s + 1) {
    __syncwarp();  // every lane is done reading the stage about to be refilled
    if (k + D - 1 < ke) issue(k + D - 1, (s == 0) ? D - 1 : s - 1);
    cp_async_commit();
    cp_async_wait<D - 1>();  // latitude k's copies have landed
    __syncwarp();            // and so have the other lanes' (each lane reads all columns)
    const unsigned char* st = stage(s);
    const float x = *reinterpret_cast<const float*>(st + 32 * 16);
    const float4 sk = reinterpret_cast<const float4*>(st)[lane];
    float qm0 = sk.x, qm1 = sk.y, qp0 = sk.z, qp1 = sk.w;
    const float2* cur = reinterpret_cast<const float2*>(st + 32 * 16 + 16) + mi;
    float2 u[kNB], v[kNB], um[kNB], vm[kNB];
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      const float2 c0 = cur[(PB * b + 0) * 32], c1 = cur[(PB * b + 1) * 32];
      u[b] = make_float2(c0.x - c1.y, c0.y + c1.x);
      v[b] = make_float2(c0.x + c1.y, c0.y - c1.x);
      if (PAR) {  // zero for the equatorial row of an odd nlat
        const float2 d0 = cur[(PB * b + 2) * 32], d1 = cur[(PB * b + 3) * 32];
        um[b] = make_float2(d0.x - d1.y, d0.y + d1.x);
        vm[b] = make_float2(d0.x + d1.y, d0.y - d1.x);
      }
    }
#pragma unroll
    for (int q = 0; q < QN; ++q) {
      const float4 ab = cfs[(2 * q) * 32 + lane];
      if (q >= Q0) {
        const float4 g = cfs[(2 * q + 1) * 32 + lane];
        const float w0 = fmaf(g.x, qm0, __fmul_rn(g.y, qp0));
        const float w1 = fmaf(g.z, qm1, __fmul_rn(g.w, qp1));
        const float wp = w0 + w1, wm = w0 - w1;
        const float2 pp = make_float2(wp, wp), mm = make_float2(wm, wm);
#pragma unroll
        for (int b = 0; b < kNB; ++b) {
          S[q - Q0][b] = __ffma2_rn(pp, u[b], S[q - Q0][b]);
          Dd[q - Q0][b] = __ffma2_rn(mm, v[b], Dd[q - Q0][b]);
        }
        if (PAR) {
          // s = (-1)^q: even q subtracts the mirror terms, odd q adds them
          const float2 ms = (q & 1) ? mm : make_float2(-wm, -wm);
          const float2 ps = (q & 1) ? pp : make_float2(-wp, -wp);
#pragma unroll
          for (int b = 0; b < kNB; ++b) {
            S[q - Q0][b] = __ffma2_rn(ms, um[b], S[q - Q0][b]);
            Dd[q - Q0][b] = __ffma2_rn(ps, vm[b], Dd[q - Q0][b]);
          }
        }
      }
      if (q + 1 < QN) {  // both recurrences to degree l + 2
        const float nm = fmaf(ab.x, __fmul_rn(x, qm1), __fmul_rn(ab.y, qm0));
        const float np = fmaf(ab.z, __fmul_rn(x, qp1), __fmul_rn(ab.w, qp0));
        qm0 = qm1;
        qm1 = nm;
        qp0 = qp1;
        qp1 = np;
      }
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();  // every warp is done with the ring the reduction reuses

  // the latitude chunks meet in shared memory, 2 degrees (32 values) at a time
  constexpr int NV = 32 / NKC;
  const long long plane = (long long)p.L * p.M;
  float* red = reinterpret_cast<float*>(ring);
  float* mine = red + tid * 33;
#pragma unroll
  for (int r = 0; r < kVDB / 2; ++r) {
#pragma unroll
    for (int qq = 0; qq < 2; ++qq)
#pragma unroll
      for (int b = 0; b < kNB; ++b) {
        float* o = mine + qq * 16 + b * 4;
        o[0] = S[2 * r + qq][b].x;
        o[1] = S[2 * r + qq][b].y;
        o[2] = Dd[2 * r + qq][b].x;
        o[3] = Dd[2 * r + qq][b].y;
      }
    __syncthreads();
    const int v0 = warp * NV;
    float sum[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) sum[i] = 0.f;
#pragma unroll
    for (int w = 0; w < NKC; ++w)
#pragma unroll
      for (int i = 0; i < NV; ++i) sum[i] += red[(w * 32 + lane) * 33 + v0 + i];
    if (live) {
#pragma unroll
      for (int i = 0; i < NV; i += 4) {
        const int vv = v0 + i, qq = vv >> 4, b = (vv >> 2) & 3;
        const int l = lseg + Q0 + 2 * r + qq;
        if (l < p.L && b0 + b < p.B) {
          const float h = 0.5f * p.scale;
          float2* o = p.out + (long long)(b0 + b) * 2 * plane + (long long)l * p.M + m;
          o[0] = make_float2(h * (sum[i] + sum[i + 2]), h * (sum[i + 1] + sum[i + 3]));
          o[plane] = make_float2(h * (sum[i + 3] - sum[i + 1]), h * (sum[i] - sum[i + 2]));
        }
      }
    }
    __syncthreads();
  }
}

// grid: x = 2 x ceil(nsegs / 32) (degree block j = x % 2), y = batch group of kNB;
// dynamic shared memory vseg_smem_bytes<PAR, NKC>()
template <bool PAR, int NKC>
__global__ void __launch_bounds__(NKC * 32) recurrence_vector_forward_seg_kernel(const VecRecParams p, int mlim,
                                                                                 int nsegs, int compact) {
  static_assert(NKC == 2 || NKC == 4 || NKC == 8, "2, 4 or 8 latitude chunks");
  extern __shared__ __align__(16) unsigned char vsmem[];
  const int b0 = blockIdx.y * kNB;
  zero_upper(p.out, (long long)p.L * p.M, 2, p.B, p.L, p.M, b0);
  const int seg = (int)(blockIdx.x >> 1) * 32 + (int)(threadIdx.x & 31);
  int m, c, m_lo;
  const float* sdl;
  long long ks;
  seg_item<4>(p.seeds, compact != 0, p.nseg, p.K, mlim, p.L, nsegs, seg, m, c, m_lo, sdl, ks);
  const float4* sd4 = reinterpret_cast<const float4*>(sdl);
  const bool live = seg < nsegs;
  if (blockIdx.x & 1) vseg_forward_body<PAR, NKC, 1>(p, m, c, m_lo, live, b0, sd4, ks, vsmem);
  else vseg_forward_body<PAR, NKC, 0>(p, m, c, m_lo, live, b0, sd4, ks, vsmem);
}

// ---------------------------------------------------------------------------
// Inverse direction (InverseRealSHT's contraction) with on-the-fly functions:
//
//   out[b, k, m] = scale * sum_{l >= m} P_l^m(x_k) c[b, l, m]
//
// The reduction runs over the degree, which is the recurrence's own direction,
// so one thread owns one (order, latitude) and accumulates while it runs the
// recurrence up through the order's 8-degree checkpoint segments: no reduction across
// threads.  CTA = 8 consecutive orders (one warp each) x 64 latitudes (two per lane) x
// a group of kNB batches; blockIdx.y is the order block, so the long low-order blocks
// are issued first.  Each warp stages its order's coefficients and the
// recurrence coefficients of the next segment in shared memory (cp.async, one
// segment ahead); every lane reads them as broadcasts.  With PAR the lanes are
// northern latitudes and keep even- and odd-(l + m) sums apart: row k gets
// e + o, row K-1-k gets e - o.  The tile's results go through shared memory so
// each (batch, row) is written as one run of 8 orders.  Orders m >= mmax up to
// out_cols are written as zeros; IRFFT_PREP zeroes Im at m = 0 and m = nlon/2.
struct RecInvParams {
  const float2* spec;  // c[b, l, m] at b*sbs + l*srs + m
  long long sbs, srs;
  const float* seeds;  // [M][nseg][K][2]: P at l = m + 8c and m + 8c + 1 (inverse normalisation)
  const float* coef;   // [M][L][2]
  const float* x;      // [K]
  float2* out;         // out[b, k, m] at b*obs + k*ors + m
  long long obs, ors;
  int B, K, L, M, nseg, out_cols, nyq;  // nyq: the Nyquist column to clear, or -1
  int prep;
  int ntile;  // 64-latitude tiles per batch group (blockIdx.x = tile + ntile * group)
  float scale;
};

constexpr int kInvOrders = 8;  // orders (warps) per CTA
constexpr int kInvSeg = 8;     // degrees between the inverse kernel's checkpoints
constexpr int kInvStages = 3;  // staged segments in flight per warp

// the checkpoints of this kernel are 8 degrees apart: over a white spectrum the
// synthesis weighs the high degrees, and the fp32 drift over 16 steps reached
// 1.1e-6 relative L2 at lmax 512 (8 steps: half of it)
// each lane runs two latitudes, k and k + 32 of a 64-latitude tile: the
// staged coefficients are read once for both (half the shared-memory loads per
// multiply-add) and the two recurrences are independent chains
template <bool PAR>
__global__ void __launch_bounds__(kInvOrders * 32, 2) recurrence_inverse_kernel(const RecInvParams p) {
  __shared__ __align__(16) float2 cst[kInvOrders][kInvStages][kInvSeg][kNB];  // staged c of a segment, per warp
  __shared__ __align__(16) float2 cab[kInvOrders][kInvStages][kInvSeg];       // staged (a_l, b_l), per warp
  __shared__ __align__(16) float2 csd[kInvOrders][kInvStages][2][32];         // staged checkpoints, per latitude
  __shared__ float2 obuf[kNB][64][kInvOrders + 1];                            // rows of one latitude half
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kInvOrders, m = m0 + warp;
  const int kc = (blockIdx.x % p.ntile) * 64;
  const int Kh = PAR ? (p.K + 1) / 2 : p.K;
  bool kv[2];
  float x[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    kv[h] = kc + 32 * h + lane < Kh;
    x[h] = kv[h] ? p.x[kc + 32 * h + lane] : 0.f;
  }
  const int b0 = (blockIdx.x / p.ntile) * kNB;
  const int nseg = (m < p.M && m < p.L) ? (p.L - m + kInvSeg - 1) / kInvSeg : 0;
  const float2* sd = reinterpret_cast<const float2*>(p.seeds) + (long long)m * p.nseg * p.K + kc + lane;

  // lane i stages entry i of the segment's kInvSeg x kNB coefficients (32 of
  // them) and the checkpoints of its two latitudes, lanes 0 .. kInvSeg-1 the
  // recurrence coefficients
  static_assert(kInvSeg * kNB == 32, "one staged coefficient per lane");
  auto stage = [&](int c, int slot) {
    const int lseg = m + c * kInvSeg;
    const int q = lane / kNB, b = lane % kNB;
    const bool v = b0 + b < p.B && lseg + q < p.L;
    cp_async8(&cst[warp][slot][q][b],
              v ? p.spec + (long long)(b0 + b) * p.sbs + (long long)(lseg + q) * p.srs + m : p.spec, v);
    if (lane < kInvSeg) {
      const bool w = lseg + lane < p.L;
      cp_async8(&cab[warp][slot][lane], w ? p.coef + ((long long)m * p.L + lseg + lane) * 2 : p.coef, w);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
      cp_async8(&csd[warp][slot][h][lane],
                kv[h] ? static_cast<const void*>(sd + (long long)c * p.K + 32 * h) : static_cast<const void*>(p.seeds),
                kv[h]);
  };
  float2 e[2][kNB], o[2][kNB];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int b = 0; b < kNB; ++b) e[h][b] = o[h][b] = make_float2(0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kInvStages - 1; ++s) {
    if (s < nseg) stage(s, s);
    cp_async_commit();
  }
  for (int c = 0, slot = 0; c < nseg; ++c, slot = (slot + 1 == kInvStages) ? 0 : slot + 1) {
    __syncwarp();  // every lane is done with the slot the next stage refills
    if (c + kInvStages - 1 < nseg) stage(c + kInvStages - 1, slot == 0 ? kInvStages - 1 : slot - 1);
    cp_async_commit();
    cp_async_wait<kInvStages - 1>();
    __syncwarp();
    float p2[2], p1[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 sk = csd[warp][slot][h][lane];  // zero for a latitude past the tile
      p2[h] = sk.x;
      p1[h] = sk.y;
    }
    const float4* cs4 = reinterpret_cast<const float4*>(&cst[warp][slot][0][0]);
    const float4* ab4 = reinterpret_cast<const float4*>(&cab[warp][slot][0]);
#pragma unroll
    for (int q = 0; q < kInvSeg; ++q) {
      const float4 c01 = cs4[2 * q], c23 = cs4[2 * q + 1];  // batches 0, 1 and 2, 3 (zero past lmax / B)
      float a = 0.f, bb = 0.f;
      if (q >= 2) {
        // (a, b) as staged: P_l = a x P_{l-1} - b P_{l-2}; both 0 beyond lmax
        const float4 ab2 = ab4[q >> 1];
        a = (q & 1) ? ab2.z : ab2.x;
        bb = (q & 1) ? ab2.w : ab2.y;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float pl;
        if (q == 0) {
          pl = p2[h];
        } else if (q == 1) {
          pl = p1[h];
        } else {
          pl = fmaf(a, __fmul_rn(x[h], p1[h]), -__fmul_rn(bb, p2[h]));
          p2[h] = p1[h];
          p1[h] = pl;
        }
        const float2 pp = make_float2(pl, pl);
        static_assert(kNB == 4, "four batches per group");
        if (q & 1) {
          o[h][0] = __ffma2_rn(pp, make_float2(c01.x, c01.y), o[h][0]);
          o[h][1] = __ffma2_rn(pp, make_float2(c01.z, c01.w), o[h][1]);
          o[h][2] = __ffma2_rn(pp, make_float2(c23.x, c23.y), o[h][2]);
          o[h][3] = __ffma2_rn(pp, make_float2(c23.z, c23.w), o[h][3]);
        } else {
          e[h][0] = __ffma2_rn(pp, make_float2(c01.x, c01.y), e[h][0]);
          e[h][1] = __ffma2_rn(pp, make_float2(c01.z, c01.w), e[h][1]);
          e[h][2] = __ffma2_rn(pp, make_float2(c23.x, c23.y), e[h][2]);
          e[h][3] = __ffma2_rn(pp, make_float2(c23.z, c23.w), e[h][3]);
        }
      }
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");

  // rows k (e + o) and K-1-k (e - o), the irfft preparation, the scale; one
  // latitude half at a time through shared memory
  const bool clear_im = p.prep && (m == 0 || m == p.nyq);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (h) __syncthreads();  // the first half's rows are written out
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float2 y = make_float2((e[h][b].x + o[h][b].x) * p.scale, (e[h][b].y + o[h][b].y) * p.scale);
      float2 ym = make_float2((e[h][b].x - o[h][b].x) * p.scale, (e[h][b].y - o[h][b].y) * p.scale);
      if (clear_im) y.y = ym.y = 0.f;
      obuf[b][lane][warp] = y;
      obuf[b][32 + lane][warp] = ym;
    }
    __syncthreads();
    const int kh = kc + 32 * h;
    for (int idx = threadIdx.x; idx < kNB * 64 * kInvOrders; idx += blockDim.x) {
      const int j = idx % kInvOrders, r = (idx / kInvOrders) % 64, b = idx / (64 * kInvOrders);
      const int mm = m0 + j;
      if (mm >= p.out_cols || b0 + b >= p.B) continue;
      int row;
      if (r < 32) {
        if (kh + r >= Kh) continue;
        row = kh + r;
      } else {
        if (!PAR || kh + r - 32 >= Kh) continue;
        row = p.K - 1 - (kh + r - 32);
        if (row == kh + r - 32) continue;  // the equator of an odd nlat is its own mirror
      }
      p.out[(long long)(b0 + b) * p.obs + (long long)row * p.ors + mm] = obuf[b][r][j];
    }
  }
}

// sets the kernel's dynamic shared-memory limit once per device, then launches
template <typename Kern, typename Params>
inline cudaError_t launch_with_smem(Kern kernel, int bytes, std::atomic<unsigned long long>& configured, dim3 grid,
                                    int threads, cudaStream_t st, const Params& p, int mlim, int nsegs, int compact) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kernel<<<grid, threads, bytes, st>>>(p, mlim, nsegs, compact);
  return cudaSuccess;
}

template <int DB, bool PAR, int NKC>
inline cudaError_t launch_seg(const RecParams& p, dim3 grid, int mlim, int nsegs, int compact, cudaStream_t st) {
  static std::atomic<unsigned long long> configured{0};
  return launch_with_smem(recurrence_forward_seg_kernel<DB, PAR, NKC>, seg_smem_bytes<PAR, NKC>(), configured, grid,
                          NKC * 32, st, p, mlim, nsegs, compact);
}

template <int DB, bool PAR>
inline cudaError_t launch_seg_forward(const RecParams& p, int nkc, dim3 grid, int mlim, int nsegs, int compact,
                                      cudaStream_t st) {
  if (nkc == 2) return launch_seg<DB, PAR, 2>(p, grid, mlim, nsegs, compact, st);
  if (nkc == 8) return launch_seg<DB, PAR, 8>(p, grid, mlim, nsegs, compact, st);
  return launch_seg<DB, PAR, 4>(p, grid, mlim, nsegs, compact, st);
}

template <bool PAR, int NKC>
inline cudaError_t launch_vseg(const VecRecParams& p, dim3 grid, int mlim, int nsegs, int compact, cudaStream_t st) {
  static std::atomic<unsigned long long> configured{0};
  return launch_with_smem(recurrence_vector_forward_seg_kernel<PAR, NKC>, vseg_smem_bytes<PAR, NKC>(), configured,
                          grid, NKC * 32, st, p, mlim, nsegs, compact);
}

template <bool PAR>
inline cudaError_t launch_vseg_forward(const VecRecParams& p, int nkc, dim3 grid, int mlim, int nsegs,
                                       int compact, cudaStream_t st) {
  if (nkc == 2) return launch_vseg<PAR, 2>(p, grid, mlim, nsegs, compact, st);
  if (nkc == 8) return launch_vseg<PAR, 8>(p, grid, mlim, nsegs, compact, st);
  return launch_vseg<PAR, 4>(p, grid, mlim, nsegs, compact, st);
}

}  // namespace rec
}  // namespace hsb
