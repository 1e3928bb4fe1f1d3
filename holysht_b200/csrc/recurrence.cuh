// Scalar forward Legendre transform with on-the-fly associated Legendre
// functions (the "recurrence" variant): no table stream.
//
//   out[b, l, m] = scale * sum_k X[b, k, m] * w_k P_l^m(x_k)        (l >= m)
//
// P is generated in registers by the three-term recurrence in l
//   P_l = a_lm x P_{l-1} - b_lm P_{l-2}
// in fp32, re-seeded every kSeg degrees from checkpoints (P_{l0}, P_{l0+1})
// computed in float64 on the host (quadrature weight folded in; values below
// fp32 range are exact zeros, which is what they contribute).  Re-seeding
// bounds the fp32 drift of the recurrence: with 16-degree segments the
// coefficients stay within ~5e-7 relative L2 of the float64 transform at
// lmax = 512.
//
// CTA: one order m, 4 checkpoint segments (64 degrees), a group of 4 batches,
// threads over latitude (kKpt latitudes per thread, in registers with the
// kKpt x 4 complex spectrum values they multiply).  Per degree each thread forms 8 partial sums (4 batches x re/im);
// every 4 degrees a warp transposes-and-reduces its 32 values with shuffles
// (lane j ends with value j summed over the warp's latitudes) and the warps'
// results are summed through shared memory.
#pragma once

#include <cuda_runtime.h>

namespace hsb {
namespace rec {

constexpr int kSeg = 16;      // degrees per checkpoint segment
#ifndef HSB_REC_KPT
#define HSB_REC_KPT 4
#endif
constexpr int kKpt = HSB_REC_KPT;  // latitudes per thread
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

// grid: x = order m, y = block of kSegPerCta segments, z = batch group
__global__ void __launch_bounds__(kMaxWarps * 32) recurrence_forward_kernel(const RecParams p) {
  __shared__ float red[kMaxWarps][32];
  const int m = blockIdx.x;
  const int b0 = blockIdx.z * kNB;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int lm = p.L - m;  // degrees l = m .. L-1
  const int nseg = lm > 0 ? (lm + kSeg - 1) / kSeg : 0;
  const int c_begin = blockIdx.y * kSegPerCta;

  if (blockIdx.y == 0) {
    // rows l < m (and every row of an order without degrees) are exact zeros
    const int zrows = lm > 0 ? m : p.L;
    for (int e = tid; e < zrows * kNB; e += blockDim.x) {
      const int l = e / kNB, b = b0 + e % kNB;
      if (b < p.B) p.out[((long long)b * p.L + l) * p.M + m] = make_float2(0.f, 0.f);
    }
  }
  if (c_begin >= nseg) return;  // uniform per CTA
  const int c_end = min(nseg, c_begin + kSegPerCta);

  // this thread's latitudes, their cos(theta) and scaled spectrum values
  const int k0 = tid * kKpt;
  float xk[kKpt];
  float2 X[kKpt][kNB];
#pragma unroll
  for (int i = 0; i < kKpt; ++i) {
    const int k = k0 + i;
    xk[i] = k < p.K ? p.x[k] : 0.f;
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float2 v = make_float2(0.f, 0.f);
      if (k < p.K && b0 + b < p.B) v = p.spec[(long long)(b0 + b) * p.sbs + (long long)k * p.srs + m];
      X[i][b] = make_float2(v.x * p.scale, v.y * p.scale);
    }
  }

  const float* coef_m = p.coef + (long long)m * p.L * 2;
  for (int c = c_begin; c < c_end; ++c) {
    const int lseg = m + c * kSeg;
    // the segment's seeds and recurrence coefficients, loaded up front
    const float* sd = p.seeds + (((long long)m * p.nseg + c) * p.K + k0) * 2;
    float p1[kKpt], p2[kKpt];
    float ca[kSeg], cb[kSeg];
#pragma unroll
    for (int q = 2; q < kSeg; ++q) {
      const int l = lseg + q;
      ca[q] = l < p.L ? coef_m[2 * l] : 0.f;
      cb[q] = l < p.L ? coef_m[2 * l + 1] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kKpt; ++i) {
      const bool ok = k0 + i < p.K;
      p2[i] = ok ? sd[2 * i] : 0.f;      // P at lseg
      p1[i] = ok ? sd[2 * i + 1] : 0.f;  // P at lseg + 1
    }
#pragma unroll
    for (int qb = 0; qb < kSeg; qb += 4) {
      float v[32];  // 4 degrees x (4 batches x re/im)
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int q = qb + q4;
        float pl[kKpt];
        if (q == 0) {
#pragma unroll
          for (int i = 0; i < kKpt; ++i) pl[i] = p2[i];
        } else if (q == 1) {
#pragma unroll
          for (int i = 0; i < kKpt; ++i) pl[i] = p1[i];
        } else {
#pragma unroll
          for (int i = 0; i < kKpt; ++i) {
            pl[i] = fmaf(ca[q] * xk[i], p1[i], -cb[q] * p2[i]);
            p2[i] = p1[i];
            p1[i] = pl[i];
          }
        }
        float2 acc[kNB];
#pragma unroll
        for (int b = 0; b < kNB; ++b) acc[b] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < kKpt; ++i)
#pragma unroll
          for (int b = 0; b < kNB; ++b) acc[b] = __ffma2_rn(make_float2(pl[i], pl[i]), X[i][b], acc[b]);
#pragma unroll
        for (int b = 0; b < kNB; ++b) {
          v[q4 * 8 + 2 * b] = acc[b].x;
          v[q4 * 8 + 2 * b + 1] = acc[b].y;
        }
      }
      // warp transpose-reduce: lane j ends with value j summed over the warp
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
      if (nwarps == 1) {
        const int q4 = lane >> 3, b = (lane >> 1) & 3, ri = lane & 1;
        const int l = lseg + qb + q4;
        if (l < p.L && b0 + b < p.B)
          reinterpret_cast<float*>(p.out)[(((long long)(b0 + b) * p.L + l) * p.M + m) * 2 + ri] = v[0];
      } else {
        red[warp][lane] = v[0];
        __syncthreads();
        if (warp == 0) {
          float sum = 0.f;
          for (int w = 0; w < nwarps; ++w) sum += red[w][lane];
          const int q4 = lane >> 3, b = (lane >> 1) & 3, ri = lane & 1;
          const int l = lseg + qb + q4;
          if (l < p.L && b0 + b < p.B)
            reinterpret_cast<float*>(p.out)[(((long long)(b0 + b) * p.L + l) * p.M + m) * 2 + ri] = sum;
        }
        __syncthreads();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Paired-latitude scalar kernel (the one the library launches).  Same maths
// and checkpoints as recurrence_forward_kernel, organised for the FP32 pipe:
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

// grid: x = order m, y = block of kSegPerCta segments, z = batch group of kNB
__global__ void __launch_bounds__(kMaxWarps * 32) recurrence_vector_forward_kernel(const VecRecParams p) {
  __shared__ float red[kMaxWarps][32];
  __shared__ float cf[kSegPerCta * kSeg][8];
  const int m = blockIdx.x;
  const int b0 = blockIdx.z * kNB;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int lm = p.L - m;
  const int nseg = lm > 0 ? (lm + kSeg - 1) / kSeg : 0;
  const int c_begin = blockIdx.y * kSegPerCta;
  const long long plane = (long long)p.L * p.M;

  if (blockIdx.y == 0) {
    // rows l < m of both components (every row of an order without degrees) are exact zeros
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
    cf[dl][f] = dl < ndeg ? p.coef[((long long)m * p.L + l_first + dl) * 8 + f] : 0.f;
  }

  // this thread's latitudes and u, v of its kNB batches (scaled)
  const int k0 = tid * kKpt;
  float xk[kKpt];
  float2 U[kKpt][kNB], V[kKpt][kNB];
#pragma unroll
  for (int i = 0; i < kKpt; ++i) {
    const int k = k0 + i;
    xk[i] = k < p.K ? p.x[k] : 0.f;
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float2 c0 = make_float2(0.f, 0.f), c1 = c0;
      if (k < p.K && b0 + b < p.B) {
        const float2* s = p.spec + (long long)(b0 + b) * p.sbs + (long long)k * p.srs + m;
        c0 = s[0];
        c1 = s[p.sps];
      }
      U[i][b] = make_float2((c0.x - c1.y) * p.scale, (c0.y + c1.x) * p.scale);
      V[i][b] = make_float2((c0.x + c1.y) * p.scale, (c0.y - c1.x) * p.scale);
    }
  }
  __syncthreads();  // coefficients staged

  for (int c = c_begin; c < c_end; ++c) {
    const int lseg = m + c * kSeg;
    const float* sd = p.seeds + (((long long)m * p.nseg + c) * p.K + k0) * 4;
    float qm0[kKpt], qm1[kKpt], qp0[kKpt], qp1[kKpt];
#pragma unroll
    for (int i = 0; i < kKpt; ++i) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + i < p.K) s4 = reinterpret_cast<const float4*>(sd)[i];
      qm0[i] = s4.x;
      qm1[i] = s4.y;
      qp0[i] = s4.z;
      qp1[i] = s4.w;
    }
#pragma unroll
    for (int qb = 0; qb < kSeg; qb += 2) {
      float v[32];  // 2 degrees x (4 batches x (u, v) x re/im)
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        const float* k8 = cf[lseg + qb + q2 - l_first];
        const float am = k8[0], bm = k8[1], ap = k8[2], bp = k8[3];
        const float al = k8[4], be = k8[5], ga = k8[6], de = k8[7];
        float2 au[kNB], av[kNB];
#pragma unroll
        for (int b = 0; b < kNB; ++b) au[b] = av[b] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < kKpt; ++i) {
          const float w0 = fmaf(al, qm0[i], be * qp0[i]);
          const float w1 = fmaf(ga, qm1[i], de * qp1[i]);
          const float wp = w0 + w1, wm = w0 - w1;
#pragma unroll
          for (int b = 0; b < kNB; ++b) {
            au[b] = __ffma2_rn(make_float2(wp, wp), U[i][b], au[b]);
            av[b] = __ffma2_rn(make_float2(wm, wm), V[i][b], av[b]);
          }
          // both recurrences to degree l + 2
          const float nm = fmaf(am * xk[i], qm1[i], -bm * qm0[i]);
          const float np = fmaf(ap * xk[i], qp1[i], -bp * qp0[i]);
          qm0[i] = qm1[i];
          qm1[i] = nm;
          qp0[i] = qp1[i];
          qp1[i] = np;
        }
#pragma unroll
        for (int b = 0; b < kNB; ++b) {
          v[q2 * 16 + b * 4 + 0] = au[b].x;
          v[q2 * 16 + b * 4 + 1] = au[b].y;
          v[q2 * 16 + b * 4 + 2] = av[b].x;
          v[q2 * 16 + b * 4 + 3] = av[b].y;
        }
      }
      // warp transpose-reduce: lane j ends with value j summed over the warp
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
        // lane j: degree qb + (j >> 4), batch (j >> 2) & 3, (u, v) product (j >> 1) & 1, re/im j & 1
        const float other = __shfl_xor_sync(0xffffffffu, sum, 2);
        const int q2 = lane >> 4, b = (lane >> 2) & 3, which = (lane >> 1) & 1, ri = lane & 1;
        const int l = lseg + qb + q2;
        if (which == 0 && l < p.L && b0 + b < p.B) {
          const float pu = sum, mv = other;  // Wp u and Wm v, component ri
          float* o = reinterpret_cast<float*>(p.out + (long long)(b0 + b) * 2 * plane + (long long)l * p.M + m);
          o[ri] = 0.5f * (mv + pu);  // sph = (Wm v + Wp u) / 2
          // tor = -i (Wm v - Wp u) / 2: re from the imaginary parts, im from the real parts
          o[2 * plane + (1 - ri)] = ri ? 0.5f * (mv - pu) : -0.5f * (mv - pu);
        }
      }
      if (nwarps > 1) __syncthreads();
    }
  }
}

// Paired-latitude vector kernel (the one the library launches): the maths of
// recurrence_vector_forward_kernel with both recurrences, the table
// combinations and the contraction on packed f32x2 operations over latitude
// pairs (no operand duplication) and KPT latitudes per thread, which halves the
// share of the per-degree warp reductions relative to 4 latitudes per thread.
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

}  // namespace rec
}  // namespace hsb
