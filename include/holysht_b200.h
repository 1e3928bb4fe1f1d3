/*
 * holysht_b200 -- C ABI of the B200 (sm_100a) Legendre kernels.
 *
 * Drop-in boundary for the HOLYSHT hot path.  Each reference-named entry point
 * below replaces one operator of the reference's torch binding
 * (chrisvoncsefalvay/holysht, torch-ext/torch_binding.cpp:12-24, implemented
 * in cuda/fused_legendre.cu:3354-3545 and cuda/fused_sht.cu:74-98) with the
 * same argument meaning, expressed as plain device pointers and sizes:
 *
 *   - every pointer is a device pointer on the CURRENT CUDA device;
 *   - complex tensors are interleaved float pairs (complex64);
 *   - all tensors are dense and contiguous in the reference's layouts
 *     (input [B,K,M], output [B,L,M], tables weight_t [L,K,M] float32,
 *     vector tensors [B,2,.,M]); tables hold zeros above the diagonal (m > l)
 *     and those entries are never read;
 *   - the caller allocates every output (as the reference's Python does);
 *     forward entry points write the exact zeros for m > l themselves;
 *   - work is enqueued on `stream` (cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous; no entry point synchronises or allocates.
 *
 * Every function returns HOLYSHT_OK (0) or an error code; the matching
 * message is available from holysht_last_error() on the calling thread
 * (the reference raises the same conditions as c10::Error via TORCH_CHECK,
 * cuda/fused_legendre.cu:3157-3335).
 */
#ifndef HOLYSHT_B200_H_
#define HOLYSHT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HOLYSHT_OK 0
#define HOLYSHT_ERR_INVALID 1     /* bad pointer, shape, stride or flag */
#define HOLYSHT_ERR_CUDA 2        /* CUDA runtime error at launch */
#define HOLYSHT_ERR_UNSUPPORTED 3 /* no kernel for this device / configuration */

/* backend hints of the reference's *_ex operators (cuda/fused_legendre.cu:59-80).
 * Accepted for compatibility; every hint runs the FP32 sm_100a kernel. */
#define HOLYSHT_BACKEND_AUTO 0
#define HOLYSHT_BACKEND_FMA 1
#define HOLYSHT_BACKEND_TMA 2
#define HOLYSHT_BACKEND_TC_TF32 3
#define HOLYSHT_BACKEND_TC_BF16 4

#define HOLYSHT_DTYPE_C64 0  /* complex64 */
#define HOLYSHT_DTYPE_F32 1  /* float32 */
#define HOLYSHT_DTYPE_BF16 2 /* bfloat16 */

#define HOLYSHT_KIND_SCALAR 0 /* complex input, one table */
#define HOLYSHT_KIND_VECTOR 1 /* complex input [.,2,.,.], tables W0 and W1 */
#define HOLYSHT_KIND_REAL 2   /* real input, one table */

#define HOLYSHT_DIR_FORWARD 0 /* out rows are l, reduce over k */
#define HOLYSHT_DIR_INVERSE 1 /* out rows are k, reduce over l >= m */

#define HOLYSHT_FLAG_CONJ_W1 1    /* vector: use -W1 (conjugate-transpose map for autograd) */
#define HOLYSHT_FLAG_ROUND_BF16 2 /* round the input to bfloat16 before the contraction */
#define HOLYSHT_FLAG_IRFFT_PREP 4 /* complex output: Im(m=0)=0 and, even nlon, Im(m=nlon/2)=0 */

/* Version of this ABI (major*10000 + minor*100 + patch). */
int holysht_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* holysht_last_error(void);

/* ---------------------------------------------------------------------------
 * Reference operator mirrors
 * ------------------------------------------------------------------------- */

/* fused_legendre_forward (torch_binding.cpp:12; fused_legendre.cu:3354-3370):
 * out[b,l,m] = sum_k weight_t[l,k,m] * in[b,k,m] for l >= m, 0 for m > l.
 * out [B,L,M] c64, in [B,K,M] c64, weight_t [L,K,M] f32. */
int holysht_fused_legendre_forward(void* out, const void* in, const float* weight_t, int64_t batch,
                                   int64_t nlat, int64_t lmax, int64_t mmax, void* stream);

/* fused_legendre_inverse (torch_binding.cpp:13; fused_legendre.cu:3372-3388):
 * out[b,k,m] = sum_{l>=m} weight_t[l,k,m] * in[b,l,m].
 * out [B,K,M] c64, in [B,L,M] c64, weight_t [L,K,M] f32. */
int holysht_fused_legendre_inverse(void* out, const void* in, const float* weight_t, int64_t batch,
                                   int64_t nlat, int64_t lmax, int64_t mmax, void* stream);

/* fused_legendre_forward_real and fused_legendre_forward_real_ex
 * (torch_binding.cpp:14,16; fused_legendre.cu:3390-3424): real input
 * (in_dtype HOLYSHT_DTYPE_F32 or HOLYSHT_DTYPE_BF16), FP32 accumulation.
 * out [B,L,M] f32, in [B,K,M], weight_t [L,K,M] f32. */
int holysht_fused_legendre_forward_real(float* out, const void* in, int in_dtype,
                                        const float* weight_t, int64_t batch, int64_t nlat,
                                        int64_t lmax, int64_t mmax, int backend_hint,
                                        void* stream);

/* fused_legendre_inverse_real (torch_binding.cpp:15; fused_legendre.cu:3426-3450):
 * out [B,K,M] f32, in [B,L,M] f32, weight_t [L,K,M] f32. */
int holysht_fused_legendre_inverse_real(float* out, const float* in, const float* weight_t,
                                        int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                        void* stream);

/* fused_vector_legendre_forward and _ex (torch_binding.cpp:17-18;
 * fused_legendre.cu:3452-3480):
 *   sph = sum_k (W0 c0 + i W1 c1),  tor = sum_k (i W1 c0 - W0 c1).
 * out [B,2,L,M] c64, in [B,2,K,M] c64, w0_t / w1_t [L,K,M] f32. */
int holysht_fused_vector_legendre_forward(void* out, const void* in, const float* w0_t,
                                          const float* w1_t, int64_t batch, int64_t nlat,
                                          int64_t lmax, int64_t mmax, int backend_hint,
                                          void* stream);

/* fused_vector_legendre_inverse (torch_binding.cpp:19; fused_legendre.cu:3482-3499):
 *   c0 = sum_{l>=m} (W0 sph + i W1 tor),  c1 = sum_{l>=m} (i W1 sph - W0 tor).
 * out [B,2,K,M] c64, in [B,2,L,M] c64. */
int holysht_fused_vector_legendre_inverse(void* out, const void* in, const float* w0_t,
                                          const float* w1_t, int64_t batch, int64_t nlat,
                                          int64_t lmax, int64_t mmax, void* stream);

/* fused_vector_forward_pack_real (torch_binding.cpp:20; fused_legendre.cu:3501-3522):
 * in [B,2,K,M] c64 -> stacked_w0, stacked_w1 [4B,K,M] f32. */
int holysht_fused_vector_forward_pack_real(float* stacked_w0, float* stacked_w1, const void* in,
                                           int64_t batch, int64_t nlat, int64_t mmax,
                                           void* stream);

/* fused_vector_forward_recompose_real (torch_binding.cpp:21; fused_legendre.cu:3524-3545):
 * out_w0, out_w1 [4B,L,M] f32 -> out [B,2,L,M] c64. */
int holysht_fused_vector_forward_recompose_real(void* out, const float* out_w0,
                                                const float* out_w1, int64_t batch, int64_t lmax,
                                                int64_t mmax, void* stream);

/* sht_prepare_irfft (torch_binding.cpp:24; fused_sht.cu:74-98): in place on
 * data [rows, width] c64 with width = nlon/2+1: zero columns >= mmax, zero
 * Im at m = 0 and, for even nlon, at m = nlon/2. */
int holysht_sht_prepare_irfft(void* data, int64_t rows, int64_t width, int64_t mmax,
                              int64_t nlon, void* stream);

/* ---------------------------------------------------------------------------
 * Strided contraction (no counterpart operator in the reference; it is what
 * the module fast paths use to read the rfft output in place, fold the 2*pi
 * spectrum scale, write straight into an irfft-ready buffer, and run the
 * conjugate-transpose vector map for autograd).  Strides are in elements of
 * the input/output type; the table is [L,K,M]-shaped with its own strides
 * and contiguous m.
 * ------------------------------------------------------------------------- */
typedef struct holysht_contract_desc {
  int kind;      /* HOLYSHT_KIND_* */
  int direction; /* HOLYSHT_DIR_* */
  int in_dtype;  /* HOLYSHT_DTYPE_*: C64 for SCALAR/VECTOR; F32 or BF16 for REAL */
  int flags;     /* HOLYSHT_FLAG_* */
  const void* in;
  void* out;
  const float* w0;
  const float* w1; /* VECTOR only */
  int64_t batch, nlat, lmax, mmax;
  int64_t in_batch_stride, in_comp_stride, in_row_stride;
  int64_t out_batch_stride, out_comp_stride, out_row_stride;
  int64_t out_cols; /* columns written, >= mmax; columns >= mmax are written as 0 */
  int64_t w_l_stride, w_k_stride;
  int64_t nlon;  /* used with HOLYSHT_FLAG_IRFFT_PREP */
  float scale;   /* multiplies every output */
  int ksplit;    /* reduction split across a CTA cluster: 0 = auto, else 1,2,4,8 */
  int64_t w_m_tile_stride; /* table stride of one 32-order m tile; 0 = 32 (dense, m contiguous).
                              The m-tiled layout [L][ceil(M/32)][K][32] (k stride 32) keeps
                              every 32-order row segment on one 128-byte line. */
  int table_layout;         /* HOLYSHT_TABLE_STRIDED (the strides above) or
                               HOLYSHT_TABLE_GROUPED / HOLYSHT_TABLE_GROUPED8 (see below;
                               strides ignored) */
  int64_t m_offset;         /* global order of column 0 of the input, output and tables
                               (a multiple of 32; 0 for whole transforms).  Lets one GPU
                               contract a slice of the orders with the global l >= m
                               triangle, for the order-partitioned multi-GPU transform. */
} holysht_contract_desc;

/* Table layouts of holysht_contract_desc.table_layout.
 * GROUPED (SCALAR and VECTOR kinds): output rows in groups of 4 (rows = l for
 * HOLYSHT_DIR_FORWARD, k for HOLYSHT_DIR_INVERSE), reduction steps s (k resp. l):
 *   T[g][mt][s][lane][r][t] = W_t(row = 4g + r, step = s, m = 32 mt + lane), table t
 * with g < ceil(R/4), mt < ceil(M/32), lane < 32, r < 4, t < (VECTOR ? 2 : 1);
 * entries outside the tables (and above the diagonal) are zero.  w0 points at
 * the start; w1 is ignored (both tables are interleaved).  For VECTOR the two
 * interleaved tables are t = 0: W0 + W1 and t = 1: W0 - W1 (the kernel applies
 * sph - i tor = (W0 + W1)(c0 + i c1) and sph + i tor = (W0 - W1)(c0 - i c1),
 * half the multiplies of the direct form); the conjugate map is a table built
 * from (W0, -W1), and HOLYSHT_FLAG_CONJ_W1 is rejected with this layout. */
/* GROUPED8 (SCALAR and VECTOR kinds, complex64 input, no CONJ_W1 flag): rows in groups of 8, each lane's 8 rows x T tables as quads of 4 floats:
 *   T8[g][mt][s][q][lane][4], g < ceil(R/8), q < 2T,
 *   VECTOR: quad q = (row 2q: t0, t1, row 2q+1: t0, t1), t0 = W0 + W1, t1 = W0 - W1
 *   SCALAR: quad q = rows 4q .. 4q+3
 * zero outside the tables and above the diagonal.  A warp's step is one
 * contiguous 1 KB (SCALAR) / 2 KB (VECTOR) block, which the streaming kernel
 * moves into shared memory with bulk asynchronous copies (cp.async.bulk),
 * 64 output rows per CTA.  Bit 0 of holysht_stream_error_word reports a
 * pipeline wait that gave up. */
#define HOLYSHT_TABLE_STRIDED 0
#define HOLYSHT_TABLE_GROUPED 1
#define HOLYSHT_TABLE_GROUPED8 2
/* GROUPED8_PARITY (forward direction, SCALAR and VECTOR kinds): the GROUPED8
 * layout of the northern rows k < ceil(nlat/2) only (S = ceil(nlat/2) steps),
 * for grids symmetric about the equator, where the table obeys
 * W(nlat-1-k) = (-1)^(l+m) W(k) (scalar, and W1 of the vector map) and
 * W0(nlat-1-k) = -(-1)^(l+m) W0(k).  The vector tables are stored as
 * t0 = W0 + W1, t1 = -(-1)^l (W0 - W1) (row l; the conjugate map: W1 -> -W1).
 * The kernel reads input rows k and nlat-1-k together (half the table bytes,
 * and for the scalar kind half the multiply-adds).  No counterpart in the
 * reference. */
#define HOLYSHT_TABLE_GROUPED8_PARITY 3

int holysht_legendre_contract(const holysht_contract_desc* desc, void* stream);

/* Forward transform from the real field in one call: the longitude rFFT of
 * `rows` contiguous rows of `nlon` float32 (unnormalised, cuFFT R2C on
 * `stream`) into `spec` (caller-allocated, rows x (nlon/2+1) complex64), then
 * holysht_legendre_contract(desc) with desc->in replaced by `spec` (desc's
 * input strides describe `spec`; forward direction, complex input).  cuFFT is
 * opened at run time (libcufft.so.11, the process's copy when one is loaded);
 * HOLYSHT_ERR_UNSUPPORTED when it cannot be.  No counterpart operator in the
 * reference, whose module calls torch.fft.rfft and then the Legendre operator
 * (torch-ext/holysht/__init__.py:1288-1389, :1504-1693): this entry is those
 * two steps.  fft_work: at least holysht_rfft_workspace() bytes (may be NULL
 * when that is 0), from the caller's allocator on the same stream. */
int holysht_rfft_workspace(int64_t rows, int64_t nlon, int64_t* bytes);
int holysht_rfft_contract(const float* field, int64_t rows, int64_t nlon, void* spec, void* fft_work,
                          int64_t fft_work_bytes, const holysht_contract_desc* desc, void* stream);

/* The same contraction (HOLYSHT_TABLE_GROUPED8 layout only) with its output
 * stored on several GPUs at once: no counterpart in the reference, which has
 * no multi-GPU code; it is the fused "contract + all-gather" step of the
 * order-partitioned transform.  Every output element (b, c, row, m) is stored
 * at column out_col_offset + m of each of the n_peers (1..8) buffers in
 * peer_out (device pointers valid in the calling context: this GPU's own
 * buffer and the peers' buffers mapped into it, all with desc's output
 * strides), by plain stores over NVLink; when multicast_out is not null it is
 * the NVLink multicast address of those buffers and each element is stored
 * once through it (multimem.st), the switch delivering it to every GPU.
 * desc->out is ignored.  The call only launches: the caller orders the
 * stores with every peer (for example a cross-GPU barrier on the same stream)
 * before any GPU reads its buffer. */
/* Cross-GPU barrier on `stream` for the ranks that share the stores of
 * holysht_legendre_contract_peers (no counterpart in the reference).
 * signal[q] is rank q's array of n_ranks (1..8) 32-bit words as mapped on this
 * GPU (zero-initialised once; epochs start at 1 and increase by one per
 * barrier).  Each rank stores `epoch` into word `rank` of every array with
 * system-scope release semantics (ordering its earlier stores, the peer
 * stores of the contraction included) and waits with acquire semantics until
 * every word of its own array has reached `epoch`.  The wait is bounded: a
 * peer that does not arrive sets bit 0 of the word holysht_peer_error_word
 * reads, and the kernel returns instead of hanging. */
int holysht_peer_barrier(void* const* signal, int n_ranks, int rank, unsigned epoch, void* stream);

/* Reads and clears the peer barrier's device error word (synchronous). */
int holysht_peer_error_word(unsigned* value);

int holysht_legendre_contract_peers(const holysht_contract_desc* desc, void* const* peer_out, int n_peers,
                                    int64_t out_col_offset, void* multicast_out, void* stream);

/* ---------------------------------------------------------------------------
 * Dense tensor-core contraction (no counterpart operator in the reference; the
 * reference's TF32 wmma forward, cuda/fused_legendre.cu:635-714, is its
 * approximate analogue).  For large batches the per-order contraction is a
 * GEMM; this entry runs it on tcgen05 tensor cores with a three-product
 * split-TF32 scheme (fp32-level accuracy), for the SCALAR kind:
 *   forward: out[b,l,m] = scale * sum_k W[m,l,k] in[b,k,m]        (l >= m; 0 otherwise)
 *   inverse: out[b,k,m] = scale * sum_{l>=m} W[m,l,k] in[b,l,m]
 * in / out: complex64, element (b,row,m) at ptr + b*batch_stride + row*row_stride + m
 * (the rfft output and the irfft input buffers can be passed as they are);
 * columns out_cols > mmax of out are written as zeros; HOLYSHT_FLAG_IRFFT_PREP
 * (inverse) also zeroes Im at m = 0 and, for even nlon, m = nlon/2;
 * HOLYSHT_FLAG_ROUND_BF16 rounds the scaled input to bfloat16 first.
 * table: float32, forward [mmax][lmax][nlat] (the torch-harmonics `weights`
 * layout), inverse [mmax][nlat][lmax] (the same table transposed per order);
 * the reduction extent (nlat forward, lmax inverse) must be a multiple of 4.
 * workspace: caller-allocated device memory (256-byte aligned) of at least
 * the size holysht_legendre_dense_tc_workspace reports; it holds the split
 * table (unless HOLYSHT_FLAG_TABLE_SPLIT), the transposed input split into
 * tf32 and residual planes, and the GEMM output between the launches. */
/* HOLYSHT_FLAG_TABLE_SPLIT (holysht_legendre_dense_tc only): `table` is the
 * split table [2][mmax][R][S] that holysht_legendre_dense_tc_split_table
 * writes (plane 0: the tf32-rounded table, plane 1: the fp32 residual), so
 * the call does not split it again; the workspace then needs only the size
 * holysht_legendre_dense_tc_workspace_ex reports with this flag. */
#define HOLYSHT_FLAG_TABLE_SPLIT 16

/* Split a dense-path table of `count` floats for HOLYSHT_FLAG_TABLE_SPLIT:
 * split[i] = rna_tf32(table[i]), split[count + i] = table[i] - split[i].
 * No counterpart in the reference (its tensor-core path rounds to TF32). */
int holysht_legendre_dense_tc_split_table(const float* table, float* split, int64_t count, void* stream);

/* Workspace bytes of holysht_legendre_dense_tc for the given flags (only
 * HOLYSHT_FLAG_TABLE_SPLIT changes the size).  Host-only. */
int holysht_legendre_dense_tc_workspace_ex(int direction, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                           int flags, int64_t* bytes);

int holysht_legendre_dense_tc_workspace(int direction, int64_t batch, int64_t nlat, int64_t lmax,
                                        int64_t mmax, int64_t* bytes);
int holysht_legendre_dense_tc(int direction, void* out, int64_t out_batch_stride,
                              int64_t out_row_stride, int64_t out_cols, const void* in,
                              int64_t in_batch_stride, int64_t in_row_stride, const float* table,
                              int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax, float scale,
                              int flags, int64_t nlon, void* workspace, int64_t workspace_bytes,
                              void* stream);

/* Scalar forward with on-the-fly Legendre functions (the recurrence variant;
 * no counterpart operator in the reference, whose kernels all stream a table):
 *   out[b,l,m] = scale * sum_k spec[b,k,m] * w_k P_l^m(cos theta_k)   (l >= m; 0 otherwise)
 * P comes from the three-term recurrence in fp32 registers, re-seeded every
 * 16 degrees from float64 checkpoints:
 *   seeds     float32 [mmax][ceil(lmax/16)][nlat][2]: w_k P_l^m at l = m + 16c and
 *             m + 16c + 1 (normalisation, Condon-Shortley phase and quadrature
 *             weight included);
 *   coef      float32 [mmax][lmax][2]: the recurrence coefficients (a_lm, b_lm);
 *   cos_theta float32 [nlat].
 * spec: complex64, element (b,k,m) at spec + b*spec_batch_stride + k*spec_row_stride + m;
 * out: complex64 [B][lmax][mmax].  (holysht_b200.weights builds
 * the three inputs.) */
int holysht_legendre_forward_recurrence(void* out, const void* spec, int64_t spec_batch_stride,
                                        int64_t spec_row_stride, const float* seeds,
                                        const float* coef, const float* cos_theta, int64_t batch,
                                        int64_t nlat, int64_t lmax, int64_t mmax, float scale,
                                        void* stream);

/* HOLYSHT_FLAG_EQUATORIAL_PARITY (recurrence entries): the grid is symmetric
 * about the equator (cos theta_{nlat-1-k} = -cos theta_k, equal quadrature
 * weights), so P_l^m(-x) = (-1)^(l+m) P_l^m(x): only the northern latitudes'
 * Legendre functions are generated, contracted with the sum (l + m even) or
 * difference (l + m odd) of each latitude's spectrum and its mirror's.  Every
 * grid holysht_b200.weights builds is symmetric; the result is undefined for
 * seeds of an asymmetric grid. */
#define HOLYSHT_FLAG_EQUATORIAL_PARITY 32

/* HOLYSHT_FLAG_SEEDS_COMPACT (recurrence entries): `seeds` is in the compact,
 * latitude-major layout [nlat][nsegs][S] (S = 2 scalar, 4 vector) holding only
 * the segments that exist: for each order m < min(mmax, lmax) in turn, its
 * segments c = 0 .. ceil((lmax - m) / 16) - 1, nsegs their total
 * (holysht_b200.weights.compact_recurrence_seeds builds it).  The default
 * layout is [mmax][ceil(lmax/16)][nlat][S]. */
#define HOLYSHT_FLAG_SEEDS_COMPACT 64

/* holysht_legendre_forward_recurrence with flags (HOLYSHT_FLAG_EQUATORIAL_PARITY,
 * HOLYSHT_FLAG_SEEDS_COMPACT); the plain entry is flags = 0.  seeds, spec and
 * out must be 8-byte aligned; any nlat. */
int holysht_legendre_forward_recurrence_ex(void* out, const void* spec, int64_t spec_batch_stride,
                                           int64_t spec_row_stride, const float* seeds,
                                           const float* coef, const float* cos_theta, int64_t batch,
                                           int64_t nlat, int64_t lmax, int64_t mmax, float scale,
                                           int flags, void* stream);

/* Vector forward (RealVectorSHT's contraction) with on-the-fly tables: the
 * orders m - 1 and m + 1 Legendre recurrences run in fp32 from float64
 * checkpoints every 16 degrees and are combined by the ladder identities into
 * (W0 + W1, W0 - W1) per degree.  out [B][2][lmax][mmax] complex64 (contiguous),
 * spec: element (b, component, k, m) at b*spec_batch_stride +
 * c*spec_comp_stride + k*spec_row_stride + m (the rfft layout), seeds
 * [mmax][ceil(lmax/16)][nlat][4] (16-byte aligned), coef [mmax][lmax][8],
 * cos_theta [nlat], all from holysht_b200.weights.vector_recurrence_tables.
 * Output = scale * contraction; exact zeros for m > l. */
int holysht_legendre_vector_forward_recurrence(void* out, const void* spec, int64_t spec_batch_stride,
                                               int64_t spec_comp_stride, int64_t spec_row_stride, const float* seeds,
                                               const float* coef, const float* cos_theta, int64_t batch,
                                               int64_t nlat, int64_t lmax, int64_t mmax, float scale, void* stream);

/* holysht_legendre_vector_forward_recurrence with flags
 * (HOLYSHT_FLAG_EQUATORIAL_PARITY, HOLYSHT_FLAG_SEEDS_COMPACT); the plain entry
 * is flags = 0.  seeds and coef 16-byte aligned, spec and out 8-byte aligned;
 * any nlat. */
int holysht_legendre_vector_forward_recurrence_ex(void* out, const void* spec, int64_t spec_batch_stride,
                                                  int64_t spec_comp_stride, int64_t spec_row_stride,
                                                  const float* seeds, const float* coef,
                                                  const float* cos_theta, int64_t batch, int64_t nlat,
                                                  int64_t lmax, int64_t mmax, float scale, int flags,
                                                  void* stream);

/* Scalar inverse contraction (InverseRealSHT's) with on-the-fly Legendre
 * functions (the recurrence variant; no counterpart operator in the reference):
 *   out[b,k,m] = scale * sum_{l >= m} P_l^m(cos theta_k) * spec[b,l,m],  m < mmax;
 * columns mmax .. out_cols-1 are written as zeros.  One thread per (order,
 * latitude) runs the recurrence through the order's 8-degree checkpoint
 * segments; the reduction over l needs no exchange between threads.
 *   seeds float32 [mmax][ceil(lmax/8)][nlat][2]: P at l = m + 8c, m + 8c + 1
 *         in the inverse normalisation (holysht_b200.weights.scalar_recurrence_tables(
 *         ..., inverse=True, segment=8)); coef [mmax][lmax][2]; cos_theta [nlat];
 *   flags: HOLYSHT_FLAG_EQUATORIAL_PARITY (symmetric grids), HOLYSHT_FLAG_IRFFT_PREP
 *         (Im = 0 at m = 0 and, even nlon, at m = nlon/2; out_cols <= nlon/2+1).
 * spec: complex64, element (b,l,m) at spec + b*spec_batch_stride + l*spec_row_stride + m;
 * out: complex64, element (b,k,m) at out + b*out_batch_stride + k*out_row_stride + m.
 * spec, out, seeds and coef must be 8-byte aligned. */
int holysht_legendre_inverse_recurrence(void* out, int64_t out_batch_stride, int64_t out_row_stride,
                                        int64_t out_cols, const void* spec, int64_t spec_batch_stride,
                                        int64_t spec_row_stride, const float* seeds, const float* coef,
                                        const float* cos_theta, int64_t batch, int64_t nlat, int64_t lmax,
                                        int64_t mmax, float scale, int flags, int64_t nlon, void* stream);

/* Same contraction as holysht_legendre_dense_tc, for callers that cannot
 * allocate device memory (a host whose own allocator owns the GPU memory, a
 * loop that must not allocate per call, a plugin handed no allocator).  No
 * counterpart in the reference.  The scratch is a 64 MiB array built into the
 * library (held on every GPU that loads it until the process exits); problems
 * whose holysht_legendre_dense_tc_workspace size exceeds 64 MiB are rejected
 * with HOLYSHT_ERR_INVALID.  Every call looks the array's device address up
 * in the current context (cudaGetSymbolAddress), so after cudaDeviceReset the
 * next call uses the re-created context's copy of the array; make the first
 * call on a device before any stream capture.  All calls share the one array: calls that overlap on the
 * GPU (other streams, other host threads) race on it and must be serialised
 * by the caller.  Nothing in the array carries over between calls: every
 * scratch element a call reads was written earlier in the same call.  No
 * cudaMalloc, cudaFree or other allocating routine is called. */
int holysht_legendre_dense_tc_noalloc(int direction, void* out, int64_t out_batch_stride,
                                      int64_t out_row_stride, int64_t out_cols, const void* in,
                                      int64_t in_batch_stride, int64_t in_row_stride,
                                      const float* table, int64_t batch, int64_t nlat, int64_t lmax,
                                      int64_t mmax, float scale, int flags, int64_t nlon, void* stream);

/* Diagnostics: reads and clears the tensor-core kernel's device error word
 * (bit 0: a pipeline wait gave up instead of hanging).  Synchronous. */
int holysht_tc_error_word(unsigned* value);

/* Diagnostics: reads and clears the streaming kernel's device error word
 * (HOLYSHT_TABLE_GROUPED8; bit 0: a pipeline wait gave up instead of hanging).
 * Synchronous. */
int holysht_stream_error_word(unsigned* value);

/* Launch plan of the streaming kernel (HOLYSHT_TABLE_GROUPED8) for a contraction
 * of the given extents: reduction split *ks_out (cluster size), number of
 * clusters *clusters_out and work items *items_out (compute tile x batch group).
 * Clusters walk the items in snake order, longest reduction first; the plan is
 * the split with the smallest simulated makespan.  sm_count > 0 plans for that
 * many SMs without touching the GPU; 0 uses the current device.  ksplit 0
 * chooses, else 1/2/4/8 is kept.  Host-only, no launch. */
int holysht_stream_launch_plan(int kind, int direction, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                               int64_t out_cols, int64_t m_offset, int ksplit, int sm_count, int* ks_out,
                               int* clusters_out, int* items_out);

#ifdef __cplusplus
}
#endif

#endif /* HOLYSHT_B200_H_ */
