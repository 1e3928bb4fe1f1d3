// C ABI of libholysht_b200.so: argument validation, launch configuration and
// dispatch to the sm_100a kernels.  The checks mirror the reference's
// TORCH_CHECK set (cuda/fused_legendre.cu:3157-3335): non-null pointers,
// non-negative extents, table/input extents that agree, and extents that fit
// the kernels' 32-bit tile arithmetic.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <array>
#include <map>
#include <mutex>
#include <utility>
#include <vector>
#include <string>

#include "../../include/holysht_b200.h"
#include "contract.cuh"
#include "elementwise.cuh"
#include "tc_dense.cuh"
#include "recurrence.cuh"
#include "stream.cuh"
#include "peer.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return HOLYSHT_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HOLYSHT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

constexpr int kMaxDevices = 64;

int sm_count_of_current_device() {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Test hook of the streaming kernel (HOLYSHT_TEST_STALL_CHUNK, read once): the
// first CTA's warp 0 skips this table stage, so a bounded wait runs out and the
// error word is set; the kernel still finishes.  Off (-1) by default.
int env_stall_chunk() {
  static int v = [] {
    const char* s = std::getenv("HOLYSHT_TEST_STALL_CHUNK");
    return (s && *s) ? std::atoi(s) : -1;
  }();
  return v;
}

// Integer environment variable (read on every call: experiment switches that
// a process may flip between launches).
int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}

int env_ksplit() {
  static int v = [] {
    const char* s = std::getenv("HOLYSHT_KSPLIT");
    if (!s || !*s) return 0;
    int k = std::atoi(s);
    return (k == 1 || k == 2 || k == 4 || k == 8) ? k : 0;
  }();
  return v;
}

template <int KIND, int DIR, int NB, typename TIN, bool GROUPED>
int launch_contract(const hsb::ContractParams& p_in, int grid_tiles, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  auto kernel = hsb::contract_kernel<KIND, DIR, NB, TIN, GROUPED>;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         hsb::kSmemBytes);
    if (e != cudaSuccess)
      return fail(HOLYSHT_ERR_UNSUPPORTED, "cannot configure the Legendre kernel: %s",
                  cudaGetErrorString(e));
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  hsb::ContractParams p = p_in;
  if (p.ks == 0) {
    // one resident wave: the largest split whose CTAs all fit on the GPU at
    // once (zero tiles are short-lived and not counted), each cluster rank
    // keeping at least two staged chunks of the reduction
    static std::atomic<int> occ_cache[kMaxDevices];
    int occ = (dev >= 0 && dev < kMaxDevices) ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
    if (occ <= 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, hsb::kThreads, hsb::kSmemBytes) !=
              cudaSuccess ||
          occ <= 0)
        occ = 1;
      if (dev >= 0 && dev < kMaxDevices) occ_cache[dev].store(occ, std::memory_order_relaxed);
    }
    const long long slots = (long long)occ * sm_count_of_current_device();
    const long long tiles = (long long)p.n_compute * p.n_bg;
    int ks = 1;
    while (ks < 8 && tiles * ks * 2 <= slots && p.S / (2LL * ks) >= 2LL * hsb::kChunk) ks *= 2;
    p.ks = ks;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid_tiles) * static_cast<unsigned>(p.ks), 1, 1);
  cfg.blockDim = dim3(hsb::kThreads, 1, 1);
  cfg.dynamicSmemBytes = hsb::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(HOLYSHT_ERR_CUDA, "Legendre kernel launch failed: %s", cudaGetErrorString(e));
  }
  return ok();
}

int next_pow2_at_least(long long v, int lo, int hi) {
  int r = lo;
  while (r < hi && r < v) r *= 2;
  return r;
}

bool fits_int(long long v) { return v >= 0 && v <= (INT_MAX / 4); }

// Normalised description handed to the dispatcher.
struct Job {
  int kind, dir, in_dtype, flags;
  const void* in;
  void* out;
  const float* w0;
  const float* w1;
  long long B, K, L, M;
  long long in_bs, in_ps, in_rs, out_bs, out_ps, out_rs, out_cols, w_ls, w_ks, w_mt, nlon;
  float scale;
  int ksplit;
  int grouped;   // HOLYSHT_TABLE_GROUPED
  int grouped8;  // HOLYSHT_TABLE_GROUPED8 / _PARITY (streaming kernel)
  int parity;    // HOLYSHT_TABLE_GROUPED8_PARITY: northern-half table, reduction over ceil(K/2) rows
  long long m_off;
  // output to several GPUs (holysht_legendre_contract_peers); n_peers == 0: out only
  void* const* peers;
  int n_peers;
  long long col_off;
  void* mc;
};

template <int KIND, int DIR, typename TIN, bool GROUPED>
int dispatch_nb(const hsb::ContractParams& p0, int nb, cudaStream_t stream) {
  hsb::ContractParams p = p0;
  p.n_bg = (p.B + nb - 1) / nb;
  const long long tiles = (long long)(p.n_compute + p.n_zero) * p.n_bg;
  if (tiles == 0) return ok();
  if (tiles * 8 > INT_MAX / 2) return fail(HOLYSHT_ERR_INVALID, "problem too large for one launch");
  const int grid_tiles = static_cast<int>(tiles);
  if constexpr (KIND == hsb::KIND_VECTOR) {
    switch (nb) {
      case 1: return launch_contract<KIND, DIR, 1, TIN, GROUPED>(p, grid_tiles, stream);
      case 2: return launch_contract<KIND, DIR, 2, TIN, GROUPED>(p, grid_tiles, stream);
      default: return launch_contract<KIND, DIR, 4, TIN, GROUPED>(p, grid_tiles, stream);
    }
  } else if constexpr (KIND == hsb::KIND_SCALAR) {
    switch (nb) {
      case 1: return launch_contract<KIND, DIR, 1, TIN, GROUPED>(p, grid_tiles, stream);
      case 2: return launch_contract<KIND, DIR, 2, TIN, GROUPED>(p, grid_tiles, stream);
      case 4: return launch_contract<KIND, DIR, 4, TIN, GROUPED>(p, grid_tiles, stream);
      default: return launch_contract<KIND, DIR, 8, TIN, GROUPED>(p, grid_tiles, stream);
    }
  } else {
    switch (nb) {
      case 2: return launch_contract<KIND, DIR, 2, TIN, false>(p, grid_tiles, stream);
      case 4: return launch_contract<KIND, DIR, 4, TIN, false>(p, grid_tiles, stream);
      case 8: return launch_contract<KIND, DIR, 8, TIN, false>(p, grid_tiles, stream);
      default: return launch_contract<KIND, DIR, 16, TIN, false>(p, grid_tiles, stream);
    }
  }
}

template <int KIND, typename TIN, bool GROUPED>
int dispatch_dir(const hsb::ContractParams& p, int dir, int nb, cudaStream_t stream) {
  return dir == HOLYSHT_DIR_FORWARD ? dispatch_nb<KIND, hsb::DIR_FWD, TIN, GROUPED>(p, nb, stream)
                                    : dispatch_nb<KIND, hsb::DIR_INV, TIN, GROUPED>(p, nb, stream);
}

int run_job_resolved(const Job& j, long long R, long long S, cudaStream_t stream);
int run_stream_job(const Job& j, long long R, long long S, cudaStream_t stream);

int run_job(const Job& j, cudaStream_t stream) {
  if (j.kind < 0 || j.kind > 2) return fail(HOLYSHT_ERR_INVALID, "unknown kind %d", j.kind);
  if (j.dir != HOLYSHT_DIR_FORWARD && j.dir != HOLYSHT_DIR_INVERSE)
    return fail(HOLYSHT_ERR_INVALID, "unknown direction %d", j.dir);
  if (j.flags & ~(HOLYSHT_FLAG_CONJ_W1 | HOLYSHT_FLAG_ROUND_BF16 | HOLYSHT_FLAG_IRFFT_PREP))
    return fail(HOLYSHT_ERR_INVALID, "unknown flags 0x%x", j.flags);
  if (j.B < 0 || j.K < 0 || j.L < 0 || j.M < 0)
    return fail(HOLYSHT_ERR_INVALID, "negative extent (batch=%lld nlat=%lld lmax=%lld mmax=%lld)",
                j.B, j.K, j.L, j.M);
  if (!fits_int(j.B) || !fits_int(j.K) || !fits_int(j.L) || !fits_int(j.M) || !fits_int(j.out_cols))
    return fail(HOLYSHT_ERR_INVALID, "extent exceeds the 32-bit tile range");
  if (j.out_cols < j.M) return fail(HOLYSHT_ERR_INVALID, "out_cols (%lld) < mmax (%lld)", j.out_cols, j.M);
  const long long R = j.dir == HOLYSHT_DIR_FORWARD ? j.L : j.K;
  const long long S = j.dir == HOLYSHT_DIR_FORWARD ? j.K : j.L;
  if (j.B == 0 || R == 0 || j.out_cols == 0) return ok();
  if (!j.out && j.n_peers == 0) return fail(HOLYSHT_ERR_INVALID, "output pointer is null");
  if (S > 0 && j.M > 0 && (!j.in || !j.w0)) return fail(HOLYSHT_ERR_INVALID, "input or table pointer is null");
  if (j.kind == HOLYSHT_KIND_VECTOR && !j.grouped && !j.grouped8 && S > 0 && j.M > 0 && !j.w1)
    return fail(HOLYSHT_ERR_INVALID, "vector contraction needs both tables");
  if (j.kind == HOLYSHT_KIND_REAL) {
    if (j.in_dtype != HOLYSHT_DTYPE_F32 && j.in_dtype != HOLYSHT_DTYPE_BF16)
      return fail(HOLYSHT_ERR_INVALID, "input must be float32 or bfloat16");
    if (j.flags & (HOLYSHT_FLAG_CONJ_W1 | HOLYSHT_FLAG_IRFFT_PREP))
      return fail(HOLYSHT_ERR_INVALID, "flag not valid for a real contraction");
  } else if (j.in_dtype != HOLYSHT_DTYPE_C64) {
    return fail(HOLYSHT_ERR_INVALID, "input must be complex64");
  }
  if (j.grouped && j.kind == HOLYSHT_KIND_REAL)
    return fail(HOLYSHT_ERR_INVALID, "the row-grouped table layout is for complex contractions");
  if (j.grouped && j.kind == HOLYSHT_KIND_VECTOR && (j.flags & HOLYSHT_FLAG_CONJ_W1))
    return fail(HOLYSHT_ERR_INVALID,
                "grouped vector tables carry the sign of W1 (W0 + W1, W0 - W1); build the "
                "conjugate map's table from (W0, -W1) instead of passing HOLYSHT_FLAG_CONJ_W1");
  if (j.grouped8) {
    if (j.kind == HOLYSHT_KIND_REAL)
      return fail(HOLYSHT_ERR_INVALID, "the GROUPED8 table layout is for complex contractions");
    if (j.flags & HOLYSHT_FLAG_CONJ_W1)
      return fail(HOLYSHT_ERR_INVALID,
                  "the GROUPED8 layout does not take HOLYSHT_FLAG_CONJ_W1 (build the table from (W0, -W1))");
    if (j.parity) {
      if (j.dir == HOLYSHT_DIR_FORWARD) return run_stream_job(j, R, (S + 1) / 2, stream);  // northern steps
      if (j.kind != HOLYSHT_KIND_SCALAR)
        return fail(HOLYSHT_ERR_INVALID, "the GROUPED8_PARITY inverse is for the scalar kind");
      return run_stream_job(j, (R + 1) / 2, S, stream);  // northern output rows, mirrored in the epilogue
    }
    return run_stream_job(j, R, S, stream);
  }
  Job jj = j;
  if (j.grouped) {
    // row-grouped layout: [R/4 groups][ceil(M/32) tiles][S steps][32 lanes][4 rows][tables]
    const long long G = (long long)hsb::kRowsPerWarp * (j.kind == HOLYSHT_KIND_VECTOR ? 2 : 1);
    const long long mt = (j.M + hsb::kMTile - 1) / hsb::kMTile;
    const long long groups = (R + hsb::kRowsPerWarp - 1) / hsb::kRowsPerWarp;
    jj.w_ks = 32 * G;
    jj.w_mt = S * 32 * G;
    jj.w_ls = mt * S * 32 * G;
    if (groups * jj.w_ls >= (1LL << 32))
      return fail(HOLYSHT_ERR_INVALID, "grouped table exceeds 2^32 floats");
  }
  return run_job_resolved(jj, R, S, stream);
}

int run_job_resolved(const Job& j, long long R, long long S, cudaStream_t stream) {
  if (!j.grouped) {
    // the kernel addresses a table with 32-bit float offsets
    const long long n_mt_tab = (j.M + hsb::kMTile - 1) / hsb::kMTile;
    const long long span = (j.L > 0 ? (j.L - 1) * j.w_ls : 0) + (j.K > 0 ? (j.K - 1) * j.w_ks : 0) +
                           (n_mt_tab > 0 ? (n_mt_tab - 1) * j.w_mt : 0) + hsb::kMTile;
    if (j.w_ls < 0 || j.w_ks < 0 || j.w_mt < 0 || span >= (1LL << 32))
      return fail(HOLYSHT_ERR_INVALID, "table strides must be non-negative and span < 2^32 floats");
  }
  if (j.ksplit != 0 && j.ksplit != 1 && j.ksplit != 2 && j.ksplit != 4 && j.ksplit != 8)
    return fail(HOLYSHT_ERR_INVALID, "ksplit must be 0, 1, 2, 4 or 8");

  hsb::ContractParams p = {};
  p.in = j.in;
  p.out = j.out;
  p.w0 = j.w0;
  p.w1 = j.w1;
  p.in_bs = j.in_bs;
  p.in_ps = j.in_ps;
  p.in_rs = j.in_rs;
  p.out_bs = j.out_bs;
  p.out_ps = j.out_ps;
  p.out_rs = j.out_rs;
  p.w_ls = j.w_ls;
  p.w_ks = j.w_ks;
  p.w_mt = j.w_mt;
  p.B = (int)j.B;
  p.K = (int)j.K;
  p.L = (int)j.L;
  p.M = (int)j.M;
  p.out_cols = (int)j.out_cols;
  p.R = (int)R;
  p.S = (int)S;
  p.scale = j.scale;
  p.w1_sign = (j.flags & HOLYSHT_FLAG_CONJ_W1) ? -1.f : 1.f;
  p.zero_imag_col0 = (j.flags & HOLYSHT_FLAG_IRFFT_PREP) ? 1 : 0;
  p.nyquist = ((j.flags & HOLYSHT_FLAG_IRFFT_PREP) && j.nlon > 0 && j.nlon % 2 == 0) ? (int)(j.nlon / 2) : -1;
  p.round_bf16 = (j.flags & HOLYSHT_FLAG_ROUND_BF16) ? 1 : 0;

  p.n_rt = (int)((R + hsb::kRows - 1) / hsb::kRows);
  p.n_mt = (int)((j.out_cols + hsb::kMTile - 1) / hsb::kMTile);
  // active m tiles: inside the table columns and with some l >= m below L
  const long long act_cols = (S > 0) ? j.M : 0;
  const long long act_l = (S > 0 && j.L > j.m_off) ? j.L - j.m_off : 0;
  const long long act = act_cols < act_l ? act_cols : act_l;
  p.j_act = (int)((act + hsb::kMTile - 1) / hsb::kMTile);
  p.m_off = (int)j.m_off;
  p.mt_off = (int)(j.m_off / hsb::kMTile);
  if (p.j_act > p.n_mt) p.j_act = p.n_mt;
  long long n_compute = 0, n_zero = 0;
  for (int jt = 0; jt < p.n_mt; ++jt) {
    if (jt < p.j_act) {
      const int first = j.dir == HOLYSHT_DIR_FORWARD ? jt + p.mt_off : 0;
      n_compute += p.n_rt > first ? p.n_rt - first : 0;
      n_zero += j.dir == HOLYSHT_DIR_FORWARD ? (first < p.n_rt ? first : p.n_rt) : 0;
    } else {
      n_zero += p.n_rt;
    }
  }
  p.n_compute = (int)n_compute;
  p.n_zero = (int)n_zero;

  int nb;
  if (j.kind == HOLYSHT_KIND_VECTOR)
    nb = next_pow2_at_least(j.B, 1, 4);
  else if (j.kind == HOLYSHT_KIND_SCALAR)
    nb = next_pow2_at_least(j.B, 1, 8);
  else
    nb = next_pow2_at_least(j.B, 2, 16);

  // reduction split (cluster size): 0 = choose at launch from the occupancy
  int ks = j.ksplit ? j.ksplit : env_ksplit();
  p.ks = ks;

  if (j.kind == HOLYSHT_KIND_SCALAR)
    return j.grouped ? dispatch_dir<hsb::KIND_SCALAR, float2, true>(p, j.dir, nb, stream)
                     : dispatch_dir<hsb::KIND_SCALAR, float2, false>(p, j.dir, nb, stream);
  if (j.kind == HOLYSHT_KIND_VECTOR)
    return j.grouped ? dispatch_dir<hsb::KIND_VECTOR, float2, true>(p, j.dir, nb, stream)
                     : dispatch_dir<hsb::KIND_VECTOR, float2, false>(p, j.dir, nb, stream);
  if (j.in_dtype == HOLYSHT_DTYPE_BF16)
    return dispatch_dir<hsb::KIND_REAL, __nv_bfloat16, false>(p, j.dir, nb, stream);
  return dispatch_dir<hsb::KIND_REAL, float, false>(p, j.dir, nb, stream);
}

// ---- streaming kernel (GROUPED8 tables) ----

// Reduction split (cluster size) and number of clusters of a streaming launch.
// One CTA per SM; clusters walk the work items (compute tile x batch group,
// ordered by decreasing reduction length) in a snake order, so the split and
// cluster count are chosen by simulating that assignment: the smallest
// makespan in chunks (plus a fixed per-item cost for the pipeline ramp and the
// epilogue), the smaller split on a tie.  An explicit ksplit is kept.
std::pair<int, int> simulate_stream_grid(const hsb::stream::Params& p, int chunk, bool forward, int sms);

// The plan depends on a handful of extents only: cached (the simulation walks every item).
std::pair<int, int> choose_stream_grid(const hsb::stream::Params& p, int chunk, bool forward, int sms) {
  using Key = std::array<long long, 10>;
  static std::mutex mu;
  static std::map<Key, std::pair<int, int>> cache;
  const Key key = {p.R, p.S, p.M, p.j_act, p.mt_off, p.n_bg, p.ks, chunk, forward ? 1 : 0, sms};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const std::pair<int, int> plan = simulate_stream_grid(p, chunk, forward, sms);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 1024) cache.clear();
  cache[key] = plan;
  return plan;
}

std::pair<int, int> simulate_stream_grid(const hsb::stream::Params& p, int chunk, bool forward, int sms) {
  namespace st = hsb::stream;
  std::vector<int> steps;  // reduction steps of every item, in item order
  for (int jt = 0; jt < p.j_act; ++jt) {
    const long long diag = std::min<long long>(32LL * (jt + p.mt_off), p.R);
    const long long first = forward ? diag : 0;
    const long long cnt = (p.R - first + st::kRows - 1) / st::kRows;
    const int s = forward ? p.S : (int)(p.S - std::min<long long>(32LL * (jt + p.mt_off), p.S));
    for (long long t = 0; t < cnt * p.n_bg; ++t) steps.push_back(s);
  }
  const long long items = (long long)steps.size();
  constexpr long long kItemCost = 2;  // chunks: pipeline ramp-up and the cluster epilogue
  long long best = LLONG_MAX;
  std::pair<int, int> choice{1, (int)std::max<long long>(1, std::min<long long>(items, sms))};
  for (int ks = 1; ks <= 8; ks *= 2) {
    if (p.ks != 0 && ks != p.ks) continue;
    if (p.ks == 0 && ks > 1 && p.S / (2LL * ks) < 2LL * st::kMaxChunk) break;
    const long long G = std::max<long long>(1, std::min<long long>(items, sms / ks));
    std::vector<long long> load((size_t)G, 0);
    for (long long i = 0; i < items; ++i) {
      const long long round = i / G, pos = i % G;
      const long long c = (round & 1) ? G - 1 - pos : pos;
      const long long per = (steps[(size_t)i] + ks - 1) / ks;
      load[(size_t)c] += (per + chunk - 1) / chunk + kItemCost;
    }
    const long long mk = *std::max_element(load.begin(), load.end());
    if (mk < best) {
      best = mk;
      choice = {ks, (int)G};
    }
  }
  return choice;
}

template <int KIND, int DIR, int NB, int FOLD = 0>
int launch_stream(const hsb::stream::Params& p_in, long long grid_tiles, cudaStream_t stream) {
  using Sm = hsb::stream::Smem<KIND, NB, FOLD>;
  static std::atomic<unsigned long long> configured{0};
  auto kernel = hsb::stream::stream_kernel<KIND, DIR, NB, FOLD>;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Sm::kBytes);
    if (e != cudaSuccess)
      return fail(HOLYSHT_ERR_UNSUPPORTED, "cannot configure the streaming Legendre kernel: %s",
                  cudaGetErrorString(e));
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  hsb::stream::Params p = p_in;
  long long grid = 0;
  if (p.n_compute == 0) {
    p.ks = 1;  // a grid of zero writers only
    grid = grid_tiles;
  } else {
    const std::pair<int, int> plan =
        choose_stream_grid(p, hsb::stream::Shape<KIND, FOLD>::kChunk, DIR == 0, sm_count_of_current_device());
    p.ks = plan.first;
    grid = (long long)plan.second * p.ks;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(hsb::stream::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Sm::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(HOLYSHT_ERR_CUDA, "streaming Legendre kernel launch failed: %s", cudaGetErrorString(e));
  }
  return ok();
}

template <int KIND, int DIR>
int stream_nb(const hsb::stream::Params& p, int nb, long long grid_tiles, cudaStream_t stream) {
  if constexpr (DIR == 0) {
    if (p.kfull > 0) {  // parity-folded forward
      switch (nb) {
        case 1: return launch_stream<KIND, DIR, 1, 1>(p, grid_tiles, stream);
        case 2: return launch_stream<KIND, DIR, 2, 1>(p, grid_tiles, stream);
        case 4: return launch_stream<KIND, DIR, 4, 1>(p, grid_tiles, stream);
        default:
          if constexpr (KIND == hsb::KIND_SCALAR) return launch_stream<KIND, DIR, 8, 1>(p, grid_tiles, stream);
          return launch_stream<KIND, DIR, 4, 1>(p, grid_tiles, stream);
      }
    }
  } else if constexpr (KIND == hsb::KIND_SCALAR) {
    if (p.kfull > 0) {  // parity-folded scalar inverse (at most 4 batches per CTA: twice the accumulators)
      switch (nb) {
        case 1: return launch_stream<KIND, DIR, 1, 2>(p, grid_tiles, stream);
        case 2: return launch_stream<KIND, DIR, 2, 2>(p, grid_tiles, stream);
        default: return launch_stream<KIND, DIR, 4, 2>(p, grid_tiles, stream);
      }
    }
  }
  switch (nb) {
    case 1: return launch_stream<KIND, DIR, 1>(p, grid_tiles, stream);
    case 2: return launch_stream<KIND, DIR, 2>(p, grid_tiles, stream);
    case 4: return launch_stream<KIND, DIR, 4>(p, grid_tiles, stream);
    default:
      if constexpr (KIND == hsb::KIND_SCALAR) return launch_stream<KIND, DIR, 8>(p, grid_tiles, stream);
      return launch_stream<KIND, DIR, 4>(p, grid_tiles, stream);
  }
}

// Kernel parameters of a streaming job (no CUDA call); *nb_out = batches per CTA.
hsb::stream::Params make_stream_params(const Job& j, long long R, long long S, int* nb_out) {
  namespace st = hsb::stream;
  const long long T = j.kind == HOLYSHT_KIND_VECTOR ? 2 : 1;
  const long long step = 32LL * st::kRowsPerWarp * T;  // floats per (group, m tile, step)
  const long long mt_tab = (j.M + st::kMTile - 1) / st::kMTile;
  st::Params p = {};
  p.in = static_cast<const float2*>(j.in);
  p.out = j.out;
  p.table = j.w0;
  p.in_bs = j.in_bs;
  p.in_ps = j.in_ps;
  p.in_rs = j.in_rs;
  p.out_bs = j.out_bs;
  p.out_ps = j.out_ps;
  p.out_rs = j.out_rs;
  p.t_mt = S * step;
  p.t_group = mt_tab * S * step;
  p.B = (int)j.B;
  p.M = (int)j.M;
  p.R = (int)R;
  p.S = (int)S;
  p.out_cols = (int)j.out_cols;
  p.scale = j.scale;
  p.zero_imag_col0 = (j.flags & HOLYSHT_FLAG_IRFFT_PREP) ? 1 : 0;
  p.nyquist = ((j.flags & HOLYSHT_FLAG_IRFFT_PREP) && j.nlon > 0 && j.nlon % 2 == 0) ? (int)(j.nlon / 2) : -1;
  p.n_mt = (int)((j.out_cols + st::kMTile - 1) / st::kMTile);
  const long long act_cols = (S > 0) ? j.M : 0;
  const long long act_l = (S > 0 && j.L > j.m_off) ? j.L - j.m_off : 0;
  const long long act = act_cols < act_l ? act_cols : act_l;
  p.j_act = (int)std::min<long long>((act + st::kMTile - 1) / st::kMTile, p.n_mt);
  p.m_off = (int)j.m_off;
  p.mt_off = (int)(j.m_off / st::kMTile);
  long long n_compute = 0, n_zero = 0;
  for (int jt = 0; jt < p.n_mt; ++jt) {
    const long long first =
        jt < p.j_act ? (j.dir == HOLYSHT_DIR_FORWARD ? std::min<long long>(32LL * (jt + p.mt_off), R) : 0) : R;
    if (jt < p.j_act) n_compute += (R - first + st::kRows - 1) / st::kRows;
    n_zero += (first + st::kRows - 1) / st::kRows;
  }
  p.n_compute = (int)n_compute;
  p.n_zero = (int)n_zero;
  const bool fold_inv = j.parity && j.dir == HOLYSHT_DIR_INVERSE;  // twice the accumulators: at most 4 batches
  const int nb = next_pow2_at_least(j.B, 1, (j.kind == HOLYSHT_KIND_VECTOR || fold_inv) ? 4 : 8);
  p.n_bg = (int)((j.B + nb - 1) / nb);
  p.ks = j.ksplit ? j.ksplit : env_ksplit();
  p.stall_chunk = env_stall_chunk();
  p.kfull = j.parity ? (int)j.K : 0;
  p.round_bf16 = (j.flags & HOLYSHT_FLAG_ROUND_BF16) ? 1 : 0;
  p.n_peers = j.n_peers;
  p.col_off = (int)j.col_off;
  p.mc = static_cast<float2*>(j.mc);
  for (int q = 0; q < j.n_peers; ++q) p.peer[q] = static_cast<float2*>(j.peers[q]);
  *nb_out = nb;
  return p;
}

int run_stream_job(const Job& j, long long R, long long S, cudaStream_t stream) {
  if (j.ksplit != 0 && j.ksplit != 1 && j.ksplit != 2 && j.ksplit != 4 && j.ksplit != 8)
    return fail(HOLYSHT_ERR_INVALID, "ksplit must be 0, 1, 2, 4 or 8");
  int nb = 1;
  const hsb::stream::Params p = make_stream_params(j, R, S, &nb);
  const long long n_compute = p.n_compute, n_zero = p.n_zero;
  // the grid holds the compute tiles; their CTAs also write the zero tiles
  if (n_compute + n_zero == 0) return ok();
  const long long grid_tiles = n_compute > 0 ? n_compute * p.n_bg : std::min<long long>(n_zero * p.n_bg, 148);
  if (j.kind == HOLYSHT_KIND_VECTOR)
    return j.dir == HOLYSHT_DIR_FORWARD ? stream_nb<hsb::KIND_VECTOR, 0>(p, nb, grid_tiles, stream)
                                        : stream_nb<hsb::KIND_VECTOR, 1>(p, nb, grid_tiles, stream);
  return j.dir == HOLYSHT_DIR_FORWARD ? stream_nb<hsb::KIND_SCALAR, 0>(p, nb, grid_tiles, stream)
                                      : stream_nb<hsb::KIND_SCALAR, 1>(p, nb, grid_tiles, stream);
}

// Dense contiguous job in the reference layouts.
Job dense_job(int kind, int dir, int in_dtype, const void* in, void* out, const float* w0,
              const float* w1, long long B, long long K, long long L, long long M) {
  Job j = {};
  j.kind = kind;
  j.dir = dir;
  j.in_dtype = in_dtype;
  j.flags = 0;
  j.in = in;
  j.out = out;
  j.w0 = w0;
  j.w1 = w1;
  j.B = B;
  j.K = K;
  j.L = L;
  j.M = M;
  const long long P = kind == HOLYSHT_KIND_VECTOR ? 2 : 1;
  const long long in_rows = dir == HOLYSHT_DIR_FORWARD ? K : L;
  const long long out_rows = dir == HOLYSHT_DIR_FORWARD ? L : K;
  j.in_rs = M;
  j.in_ps = in_rows * M;
  j.in_bs = P * in_rows * M;
  j.out_rs = M;
  j.out_ps = out_rows * M;
  j.out_bs = P * out_rows * M;
  j.out_cols = M;
  j.w_ks = M;
  j.w_ls = K * M;
  j.w_mt = hsb::kMTile;
  j.nlon = 0;
  j.scale = 1.f;
  j.ksplit = 0;
  j.grouped = 0;
  j.m_off = 0;
  return j;
}

// ---- tcgen05 dense path: host side ----

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// 3-D fp32 tensor map (inner dim contiguous), 128-byte swizzle, zero OOB fill
bool make_map_3d(CUtensorMap* map, const void* base, unsigned long long d0, unsigned long long d1,
                 unsigned long long d2, unsigned box0, unsigned box1,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 4, d0 * d1 * 4};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

long long align256(long long v) { return (v + 255) & ~255LL; }

// Bytes of the dense path's scratch: the split spectrum Xt hi/lo [2][M][2B][S],
// the GEMM output D [M][R][2B] and, unless the caller passes a split table, the
// split table [2][M][R][S] (fp32 each); -1 when the size does not fit in 62
// bits (each product is checked factor by factor).
long long tc_workspace(long long B, long long R, long long S, long long M, bool split_table = true) {
  const long long lim = 1LL << 62;
  auto mul = [lim](long long a, long long b, long long* r) {
    return !__builtin_mul_overflow(a, b, r) && *r < lim;
  };
  long long a = 0, b = 0, c = 0;
  if (!mul(M, 2, &a) || !mul(a, B, &a) || !mul(a, S, &a) || !mul(a, 4, &a)) return -1;
  if (!mul(M, R, &b) || !mul(b, 2, &b) || !mul(b, B, &b) || !mul(b, 4, &b)) return -1;
  if (!mul(M, R, &c) || !mul(c, S, &c) || !mul(c, 4, &c)) return -1;
  const long long total = 2 * align256(a) + align256(b) + (split_table ? 2 * align256(c) : 0);
  return total < lim ? total : -1;
}

}  // namespace

// ---- longitude rFFT through cuFFT (loaded at run time) ----------------------
// The library does not link cuFFT: it opens libcufft.so.11 on first use,
// preferring a copy the process has already loaded (torch's), so both share one
// cuFFT.  Plans are cached per (device, rows, nlon) with auto-allocation off:
// every execution takes its work area from the caller, as torch's own rFFT
// does, so a plan may run on several streams at once.
namespace {
typedef int cufft_handle;
struct CufftApi {
  int (*create)(cufft_handle*) = nullptr;
  int (*set_auto_alloc)(cufft_handle, int) = nullptr;
  int (*make_plan_many)(cufft_handle, int, int*, int*, int, int, int*, int, int, int, int, size_t*) = nullptr;
  int (*set_stream)(cufft_handle, cudaStream_t) = nullptr;
  int (*set_work_area)(cufft_handle, void*) = nullptr;
  int (*exec_r2c)(cufft_handle, float*, float2*) = nullptr;
  bool ok = false;
};
constexpr int kCufftR2C = 0x2a;  // CUFFT_R2C

const CufftApi& cufft_api() {
  static CufftApi api = [] {
    CufftApi a;
    void* h = dlopen("libcufft.so.11", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libcufft.so.11", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libcufft.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.create = reinterpret_cast<decltype(a.create)>(dlsym(h, "cufftCreate"));
    a.set_auto_alloc = reinterpret_cast<decltype(a.set_auto_alloc)>(dlsym(h, "cufftSetAutoAllocation"));
    a.make_plan_many = reinterpret_cast<decltype(a.make_plan_many)>(dlsym(h, "cufftMakePlanMany"));
    a.set_stream = reinterpret_cast<decltype(a.set_stream)>(dlsym(h, "cufftSetStream"));
    a.set_work_area = reinterpret_cast<decltype(a.set_work_area)>(dlsym(h, "cufftSetWorkArea"));
    a.exec_r2c = reinterpret_cast<decltype(a.exec_r2c)>(dlsym(h, "cufftExecR2C"));
    a.ok = a.create && a.set_auto_alloc && a.make_plan_many && a.set_stream && a.set_work_area && a.exec_r2c;
    return a;
  }();
  return api;
}

struct RfftPlan {
  cufft_handle h;
  size_t work;
};
std::mutex g_fft_mu;
std::map<std::array<long long, 3>, RfftPlan> g_fft_plans;  // (device, rows, nlon)
constexpr size_t kMaxFftPlans = 64;  // plans live until exit (a plan in flight is never destroyed)

// plan for `rows` transforms of nlon points (contiguous rows in, rows of
// nlon/2+1 complex out) on the current device; call with g_fft_mu held
int rfft_plan(long long rows, long long nlon, RfftPlan* out) {
  const CufftApi& api = cufft_api();
  if (!api.ok) return fail(HOLYSHT_ERR_UNSUPPORTED, "libcufft.so.11 could not be loaded");
  int dev = 0;
  // cuFFT needs the device's context current on this thread; a thread that
  // has made no runtime call yet has none (cudaSetDevice makes the primary
  // context current)
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess)
    return fail(HOLYSHT_ERR_CUDA, "no current CUDA device");
  const std::array<long long, 3> key = {dev, rows, nlon};
  auto it = g_fft_plans.find(key);
  if (it != g_fft_plans.end()) {
    *out = it->second;
    return ok();
  }
  if (g_fft_plans.size() >= kMaxFftPlans) return fail(HOLYSHT_ERR_UNSUPPORTED, "too many rFFT shapes");
  RfftPlan p{};
  if (api.create(&p.h) != 0) return fail(HOLYSHT_ERR_CUDA, "cufftCreate failed");
  int n[1] = {(int)nlon};
  int onembed[1] = {(int)(nlon / 2 + 1)};
  if (api.set_auto_alloc(p.h, 0) != 0 ||
      api.make_plan_many(p.h, 1, n, n, 1, (int)nlon, onembed, 1, (int)(nlon / 2 + 1), kCufftR2C, (int)rows,
                         &p.work) != 0)
    return fail(HOLYSHT_ERR_CUDA, "cufftMakePlanMany failed for %lld x %lld", rows, nlon);
  g_fft_plans[key] = p;
  *out = p;
  return ok();
}
}  // namespace

extern "C" {

int holysht_legendre_dense_tc_workspace_ex(int direction, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                           int flags, int64_t* bytes) {
  if (!bytes) return fail(HOLYSHT_ERR_INVALID, "bytes pointer is null");
  if (direction != HOLYSHT_DIR_FORWARD && direction != HOLYSHT_DIR_INVERSE)
    return fail(HOLYSHT_ERR_INVALID, "unknown direction %d", direction);
  if (batch < 0 || nlat < 0 || lmax < 0 || mmax < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  const bool fwd = direction == HOLYSHT_DIR_FORWARD;
  const long long Mrows = mmax < lmax ? mmax : lmax;
  const long long need = tc_workspace(batch, fwd ? lmax : nlat, fwd ? nlat : lmax, Mrows,
                                      !(flags & HOLYSHT_FLAG_TABLE_SPLIT));
  if (need < 0) return fail(HOLYSHT_ERR_INVALID, "extents too large: the workspace size overflows");
  *bytes = need;
  return ok();
}

int holysht_legendre_dense_tc_split_table(const float* table, float* split, int64_t count, void* stream) {
  if (count < 0) return fail(HOLYSHT_ERR_INVALID, "negative count");
  if (count == 0) return ok();
  if (!table || !split) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  const long long blocks = std::min<long long>((count + 255) / 256, 148LL * 16);
  hsb::tc::split_tf32_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(table, split,
                                                                                             split + count, count);
  return check_launch("split_tf32");
}

int holysht_legendre_dense_tc_workspace(int direction, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                        int64_t* bytes) {
  if (!bytes) return fail(HOLYSHT_ERR_INVALID, "bytes pointer is null");
  if (direction != HOLYSHT_DIR_FORWARD && direction != HOLYSHT_DIR_INVERSE)
    return fail(HOLYSHT_ERR_INVALID, "unknown direction %d", direction);
  if (batch < 0 || nlat < 0 || lmax < 0 || mmax < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  const bool fwd = direction == HOLYSHT_DIR_FORWARD;
  const long long Mrows = mmax < lmax ? mmax : lmax;
  const long long need = tc_workspace(batch, fwd ? lmax : nlat, fwd ? nlat : lmax, Mrows);
  if (need < 0) return fail(HOLYSHT_ERR_INVALID, "extents too large: the workspace size overflows");
  *bytes = need;
  return ok();
}

int holysht_legendre_dense_tc(int direction, void* out, int64_t out_batch_stride, int64_t out_row_stride,
                              int64_t out_cols, const void* in, int64_t in_batch_stride, int64_t in_row_stride,
                              const float* table, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                              float scale, int flags, int64_t nlon, void* workspace, int64_t workspace_bytes,
                              void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (direction != HOLYSHT_DIR_FORWARD && direction != HOLYSHT_DIR_INVERSE)
    return fail(HOLYSHT_ERR_INVALID, "unknown direction %d", direction);
  if (flags & ~(HOLYSHT_FLAG_ROUND_BF16 | HOLYSHT_FLAG_IRFFT_PREP | HOLYSHT_FLAG_TABLE_SPLIT))
    return fail(HOLYSHT_ERR_INVALID, "unsupported flags 0x%x", flags);
  const bool fwd = direction == HOLYSHT_DIR_FORWARD;
  const bool presplit = (flags & HOLYSHT_FLAG_TABLE_SPLIT) != 0;
  const long long B = batch, K = nlat, L = lmax, M = mmax;
  if (B < 0 || K < 0 || L < 0 || M < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  if (out_cols < M) return fail(HOLYSHT_ERR_INVALID, "out_cols (%lld) < mmax (%lld)", (long long)out_cols, M);
  const long long R = fwd ? L : K, S = fwd ? K : L;
  if (B == 0 || R == 0 || out_cols == 0) return ok();
  if (!out || !in || !table || !workspace) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (S % 4 != 0 || S == 0)
    return fail(HOLYSHT_ERR_UNSUPPORTED, "tensor-core path needs the reduction extent to be a multiple of 4");
  if ((reinterpret_cast<uintptr_t>(table) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(HOLYSHT_ERR_INVALID, "table must be 16-byte and workspace 256-byte aligned");
  if (2 * B > (1LL << 30) || B > 65535 || !fits_int(K) || !fits_int(L) || !fits_int(M) || R > 65535 ||
      !fits_int(out_cols))
    return fail(HOLYSHT_ERR_INVALID, "extent out of range for the tensor-core path");
  if ((flags & HOLYSHT_FLAG_IRFFT_PREP) && (fwd || nlon <= 0 || out_cols > nlon / 2 + 1))
    return fail(HOLYSHT_ERR_INVALID, "irfft preparation is for the inverse with out_cols <= nlon/2+1");
  const long long Mrows = M < L ? M : L;
  const long long need = tc_workspace(B, R, S, Mrows, !presplit);
  if (need < 0 || workspace_bytes < need) return fail(HOLYSHT_ERR_INVALID, "workspace too small");
  if (in_row_stride < M || in_batch_stride < S * in_row_stride || out_row_stride < out_cols ||
      out_batch_stride < R * out_row_stride)
    return fail(HOLYSHT_ERR_INVALID, "input or output strides too small");
  const long long N = 2 * B;
  char* ws = static_cast<char*>(workspace);
  float* xt = reinterpret_cast<float*>(ws);
  float* xt_lo = reinterpret_cast<float*>(ws + align256(Mrows * N * S * 4));
  float* D = reinterpret_cast<float*>(ws + 2 * align256(Mrows * N * S * 4));
  const float* a_hi = table;
  const float* a_lo = table + M * R * S;  // a split table: [2][mmax][R][S]

  if (Mrows > 0) {  // input -> Xt [Mrows][2B][S], split into tf32 hi and residual lo
    if (!presplit) {  // split the table's first Mrows orders into the workspace
      float* t_hi = reinterpret_cast<float*>(ws + 2 * align256(Mrows * N * S * 4) + align256(Mrows * R * N * 4));
      float* t_lo = reinterpret_cast<float*>(reinterpret_cast<char*>(t_hi) + align256(Mrows * R * S * 4));
      const long long cnt = Mrows * R * S;
      const long long blocks = std::min<long long>((cnt + 255) / 256, 148LL * 16);
      hsb::tc::split_tf32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(table, t_hi, t_lo, cnt);
      if (int st = check_launch("split_tf32")) return st;
      a_hi = t_hi;
      a_lo = t_lo;
    }
    // kernels: 0 = split B in shared memory (default), 1 = pre-split B planes,
    // 2 = the first 8-warp kernel (HSB_TC_MODE selects; 1 and 2 for comparison)
    const int mode = env_int("HSB_TC_MODE", env_int("HSB_TC_LEGACY", 0) ? 2 : 1);
    dim3 grid((unsigned)((Mrows + 31) / 32), (unsigned)((S + 31) / 32), (unsigned)B), block(32, 8);
    hsb::tc::transpose_in_kernel<<<grid, block, 0, stream>>>(static_cast<const float2*>(in), xt,
                                                             mode == 0 ? nullptr : xt_lo, (int)B,
                                                             (int)S, (int)Mrows, in_batch_stride, in_row_stride,
                                                             scale, (flags & HOLYSHT_FLAG_ROUND_BF16) ? 1 : 0);
    if (int st = check_launch("transpose_in")) return st;
    // table: forward [M][L][K] (rows l, reduce k); inverse [M][K][L] (rows k, reduce l)
    // the warp-specialised kernel moves 16-wide k blocks (64-byte swizzle);
    // HSB_TC_LEGACY=1 runs the earlier 32-wide, 8-warp kernel
    const bool legacy = mode == 2;
    const unsigned bk = legacy ? hsb::tc::kBK : hsb::tc::kBK2;
    const CUtensorMapSwizzle sw = legacy ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap map_a, map_b, map_a_lo, map_b_lo;
    if (!make_map_3d(&map_a, a_hi, S, R, Mrows, bk, hsb::tc::kBM, sw) ||
        !make_map_3d(&map_a_lo, a_lo, S, R, Mrows, bk, hsb::tc::kBM, sw) ||
        !make_map_3d(&map_b, xt, S, N, Mrows, bk, hsb::tc::kBN, sw) ||
        !make_map_3d(&map_b_lo, xt_lo, S, N, Mrows, bk, hsb::tc::kBN, sw))
      return fail(HOLYSHT_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable or rejected the tensors");
    hsb::tc::DenseParams p;
    p.R = (int)R;
    p.S = (int)S;
    p.M = (int)Mrows;
    p.N = (int)N;
    p.inverse = fwd ? 0 : 1;
    p.n_nt = (int)((N + hsb::tc::kBN - 1) / hsb::tc::kBN);
    p.n_bands = (int)((R + hsb::tc::kBM - 1) / hsb::tc::kBM);
    p.D = D;
    long long tiles = 0;
    if (fwd) {
      for (int q = 0; q < p.n_bands; ++q) {
        const long long m_hi = std::min<long long>(Mrows, R - (long long)hsb::tc::kBM * q);
        const long long m_lo = std::max<long long>(0, R - (long long)hsb::tc::kBM * (q + 1));
        if (m_hi > m_lo) tiles += (m_hi - m_lo) * (q + 1) * p.n_nt;
      }
    } else {
      tiles = Mrows * p.n_bands * p.n_nt;
    }
    if (tiles > INT_MAX) return fail(HOLYSHT_ERR_INVALID, "too many tiles");
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
      if (cudaFuncSetAttribute(hsb::tc::dense_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               hsb::tc::kSmemBytes) != cudaSuccess ||
          cudaFuncSetAttribute(hsb::tc::dense_ws3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               hsb::tc::kWs3SmemBytes) != cudaSuccess ||
          cudaFuncSetAttribute(hsb::tc::dense_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               hsb::tc::kWsSmemBytes) != cudaSuccess)
        return fail(HOLYSHT_ERR_UNSUPPORTED, "cannot configure the tensor-core kernel");
      configured.fetch_or(bit);
    }
    if (tiles > 0) {
      if (legacy)
        hsb::tc::dense_tf32x3_kernel<<<(unsigned)tiles, hsb::tc::kThreads, hsb::tc::kSmemBytes, stream>>>(
            map_a, map_b, map_a_lo, map_b_lo, p);
      else if (mode == 1)
        hsb::tc::dense_ws_kernel<<<(unsigned)tiles, hsb::tc::kWsThreads, hsb::tc::kWsSmemBytes, stream>>>(
            map_a, map_b, map_a_lo, map_b_lo, p);
      else
        hsb::tc::dense_ws3_kernel<<<(unsigned)tiles, hsb::tc::kWsThreads, hsb::tc::kWs3SmemBytes, stream>>>(
            map_a, map_b, map_a_lo, map_b_lo, p);
      if (int st = check_launch("dense tcgen05 kernel")) return st;
    }
  }
  {  // D [Mrows][R][2B] -> out [B][R][out_cols]
    dim3 grid((unsigned)((out_cols + 31) / 32), (unsigned)((B + 31) / 32), (unsigned)R), block(32, 8);
    const int prep = (flags & HOLYSHT_FLAG_IRFFT_PREP) ? 1 : 0;
    const int nyq = (prep && nlon % 2 == 0) ? (int)(nlon / 2) : -1;
    hsb::tc::transpose_out_kernel<<<grid, block, 0, stream>>>(D, static_cast<float2*>(out), (int)B, (int)R,
                                                              (int)out_cols, (int)Mrows, out_batch_stride,
                                                              out_row_stride, fwd ? 1 : 0, prep, nyq);
    if (int st = check_launch("transpose_out")) return st;
  }
  return ok();
}

int holysht_legendre_forward_recurrence(void* out, const void* spec, int64_t spec_batch_stride,
                                        int64_t spec_row_stride, const float* seeds, const float* coef,
                                        const float* cos_theta, int64_t batch, int64_t nlat, int64_t lmax,
                                        int64_t mmax, float scale, void* stream) {
  return holysht_legendre_forward_recurrence_ex(out, spec, spec_batch_stride, spec_row_stride, seeds, coef,
                                                cos_theta, batch, nlat, lmax, mmax, scale, 0, stream);
}

int holysht_legendre_forward_recurrence_ex(void* out, const void* spec, int64_t spec_batch_stride,
                                           int64_t spec_row_stride, const float* seeds, const float* coef,
                                           const float* cos_theta, int64_t batch, int64_t nlat, int64_t lmax,
                                           int64_t mmax, float scale, int flags, void* stream) {
  const long long B = batch, K = nlat, L = lmax, M = mmax;
  if (B < 0 || K < 0 || L < 0 || M < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  if ((flags & ~(HOLYSHT_FLAG_EQUATORIAL_PARITY | HOLYSHT_FLAG_SEEDS_COMPACT)) != 0)
    return fail(HOLYSHT_ERR_INVALID, "unknown flag");
  if (B == 0 || L == 0 || M == 0) return ok();
  if (!out || !spec || !seeds || !coef || !cos_theta) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (K < 1 || !fits_int(B) || !fits_int(K) || !fits_int(L) || !fits_int(M) || (B + 3) / 4 > 65535)
    return fail(HOLYSHT_ERR_INVALID, "extent out of range");
  if (spec_row_stride < M || spec_batch_stride < K * spec_row_stride)
    return fail(HOLYSHT_ERR_INVALID, "spectrum strides too small");
  if ((reinterpret_cast<uintptr_t>(seeds) & 7) != 0) return fail(HOLYSHT_ERR_INVALID, "seeds must be 8-byte aligned");
  // the spectrum is copied and the output written as 8-byte complex values
  if ((reinterpret_cast<uintptr_t>(spec) & 7) || (reinterpret_cast<uintptr_t>(out) & 7))
    return fail(HOLYSHT_ERR_INVALID, "spec and out must be 8-byte aligned");
  hsb::rec::RecParams p;
  p.spec = static_cast<const float2*>(spec);
  p.sbs = spec_batch_stride;
  p.srs = spec_row_stride;
  p.seeds = seeds;
  p.coef = coef;
  p.x = cos_theta;
  p.out = static_cast<float2*>(out);
  p.B = (int)B;
  p.K = (int)K;
  p.L = (int)L;
  p.M = (int)M;
  p.nseg = (int)((L + hsb::rec::kSeg - 1) / hsb::rec::kSeg);
  p.scale = scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool par = (flags & HOLYSHT_FLAG_EQUATORIAL_PARITY) != 0;
  const int compact = (flags & HOLYSHT_FLAG_SEEDS_COMPACT) ? 1 : 0;
  if (env_int("HSB_REC_PAIR", 0) && !par && !compact) {
    // the earlier latitude-pair kernel (per-degree shuffle reductions), kept for comparison
    if (K > (long long)hsb::rec::kMaxWarps * 32 * 16)
      return fail(HOLYSHT_ERR_UNSUPPORTED, "the pair kernel supports nlat <= %d", hsb::rec::kMaxWarps * 32 * 16);
    const int kpt = K > 2048 ? 16 : 8;
    const int threads = (int)(((K + kpt - 1) / kpt + 31) / 32 * 32);
    const long long seg_blocks = (p.nseg + hsb::rec::kSegPerCta - 1) / hsb::rec::kSegPerCta;
    dim3 grid((unsigned)M, (unsigned)seg_blocks, (unsigned)((B + hsb::rec::kNB - 1) / hsb::rec::kNB));
    if (kpt == 8) hsb::rec::recurrence_forward_pair_kernel<8><<<grid, threads, 0, st>>>(p);
    else hsb::rec::recurrence_forward_pair_kernel<16><<<grid, threads, 0, st>>>(p);
    return check_launch("recurrence forward kernel");
  }
  // segment-per-thread kernel: degree block (16, or 8 for more resident warps)
  // and latitude chunks per item (warps per CTA)
  const int mlim = (int)std::min(M, L);
  const long long nsegs = hsb::rec::segs_before(mlim, (int)L);
  const int db = env_int("HSB_REC_DB", 16) == 8 ? 8 : 16;
  const int nkc = env_int("HSB_REC_NKC", 4);
  if (!fits_int(nsegs) || (nsegs + 31) / 32 * (16 / db) > 0x7fffffffLL)
    return fail(HOLYSHT_ERR_INVALID, "extent out of range");
  dim3 grid((unsigned)((nsegs + 31) / 32 * (16 / db)), (unsigned)((B + hsb::rec::kNB - 1) / hsb::rec::kNB));
  cudaError_t e;
  if (db == 16)
    e = par ? hsb::rec::launch_seg_forward<16, true>(p, nkc, grid, mlim, (int)nsegs, compact, st)
            : hsb::rec::launch_seg_forward<16, false>(p, nkc, grid, mlim, (int)nsegs, compact, st);
  else
    e = par ? hsb::rec::launch_seg_forward<8, true>(p, nkc, grid, mlim, (int)nsegs, compact, st)
            : hsb::rec::launch_seg_forward<8, false>(p, nkc, grid, mlim, (int)nsegs, compact, st);
  if (e != cudaSuccess) return fail(HOLYSHT_ERR_CUDA, "recurrence forward: %s", cudaGetErrorString(e));
  return check_launch("recurrence forward kernel");
}

int holysht_legendre_vector_forward_recurrence(void* out, const void* spec, int64_t spec_batch_stride,
                                               int64_t spec_comp_stride, int64_t spec_row_stride, const float* seeds,
                                               const float* coef, const float* cos_theta, int64_t batch,
                                               int64_t nlat, int64_t lmax, int64_t mmax, float scale, void* stream) {
  return holysht_legendre_vector_forward_recurrence_ex(out, spec, spec_batch_stride, spec_comp_stride,
                                                       spec_row_stride, seeds, coef, cos_theta, batch, nlat, lmax,
                                                       mmax, scale, 0, stream);
}

int holysht_legendre_vector_forward_recurrence_ex(void* out, const void* spec, int64_t spec_batch_stride,
                                                  int64_t spec_comp_stride, int64_t spec_row_stride,
                                                  const float* seeds, const float* coef, const float* cos_theta,
                                                  int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                                  float scale, int flags, void* stream) {
  const long long B = batch, K = nlat, L = lmax, M = mmax;
  if (B < 0 || K < 0 || L < 0 || M < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  if ((flags & ~(HOLYSHT_FLAG_EQUATORIAL_PARITY | HOLYSHT_FLAG_SEEDS_COMPACT)) != 0)
    return fail(HOLYSHT_ERR_INVALID, "unknown flag");
  if (B == 0 || L == 0 || M == 0) return ok();
  if (!out || !spec || !seeds || !coef || !cos_theta) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (K < 1 || !fits_int(B) || !fits_int(K) || !fits_int(L) || !fits_int(M) ||
      (B + hsb::rec::kNB - 1) / hsb::rec::kNB > 65535)
    return fail(HOLYSHT_ERR_INVALID, "extent out of range");
  if (spec_row_stride < M || spec_comp_stride < K * spec_row_stride || spec_batch_stride < 2 * spec_comp_stride)
    return fail(HOLYSHT_ERR_INVALID, "spectrum strides too small");
  if ((reinterpret_cast<uintptr_t>(seeds) & 15) != 0 || (reinterpret_cast<uintptr_t>(coef) & 15) != 0)
    return fail(HOLYSHT_ERR_INVALID, "seeds and coef must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(spec) & 7) || (reinterpret_cast<uintptr_t>(out) & 7))
    return fail(HOLYSHT_ERR_INVALID, "spec and out must be 8-byte aligned");
  hsb::rec::VecRecParams p;
  p.spec = static_cast<const float2*>(spec);
  p.sbs = spec_batch_stride;
  p.sps = spec_comp_stride;
  p.srs = spec_row_stride;
  p.seeds = seeds;
  p.coef = coef;
  p.x = cos_theta;
  p.out = static_cast<float2*>(out);
  p.B = (int)B;
  p.K = (int)K;
  p.L = (int)L;
  p.M = (int)M;
  p.nseg = (int)((L + hsb::rec::kSeg - 1) / hsb::rec::kSeg);
  p.scale = scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool par = (flags & HOLYSHT_FLAG_EQUATORIAL_PARITY) != 0;
  const int compact = (flags & HOLYSHT_FLAG_SEEDS_COMPACT) ? 1 : 0;
  if (env_int("HSB_REC_PAIR", 0) && !par && !compact) {
    // the earlier latitude-pair kernel (per-degree shuffle reductions), kept for comparison
    if (K > (long long)hsb::rec::kMaxWarps * 32 * 8)
      return fail(HOLYSHT_ERR_UNSUPPORTED, "the pair kernel supports nlat <= %d", hsb::rec::kMaxWarps * 32 * 8);
    const long long seg_blocks = (p.nseg + hsb::rec::kSegPerCta - 1) / hsb::rec::kSegPerCta;
    dim3 grid((unsigned)M, (unsigned)seg_blocks, (unsigned)((B + hsb::rec::kNB - 1) / hsb::rec::kNB));
    const int t8 = (int)(((K + 7) / 8 + 31) / 32 * 32);
    hsb::rec::recurrence_vector_forward_pair_kernel<8><<<grid, t8, 0, st>>>(p);
    return check_launch("recurrence_vector_forward");
  }
  const int mlim = (int)std::min(M, L);
  const long long nsegs = hsb::rec::segs_before(mlim, (int)L);
  const int nkc = env_int("HSB_REC_NKC", 4);
  if (!fits_int(nsegs) || (nsegs + 31) / 32 * 2 > 0x7fffffffLL) return fail(HOLYSHT_ERR_INVALID, "extent out of range");
  dim3 grid((unsigned)((nsegs + 31) / 32 * 2), (unsigned)((B + hsb::rec::kNB - 1) / hsb::rec::kNB));
  const cudaError_t e = par ? hsb::rec::launch_vseg_forward<true>(p, nkc, grid, mlim, (int)nsegs, compact, st)
                            : hsb::rec::launch_vseg_forward<false>(p, nkc, grid, mlim, (int)nsegs, compact, st);
  if (e != cudaSuccess) return fail(HOLYSHT_ERR_CUDA, "recurrence vector forward: %s", cudaGetErrorString(e));
  return check_launch("recurrence vector forward kernel");
}

int holysht_legendre_inverse_recurrence(void* out, int64_t out_batch_stride, int64_t out_row_stride,
                                        int64_t out_cols, const void* spec, int64_t spec_batch_stride,
                                        int64_t spec_row_stride, const float* seeds, const float* coef,
                                        const float* cos_theta, int64_t batch, int64_t nlat, int64_t lmax,
                                        int64_t mmax, float scale, int flags, int64_t nlon, void* stream) {
  const long long B = batch, K = nlat, L = lmax, M = mmax;
  if (B < 0 || K < 0 || L < 0 || M < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  if ((flags & ~(HOLYSHT_FLAG_EQUATORIAL_PARITY | HOLYSHT_FLAG_IRFFT_PREP)) != 0)
    return fail(HOLYSHT_ERR_INVALID, "unknown flag");
  if (out_cols < M) return fail(HOLYSHT_ERR_INVALID, "out_cols (%lld) < mmax (%lld)", (long long)out_cols, M);
  if (B == 0 || K == 0 || out_cols == 0) return ok();
  if (!out || !seeds || !coef || !cos_theta || (M > 0 && L > 0 && !spec)) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (!fits_int(B) || !fits_int(K) || !fits_int(L) || !fits_int(M) || !fits_int(out_cols) ||
      (B + hsb::rec::kNB - 1) / hsb::rec::kNB > 65535)
    return fail(HOLYSHT_ERR_INVALID, "extent out of range");
  if ((flags & HOLYSHT_FLAG_IRFFT_PREP) && (nlon <= 0 || out_cols > nlon / 2 + 1))
    return fail(HOLYSHT_ERR_INVALID, "irfft preparation needs out_cols <= nlon/2+1");
  if (spec_row_stride < M || spec_batch_stride < L * spec_row_stride || out_row_stride < out_cols ||
      out_batch_stride < K * out_row_stride)
    return fail(HOLYSHT_ERR_INVALID, "input or output strides too small");
  if ((reinterpret_cast<uintptr_t>(seeds) & 7) || (reinterpret_cast<uintptr_t>(coef) & 7))
    return fail(HOLYSHT_ERR_INVALID, "seeds and coef must be 8-byte aligned");
  // spec is copied and out written as 8-byte complex values
  if ((reinterpret_cast<uintptr_t>(spec) & 7) || (reinterpret_cast<uintptr_t>(out) & 7))
    return fail(HOLYSHT_ERR_INVALID, "spec and out must be 8-byte aligned");
  const bool par = (flags & HOLYSHT_FLAG_EQUATORIAL_PARITY) != 0;
  hsb::rec::RecInvParams p;
  p.spec = static_cast<const float2*>(spec);
  p.sbs = spec_batch_stride;
  p.srs = spec_row_stride;
  p.seeds = seeds;
  p.coef = coef;
  p.x = cos_theta;
  p.out = static_cast<float2*>(out);
  p.obs = out_batch_stride;
  p.ors = out_row_stride;
  p.B = (int)B;
  p.K = (int)K;
  p.L = (int)L;
  p.M = (int)M;
  p.nseg = (int)((L + hsb::rec::kInvSeg - 1) / hsb::rec::kInvSeg);
  p.out_cols = (int)out_cols;
  p.prep = (flags & HOLYSHT_FLAG_IRFFT_PREP) ? 1 : 0;
  p.nyq = (p.prep && nlon % 2 == 0) ? (int)(nlon / 2) : -1;
  p.scale = scale;
  const long long Kh = par ? (K + 1) / 2 : K;
  // x runs over (latitude tile, batch group) and y over the order blocks, so the
  // block scheduler issues every tile of the long low-order blocks first
  const long long ntile = (Kh + 63) / 64, ngroup = (B + hsb::rec::kNB - 1) / hsb::rec::kNB;
  const long long nblk = (out_cols + hsb::rec::kInvOrders - 1) / hsb::rec::kInvOrders;
  if (nblk > 65535) return fail(HOLYSHT_ERR_INVALID, "out_cols out of range");
  if (ntile * ngroup > 0x7fffffffLL) return fail(HOLYSHT_ERR_INVALID, "nlat x batch out of range");
  p.ntile = (int)ntile;
  dim3 grid((unsigned)(ntile * ngroup), (unsigned)nblk, 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (par) hsb::rec::recurrence_inverse_kernel<true><<<grid, hsb::rec::kInvOrders * 32, 0, st>>>(p);
  else hsb::rec::recurrence_inverse_kernel<false><<<grid, hsb::rec::kInvOrders * 32, 0, st>>>(p);
  return check_launch("recurrence inverse kernel");
}

int holysht_tc_error_word(unsigned* value) {
  if (!value) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  unsigned zero = 0;
  if (cudaMemcpyFromSymbol(value, hsb::tc::g_tc_error, sizeof(unsigned)) != cudaSuccess ||
      cudaMemcpyToSymbol(hsb::tc::g_tc_error, &zero, sizeof(unsigned)) != cudaSuccess)
    return fail(HOLYSHT_ERR_CUDA, "cannot read the tensor-core error word");
  return ok();
}


int holysht_stream_launch_plan(int kind, int direction, int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                               int64_t out_cols, int64_t m_offset, int ksplit, int sm_count, int* ks_out,
                               int* clusters_out, int* items_out) {
  if (!ks_out || !clusters_out || !items_out) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (kind != HOLYSHT_KIND_SCALAR && kind != HOLYSHT_KIND_VECTOR)
    return fail(HOLYSHT_ERR_INVALID, "the streaming kernel serves the SCALAR and VECTOR kinds");
  if (direction != HOLYSHT_DIR_FORWARD && direction != HOLYSHT_DIR_INVERSE)
    return fail(HOLYSHT_ERR_INVALID, "unknown direction %d", direction);
  if (batch <= 0 || nlat <= 0 || lmax <= 0 || mmax <= 0 || out_cols < mmax || !fits_int(batch) || !fits_int(nlat) ||
      !fits_int(lmax) || !fits_int(mmax) || !fits_int(out_cols))
    return fail(HOLYSHT_ERR_INVALID, "extents must be positive, fit the tile range, out_cols >= mmax");
  if (m_offset < 0 || m_offset % 32 != 0) return fail(HOLYSHT_ERR_INVALID, "m_offset must be a multiple of 32");
  if (ksplit != 0 && ksplit != 1 && ksplit != 2 && ksplit != 4 && ksplit != 8)
    return fail(HOLYSHT_ERR_INVALID, "ksplit must be 0, 1, 2, 4 or 8");
  Job j = {};
  j.kind = kind;
  j.dir = direction;
  j.B = batch;
  j.K = nlat;
  j.L = lmax;
  j.M = mmax;
  j.out_cols = out_cols;
  j.m_off = m_offset;
  j.ksplit = ksplit;
  const long long R = direction == HOLYSHT_DIR_FORWARD ? lmax : nlat;
  const long long S = direction == HOLYSHT_DIR_FORWARD ? nlat : lmax;
  int nb = 1;
  hsb::stream::Params p = make_stream_params(j, R, S, &nb);
  p.ks = ksplit;  // the environment override is a launch-time setting
  *items_out = p.n_compute * p.n_bg;
  if (p.n_compute == 0) {
    *ks_out = 1;
    *clusters_out = 0;
    return ok();
  }
  const int chunk = kind == HOLYSHT_KIND_VECTOR ? hsb::stream::Shape<hsb::KIND_VECTOR>::kChunk
                                                : hsb::stream::Shape<hsb::KIND_SCALAR>::kChunk;
  const std::pair<int, int> plan =
      choose_stream_grid(p, chunk, direction == HOLYSHT_DIR_FORWARD, sm_count > 0 ? sm_count : sm_count_of_current_device());
  *ks_out = plan.first;
  *clusters_out = plan.second;
  return ok();
}

int holysht_stream_error_word(unsigned* value) {
  if (!value) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  unsigned zero = 0;
  if (cudaMemcpyFromSymbol(value, hsb::stream::g_stream_error, sizeof(unsigned)) != cudaSuccess ||
      cudaMemcpyToSymbol(hsb::stream::g_stream_error, &zero, sizeof(unsigned)) != cudaSuccess)
    return fail(HOLYSHT_ERR_CUDA, "cannot read the streaming kernel's error word");
  return ok();
}

int holysht_peer_barrier(void* const* signal, int n_ranks, int rank, unsigned epoch, void* stream) {
  if (!signal) return fail(HOLYSHT_ERR_INVALID, "signal is null");
  if (n_ranks < 1 || n_ranks > 8 || rank < 0 || rank >= n_ranks)
    return fail(HOLYSHT_ERR_INVALID, "rank %d of %d ranks (1..8)", rank, n_ranks);
  if (epoch == 0) return fail(HOLYSHT_ERR_INVALID, "epoch starts at 1");
  hsb::peer::BarrierParams p = {};
  for (int q = 0; q < n_ranks; ++q) {
    if (!signal[q] || (reinterpret_cast<uintptr_t>(signal[q]) & 3))
      return fail(HOLYSHT_ERR_INVALID, "signal[%d] is null or misaligned", q);
    p.signal[q] = static_cast<unsigned*>(signal[q]);
  }
  p.n_ranks = n_ranks;
  p.rank = rank;
  p.epoch = epoch;
  hsb::peer::barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("peer_barrier");
}

int holysht_peer_error_word(unsigned* value) {
  if (!value) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  unsigned zero = 0;
  if (cudaMemcpyFromSymbol(value, hsb::peer::g_peer_error, sizeof(unsigned)) != cudaSuccess ||
      cudaMemcpyToSymbol(hsb::peer::g_peer_error, &zero, sizeof(unsigned)) != cudaSuccess)
    return fail(HOLYSHT_ERR_CUDA, "cannot read the peer barrier's error word");
  return ok();
}

int holysht_version(void) { return 100; }

const char* holysht_last_error(void) { return g_last_error.c_str(); }

int holysht_fused_legendre_forward(void* out, const void* in, const float* weight_t, int64_t batch,
                                   int64_t nlat, int64_t lmax, int64_t mmax, void* stream) {
  Job j = dense_job(HOLYSHT_KIND_SCALAR, HOLYSHT_DIR_FORWARD, HOLYSHT_DTYPE_C64, in, out, weight_t,
                    nullptr, batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

int holysht_fused_legendre_inverse(void* out, const void* in, const float* weight_t, int64_t batch,
                                   int64_t nlat, int64_t lmax, int64_t mmax, void* stream) {
  Job j = dense_job(HOLYSHT_KIND_SCALAR, HOLYSHT_DIR_INVERSE, HOLYSHT_DTYPE_C64, in, out, weight_t,
                    nullptr, batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

int holysht_fused_legendre_forward_real(float* out, const void* in, int in_dtype,
                                        const float* weight_t, int64_t batch, int64_t nlat,
                                        int64_t lmax, int64_t mmax, int backend_hint,
                                        void* stream) {
  if (backend_hint < HOLYSHT_BACKEND_AUTO || backend_hint > HOLYSHT_BACKEND_TC_BF16)
    return fail(HOLYSHT_ERR_INVALID, "unknown backend_hint %d", backend_hint);
  Job j = dense_job(HOLYSHT_KIND_REAL, HOLYSHT_DIR_FORWARD, in_dtype, in, out, weight_t, nullptr,
                    batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

int holysht_fused_legendre_inverse_real(float* out, const float* in, const float* weight_t,
                                        int64_t batch, int64_t nlat, int64_t lmax, int64_t mmax,
                                        void* stream) {
  Job j = dense_job(HOLYSHT_KIND_REAL, HOLYSHT_DIR_INVERSE, HOLYSHT_DTYPE_F32, in, out, weight_t,
                    nullptr, batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

int holysht_fused_vector_legendre_forward(void* out, const void* in, const float* w0_t,
                                          const float* w1_t, int64_t batch, int64_t nlat,
                                          int64_t lmax, int64_t mmax, int backend_hint,
                                          void* stream) {
  if (backend_hint < HOLYSHT_BACKEND_AUTO || backend_hint > HOLYSHT_BACKEND_TC_BF16)
    return fail(HOLYSHT_ERR_INVALID, "unknown backend_hint %d", backend_hint);
  Job j = dense_job(HOLYSHT_KIND_VECTOR, HOLYSHT_DIR_FORWARD, HOLYSHT_DTYPE_C64, in, out, w0_t,
                    w1_t, batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

int holysht_fused_vector_legendre_inverse(void* out, const void* in, const float* w0_t,
                                          const float* w1_t, int64_t batch, int64_t nlat,
                                          int64_t lmax, int64_t mmax, void* stream) {
  Job j = dense_job(HOLYSHT_KIND_VECTOR, HOLYSHT_DIR_INVERSE, HOLYSHT_DTYPE_C64, in, out, w0_t,
                    w1_t, batch, nlat, lmax, mmax);
  return run_job(j, static_cast<cudaStream_t>(stream));
}

namespace {
int contract_impl(const holysht_contract_desc* d, void* const* peers, int n_peers, long long col_off, void* mc,
                  void* stream);
}  // namespace

int holysht_legendre_contract(const holysht_contract_desc* desc, void* stream) {
  return contract_impl(desc, nullptr, 0, 0, nullptr, stream);
}

int holysht_rfft_workspace(int64_t rows, int64_t nlon, int64_t* bytes) {
  if (!bytes) return fail(HOLYSHT_ERR_INVALID, "bytes pointer is null");
  if (rows < 1 || nlon < 2 || !fits_int(rows) || !fits_int(nlon)) return fail(HOLYSHT_ERR_INVALID, "bad rFFT extents");
  std::lock_guard<std::mutex> g(g_fft_mu);
  RfftPlan p;
  if (int st = rfft_plan(rows, nlon, &p)) return st;
  *bytes = (int64_t)p.work;
  return ok();
}

int holysht_rfft_contract(const float* field, int64_t rows, int64_t nlon, void* spec, void* fft_work,
                          int64_t fft_work_bytes, const holysht_contract_desc* desc, void* stream) {
  if (!field || !spec || !desc) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  if (rows < 1 || nlon < 2 || !fits_int(rows) || !fits_int(nlon)) return fail(HOLYSHT_ERR_INVALID, "bad rFFT extents");
  if (desc->direction != HOLYSHT_DIR_FORWARD || desc->in_dtype != HOLYSHT_DTYPE_C64)
    return fail(HOLYSHT_ERR_INVALID, "the rFFT feeds a forward contraction of complex input");
  {
    std::lock_guard<std::mutex> g(g_fft_mu);
    RfftPlan p;
    if (int st = rfft_plan(rows, nlon, &p)) return st;
    if (p.work > 0 && (!fft_work || fft_work_bytes < (int64_t)p.work))
      return fail(HOLYSHT_ERR_INVALID, "rFFT work area of %lld bytes needed", (long long)p.work);
    const CufftApi& api = cufft_api();
    if (api.set_stream(p.h, static_cast<cudaStream_t>(stream)) != 0 ||
        (p.work > 0 && api.set_work_area(p.h, fft_work) != 0) ||
        api.exec_r2c(p.h, const_cast<float*>(field), static_cast<float2*>(spec)) != 0)
      return fail(HOLYSHT_ERR_CUDA, "cufftExecR2C failed");
  }
  holysht_contract_desc d = *desc;
  d.in = spec;
  return contract_impl(&d, nullptr, 0, 0, nullptr, stream);
}

int holysht_legendre_contract_peers(const holysht_contract_desc* desc, void* const* peer_out, int n_peers,
                                    int64_t out_col_offset, void* multicast_out, void* stream) {
  if (!desc) return fail(HOLYSHT_ERR_INVALID, "descriptor is null");
  if (n_peers < 1 || n_peers > 8) return fail(HOLYSHT_ERR_INVALID, "n_peers must be 1..8 (got %d)", n_peers);
  if (!peer_out) return fail(HOLYSHT_ERR_INVALID, "peer_out is null");
  for (int q = 0; q < n_peers; ++q)
    if (!peer_out[q]) return fail(HOLYSHT_ERR_INVALID, "peer_out[%d] is null", q);
  if (desc->table_layout != HOLYSHT_TABLE_GROUPED8)
    return fail(HOLYSHT_ERR_INVALID, "output to several GPUs needs the GROUPED8 table layout");
  if (out_col_offset < 0 || !fits_int(out_col_offset + desc->out_cols))
    return fail(HOLYSHT_ERR_INVALID, "out_col_offset out of range");
  if (multicast_out && (reinterpret_cast<uintptr_t>(multicast_out) & 7))
    return fail(HOLYSHT_ERR_INVALID, "multicast_out must be 8-byte aligned");
  return contract_impl(desc, peer_out, n_peers, out_col_offset, multicast_out, stream);
}

namespace {
int contract_impl(const holysht_contract_desc* d, void* const* peers, int n_peers, long long col_off, void* mc,
                  void* stream) {
  if (!d) return fail(HOLYSHT_ERR_INVALID, "descriptor is null");
  Job j = {};
  j.peers = peers;
  j.n_peers = n_peers;
  j.col_off = col_off;
  j.mc = mc;
  j.kind = d->kind;
  j.dir = d->direction;
  j.in_dtype = d->in_dtype;
  j.flags = d->flags;
  j.in = d->in;
  j.out = d->out;
  j.w0 = d->w0;
  j.w1 = d->w1;
  j.B = d->batch;
  j.K = d->nlat;
  j.L = d->lmax;
  j.M = d->mmax;
  j.in_bs = d->in_batch_stride;
  j.in_ps = d->in_comp_stride;
  j.in_rs = d->in_row_stride;
  j.out_bs = d->out_batch_stride;
  j.out_ps = d->out_comp_stride;
  j.out_rs = d->out_row_stride;
  j.out_cols = d->out_cols;
  j.w_ls = d->w_l_stride;
  j.w_ks = d->w_k_stride;
  j.w_mt = d->w_m_tile_stride ? d->w_m_tile_stride : hsb::kMTile;
  j.grouped = d->table_layout == HOLYSHT_TABLE_GROUPED;
  j.grouped8 = d->table_layout == HOLYSHT_TABLE_GROUPED8 || d->table_layout == HOLYSHT_TABLE_GROUPED8_PARITY;
  j.parity = d->table_layout == HOLYSHT_TABLE_GROUPED8_PARITY;
  j.m_off = d->m_offset;
  if (j.m_off < 0 || j.m_off % hsb::kMTile != 0 || !fits_int(j.m_off))
    return fail(HOLYSHT_ERR_INVALID, "m_offset must be a non-negative multiple of 32");
  if (d->table_layout != HOLYSHT_TABLE_STRIDED && d->table_layout != HOLYSHT_TABLE_GROUPED &&
      d->table_layout != HOLYSHT_TABLE_GROUPED8 && d->table_layout != HOLYSHT_TABLE_GROUPED8_PARITY)
    return fail(HOLYSHT_ERR_INVALID, "unknown table_layout %d", d->table_layout);
  j.nlon = d->nlon;
  j.scale = d->scale;
  j.ksplit = d->ksplit;
  if ((j.flags & HOLYSHT_FLAG_IRFFT_PREP) && (j.nlon <= 0 || j.out_cols > j.nlon / 2 + 1))
    return fail(HOLYSHT_ERR_INVALID, "irfft preparation needs nlon > 0 and out_cols <= nlon/2+1");
  return run_job(j, static_cast<cudaStream_t>(stream));
}
}  // namespace

int holysht_fused_vector_forward_pack_real(float* s0, float* s1, const void* in, int64_t batch,
                                           int64_t nlat, int64_t mmax, void* stream) {
  if (batch < 0 || nlat < 0 || mmax < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  const long long plane = (long long)nlat * mmax;
  if (batch == 0 || plane == 0) return ok();
  if (!s0 || !s1 || !in) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  const long long total = batch * plane;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  hsb::vector_pack_real_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      s0, s1, static_cast<const float2*>(in), (int)batch, plane);
  return check_launch("fused_vector_forward_pack_real");
}

int holysht_fused_vector_forward_recompose_real(void* out, const float* o0, const float* o1,
                                                int64_t batch, int64_t lmax, int64_t mmax,
                                                void* stream) {
  if (batch < 0 || lmax < 0 || mmax < 0) return fail(HOLYSHT_ERR_INVALID, "negative extent");
  const long long plane = (long long)lmax * mmax;
  if (batch == 0 || plane == 0) return ok();
  if (!out || !o0 || !o1) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  const long long total = batch * plane;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  hsb::vector_recompose_real_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<float2*>(out), o0, o1, (int)batch, plane);
  return check_launch("fused_vector_forward_recompose_real");
}

int holysht_sht_prepare_irfft(void* data, int64_t rows, int64_t width, int64_t mmax, int64_t nlon,
                              void* stream) {
  if (rows < 0 || width < 0 || mmax < 0 || nlon <= 0)
    return fail(HOLYSHT_ERR_INVALID, "invalid extents (rows=%lld width=%lld mmax=%lld nlon=%lld)",
                (long long)rows, (long long)width, (long long)mmax, (long long)nlon);
  if (width > INT_MAX) return fail(HOLYSHT_ERR_INVALID, "width too large");
  const long long total = rows * width;
  if (total == 0) return ok();
  if (!data) return fail(HOLYSHT_ERR_INVALID, "null pointer");
  const int nyq = (nlon % 2 == 0) ? (int)(nlon / 2) : -1;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  hsb::prepare_irfft_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<float2*>(data), rows, (int)width, (int)(mmax < width ? mmax : width), nyq);
  return check_launch("sht_prepare_irfft");
}

// ---------------------------------------------------------------------------
// Dense tensor-core contraction without any allocation.
//
// Some callers cannot allocate device memory themselves: code embedded in a
// host whose allocator owns all GPU memory (a raw cudaMalloc there would bypass
// its memory budget), or a latency-critical loop that must not pay for an
// allocation on every call, or a plugin loaded through a bare C ABI that was
// given no allocator.  For them the scratch the dense path needs (the
// transposed input and the GEMM output) lives in the static device array below.
// It has a fixed size of kNoAllocScratchBytes and occupies that much memory on
// every GPU that loads this library, until the process exits.
// ---------------------------------------------------------------------------

constexpr long long kNoAllocScratchBytes = 64LL << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
// Device address of the scratch array in the current device's context.  The
// host-side name of the array is not a device address.  It is looked up on
// every call (a cheap host-side query), so a context that was destroyed and
// re-created (cudaDeviceReset) never receives a stale address.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    return fail(HOLYSHT_ERR_CUDA, "cannot get the address of the built-in scratch: %s", cudaGetErrorString(e));
  }
  *out = p;
  return HOLYSHT_OK;
}
}  // namespace

int holysht_legendre_dense_tc_noalloc(int direction, void* out, int64_t out_batch_stride, int64_t out_row_stride,
                                      int64_t out_cols, const void* in, int64_t in_batch_stride,
                                      int64_t in_row_stride, const float* table, int64_t batch, int64_t nlat,
                                      int64_t lmax, int64_t mmax, float scale, int flags, int64_t nlon,
                                      void* stream) {
  int64_t need = 0;
  if (int st = holysht_legendre_dense_tc_workspace(direction, batch, nlat, lmax, mmax, &need)) return st;
  if (need > kNoAllocScratchBytes)
    return fail(HOLYSHT_ERR_INVALID,
                "problem needs %lld bytes of scratch but the built-in scratch holds %lld bytes (64 MiB); "
                "call holysht_legendre_dense_tc with a workspace instead",
                (long long)need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  return holysht_legendre_dense_tc(direction, out, out_batch_stride, out_row_stride, out_cols, in, in_batch_stride,
                                   in_row_stride, table, batch, nlat, lmax, mmax, scale, flags, nlon, scratch,
                                   kNoAllocScratchBytes, stream);
}

}  // extern "C"
