// fo_api.cu -- the extern "C" boundary of libb200fo.so (declared in include/b200fo.h):
// argument validation, TMA tensor-map encoding, config legality, kernel selection and
// the device status word.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/b200fo.h"
#include "fo_launch.cuh"
#include "fo_direct.cuh"

namespace {

thread_local std::string g_err;
thread_local int g_err_code = 0;
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_timeout_ns{2000000000ull};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  g_err_code = code;
  return code;
}

int ok() {
  g_err.clear();
  g_err_code = 0;
  return FO_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // legal under a capture
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaThreadExchangeStreamCaptureMode(&mode);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int* g_status[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};

struct DevInfo {
  int dev;
  int sms;
  int* status;
};

// The status word lives in this module's own device memory (zero at module load), so
// the first call on a device allocates and synchronises nothing: a first call made
// while the caller's stream is being captured into a CUDA graph stays legal.
__device__ int g_status_words[4];

int device_info(DevInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(FO_ENODEVICE, "no current CUDA device");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_status[dev] == nullptr) {
    // Attribute and symbol queries enqueue nothing; relaxed mode keeps them legal under
    // a global-mode capture on another thread's stream.
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    int major = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    void* st = nullptr;
    const cudaError_t e = major == 10 ? cudaGetSymbolAddress(&st, g_status_words) : cudaSuccess;
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (major != 10)
      return fail(FO_ENODEVICE, "device %d has compute capability %d.x; this library is built for sm_100a",
                  dev, major);
    if (e != cudaSuccess || st == nullptr)
      return fail(FO_ECUDA, "locating the device status word failed: %s", cudaGetErrorString(e));
    g_status[dev] = static_cast<int*>(st);
    g_sms[dev] = sms;
  }
  out->dev = dev;
  out->sms = g_sms[dev];
  out->status = g_status[dev];
  return FO_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int esize(int dt) { return dt == FO_DT_F32 ? 4 : 2; }
bool valid_dt(int dt) { return dt == FO_DT_F16 || dt == FO_DT_BF16 || dt == FO_DT_F32; }

CUtensorMapDataType tma_dt(int dt) {
  switch (dt) {
    case FO_DT_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case FO_DT_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

// 2-D row-major tensor [outer, inner] with row stride `row_bytes`, 128-byte swizzled
// boxes of box_inner x box_outer elements.  Out-of-range elements load as zero and are
// skipped by stores.
int make_tmap(CUtensorMap* m, int dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, const char* what,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(FO_ECUDA, "cuTensorMapEncodeTiled is unavailable in the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, tma_dt(dt), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FO_EINVAL, "tensor map for %s rejected by the driver (CUresult %d; dims %llu x %llu, row %llu B)",
                what, static_cast<int>(r), static_cast<unsigned long long>(outer),
                static_cast<unsigned long long>(inner), static_cast<unsigned long long>(row_bytes));
  return FO_OK;
}

PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // legal under a capture
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
    cudaThreadExchangeStreamCaptureMode(&mode);
  });
  return fn;
}

// im2col-mode map over x[n][h][w][c]: each load walks 128 consecutive filter-origin
// positions through the bounding box [-pad, dim - 1 + pad - (k - 1) * dil] of W, then
// H, then N (stepping by the conv stride) and fetches 64 channels per position.  Returns
// false when the driver rejects the geometry (the gather producer is used instead).
bool make_im2col_map(CUtensorMap* m, const FoConvDesc* d, uint32_t pixels) {
  auto fn = encode_im2col_fn();
  if (fn == nullptr) return false;
  const int lw = -d->pad, lh = -d->pad;
  const int uw = d->pad - (d->kw - 1) * d->dil, uh = d->pad - (d->kh - 1) * d->dil;
  if (lw < -128 || uw > 127 || uh > 127 || uw < -128 || uh < -128) return false;
  if ((d->kw - 1) * d->dil > 255 || (d->kh - 1) * d->dil > 255) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d->c), static_cast<cuuint64_t>(d->w),
                        static_cast<cuuint64_t>(d->h), static_cast<cuuint64_t>(d->n)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d->c) * 2, static_cast<cuuint64_t>(d->w) * d->c * 2,
                           static_cast<cuuint64_t>(d->h) * d->w * d->c * 2};
  int lower[2] = {lw, lh};
  int upper[2] = {uw, uh};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(d->stride), static_cast<cuuint32_t>(d->stride), 1};
  CUresult r = fn(m, tma_dt(d->in_dtype), 4, const_cast<void*>(d->x), dims, strides, lower, upper, 64, pixels, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool conv_gather_forced() {
  static const bool v = [] {
    const char* e = getenv("FO_CONV_GATHER");
    return e != nullptr && e[0] == '1';
  }();
  return v;
}

int check_cfg(int op, int out_dtype, const FoTileCfg* cfg, char* why, size_t why_len) {
  auto say = [&](const char* fmt, int v) {
    if (why != nullptr && why_len > 0) snprintf(why, why_len, fmt, v);
    return FO_EINVAL;
  };
  if (cfg == nullptr) return say("null config%d", 0);
  if (cfg->block_m != 128 && cfg->block_m != 256)
    return say("block_m must be 128 (one CTA) or 256 (a CTA pair, tcgen05 cta_group::2), got %d", cfg->block_m);
  if (cfg->block_m == 256 && cfg->block_n < 128) return say("CTA pairs (block_m 256) need block_n >= 128, got %d", cfg->block_n);
  if (cfg->block_n != 64 && cfg->block_n != 128 && cfg->block_n != 256)
    return say("block_n must be 64, 128 or 256, got %d", cfg->block_n);
  if (cfg->block_k != 64 && cfg->block_k != 128 && !(cfg->block_k == 192 && cfg->swap_ab == 2))
    return say("block_k must be 64 or 128 (one or two 128-byte swizzle rows per stage; 192, three filter taps "
               "per weight stage, for the direct conv), got %d", cfg->block_k);
  const int min_stages = op == 1 && cfg->swap_ab != 2 ? 3 : 2;
  if (cfg->stages < min_stages || cfg->stages > fo::kMaxStages)
    return say("stages out of range: %d", cfg->stages);
  if (cfg->group_m < 0) return say("group_m must be >= 0, got %d", cfg->group_m);
  if (cfg->swap_ab < 0 || cfg->swap_ab > 2) return say("swap_ab must be 0, 1 or 2 (direct conv), got %d", cfg->swap_ab);
  if (cfg->swap_ab && (op != 1 || cfg->block_m != 128 || cfg->block_n < 128))
    return say("swap_ab is a conv2d mode with block_m 128 and block_n >= 128 (block_n %d)", cfg->block_n);
  if (cfg->max_ctas < 0) return say("max_ctas must be >= 0, got %d", cfg->max_ctas);
  if (cfg->split_k < 0 || cfg->split_k > 16) return say("split_k must be 0 (automatic) .. 16, got %d", cfg->split_k);
  if (cfg->split_mode < 0 || cfg->split_mode > 2)
    return say("split_mode must be 0 (automatic), 1 (workspace) or 2 (cluster), got %d", cfg->split_mode);
  if (cfg->ln_mode < 0 || cfg->ln_mode > 3)
    return say("ln_mode must be 0 (automatic), 1 (two kernels), 2 (one kernel) or 3 (one kernel, slices held in "
               "TMEM), got %d", cfg->ln_mode);
  // (the direct conv's shared memory depends on the image width: fo_conv2d checks it)
  const int smem = fo::smem_bytes_for(cfg->block_n, cfg->stages, cfg->block_m == 256, cfg->block_k / 64);
  if (cfg->swap_ab != 2 && smem > 232448) return say("shared memory %d B exceeds the 227 KB per-block limit", smem);
  // TMEM: two fp32 accumulators of block_n columns each, <= 512 columns.
  if (2 * cfg->block_n > 512) return say("TMEM columns %d exceed 512", 2 * cfg->block_n);
  if (out_dtype < 0 || out_dtype > 2) return say("bad output dtype %d", out_dtype);
  return FO_OK;
}

int act_of(int epi, int* has_bias) {
  switch (epi) {
    case FO_EPI_NONE: *has_bias = 0; return fo::ACT_NONE;
    case FO_EPI_BIAS: *has_bias = 1; return fo::ACT_NONE;
    case FO_EPI_BIAS_RELU: *has_bias = 1; return fo::ACT_RELU;
    case FO_EPI_BIAS_GELU_TANH: *has_bias = 1; return fo::ACT_GELU_TANH;
    case FO_EPI_BIAS_GELU_ERF: *has_bias = 1; return fo::ACT_GELU_ERF;
    case FO_EPI_BIAS_LN: *has_bias = 1; return fo::ACT_NONE;
    case FO_EPI_RELU: *has_bias = 0; return fo::ACT_RELU;
    case FO_EPI_BIAS_RESIDUAL_LN: *has_bias = 1; return fo::ACT_NONE;
    case FO_EPI_BN: *has_bias = 0; return fo::ACT_NONE;
    case FO_EPI_BN_RELU: *has_bias = 0; return fo::ACT_RELU;
    case FO_EPI_BN_ADD_RELU: *has_bias = 0; return fo::ACT_RELU;
  }
  return -1;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Work split of a GEMM over `cap` persistent CTAs.  Whole tiles fill as many complete
// waves as they can; the tiles of a last, less than half-full wave (or of a problem with
// fewer tiles than CTAs) are split along K (`forced` 0) into the number of parts that
// minimises the measured cost of a split tile on B200:
//   parts x k-blocks-per-part x t_kb  +  (parts - 1) x bn x 512 B / 30 GB/s  +  2 us,
// where t_kb is one k-block of a 128 x bn tile (0.45 us x bn/256 / tensor rate of bn:
// 1, 0.66, 0.37 for 256, 128, 64; conv's im2col producer at 0.7 of that), the second
// term the last-arriving CTA reading the other parts' fp32 partials (about 30 GB/s per
// SM), the third the write -> fence -> atomic chain.  The parts must fit the idle CTAs
// (left x parts <= cap), at most 8.  forced = 1 never splits; forced = s >= 2 splits the
// last partial wave into s parts regardless of cost.
struct SplitPlan {
  int grid, num_units, dp_units, split, kb_per_part, split_tiles;
};

int best_split(int k_blocks, int max_split, int bn, bool conv) {
  const double rate = bn >= 256 ? 1.0 : bn >= 128 ? 0.66 : 0.37;
  const double t_kb = 0.45e-6 * (bn / 256.0) / rate / (conv ? 0.7 : 1.0);
  const double part_s = bn * 512.0 / 30e9;
  int best = 1;
  double best_t = k_blocks * t_kb;
  for (int s = 2; s <= max_split; ++s) {
    const int kbp = (k_blocks + s - 1) / s;
    const int parts = (k_blocks + kbp - 1) / kbp;
    const double t = kbp * t_kb + (parts - 1) * part_s + 2e-6;
    if (t < best_t) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

SplitPlan plan_split(int tiles, int k_blocks, int cap, bool allow, int forced = 0, int bn = 256, bool conv = false) {
  SplitPlan pl{tiles < cap ? tiles : cap, tiles, tiles, 1, k_blocks, 0};
  if (!allow || forced == 1 || k_blocks < 2 || tiles <= 0) return pl;
  const int full = tiles >= cap ? tiles / cap : 0;
  const int left = tiles - full * cap;
  if (left == 0) return pl;
  int split;
  if (forced >= 2) {
    split = forced < k_blocks ? forced : k_blocks;
  } else {
    if (2 * left > cap) return pl;
    int max_split = cap / left;
    if (max_split > 8) max_split = 8;
    if (max_split > k_blocks) max_split = k_blocks;
    split = best_split(k_blocks, max_split, bn, conv);
  }
  if (split < 2) return pl;
  const int kbp = (k_blocks + split - 1) / split;
  split = (k_blocks + kbp - 1) / kbp;  // no empty parts
  if (split < 2) return pl;
  pl.split = split;
  pl.kb_per_part = kbp;
  pl.split_tiles = left;
  pl.dp_units = full * cap;
  pl.num_units = pl.dp_units + left * split;
  pl.grid = pl.num_units < cap ? pl.num_units : cap;
  return pl;
}

// Cluster split of a single-CTA GEMM with fewer than half a wave of tiles: the s parts
// of each tile run as one cluster (s <= 8 CTAs, all co-resident) and reduce-scatter their
// fp32 partials through distributed shared memory, so a split costs no workspace, no
// global round trip and no fence / atomic chain.  Candidates are ranked by the cost
// fitted to B200 sweeps of single-wave problems (M = 64..512, K = 768..8192):
//   stages-per-part x kps x 0.30 us  +  c0(bn) + c1(bn) x s
// where 0.30 us is one 64-wide k-block of a 128-row tile whatever block_n (these tiles
// are bound by load latency, not by the tensor pipe), and (c0, c1) = (0.9, 0.32),
// (1.9, 0.5), (2.3, 1.1) us for block_n 64, 128, 256 is the cluster's start, the
// exchange of (s - 1) / s of the tile's fp32 partials and the exit (the exchanged bytes
// grow with block_n).  A split must beat the unsplit tile by 20%.  Every part holds at
// least one stage and the shared memory of a CTA (pipeline + receive area) must fit
// 227 KB: a part's short K loop needs no deep pipeline, so the stages drop (not below
// 2) until it does (cluster_stages).  forced = s >= 2 asks for exactly s parts.  Fills
// `cand` best first; returns how many (0: no cluster split).
int cluster_stages(int bn, int stages, int kps, int s) {
  while (stages > 2 && fo::smem_bytes_for(bn, stages, false, kps, s) > 232448) --stages;
  return fo::smem_bytes_for(bn, stages, false, kps, s) <= 232448 ? stages : 0;
}

int plan_cluster_split(int tiles, int k_blocks, int kps, int cap, int bn, int stages, int forced, int cand[8],
                       const char** why) {
  *why = nullptr;
  if (forced == 1) return 0;
  const int nst = (k_blocks + kps - 1) / kps;
  auto fits = [&](int s) {
    return s >= 2 && s <= 8 && tiles * s <= cap && s <= nst && cluster_stages(bn, stages, kps, s) > 0;
  };
  if (forced >= 2) {
    if (!fits(forced)) {
      *why = "cluster split needs parts <= 8, tiles x parts <= the CTA cap, a stage per part and the receive area "
             "to fit shared memory";
      return 0;
    }
    cand[0] = forced;
    return 1;
  }
  if (2 * tiles > cap || nst < 2) return 0;
  const double t_kb = 0.30e-6;
  const double c0 = bn >= 256 ? 2.3e-6 : bn >= 128 ? 1.9e-6 : 0.9e-6;
  const double c1 = bn >= 256 ? 1.1e-6 : bn >= 128 ? 0.5e-6 : 0.32e-6;
  const double t1 = k_blocks * t_kb;
  double cost[8];
  int n = 0;
  for (int s = 2; s <= 8; ++s) {
    if (!fits(s)) continue;
    const double t = (nst + s - 1) / s * kps * t_kb + c0 + c1 * s;
    if (t >= 0.8 * t1) continue;
    int k = n++;
    while (k > 0 && cost[k - 1] > t) {  // insertion: best first
      cost[k] = cost[k - 1];
      cand[k] = cand[k - 1];
      --k;
    }
    cost[k] = t;
    cand[k] = s;
  }
  return n;
}

// Counters (8 per slot: 4 row quarters x 2 column halves, one per epilogue warp) then
// fp32 partials, per 128-row slot of each split tile (`halves` slots per tile: 2 for
// CTA pairs).
size_t split_counter_bytes(const SplitPlan& pl, int halves) {
  return round_up(static_cast<size_t>(pl.split_tiles) * halves * 8 * sizeof(int), 256);
}

size_t split_workspace(const SplitPlan& pl, int bn, int halves = 1) {
  if (pl.split < 2) return 0;
  return split_counter_bytes(pl, halves) +
         static_cast<size_t>(pl.split_tiles) * halves * pl.split * 128 * bn * sizeof(float);
}

int sm_count_or_default() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      n > 0)
    return n;
  cudaGetLastError();
  return 148;
}

// LayerNorm workspace: the one-kernel path's counters (arrivals and finished
// normalisers per 32-row group, zero-filled, left zeroed), then the statistics: one
// float4 (two kernels) or float2 (one kernel) per row per slice, a slice being the
// column half of an N tile that one epilogue warp covers.
int ln_halves(int) { return 2; }

size_t ln_header_bytes(int64_t M) { return round_up(static_cast<size_t>((M + 31) / 32) * 2 * sizeof(int), 256); }

size_t ln_workspace(int64_t M, int64_t N, int bn) {
  const int64_t slices = (N + bn - 1) / bn * ln_halves(bn);
  return ln_header_bytes(M) + static_cast<size_t>(slices * M) * 16;
}

void fill_common(fo::KParams& p, const DevInfo& di) {
  p.status = di.status;
  p.timeout_ns = g_timeout_ns.load();

}

}  // namespace

void fo::set_last_error(int code, const char* msg) {
  g_err = msg != nullptr ? msg : "";
  g_err_code = code;
}

extern "C" {

const char* fo_version(void) { return "b200fo 0.2.0 sm_100a abi 2"; }

uint64_t fo_launch_count(void) { return g_launches.load(); }

int fo_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    strncpy(buf, g_err.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return g_err_code;
}

int fo_set_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) return fail(FO_EINVAL, "timeout must be > 0 ns");
  g_timeout_ns.store(ns);
  return ok();
}

size_t fo_config_smem_bytes(int32_t op, int32_t out_dtype, const FoTileCfg* cfg) {
  if (check_cfg(op, out_dtype, cfg, nullptr, 0) != FO_OK) return 0;
  return static_cast<size_t>(fo::smem_bytes_for(cfg->block_n, cfg->stages, cfg->block_m == 256, cfg->block_k / 64));
}

int fo_query_config_legal(int32_t op, int32_t out_dtype, const FoTileCfg* cfg, char* why,
                          size_t why_len) {
  if (why != nullptr && why_len > 0) why[0] = '\0';
  if (op != 0 && op != 1) {
    if (why != nullptr && why_len > 0) snprintf(why, why_len, "op must be 0 (gemm) or 1 (conv2d)");
    return FO_EINVAL;
  }
  return check_cfg(op, out_dtype, cfg, why, why_len);
}

size_t fo_gemm_workspace_size(const FoGemmDesc* d, const FoTileCfg* cfg) {
  if (d == nullptr || cfg == nullptr) return 0;
  if (cfg->block_n != 64 && cfg->block_n != 128 && cfg->block_n != 256) return 0;
  if (d->M <= 0 || d->N <= 0) return 0;
  if (d->epilogue == FO_EPI_BIAS_LN) return ln_workspace(d->M, d->N, cfg->block_n);
  // Other epilogues: room for the split-K tail (optional; without it there is no split).
  const int bn = cfg->block_n, bm = cfg->block_m, halves = bm / 128;
  const int tiles = static_cast<int>(((d->M + bm - 1) / bm) * ((d->N + bn - 1) / bn));
  const int sms = cfg->max_ctas > 0 ? cfg->max_ctas : sm_count_or_default();
  return split_workspace(plan_split(tiles, static_cast<int>((d->K + 63) / 64), sms / halves, true, cfg->split_k, bn), bn,
                         halves);
}

int fo_gemm(const FoGemmDesc* d, const FoTileCfg* cfg, void* stream) {
  if (d == nullptr) return fail(FO_EINVAL, "null descriptor");
  char why[256];
  if (check_cfg(0, d->out_dtype, cfg, why, sizeof(why)) != FO_OK) return fail(FO_EINVAL, "config: %s", why);
  if (d->M < 0 || d->N < 0 || d->K < 0) return fail(FO_EINVAL, "negative shape M=%lld N=%lld K=%lld",
                                                    (long long)d->M, (long long)d->N, (long long)d->K);
  if (d->M > (1ll << 31) - 1 || d->N > (1ll << 31) - 1 || d->K > (1ll << 31) - 1)
    return fail(FO_EINVAL, "shape exceeds 2^31-1");
  if (d->in_dtype != FO_DT_F16 && d->in_dtype != FO_DT_BF16)
    return fail(FO_EINVAL, "in_dtype must be FO_DT_F16 or FO_DT_BF16");
  if (!valid_dt(d->out_dtype)) return fail(FO_EINVAL, "bad out_dtype %d", d->out_dtype);
  if (d->b_layout != FO_B_KN && d->b_layout != FO_B_NK) return fail(FO_EINVAL, "bad b_layout %d", d->b_layout);
  int has_bias = 0;
  const int act = act_of(d->epilogue, &has_bias);
  if (act < 0 || d->epilogue == FO_EPI_BN || d->epilogue == FO_EPI_BN_RELU || d->epilogue == FO_EPI_BN_ADD_RELU)
    return fail(FO_EINVAL, "bad gemm epilogue %d", d->epilogue);
  const bool ln = d->epilogue == FO_EPI_BIAS_LN;
  const bool rln = d->epilogue == FO_EPI_BIAS_RESIDUAL_LN;
  if (has_bias && (d->bias == nullptr || !valid_dt(d->vec_dtype)))
    return fail(FO_EINVAL, "epilogue %d needs a bias vector and a valid vec_dtype", d->epilogue);
  if (d->M == 0 || d->N == 0) return ok();  // empty output: nothing to launch
  const int ib = 2, ob = esize(d->out_dtype);
  if (d->out == nullptr || !aligned16(d->out)) return fail(FO_EINVAL, "out must be a 16-byte aligned device pointer");
  if (d->ldo < d->N || (d->ldo * ob) % 16 != 0)
    return fail(FO_EINVAL, "ldo=%lld must be >= N=%lld and a multiple of %d elements (16-byte rows)",
                (long long)d->ldo, (long long)d->N, 16 / ob);
  if (d->K > 0) {
    if (d->a == nullptr || d->b == nullptr || !aligned16(d->a) || !aligned16(d->b))
      return fail(FO_EINVAL, "a and b must be 16-byte aligned device pointers");
    if (d->lda < d->K || (d->lda * ib) % 16 != 0)
      return fail(FO_EINVAL, "lda=%lld must be >= K=%lld and a multiple of 8 elements", (long long)d->lda,
                  (long long)d->K);
    const int64_t bmin = d->b_layout == FO_B_KN ? d->N : d->K;
    if (d->ldb < bmin || (d->ldb * ib) % 16 != 0)
      return fail(FO_EINVAL, "ldb=%lld must be >= %lld and a multiple of 8 elements", (long long)d->ldb,
                  (long long)bmin);
  }
  if (rln) {
    if (d->out_dtype == FO_DT_F32) return fail(FO_EINVAL, "LayerNorm output must be f16 or bf16");
    if (d->gamma == nullptr || d->beta == nullptr || !aligned16(d->gamma) || !aligned16(d->beta))
      return fail(FO_EINVAL, "LayerNorm needs 16-byte aligned gamma and beta");
    if (d->N % 8 != 0 || d->N > 4096)
      return fail(FO_EINVAL, "residual LayerNorm needs N %% 8 == 0 and N <= 4096, got N=%lld", (long long)d->N);
    if (d->residual == nullptr || !aligned16(d->residual) || d->ldr < d->N || (d->ldr * ob) % 16 != 0)
      return fail(FO_EINVAL, "residual must be a 16-byte aligned [M, N] tensor of the output dtype with ldr >= N");
    if (!(d->eps >= 0.0f)) return fail(FO_EINVAL, "eps must be >= 0");
  }
  if (ln) {
    if (d->out_dtype == FO_DT_F32) return fail(FO_EINVAL, "LayerNorm output must be f16 or bf16");
    if (d->gamma == nullptr || d->beta == nullptr) return fail(FO_EINVAL, "LayerNorm needs gamma and beta");
    if (!aligned16(d->gamma) || !aligned16(d->beta)) return fail(FO_EINVAL, "gamma and beta must be 16-byte aligned");
    if (d->N % 8 != 0) return fail(FO_EINVAL, "LayerNorm needs N %% 8 == 0, got N=%lld", (long long)d->N);
    const size_t need = ln_workspace(d->M, d->N, cfg->block_n);
    if (d->workspace == nullptr || d->workspace_bytes < need || !aligned16(d->workspace))
      return fail(FO_EINVAL, "LayerNorm needs a 16-byte aligned workspace of %zu bytes", need);
    if (!(d->eps >= 0.0f)) return fail(FO_EINVAL, "eps must be >= 0");
  }
  DevInfo di;
  if (int rc = device_info(&di)) return rc;

  fo::LaunchArgs la;
  memset(&la, 0, sizeof(la));
  fo::KParams& p = la.p;
  const int bn = cfg->block_n;
  p.M = static_cast<int>(d->M);
  p.N = static_cast<int>(d->N);
  p.K = static_cast<int>(d->K);
  const bool pair = cfg->block_m == 256;
  p.tiles_m = (p.M + cfg->block_m - 1) / cfg->block_m;
  p.tiles_n = (p.N + bn - 1) / bn;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (p.K + 63) / 64;
  p.group_m = cfg->group_m;
  p.stages = cfg->stages;
  p.ab_bf16 = d->in_dtype == FO_DT_BF16;
  p.b_mn = d->b_layout == FO_B_KN;
  p.has_bias = has_bias;
  p.bias = d->bias;
  p.gamma = d->gamma;
  p.beta = d->beta;
  p.vec_dtype = d->vec_dtype;
  p.eps = d->eps;
  p.out = d->out;
  p.ldo = d->ldo;
  p.residual = d->residual;
  p.ldr = d->ldr;
  if (ln) {
    char* ws = static_cast<char*>(d->workspace);
    p.ln_cnt = reinterpret_cast<int*>(ws);
    p.ln_groups = (p.M + 31) / 32;
    p.ln_stats = reinterpret_cast<float4*>(ws + ln_header_bytes(p.M));
    p.ln_st2 = reinterpret_cast<float2*>(ws + ln_header_bytes(p.M));
    // after the (mean, M2) slices, in the half of the statistics region they leave free
    p.ln_fin = p.ln_st2 + static_cast<size_t>(p.tiles_n) * ln_halves(bn) * p.M;
  }
  fill_common(p, di);

  if (p.K > 0) {
    if (int rc = make_tmap(&la.tmA, d->in_dtype, d->a, d->K, d->M, d->lda * ib, 64, 128, "A")) return rc;
    if (d->b_layout == FO_B_NK) {
      if (int rc = make_tmap(&la.tmB, d->in_dtype, d->b, d->K, d->N, d->ldb * ib, 64, pair ? bn / 2 : bn, "B"))
        return rc;
    } else {
      if (int rc = make_tmap(&la.tmB, d->in_dtype, d->b, d->N, d->K, d->ldb * ib, 64, 64, "B")) return rc;
    }
  }
  if (int rc = make_tmap(&la.tmC, d->out_dtype, d->out, d->N, d->M, d->ldo * ob, 128 / ob, 32, "out")) return rc;

  // Persistent grid: one CTA (or CTA pair) per SM (pair of SMs).
  const int cap = pair ? (cfg->max_ctas > 0 ? cfg->max_ctas / 2 : di.sms / 2) : (cfg->max_ctas > 0 ? cfg->max_ctas : di.sms);
  if (cap < 1) return fail(FO_EINVAL, "max_ctas too small for CTA pairs");
  p.kps = cfg->block_k / 64;
  la.pair = pair;
  la.stream = static_cast<cudaStream_t>(stream);
  const int out_dt = d->out_dtype == FO_DT_F16 ? fo::DT_F16 : d->out_dtype == FO_DT_BF16 ? fo::DT_BF16 : fo::DT_F32;
  auto launch = [&]() {
    return ln ? fo::launch_ln_family(bn, out_dt, la)
              : rln ? fo::launch_residual_ln(bn, out_dt, la)
                    : fo::launch_gemm_family(bn, act, out_dt, la);
  };
  cudaError_t e = cudaErrorNotReady;
  if (cfg->split_mode == 2 && (pair || ln))
    return fail(FO_EINVAL, "cluster split needs block_m 128 and an epilogue other than FO_EPI_BIAS_LN");
  // Cluster split first (automatic or asked for), then the workspace split / whole tiles.
  // A cluster size whose clusters do not all fit the GPU at once is skipped for the next.
  if (!pair && !ln && p.K > 0 && cfg->split_mode != 1) {
    const char* cwhy = nullptr;
    int cand[8];
    const int n = plan_cluster_split(p.num_tiles, p.k_blocks, p.kps, cap, bn, cfg->stages,
                                     cfg->split_mode == 2 ? (cfg->split_k >= 2 ? cfg->split_k : 0) : cfg->split_k,
                                     cand, &cwhy);
    if (cfg->split_mode == 2 && n == 0)
      return fail(FO_EINVAL, "cluster split not possible for this shape and config: %s",
                  cwhy != nullptr ? cwhy : "a whole wave of tiles or too few k-blocks (set split_k to force)");
    for (int i = 0; i < n; ++i) {
      const int s = cand[i];
      p.csplit = s;
      p.split = s;
      p.kb_per_part = 0;  // parts take ranges of stages (unit_of)
      p.dp_units = 0;
      p.num_units = p.num_tiles * s;
      la.csplit = s;
      la.grid = p.num_units;
      p.stages = cluster_stages(bn, cfg->stages, p.kps, s);
      la.smem = fo::smem_bytes_for(bn, p.stages, false, p.kps, s);
      e = launch();
      if (e != cudaErrorCooperativeLaunchTooLarge) break;
    }
    if (e == cudaErrorCooperativeLaunchTooLarge) {
      if (cfg->split_mode == 2)
        return fail(FO_EINVAL, "cluster split: %d clusters of %d CTAs do not fit the GPU at once", p.num_tiles,
                    cand[0]);
      p.csplit = 0;  // no size fits: plan without it
      la.csplit = 0;
      p.stages = cfg->stages;
    }
  }
  if (e == cudaErrorNotReady || e == cudaErrorCooperativeLaunchTooLarge) {
    SplitPlan pl = plan_split(p.num_tiles, p.k_blocks, cap, !ln, cfg->split_k, bn);
    const size_t split_need = split_workspace(pl, bn, pair ? 2 : 1);
    if (split_need == 0 || d->workspace == nullptr || d->workspace_bytes < split_need || !aligned16(d->workspace))
      pl = plan_split(p.num_tiles, p.k_blocks, cap, false);  // no room for partials: whole tiles only
    p.num_units = pl.num_units;
    p.dp_units = pl.dp_units;
    p.split = pl.split;
    p.kb_per_part = pl.kb_per_part;
    if (pl.split > 1) {
      p.split_cnt = static_cast<int*>(d->workspace);
      p.split_ws = reinterpret_cast<float*>(static_cast<char*>(d->workspace) + split_counter_bytes(pl, pair ? 2 : 1));
      p.tail_first = 1;
    }
    la.grid = pair ? 2 * pl.grid : pl.grid;
    la.smem = fo::smem_bytes_for(bn, cfg->stages, pair, p.kps);
    if (ln && cfg->ln_mode != 1) {
      // One kernel when the epilogue stages 128-byte chunks (block_n >= 128) and every
      // row block's tiles lie within kLnMaxDefer waves of units of the raster.
      const int span = p.group_m > 0 ? (p.group_m < p.tiles_m ? p.group_m : p.tiles_m) * (p.tiles_n - 1)
                                     : p.tiles_n - 1;
      const bool eligible = bn >= 128 && fo::ln_defer_for(span, pl.grid) <= fo::kLnMaxDefer;
      if (cfg->ln_mode == 2 && !eligible)
        return fail(FO_EINVAL, "one-kernel LayerNorm needs block_n >= 128 and each row block's %d tiles within %d "
                    "waves of the tile raster (use group_m 0 or ln_mode 1)", p.tiles_n, fo::kLnMaxDefer);
      // Held slices: a unit's epilogue waits for its row block's other tiles while it
      // holds its accumulator, which is cycle-free when those tiles lie within fewer
      // units of the raster than one wave has (span < units per wave).
      const bool held_ok = bn >= 128 && span < pl.grid;
      if (cfg->ln_mode == 3 && !held_ok)
        return fail(FO_EINVAL, "one-kernel LayerNorm with held slices needs block_n >= 128 and each row block's tiles "
                    "within %d units of the raster (span %d; use group_m 0, fewer column tiles or ln_mode 1)",
                    pl.grid - 1, span);
      // Automatic: one kernel from 16M outputs up.  Below that the row pass is short and
      // the one kernel's normalisation tail (wait, read-back, store after the last unit)
      // measured 3-9 us slower (B200: 2048 x 4096 +2.7 us; 16384 x 4096 -30 us).
      const bool large = static_cast<int64_t>(p.M) * p.N >= (int64_t{1} << 24);
      // Automatic, held slices: up to 4 waves of units, K >= 2048 and 4M outputs, where
      // they measured fastest (B200, 256 x 256 pair tiles: 8192 x 1024 x 4096 71.6 us vs
      // 74.8 two-kernel / 75.7 stored; 4096^3 123.4 vs 128.4 / 126.0).  With more waves a
      // late tile delays its row block's partners, and the delays add up from wave to
      // wave (16384 x 4096 x 4096: 422 vs 390 us stored).
      const int waves = (pl.num_units + pl.grid - 1) / pl.grid;
      const bool held_auto = held_ok && cfg->ln_mode == 0 && waves <= 4 && p.K >= 2048 &&
                             static_cast<int64_t>(p.M) * p.N >= (int64_t{1} << 22);
      if (cfg->ln_mode == 3 || held_auto || (eligible && (cfg->ln_mode == 2 || large))) {
        p.ln_fused = cfg->ln_mode == 3 || held_auto ? 2 : 1;
        p.ln_span = span;
        la.coop = true;
        e = launch();
        if (e != cudaSuccess && cfg->ln_mode >= 2)
          return fail(FO_ECUDA, "one-kernel LayerNorm launch failed: %s", cudaGetErrorString(e));
        if (e != cudaSuccess) {  // automatic: the two-kernel path instead
          cudaGetLastError();
          p.ln_fused = 0;
          p.ln_span = 0;
          la.coop = false;
        }
      }
    }
    if (!p.ln_fused) e = launch();
  }
  if (e != cudaSuccess) return fail(FO_ECUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  g_launches.fetch_add((ln && !p.ln_fused) || rln ? 2 : 1);  // two-kernel LayerNorm: GEMM + row kernel
  return ok();
}

// Tile grid of a conv call: (tiles, k_blocks, single-CTA?) as fo_conv2d lays it out when
// the TMA im2col path is available (the split tail needs whole-K producers per unit).
static bool conv_grid(const FoConvDesc* d, const FoTileCfg* cfg, int* tiles, int* k_blocks) {
  if (d == nullptr || cfg == nullptr || check_cfg(1, d->out_dtype, cfg, nullptr, 0) != FO_OK) return false;
  if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->f <= 0 || d->kh <= 0 || d->kw <= 0 || d->stride <= 0 ||
      d->dil <= 0 || d->pad < 0)
    return false;
  const int oh = (d->h + 2 * d->pad - d->dil * (d->kh - 1) - 1) / d->stride + 1;
  const int ow = (d->w + 2 * d->pad - d->dil * (d->kw - 1) - 1) / d->stride + 1;
  if (oh <= 0 || ow <= 0) return false;
  const int64_t M = static_cast<int64_t>(d->n) * oh * ow;
  if (cfg->block_m == 256 || cfg->swap_ab == 2) return false;  // CTA pairs and the direct conv run whole tiles
  const int bn = cfg->block_n;
  if (cfg->swap_ab)
    *tiles = static_cast<int>(((d->f + 127) / 128) * ((M + bn - 1) / bn));
  else
    *tiles = static_cast<int>(((M + 127) / 128) * ((d->f + bn - 1) / bn));
  *k_blocks = d->kh * d->kw * ((d->c + 63) / 64);
  return true;
}

extern "C" size_t fo_conv2d_workspace_size(const FoConvDesc* d, const FoTileCfg* cfg) {
  int tiles = 0, kb = 0;
  if (!conv_grid(d, cfg, &tiles, &kb)) return 0;
  const int cap = cfg->max_ctas > 0 ? cfg->max_ctas : sm_count_or_default();
  return split_workspace(plan_split(tiles, kb, cap, true, cfg->split_k, cfg->block_n, true), cfg->block_n);
}

// Geometry of the direct conv (swap_ab 2): pitch P of the padded rows (W + 2 pad rounded
// up to 32), output rows per tile (rpt: BN = rpt * P <= block_n positions), rows per pixel
// slot, and how many slots fit beside `stages` weight stages.  rpt minimises the time of
// the busiest SM, ceil(tiles / sms) x (max(BN, 240) + 32) in positions: a tile's MMAs
// (128 x BN x 16) cost BN / 2 tensor cycles each, but no less than the ~130 cycles the
// issuing thread needs per MMA, and 32 is a tile's fixed cost.  Ties go to taller tiles;
// e.g. 28 x 28 with P = 32 takes 7-row tiles (4 per image, 224 positions) over 8-row
// ones that would compute 32 rows per 28.  Returns false (with the reason) when the
// shape does not qualify.
struct DirectPlan {
  int P, Hp, nR, pslots, smem, rpt, tpi;
};

bool plan_direct(const FoConvDesc* d, int stages, int kps, int block_n, int sms, DirectPlan* pl, char* why,
                 size_t n) {
  auto no = [&](const char* msg) {
    snprintf(why, n, "%s", msg);
    return false;
  };
  if (d->stride != 1 || d->dil != 1) return no("the direct conv needs stride 1 and dilation 1");
  if (d->c % 64 != 0) return no("the direct conv needs C % 64 == 0");
  const int wp = d->w + 2 * d->pad;
  const int P = (wp + 31) / 32 * 32;
  if (P > block_n) {
    snprintf(why, n, "the direct conv needs W + 2 pad, rounded up to 32, <= %d (block_n)", block_n);
    return false;
  }
  if (d->kw - 1 >= P) return no("filter wider than the padded row");
  const int oh = d->h + 2 * d->pad - d->kh + 1;
  if (oh <= 0) return no("the filter is taller than the padded image");
  pl->P = P;
  pl->Hp = d->h + 2 * d->pad;
  const long long tiles_m = (d->f + 127) / 128;
  long long best = -1;
  for (int rpt = 1; rpt * P <= block_n; ++rpt) {
    const long long tiles = static_cast<long long>(d->n) * ((oh + rpt - 1) / rpt) * tiles_m;
    const long long cost = (tiles + sms - 1) / sms * ((rpt * P > 240 ? rpt * P : 240) + 32);
    if (best < 0 || cost <= best) {
      best = cost;
      pl->rpt = rpt;
    }
  }
  pl->tpi = (oh + pl->rpt - 1) / pl->rpt;
  const int bn = pl->rpt * P;
  pl->nR = (bn - 1 + (d->kh - 1) * P + d->kw - 1) / P + 1;
  const int slot = pl->nR * P * 128;
  for (int slots = 2; slots >= 1; --slots) {
    const int smem = fo::direct_smem_bytes(stages, slots, slot, kps);
    if (smem <= 232448) {
      pl->pslots = slots;
      pl->smem = smem;
      return true;
    }
  }
  return no("the direct conv's input rows and weight stages exceed 227 KB of shared memory; use fewer stages");
}

int make_tmap_4d(CUtensorMap* m, int dt, const void* base, const cuuint64_t (&dims)[4], const cuuint64_t (&strides)[3],
                 const cuuint32_t (&box)[4], CUtensorMapSwizzle swizzle, const char* what) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(FO_ECUDA, "cuTensorMapEncodeTiled is unavailable in the driver");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, tma_dt(dt), 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FO_EINVAL, "tensor map for %s rejected by the driver (CUresult %d)", what, static_cast<int>(r));
  return FO_OK;
}

int fo_conv2d(const FoConvDesc* d, const FoTileCfg* cfg, void* stream) {
  if (d == nullptr) return fail(FO_EINVAL, "null descriptor");
  char why[256];
  if (check_cfg(1, d->out_dtype, cfg, why, sizeof(why)) != FO_OK) return fail(FO_EINVAL, "config: %s", why);
  if (d->n < 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->f <= 0 || d->kh <= 0 || d->kw <= 0 ||
      d->stride <= 0 || d->pad < 0 || d->dil <= 0)
    return fail(FO_EINVAL, "bad conv geometry");
  if (d->in_dtype != FO_DT_F16 && d->in_dtype != FO_DT_BF16)
    return fail(FO_EINVAL, "in_dtype must be FO_DT_F16 or FO_DT_BF16");
  if (!valid_dt(d->out_dtype)) return fail(FO_EINVAL, "bad out_dtype %d", d->out_dtype);
  int has_bias = 0;
  const int act = act_of(d->epilogue, &has_bias);
  const bool bn_epi = d->epilogue == FO_EPI_BN || d->epilogue == FO_EPI_BN_RELU || d->epilogue == FO_EPI_BN_ADD_RELU;
  if (act < 0 || (act != fo::ACT_NONE && act != fo::ACT_RELU) || d->epilogue == FO_EPI_BIAS_LN ||
      d->epilogue == FO_EPI_BIAS_RESIDUAL_LN)
    return fail(FO_EINVAL, "conv2d epilogue must be NONE, BIAS, RELU, BIAS_RELU, BN, BN_RELU or BN_ADD_RELU");
  if (has_bias && (d->bias == nullptr || !valid_dt(d->vec_dtype)))
    return fail(FO_EINVAL, "conv2d bias epilogue needs a bias vector and a valid vec_dtype");
  if (bn_epi) {
    if (d->bn_gamma == nullptr || d->bn_beta == nullptr || d->bn_mean == nullptr || d->bn_var == nullptr ||
        !valid_dt(d->vec_dtype))
      return fail(FO_EINVAL, "BatchNorm epilogues need bn_gamma, bn_beta, bn_mean, bn_var and a valid vec_dtype");
    if (!(d->bn_eps >= 0.0f)) return fail(FO_EINVAL, "bn_eps must be >= 0");
  }
  if (d->epilogue == FO_EPI_BN_ADD_RELU) {
    if (d->out_dtype == FO_DT_F32) return fail(FO_EINVAL, "BN_ADD_RELU needs an f16 or bf16 output and residual");
    if (d->residual == nullptr || !aligned16(d->residual))
      return fail(FO_EINVAL, "BN_ADD_RELU needs a 16-byte aligned residual [n, oh, ow, f] of the output dtype");
  }
  const int oh = (d->h + 2 * d->pad - d->dil * (d->kh - 1) - 1) / d->stride + 1;
  const int ow = (d->w + 2 * d->pad - d->dil * (d->kw - 1) - 1) / d->stride + 1;
  if (oh <= 0 || ow <= 0) return fail(FO_EINVAL, "conv output is empty (oh=%d ow=%d)", oh, ow);
  if (d->c % 8 != 0) return fail(FO_EINVAL, "conv2d needs C %% 8 == 0 (16-byte channel chunks), got C=%d", d->c);
  const int ob = esize(d->out_dtype);
  if ((static_cast<int64_t>(d->f) * ob) % 16 != 0 || d->f % 8 != 0)
    return fail(FO_EINVAL, "conv2d needs F %% 8 == 0, got F=%d", d->f);
  const int64_t M64 = static_cast<int64_t>(d->n) * oh * ow;
  const int64_t K64 = static_cast<int64_t>(d->kh) * d->kw * d->c;
  const int64_t xelems = static_cast<int64_t>(d->n) * d->h * d->w * d->c;
  if (M64 > (1ll << 31) - 1 || xelems > (1ll << 40)) return fail(FO_EINVAL, "conv problem too large");
  if (M64 == 0) return ok();
  if (cfg->block_k != 64 && cfg->swap_ab != 2)
    return fail(FO_EINVAL, "conv2d stages one 64-wide K slice: block_k must be 64, got %d", cfg->block_k);
  if (d->x == nullptr || d->wgt == nullptr || d->out == nullptr || !aligned16(d->x) || !aligned16(d->wgt) ||
      !aligned16(d->out))
    return fail(FO_EINVAL, "x, wgt and out must be 16-byte aligned device pointers");
  DevInfo di;
  if (int rc = device_info(&di)) return rc;

  fo::LaunchArgs la;
  memset(&la, 0, sizeof(la));
  fo::KParams& p = la.p;
  const int bn = cfg->block_n;
  p.M = static_cast<int>(M64);
  p.N = d->f;
  p.K = static_cast<int>(K64);
  // CTA pairs need the TMA im2col producer; without it the conv runs as single CTAs.
  bool pair = cfg->block_m == 256;
  bool swap = cfg->swap_ab == 1;
  p.c_blocks = (d->c + 63) / 64;
  p.k_blocks = d->kh * d->kw * p.c_blocks;
  p.group_m = cfg->group_m;
  p.stages = cfg->stages;
  p.ab_bf16 = d->in_dtype == FO_DT_BF16;
  p.b_mn = 1;
  p.has_bias = has_bias;
  p.bias = d->bias;
  p.vec_dtype = d->vec_dtype;
  if (bn_epi) {
    p.bn_mode = d->epilogue == FO_EPI_BN_ADD_RELU ? 2 : 1;  // the reference clamps var there only
    p.bn_eps = d->bn_eps;
    p.bn_gamma = d->bn_gamma;
    p.bn_beta = d->bn_beta;
    p.bn_mean = d->bn_mean;
    p.bn_var = d->bn_var;
  }
  if (d->epilogue == FO_EPI_BN_ADD_RELU) {
    p.add_src = d->residual;
    p.ld_add = d->f;
  }
  p.out = d->out;
  p.ldo = d->f;
  p.x = d->x;
  p.H = d->h;
  p.W = d->w;
  p.C = d->c;
  p.OH = oh;
  p.OW = ow;
  p.KH = d->kh;
  p.KW = d->kw;
  p.stride = d->stride;
  p.pad = d->pad;
  p.dil = d->dil;
  fill_common(p, di);
  if (cfg->swap_ab == 2) {
    // direct conv: one 4-D box per padded input row, 4-D output boxes of 32 x 32
    DirectPlan dp;
    char why[160];
    const int ctas = cfg->max_ctas > 0 && cfg->max_ctas < di.sms ? cfg->max_ctas : di.sms;
    if (!plan_direct(d, cfg->stages, cfg->block_k / 64, cfg->block_n, ctas, &dp, why, sizeof(why)))
      return fail(FO_EINVAL, "%s", why);
    p.kps = cfg->block_k / 64;  // filter taps per weight stage
    p.P = dp.P;
    p.Hp = dp.Hp;
    p.nR = dp.nR;
    p.pslots = dp.pslots;
    p.nimg = d->n;
    p.rpt = dp.rpt;
    p.tpi = dp.tpi;
    p.c_blocks = d->c / 64;
    p.tiles_m = (p.N + 127) / 128;
    p.tiles_n = d->n * dp.tpi;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.num_units = p.num_tiles;
    p.dp_units = p.num_tiles;
    p.split = 1;
    const cuuint64_t xd[4] = {static_cast<cuuint64_t>(d->c), static_cast<cuuint64_t>(d->w),
                              static_cast<cuuint64_t>(d->h), static_cast<cuuint64_t>(d->n)};
    const cuuint64_t xs[3] = {static_cast<cuuint64_t>(d->c) * 2, static_cast<cuuint64_t>(d->w) * d->c * 2,
                              static_cast<cuuint64_t>(d->h) * d->w * d->c * 2};
    const cuuint32_t xb[4] = {64, static_cast<cuuint32_t>(dp.P), 1, 1};
    if (int rc = make_tmap_4d(&la.tmA, d->in_dtype, d->x, xd, xs, xb, CU_TENSOR_MAP_SWIZZLE_128B, "input rows")) return rc;
    if (int rc = make_tmap(&la.tmB, d->in_dtype, d->wgt, d->f, K64, static_cast<uint64_t>(d->f) * 2, 64, 64, "weights"))
      return rc;
    const cuuint64_t yd[4] = {static_cast<cuuint64_t>(d->f), static_cast<cuuint64_t>(ow), static_cast<cuuint64_t>(oh),
                              static_cast<cuuint64_t>(d->n)};
    const cuuint64_t ys[3] = {static_cast<cuuint64_t>(d->f) * ob, static_cast<cuuint64_t>(ow) * d->f * ob,
                              static_cast<cuuint64_t>(oh) * ow * d->f * ob};
    const cuuint32_t yb[4] = {32, 32, 1, 1};
    if (int rc = make_tmap_4d(&la.tmC, d->out_dtype, d->out, yd, ys, yb, CU_TENSOR_MAP_SWIZZLE_NONE, "output")) return rc;
    const int cap = cfg->max_ctas > 0 ? cfg->max_ctas : di.sms;
    la.grid = p.num_units < cap ? p.num_units : cap;
    la.smem = dp.smem;
    la.stream = static_cast<cudaStream_t>(stream);
    const int out_dt = d->out_dtype == FO_DT_F16 ? fo::DT_F16 : d->out_dtype == FO_DT_BF16 ? fo::DT_BF16 : fo::DT_F32;
    cudaError_t e = fo::launch_direct_conv(act, out_dt, la);
    if (e != cudaSuccess) return fail(FO_ECUDA, "kernel launch failed: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1);
    return ok();
  }
  p.conv_tma = (d->stride <= 8 && !conv_gather_forced() && make_im2col_map(&la.tmA, d, swap ? bn : 128)) ? 1 : 0;
  if (!p.conv_tma) pair = swap = false;  // both need the TMA im2col producer
  if (swap) {
    // M: output channels in blocks of 128; N: output pixels in blocks of block_n
    p.tiles_m = (p.N + 127) / 128;
    p.tiles_n = (p.M + bn - 1) / bn;
  } else {
    const int tile_m = pair ? 256 : 128;
    p.tiles_m = (p.M + tile_m - 1) / tile_m;
    p.tiles_n = (p.N + bn - 1) / bn;
  }
  p.num_tiles = p.tiles_m * p.tiles_n;
  if (int rc = make_tmap(&la.tmB, d->in_dtype, d->wgt, d->f, K64, static_cast<uint64_t>(d->f) * 2, 64, 64, "weights"))
    return rc;
  if (swap) {  // 32 channels x 32 pixels per store, unswizzled
    if (int rc = make_tmap(&la.tmC, d->out_dtype, d->out, d->f, M64, static_cast<uint64_t>(d->f) * ob, 32, 32, "out",
                           CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else if (int rc = make_tmap(&la.tmC, d->out_dtype, d->out, d->f, M64, static_cast<uint64_t>(d->f) * ob, 128 / ob,
                                32, "out")) {
    return rc;
  }
  const int cap = pair ? (cfg->max_ctas > 0 ? cfg->max_ctas / 2 : di.sms / 2) : (cfg->max_ctas > 0 ? cfg->max_ctas : di.sms);
  if (cap < 1) return fail(FO_EINVAL, "max_ctas too small for CTA pairs");
  la.pair = pair;
  la.swap = swap;
  SplitPlan pl = plan_split(p.num_tiles, p.k_blocks, cap, !pair && p.conv_tma, cfg->split_k, bn, true);
  const size_t split_need = split_workspace(pl, bn);
  if (split_need == 0 || d->workspace == nullptr || d->workspace_bytes < split_need || !aligned16(d->workspace))
    pl = plan_split(p.num_tiles, p.k_blocks, cap, false);
  p.num_units = pl.num_units;
  p.dp_units = pl.dp_units;
  p.split = pl.split;
  p.kb_per_part = pl.kb_per_part;
  if (pl.split > 1) {
    p.split_cnt = static_cast<int*>(d->workspace);
    p.split_ws = reinterpret_cast<float*>(static_cast<char*>(d->workspace) +
                                          split_counter_bytes(pl, 1));
    p.tail_first = 1;
  }
  la.grid = pl.grid * (pair ? 2 : 1);
  p.kps = 1;  // conv kernels stage one K slice (block_k 128 is a GEMM-family option)
  la.smem = fo::smem_bytes_for(bn, cfg->stages, pair, p.kps);
  la.stream = static_cast<cudaStream_t>(stream);
  const int out_dt = d->out_dtype == FO_DT_F16 ? fo::DT_F16 : d->out_dtype == FO_DT_BF16 ? fo::DT_BF16 : fo::DT_F32;
  cudaError_t e = fo::launch_conv_family(bn, act, out_dt, la);
  if (e != cudaSuccess) return fail(FO_ECUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1);
  return ok();
}

int fo_device_status(int32_t device, int32_t clear, int32_t* where) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(FO_ENODEVICE, "no CUDA device");
  if (device < 0 || device >= kMaxDevices) return fail(FO_EINVAL, "bad device %d", device);
  int* st = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    st = g_status[device];
  }
  if (where != nullptr) *where = 0;
  if (st == nullptr) return 0;  // nothing launched on this device yet
  if (prev != device) cudaSetDevice(device);
  int h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(h, st, sizeof(h), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(st, 0, sizeof(h));
  if (e == cudaSuccess && clear) e = cudaDeviceSynchronize();
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(FO_ECUDA, "reading the device status failed: %s", cudaGetErrorString(e));
  if (where != nullptr) *where = h[1];
  return h[0] == fo::kStatusTimeout ? FO_ETIMEOUT : h[0];
}

}  // extern "C"

// ---------------------------------------------------------------------- self-test
namespace {

__global__ void fo_wait_selftest_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = fo::smem_u32(&bar);
  if (threadIdx.x == 0) {
    fo::mbar_init(b, 1);
    fo::fence_mbar_init();
  }
  __syncwarp();
  // Nothing ever arrives on `bar`: the wait must run out and report it.
  bool got = true;
  if (threadIdx.x == 0) got = fo::mbar_wait(b, 0, timeout_ns, nullptr);
  if (threadIdx.x == 0 && !got) {
    status[0] = fo::kStatusTimeout;
    status[1] = 0x7e57;
  }
}

}  // namespace

extern "C" int fo_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return fail(FO_EINVAL, "timeout must be in (0, 10 s]");
  DevInfo di;
  if (int rc = device_info(&di)) return rc;
  int* st = nullptr;
  if (cudaMalloc(&st, 4 * sizeof(int)) != cudaSuccess) return fail(FO_ECUDA, "cudaMalloc failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(st, 0, 4 * sizeof(int), s);
  fo_wait_selftest_kernel<<<1, 32, 0, s>>>(st, timeout_ns);
  cudaError_t e = cudaGetLastError();
  int h[4] = {0, 0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpyAsync(h, st, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(st);
  if (e != cudaSuccess) return fail(FO_ECUDA, "self-test failed: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1);
  if (h[0] == fo::kStatusTimeout) return fail(FO_ETIMEOUT, "bounded wait ran out after %llu ns as expected",
                                              static_cast<unsigned long long>(timeout_ns));
  return ok();
}
