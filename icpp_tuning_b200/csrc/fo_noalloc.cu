// fo_noalloc.cu -- fo_gemm_bias_layernorm_noalloc: the fused GEMM + bias + LayerNorm for
// callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc (or anything that allocates) once
// they are running: a serving process that reserves its whole device-memory budget at
// start-up and must never grow it, or a host framework whose plugin interface hands the
// operator its inputs and outputs but no allocator.  fo_gemm's LayerNorm epilogue needs
// scratch memory for its per-row slice statistics, which those callers
// cannot provide.  This entry point takes that scratch from a file-scope __device__
// array of fixed size instead, and it allocates nothing: no cudaMalloc, no cudaFree, no
// allocating library routine.  (Its device status word is a static array too, separate
// from the one fo_device_status reads.)
//
// Limits and rules:
//   * the scratch holds FO_NOALLOC_LN_SCRATCH_BYTES (8 MiB); a problem whose statistics
//     need more (fo_gemm_workspace_size > 8 MiB, e.g. M * ceil(N / block_n) > ~260k, the
//     statistics coming in half-tile slices) is
//     rejected with FO_EINVAL and a message naming both sizes;
//   * every GPU that loads this library holds the 8 MiB array until the process exits;
//   * every call shares the one array per device and it keeps the last call's contents;
//     nothing in it has to start at zero (each call writes every statistic it later
//     reads), but calls whose executions overlap on the GPU (different streams, or other
//     threads) race on the array -- serialise them;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current, in relaxed
//     stream-capture mode, so that even a first call made under a capture is legal);
//   * a bounded device-side wait that runs out is recorded in this path's own static
//     status word, not in the one fo_device_status reads.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/b200fo.h"
#include "fo_launch.cuh"

namespace {

constexpr size_t kScratchBytes = FO_NOALLOC_LN_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_ln_scratch[kScratchBytes];
static __device__ __align__(256) int g_ln_status[4];

constexpr int kMaxDev = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDev] = {nullptr};
int* g_status_ptr[kMaxDev] = {nullptr};
int g_sm_count[kMaxDev] = {0};

int say(int code, const char* msg) {
  fo::set_last_error(code, msg);  // read back with fo_last_error
  return code;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Once per device, with that device current: the device addresses of the static arrays.
int setup_device(int dev, void** scratch, int** status, int* sms) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* s = nullptr;
    void* st = nullptr;
    int n = 0;
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // queries only: legal under a capture
    cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t e1 = cudaGetSymbolAddress(&s, g_ln_scratch);
    const cudaError_t e2 = cudaGetSymbolAddress(&st, g_ln_status);
    const cudaError_t e3 = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e1 != cudaSuccess) return say(FO_ECUDA, "cudaGetSymbolAddress(scratch) failed");
    if (e2 != cudaSuccess) return say(FO_ECUDA, "cudaGetSymbolAddress(status) failed");
    if (e3 != cudaSuccess) return say(FO_ECUDA, "cudaDeviceGetAttribute failed");
    g_scratch_ptr[dev] = s;
    g_status_ptr[dev] = static_cast<int*>(st);
    g_sm_count[dev] = n;
  }
  *scratch = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  *sms = g_sm_count[dev];
  return FO_OK;
}

int tmap(CUtensorMap* m, int dt, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
         uint32_t box_inner, uint32_t box_outer) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // legal under a capture
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaThreadExchangeStreamCaptureMode(&mode);
  });
  if (fn == nullptr) return say(FO_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType t = dt == FO_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                : dt == FO_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  if (fn(m, t, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return say(FO_EINVAL, "a tensor map was rejected by the driver (shape, stride or alignment)");
  return FO_OK;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int run(const FoGemmDesc* d, const FoTileCfg* cfg, void* stream) {
  if (d == nullptr || cfg == nullptr) return say(FO_EINVAL, "null descriptor or config");
  if (d->epilogue != FO_EPI_BIAS_LN) return say(FO_EINVAL, "this entry point runs only FO_EPI_BIAS_LN");
  char why[256];
  if (fo_query_config_legal(0, d->out_dtype, cfg, why, sizeof(why)) != FO_OK) return say(FO_EINVAL, why);
  if (d->M < 0 || d->N < 0 || d->K < 0 || d->M > (1ll << 31) - 1 || d->N > (1ll << 31) - 1 || d->K > (1ll << 31) - 1)
    return say(FO_EINVAL, "bad shape");
  if (d->M == 0 || d->N == 0) return FO_OK;
  if (d->in_dtype != FO_DT_F16 && d->in_dtype != FO_DT_BF16) return say(FO_EINVAL, "in_dtype must be f16 or bf16");
  if (d->out_dtype != FO_DT_F16 && d->out_dtype != FO_DT_BF16) return say(FO_EINVAL, "LayerNorm output must be f16 or bf16");
  if (d->vec_dtype < FO_DT_F16 || d->vec_dtype > FO_DT_F32) return say(FO_EINVAL, "bad vec_dtype");
  if (d->b_layout != FO_B_KN && d->b_layout != FO_B_NK) return say(FO_EINVAL, "bad b_layout");
  if (d->bias == nullptr || d->gamma == nullptr || d->beta == nullptr) return say(FO_EINVAL, "LayerNorm needs bias, gamma and beta");
  if (!a16(d->gamma) || !a16(d->beta)) return say(FO_EINVAL, "gamma and beta must be 16-byte aligned");
  if (d->N % 8 != 0) return say(FO_EINVAL, "LayerNorm needs N % 8 == 0");
  if (d->out == nullptr || !a16(d->out) || d->ldo < d->N || (d->ldo * 2) % 16 != 0)
    return say(FO_EINVAL, "out must be 16-byte aligned with ldo >= N and a multiple of 8");
  if (d->K > 0) {
    const int64_t bmin = d->b_layout == FO_B_KN ? d->N : d->K;
    if (d->a == nullptr || d->b == nullptr || !a16(d->a) || !a16(d->b) || d->lda < d->K || (d->lda * 2) % 16 != 0 ||
        d->ldb < bmin || (d->ldb * 2) % 16 != 0)
      return say(FO_EINVAL, "a / b must be 16-byte aligned with row strides that are multiples of 8 elements");
  }
  if (!(d->eps >= 0.0f)) return say(FO_EINVAL, "eps must be >= 0");
  const size_t need = fo_gemm_workspace_size(d, cfg);
  if (need > kScratchBytes) {
    snprintf(why, sizeof(why),
             "this problem needs %zu bytes of LayerNorm scratch; the static scratch holds %zu bytes "
             "(use fo_gemm with a caller-provided workspace)",
             need, kScratchBytes);
    return say(FO_EINVAL, why);
  }

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return say(FO_ENODEVICE, "no current CUDA device");
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return say(FO_ENODEVICE, "this library is built for sm_100a");
  void* scratch = nullptr;
  int* status = nullptr;
  int sms = 0;
  if (int rc = setup_device(dev, &scratch, &status, &sms)) return rc;

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
  p.group_m = 0;
  p.stages = cfg->stages;
  p.ab_bf16 = d->in_dtype == FO_DT_BF16;
  p.b_mn = d->b_layout == FO_B_KN;
  p.has_bias = 1;
  p.bias = d->bias;
  p.gamma = d->gamma;
  p.beta = d->beta;
  p.vec_dtype = d->vec_dtype;
  p.eps = d->eps;
  p.out = d->out;
  p.ldo = d->ldo;
  // Same layout as fo_gemm's workspace: a reserved 256-byte-aligned header, then the stats.
  const size_t header_bytes = round_up(static_cast<size_t>((p.M + 127) / 128) * 4, 256);
  p.ln_stats = reinterpret_cast<float4*>(static_cast<char*>(scratch) + header_bytes);
  p.status = status;
  p.timeout_ns = 2000000000ull;

  if (p.K > 0) {
    if (int rc = tmap(&la.tmA, d->in_dtype, d->a, d->K, d->M, d->lda * 2, 64, 128)) return rc;
    if (d->b_layout == FO_B_NK) {
      if (int rc = tmap(&la.tmB, d->in_dtype, d->b, d->K, d->N, d->ldb * 2, 64, pair ? bn / 2 : bn)) return rc;
    } else {
      if (int rc = tmap(&la.tmB, d->in_dtype, d->b, d->N, d->K, d->ldb * 2, 64, 64)) return rc;
    }
  }
  if (int rc = tmap(&la.tmC, d->out_dtype, d->out, d->N, d->M, d->ldo * 2, 64, 32)) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int cap = pair ? (cfg->max_ctas > 0 ? cfg->max_ctas / 2 : sms / 2) : (cfg->max_ctas > 0 ? cfg->max_ctas : sms);
  if (cap < 1) return say(FO_EINVAL, "max_ctas too small for CTA pairs");
  la.grid = (p.num_tiles < cap ? p.num_tiles : cap) * (pair ? 2 : 1);
  la.pair = pair;
  p.num_units = p.dp_units = p.num_tiles;  // whole tiles
  p.split = 1;
  p.kb_per_part = p.k_blocks;
  p.kps = cfg->block_k / 64;
  la.smem = fo::smem_bytes_for(bn, cfg->stages, pair, p.kps);
  la.stream = st;
  cudaError_t e = fo::launch_ln_family(bn, d->out_dtype == FO_DT_F16 ? fo::DT_F16 : fo::DT_BF16, la);
  if (e != cudaSuccess) {
    snprintf(why, sizeof(why), "kernel launch failed: %s", cudaGetErrorString(e));
    return say(FO_ECUDA, why);
  }
  return FO_OK;
}

}  // namespace

extern "C" int fo_gemm_bias_layernorm_noalloc(const FoGemmDesc* desc, const FoTileCfg* cfg, void* stream) {
  const int rc = run(desc, cfg, stream);
  if (rc == FO_OK) fo::set_last_error(FO_OK, "");
  return rc;
}
