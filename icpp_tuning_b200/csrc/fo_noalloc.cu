// fo_noalloc.cu -- fo_gemm_bias_layernorm_noalloc: the fused GEMM + bias + LayerNorm for
// callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc (or anything that allocates) once
// they are running: a serving process that reserves its whole device-memory budget at
// start-up and must never grow it, or a host framework whose plugin interface hands the
// operator its inputs and outputs but no allocator.  fo_gemm's LayerNorm epilogue needs
// scratch memory for its per-row slice statistics and arrival counters, which those
// callers cannot provide.  This entry point takes that scratch from a file-scope
// __device__ array of fixed size instead and runs fo_gemm on it, so its arguments,
// checks, kernels, wait limit (fo_set_wait_timeout_ns), device status word
// (fo_device_status) and launch count are fo_gemm's.  It allocates nothing: no
// cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits and rules:
//   * the scratch holds FO_NOALLOC_LN_SCRATCH_BYTES (8 MiB); a problem whose workspace
//     would need more (fo_gemm_workspace_size > 8 MiB, about M * ceil(N / block_n) >
//     260k) is rejected with FO_EINVAL and a message naming both sizes;
//   * every GPU that loads this library holds the 8 MiB array until the process exits;
//   * every call shares the one array per device and it keeps the last call's contents.
//     The counters at its head must start at zero: the kernels leave them zeroed, and
//     each call also clears them on its stream first (cudaMemsetAsync, which allocates
//     nothing), so a call after one that timed out starts clean.  Calls whose
//     executions overlap on the GPU (different streams, or other threads) race on the
//     array -- serialise them;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current, in relaxed
//     stream-capture mode).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/b200fo.h"
#include "fo_launch.cuh"

namespace {

constexpr size_t kScratchBytes = FO_NOALLOC_LN_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_ln_scratch[kScratchBytes];

constexpr int kMaxDev = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDev] = {nullptr};

int say(int code, const char* msg) {
  fo::set_last_error(code, msg);  // read back with fo_last_error
  return code;
}

// Once per device, with that device current: the device address of the static array.
int setup_device(int dev, void** scratch) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* s = nullptr;
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // a query: legal under a capture
    cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t e = cudaGetSymbolAddress(&s, g_ln_scratch);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess || s == nullptr) return say(FO_ECUDA, "cudaGetSymbolAddress(scratch) failed");
    g_scratch_ptr[dev] = s;
  }
  *scratch = g_scratch_ptr[dev];
  return FO_OK;
}

int run(const FoGemmDesc* d, const FoTileCfg* cfg, void* stream) {
  if (d == nullptr || cfg == nullptr) return say(FO_EINVAL, "null descriptor or config");
  if (d->epilogue != FO_EPI_BIAS_LN) return say(FO_EINVAL, "this entry point runs only FO_EPI_BIAS_LN");
  if (d->M <= 0 || d->N <= 0) return fo_gemm(d, cfg, stream);  // validation / empty output only
  const size_t need = fo_gemm_workspace_size(d, cfg);
  if (need == 0) return fo_gemm(d, cfg, stream);  // a bad config: fo_gemm names it
  if (need > kScratchBytes) {
    char why[256];
    snprintf(why, sizeof(why),
             "this problem needs %zu bytes of LayerNorm scratch; the static scratch holds %zu bytes "
             "(use fo_gemm with a caller-provided workspace)",
             need, kScratchBytes);
    return say(FO_EINVAL, why);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return say(FO_ENODEVICE, "no current CUDA device");
  void* scratch = nullptr;
  if (int rc = setup_device(dev, &scratch)) return rc;
  // The arrival counters at the head of the scratch start at zero (1 KB covers 128k rows).
  const size_t head = static_cast<size_t>((d->M + 31) / 32) * 2 * sizeof(int);
  if (cudaMemsetAsync(scratch, 0, head, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return say(FO_ECUDA, "clearing the scratch counters failed");
  FoGemmDesc dd = *d;
  dd.workspace = scratch;
  dd.workspace_bytes = kScratchBytes;
  return fo_gemm(&dd, cfg, stream);
}

}  // namespace

extern "C" int fo_gemm_bias_layernorm_noalloc(const FoGemmDesc* desc, const FoTileCfg* cfg, void* stream) {
  return run(desc, cfg, stream);
}
