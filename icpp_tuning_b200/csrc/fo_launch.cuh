// fo_launch.cuh -- host-side launch of one fo_tc_kernel instantiation.  Each family of
// instantiations (gemm, gemm+LayerNorm, conv) is compiled in its own translation unit.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

#include "fo_kernel.cuh"

namespace fo {

struct LaunchArgs {
  CUtensorMap tmA, tmB, tmC;
  KParams p;
  int grid;
  int smem;
  cudaStream_t stream;
};

template <int BN, int ACT, int OUT_DT, bool LN, bool CONV>
cudaError_t launch_tc(const LaunchArgs& a) {
  auto kern = fo_tc_kernel<BN, ACT, OUT_DT, LN, CONV>;
  // Opt in to the full 227 KB of dynamic shared memory once per device.
  static std::atomic<uint64_t> opted{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((opted.load(std::memory_order_acquire) & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (e != cudaSuccess) return e;
    opted.fetch_or(bit, std::memory_order_acq_rel);
  }
  constexpr int kThreads = CONV ? 288 : 192;
  kern<<<a.grid, kThreads, a.smem, a.stream>>>(a.tmA, a.tmB, a.tmC, a.p);
  return cudaGetLastError();
}

// Returns cudaErrorInvalidValue for a combination this build does not instantiate.
cudaError_t launch_gemm_family(int bn, int act, int out_dt, const LaunchArgs& a);
cudaError_t launch_ln_family(int bn, int out_dt, const LaunchArgs& a);
cudaError_t launch_conv_family(int bn, int act, int out_dt, const LaunchArgs& a);

// Sets the message fo_last_error returns on the calling thread (defined in fo_api.cu).
void set_last_error(int code, const char* msg);

}  // namespace fo
