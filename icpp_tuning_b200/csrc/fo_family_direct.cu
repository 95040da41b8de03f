// Instantiations and launch of the direct (padded-pitch) conv kernel.
#include "fo_direct.cuh"
#include "fo_launch.cuh"

namespace fo {

template <int ACT, int OUT, int KPS>
static cudaError_t launch_direct_k(const LaunchArgs& a) {
  auto kern = fo_direct_conv_kernel<ACT, OUT, KPS>;
  static std::atomic<uint64_t> opted{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((opted.load(std::memory_order_acquire) & bit) == 0) {
    RelaxedCapture relaxed;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (e != cudaSuccess) return e;
    opted.fetch_or(bit, std::memory_order_acq_rel);
  }
  kern<<<a.grid, kDirectThreads, a.smem, a.stream>>>(a.tmA, a.tmB, a.tmC, a.p);
  return cudaGetLastError();
}

// One filter tap per weight stage, two (block_k 128) or three (block_k 192).
template <int ACT, int OUT>
static cudaError_t launch_direct(const LaunchArgs& a) {
  switch (a.p.kps) {
    case 1: return launch_direct_k<ACT, OUT, 1>(a);
    case 2: return launch_direct_k<ACT, OUT, 2>(a);
    case 3: return launch_direct_k<ACT, OUT, 3>(a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_direct_conv(int act, int out_dt, const LaunchArgs& a) {
  const bool relu = act == ACT_RELU;
  if (act != ACT_NONE && !relu) return cudaErrorInvalidValue;
  switch (out_dt) {
    case DT_F16: return relu ? launch_direct<ACT_RELU, DT_F16>(a) : launch_direct<ACT_NONE, DT_F16>(a);
    case DT_BF16: return relu ? launch_direct<ACT_RELU, DT_BF16>(a) : launch_direct<ACT_NONE, DT_BF16>(a);
    case DT_F32: return relu ? launch_direct<ACT_RELU, DT_F32>(a) : launch_direct<ACT_NONE, DT_F32>(a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fo
