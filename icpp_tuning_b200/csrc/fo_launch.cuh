// fo_launch.cuh -- host-side launch of one fo_tc_kernel instantiation.  Each family of
// instantiations (gemm, gemm+LayerNorm, conv) is compiled in its own translation unit.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

#include "fo_kernel.cuh"

namespace fo {

// Function attributes and occupancy queries enqueue nothing, but a global-mode stream
// capture on another thread would refuse them: switch this thread to relaxed mode for
// the one-time setup of a kernel so that a first call under capture stays legal.
struct RelaxedCapture {
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
  ~RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
};

struct LaunchArgs {
  CUtensorMap tmA, tmB, tmC;
  KParams p;
  int grid;  // CTAs (for CTA pairs: 2 x clusters)
  int smem;
  cudaStream_t stream;
  bool pair;  // launch as clusters of two CTAs (block_m 256, tcgen05 cta_group::2)
  bool swap;  // conv: operand-swapped kernel (M = output channels, N = pixels)
  int csplit;  // gemm: parts of a cluster split (clusters of csplit CTAs), 0 or 1 = none
  bool coop;   // cooperative launch: every CTA resident at once (one-kernel LayerNorm,
               // whose CTAs wait on counters other CTAs of the grid increment)
};

template <int BN, int ACT, int OUT_DT, bool LN, bool CONV, bool PAIR, bool SWAP, int KPS>
cudaError_t launch_tc_k(const LaunchArgs& a) {
  auto kern = fo_tc_kernel<BN, ACT, OUT_DT, LN, CONV, PAIR, SWAP, KPS>;
  // Opt in to the full 227 KB of dynamic shared memory once per device.
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
  constexpr int kThreads = CONV ? 416 : 320;  // producer(s) + MMA + 8 epilogue warps
  // Every launch is a programmatic dependent of the previous kernel on the stream (the
  // kernel waits on griddepcontrol before its first global access), so its CTAs set up
  // on idle SMs while that kernel finishes.
  cudaLaunchAttribute pdl;
  pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchAttribute coop;
  coop.id = cudaLaunchAttributeCooperative;
  coop.val.cooperative = 1;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = a.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1] = pdl;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // A persistent grid larger than the number of co-resident pairs would leave a tail
    // wave: clamp to what the GPU can hold at once (queried once per device).
    static std::atomic<int> max_clusters[64];
    int mc = max_clusters[dev & 63].load(std::memory_order_relaxed);
    if (mc == 0) {
      RelaxedCapture relaxed;
      if (cudaOccupancyMaxActiveClusters(&mc, kern, &cfg) != cudaSuccess || mc <= 0) {
        cudaGetLastError();
        mc = -1;
      }
      max_clusters[dev & 63].store(mc, std::memory_order_relaxed);
    }
    if (mc > 0 && static_cast<int>(cfg.gridDim.x) > 2 * mc) cfg.gridDim.x = 2 * mc;
    // the one-kernel LayerNorm's wait depth follows the number of pairs actually launched
    if (LN && a.p.ln_fused == 1 && ln_defer_for(a.p.ln_span, static_cast<int>(cfg.gridDim.x) / 2) > kLnMaxDefer)
      return cudaErrorCooperativeLaunchTooLarge;
    if (LN && a.p.ln_fused == 2 && a.p.ln_span >= static_cast<int>(cfg.gridDim.x) / 2)
      return cudaErrorCooperativeLaunchTooLarge;  // held slices need span < pairs launched
    if (a.coop) attr[1] = coop;  // a cooperative grid is not a programmatic dependent
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a.tmA, a.tmB, a.tmC, a.p);
  } else {
    if (a.csplit > 1) {
      // Cluster split: every unit needs its own CTA and a cluster's CTAs run at once, so
      // the grid must fit the co-resident clusters of this size (queried once per size).
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(a.grid, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = a.smem;
      cfg.stream = a.stream;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = a.csplit;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1] = pdl;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      static std::atomic<int> max_clusters[64][9];
      if (a.csplit > 8) return cudaErrorInvalidValue;  // portable cluster sizes only
      std::atomic<int>& slot = max_clusters[dev & 63][a.csplit];
      int mc = slot.load(std::memory_order_relaxed);
      if (mc == 0) {
        RelaxedCapture relaxed;
        if (cudaOccupancyMaxActiveClusters(&mc, kern, &cfg) != cudaSuccess || mc <= 0) {
          cudaGetLastError();
          mc = -1;
        }
        slot.store(mc, std::memory_order_relaxed);
      }
      if (mc > 0 && a.grid > mc * a.csplit) return cudaErrorCooperativeLaunchTooLarge;
      cfg.numAttrs = 2;
      return cudaLaunchKernelEx(&cfg, kern, a.tmA, a.tmB, a.tmC, a.p);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = a.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1] = {a.coop ? coop : pdl};  // a cooperative grid is not a programmatic dependent
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a.tmA, a.tmB, a.tmC, a.p);
  }
}

// One k-block per stage, or two (p.kps == 2, block_k 128; GEMM family only).
template <int BN, int ACT, int OUT_DT, bool LN, bool CONV, bool PAIR, bool SWAP = false>
cudaError_t launch_tc(const LaunchArgs& a) {
  if constexpr (CONV) {
    if (a.p.kps != 1) return cudaErrorInvalidValue;
    return launch_tc_k<BN, ACT, OUT_DT, LN, CONV, PAIR, SWAP, 1>(a);
  } else {
    return a.p.kps == 2 ? launch_tc_k<BN, ACT, OUT_DT, LN, CONV, PAIR, SWAP, 2>(a)
                        : launch_tc_k<BN, ACT, OUT_DT, LN, CONV, PAIR, SWAP, 1>(a);
  }
}

// Returns cudaErrorInvalidValue for a combination this build does not instantiate.
// The gemm family is compiled twice (fo_family_gemm.cu with FO_PAIR 0 and 1).
cudaError_t launch_gemm_family(int bn, int act, int out_dt, const LaunchArgs& a);
cudaError_t launch_gemm_family_single(int bn, int act, int out_dt, const LaunchArgs& a);
cudaError_t launch_gemm_family_pair(int bn, int act, int out_dt, const LaunchArgs& a);
cudaError_t launch_ln_family(int bn, int out_dt, const LaunchArgs& a);
cudaError_t launch_residual_ln(int bn, int out_dt, const LaunchArgs& a);
cudaError_t launch_conv_family(int bn, int act, int out_dt, const LaunchArgs& a);
// Direct (padded-pitch) conv: tmA = input rows (4-D), tmB = weights, tmC = output (4-D).
cudaError_t launch_direct_conv(int act, int out_dt, const LaunchArgs& a);

// Sets the message fo_last_error returns on the calling thread (defined in fo_api.cu).
void set_last_error(int code, const char* msg);

}  // namespace fo
