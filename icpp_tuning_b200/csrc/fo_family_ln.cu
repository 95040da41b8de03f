// Instantiations of the GEMM + bias + LayerNorm kernels (16-bit outputs): the tcgen05
// kernel writes the biased rows and per-slice statistics, fo_ln_normalize_kernel follows.
#include "fo_launch.cuh"

namespace fo {

// GEMM + bias + slice statistics, then the stream-ordered normalisation pass.
template <int BN, int OUT>
static cudaError_t gemm_then_normalize(const LaunchArgs& a) {
  cudaError_t e;
  if constexpr (BN >= 128) {
    e = a.pair ? launch_tc<BN, ACT_NONE, OUT, true, false, true>(a) : launch_tc<BN, ACT_NONE, OUT, true, false, false>(a);
  } else {
    e = a.pair ? cudaErrorInvalidValue : launch_tc<BN, ACT_NONE, OUT, true, false, false>(a);
  }
  if (e != cudaSuccess) return e;
  const int blocks = (a.p.M + 7) / 8;
  fo_ln_normalize_kernel<OUT><<<blocks, 256, 0, a.stream>>>(a.p, BN);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t by_out(int out_dt, const LaunchArgs& a) {
  switch (out_dt) {
    case DT_F16: return gemm_then_normalize<BN, DT_F16>(a);
    case DT_BF16: return gemm_then_normalize<BN, DT_BF16>(a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_ln_family(int bn, int out_dt, const LaunchArgs& a) {
  switch (bn) {
    case 64: return by_out<64>(out_dt, a);
    case 128: return by_out<128>(out_dt, a);
    case 256: return by_out<256>(out_dt, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fo
