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

// GEMM + bias (16-bit) through the plain family, then the residual LayerNorm row pass.
cudaError_t launch_residual_ln(int bn, int out_dt, const LaunchArgs& a) {
  cudaError_t e = launch_gemm_family(bn, ACT_NONE, out_dt, a);
  if (e != cudaSuccess) return e;
  const int blocks = (a.p.M + 7) / 8;
  const int slabs = (a.p.N + 255) / 256;
  if (out_dt != DT_F16 && out_dt != DT_BF16) return cudaErrorInvalidValue;
  const bool h = out_dt == DT_F16;
  if (slabs <= 4)
    h ? fo_ln_residual_kernel<DT_F16, 4><<<blocks, 256, 0, a.stream>>>(a.p)
      : fo_ln_residual_kernel<DT_BF16, 4><<<blocks, 256, 0, a.stream>>>(a.p);
  else if (slabs <= 8)
    h ? fo_ln_residual_kernel<DT_F16, 8><<<blocks, 256, 0, a.stream>>>(a.p)
      : fo_ln_residual_kernel<DT_BF16, 8><<<blocks, 256, 0, a.stream>>>(a.p);
  else
    h ? fo_ln_residual_kernel<DT_F16, 16><<<blocks, 256, 0, a.stream>>>(a.p)
      : fo_ln_residual_kernel<DT_BF16, 16><<<blocks, 256, 0, a.stream>>>(a.p);
  return cudaGetLastError();
}

}  // namespace fo
