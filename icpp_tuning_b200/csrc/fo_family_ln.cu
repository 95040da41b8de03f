// Instantiations of the GEMM + bias + LayerNorm kernels (16-bit outputs).
#include "fo_launch.cuh"

namespace fo {

template <int BN>
static cudaError_t by_out(int out_dt, const LaunchArgs& a) {
  switch (out_dt) {
    case DT_F16: return launch_tc<BN, ACT_NONE, DT_F16, true, false>(a);
    case DT_BF16: return launch_tc<BN, ACT_NONE, DT_BF16, true, false>(a);
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
