// Instantiations of the implicit-GEMM conv2d kernels (epilogue: none / ReLU, bias optional).
#include "fo_launch.cuh"

namespace fo {

template <int BN, int ACT, bool PAIR>
static cudaError_t by_out_p(int out_dt, const LaunchArgs& a) {
  switch (out_dt) {
    case DT_F16: return launch_tc<BN, ACT, DT_F16, false, true, PAIR>(a);
    case DT_BF16: return launch_tc<BN, ACT, DT_BF16, false, true, PAIR>(a);
    case DT_F32: return launch_tc<BN, ACT, DT_F32, false, true, PAIR>(a);
  }
  return cudaErrorInvalidValue;
}

template <int BN, int ACT>
static cudaError_t by_out_swap(int out_dt, const LaunchArgs& a) {
  switch (out_dt) {
    case DT_F16: return launch_tc<BN, ACT, DT_F16, false, true, false, true>(a);
    case DT_BF16: return launch_tc<BN, ACT, DT_BF16, false, true, false, true>(a);
    case DT_F32: return launch_tc<BN, ACT, DT_F32, false, true, false, true>(a);
  }
  return cudaErrorInvalidValue;
}

template <int BN, int ACT>
static cudaError_t by_out(int out_dt, const LaunchArgs& a) {
  if constexpr (BN >= 128) {
    if (a.swap) return by_out_swap<BN, ACT>(out_dt, a);
    if (a.pair) return by_out_p<BN, ACT, true>(out_dt, a);
  } else {
    if (a.pair || a.swap) return cudaErrorInvalidValue;
  }
  return by_out_p<BN, ACT, false>(out_dt, a);
}

template <int BN>
static cudaError_t by_act(int act, int out_dt, const LaunchArgs& a) {
  switch (act) {
    case ACT_NONE: return by_out<BN, ACT_NONE>(out_dt, a);
    case ACT_RELU: return by_out<BN, ACT_RELU>(out_dt, a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_conv_family(int bn, int act, int out_dt, const LaunchArgs& a) {
  switch (bn) {
    case 64: return by_act<64>(act, out_dt, a);
    case 128: return by_act<128>(act, out_dt, a);
    case 256: return by_act<256>(act, out_dt, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fo
