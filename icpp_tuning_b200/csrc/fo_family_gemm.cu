// Instantiations of the plain / bias / activation GEMM kernels.  Compiled twice:
// FO_PAIR = 0 (one CTA per 128-row tile) and FO_PAIR = 1 (CTA pairs, 256-row tiles).
#include "fo_launch.cuh"

#ifndef FO_PAIR
#define FO_PAIR 0
#endif

namespace fo {
namespace {

constexpr bool kPair = FO_PAIR != 0;

template <int BN, int ACT>
cudaError_t by_out(int out_dt, const LaunchArgs& a) {
  switch (out_dt) {
    case DT_F16: return launch_tc<BN, ACT, DT_F16, false, false, kPair>(a);
    case DT_BF16: return launch_tc<BN, ACT, DT_BF16, false, false, kPair>(a);
    case DT_F32: return launch_tc<BN, ACT, DT_F32, false, false, kPair>(a);
  }
  return cudaErrorInvalidValue;
}

template <int BN>
cudaError_t by_act(int act, int out_dt, const LaunchArgs& a) {
  switch (act) {
    case ACT_NONE: return by_out<BN, ACT_NONE>(out_dt, a);
    case ACT_RELU: return by_out<BN, ACT_RELU>(out_dt, a);
    case ACT_GELU_TANH: return by_out<BN, ACT_GELU_TANH>(out_dt, a);
    case ACT_GELU_ERF: return by_out<BN, ACT_GELU_ERF>(out_dt, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

#if FO_PAIR
cudaError_t launch_gemm_family_pair(int bn, int act, int out_dt, const LaunchArgs& a) {
  switch (bn) {
    case 128: return by_act<128>(act, out_dt, a);
    case 256: return by_act<256>(act, out_dt, a);
  }
  return cudaErrorInvalidValue;
}
#else
cudaError_t launch_gemm_family_single(int bn, int act, int out_dt, const LaunchArgs& a) {
  switch (bn) {
    case 64: return by_act<64>(act, out_dt, a);
    case 128: return by_act<128>(act, out_dt, a);
    case 256: return by_act<256>(act, out_dt, a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_family(int bn, int act, int out_dt, const LaunchArgs& a) {
  return a.pair ? launch_gemm_family_pair(bn, act, out_dt, a) : launch_gemm_family_single(bn, act, out_dt, a);
}
#endif

}  // namespace fo

#ifdef FO_PHASE_PROBE
#define FO_PROBE_CAT2(a, b) a##b
#define FO_PROBE_CAT(a, b) FO_PROBE_CAT2(a, b)
// Copies this translation unit's phase timestamps to the host (latency studies only).
extern "C" int FO_PROBE_CAT(fo_probe_read_pair, FO_PAIR)(void* host, size_t bytes) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, fo::g_fo_probe, bytes));
}
namespace {
__global__ void fo_probe_stamp_kernel(int slot, int smem) {
  extern __shared__ uint8_t pad[];
  if (threadIdx.x == 0) {
    fo::g_fo_probe[2047][slot] = fo::global_timer_ns();
    if (smem > 0) pad[smem - 1] = 1;  // touch the requested shared memory, inside it
  }
}
}  // namespace
// One in-stream timestamp into row 2047, slot `slot`; smem > 0 asks for that much dynamic
// shared memory (the carveout a kernel needs).
extern "C" int FO_PROBE_CAT(fo_probe_stamp_pair, FO_PAIR)(int slot, int smem, void* stream) {
  if (smem > 48 * 1024) cudaFuncSetAttribute(fo_probe_stamp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  fo_probe_stamp_kernel<<<1, 32, smem, static_cast<cudaStream_t>(stream)>>>(slot, smem);
  return static_cast<int>(cudaGetLastError());
}
extern "C" int FO_PROBE_CAT(fo_probe_clear_pair, FO_PAIR)() {
  void* a = nullptr;
  if (cudaGetSymbolAddress(&a, fo::g_fo_probe) != cudaSuccess) return -1;
  return static_cast<int>(cudaMemset(a, 0, sizeof(fo::g_fo_probe)));
}
#endif
