// Instantiations of the GEMM + bias + LayerNorm kernels (16-bit outputs).  One kernel
// (p.ln_fused): the tcgen05 kernel normalises its own stored slices once their rows'
// statistics are complete.  Two kernels: it writes the biased rows and per-slice
// statistics, and a row pass (fo_ln_normalize_kernel or fo_ln_rows_kernel) follows.
#include "fo_launch.cuh"

namespace fo {

// The row pass after the GEMM kernel, launched programmatically so its launch (and, for
// the block-per-row kernel, its gamma / beta / residual reads) overlap the GEMM's tail
// (griddepcontrol; the GEMM's MMA thread signals once it has issued its last MMA).
//   M <= kSmallRows, N <= 4096: fo_ln_rows_kernel, one block per row (latency);
//   otherwise plain LayerNorm: fo_ln_normalize_kernel, one warp per row in batches of 8
//     slabs (measured 67 us on 16384 x 4096 bf16, against 70 us for the whole-row warp
//     kernel, whose registers allow fewer warps per SM);
//   otherwise residual LayerNorm (N <= 4096): fo_ln_warp_rows_kernel.
constexpr int kSmallRows = 1024;

template <typename Kern>
static cudaError_t launch_pdl(Kern kern, int grid, int threads, const LaunchArgs& a, int bn) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a.p, bn);
}

template <int OUT, bool RESID, int kChunks>
static cudaError_t rows(const LaunchArgs& a, int bn) {
  if (a.p.M <= kSmallRows) return launch_pdl(fo_ln_rows_kernel<OUT, RESID, kChunks>, a.p.M, 128, a, bn);
  if constexpr (RESID) {
    return launch_pdl(fo_ln_warp_rows_kernel<OUT, RESID, 4 * kChunks>, (a.p.M + 7) / 8, 256, a, bn);
  } else {
    return launch_pdl(fo_ln_normalize_kernel<OUT>, (a.p.M + 7) / 8, 256, a, bn);
  }
}

template <int OUT, bool RESID>
static cudaError_t row_pass(const LaunchArgs& a, int bn) {
  const int chunks = (a.p.N + 1023) / 1024;
  if (chunks <= 1) return rows<OUT, RESID, 1>(a, bn);
  if (chunks <= 2) return rows<OUT, RESID, 2>(a, bn);
  if (chunks <= 4) return rows<OUT, RESID, 4>(a, bn);
  if constexpr (RESID) {
    return cudaErrorInvalidValue;  // fo_gemm admits N <= 4096 only
  } else {
    return launch_pdl(fo_ln_normalize_kernel<OUT>, (a.p.M + 7) / 8, 256, a, bn);
  }
}

// GEMM + bias + slice statistics, then the row pass.
template <int BN, int OUT>
static cudaError_t gemm_then_normalize(const LaunchArgs& a) {
  cudaError_t e;
  if constexpr (BN >= 128) {
    e = a.pair ? launch_tc<BN, ACT_NONE, OUT, true, false, true>(a) : launch_tc<BN, ACT_NONE, OUT, true, false, false>(a);
  } else {
    e = a.pair ? cudaErrorInvalidValue : launch_tc<BN, ACT_NONE, OUT, true, false, false>(a);
  }
  if (e != cudaSuccess || a.p.ln_fused) return e;  // one kernel: no row pass
  // The statistics come in slices of half a tile (one per epilogue warp): the row pass
  // merges tiles_n x 2 slices of BN / 2 columns.
  constexpr int kHalves = 2;
  LaunchArgs r = a;
  r.p.tiles_n = a.p.tiles_n * kHalves;
  return row_pass<OUT, false>(r, BN / kHalves);
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
  if (out_dt != DT_F16 && out_dt != DT_BF16) return cudaErrorInvalidValue;
  cudaError_t e = launch_gemm_family(bn, ACT_NONE, out_dt, a);
  if (e != cudaSuccess) return e;
  return out_dt == DT_F16 ? row_pass<DT_F16, true>(a, bn) : row_pass<DT_BF16, true>(a, bn);
}

}  // namespace fo
