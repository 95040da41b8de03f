"""icpp_tuning_b200 -- B200-native (sm_100a) fused dense operators behind the
descriptor / autotuner API of leon062112/icpp-tuning.

Layout:
  autotuner/   descriptor API, cost models, search space, GPU spec (host)
  gemm/        gemm, gemm_bias_act, gemm_bias_layernorm (reference-shaped modules)
  conv/        conv2d, conv2d_relu (reference-shaped modules)
  fused.py     functional calls over the C ABI (libb200fo.so, include/b200fo.h)
  csrc/        the CUDA kernels and the C ABI
"""
__version__ = "0.1.0"
