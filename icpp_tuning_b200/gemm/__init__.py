"""GEMM-family operators (reference kernel/tilelang/gemm/)."""
