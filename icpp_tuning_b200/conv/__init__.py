"""Conv operators as implicit GEMM (reference kernel/tilelang/conv/)."""
