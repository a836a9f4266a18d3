"""The three sm_100a kernel families KernelOps lower to: pointwise, reduction, GEMM."""
