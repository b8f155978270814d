"""CUDA kernels of the CVSA step (page scoring, sparse decode, coverage)."""
