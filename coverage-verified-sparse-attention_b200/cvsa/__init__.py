"""B200-native CVSA decode step (coverage-verified sparse attention).

Drop-in for the hot path of DJ-Melvin/coverage-verified-sparse-attention:
`cvsa.backend.CVSABackend`, `cvsa.runtime.kv_cache`, the kernel functions of
`cvsa.kernels.*`, `cvsa.complement` and `cvsa.lse_merge` keep the reference's
names and signatures and run on hand-written sm_100a CUDA kernels through the
C ABI of libcvsa_b200.so (include/cvsa_b200.h).
"""

__version__ = "0.1.0"
