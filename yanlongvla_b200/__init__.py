"""B200-native (sm_100a) trellis-coded W2A8 Linear: randomized Walsh rotation, fused 2-bit trellis decode-GEMV,
per-token INT8 quantizer and W8A8 INT8 GEMM, behind the C ABI of include/tcq_b200.h.

Submodules: `kernels` (the reference's kernel-wrapper interface), `tcq_format` (packed format and layers), `modules`
(quantized Linear replacement and policy surgery). Importing `kernels` loads libtcq_b200.so and fails if it is absent.
"""
__version__ = '0.1.0'
