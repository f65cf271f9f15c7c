"""tops (B200 build): Gated Linear Attention operators on NVIDIA B200.

The Python API mirrors the reference package ``tops`` (primatrix/pallas-kernel)
for the GLA hot path -- ``tops.ops.gla`` -- and runs every operator in
``tops/_lib/libtops_gla.so`` (hand-written sm_100a CUDA behind a C ABI,
``include/tops_gla.h``).  Tensors are torch CUDA tensors.
"""
__version__ = "0.1.0"
