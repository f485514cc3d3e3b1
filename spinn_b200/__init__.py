"""spinn_b200 -- SPINN's dense-contraction hot path (Conv / Gemm / MatMul with the
Conv+BN/ReLU/SiLU/Add fusions) on NVIDIA B200 (sm_100a).

The compute lives in ``libspinn_cuda.so`` (hand-written tcgen05/TMA kernels, C ABI in
``include/spinn_cuda.h``); this package holds the ctypes binding, the ENNF format tools and
the synthetic model definitions used by the benchmark.
"""
from . import ennf, netdef  # noqa: F401

__all__ = ["ennf", "netdef", "lib", "runtime"]
__version__ = "0.1.0"
