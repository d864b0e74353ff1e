"""B200 (sm_100a) backend for the Pairformer pair-representation hot path.

The compute path is the C-ABI library ``libfireprot_b200.so`` (hand-written
tcgen05/TMA CUDA kernels) loaded through :mod:`fireprot_b200._lib`; there is
no CPU fallback inside this package.
"""
__version__ = "0.1.0"
BACKEND_NAME = "b200"
