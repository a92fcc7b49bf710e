"""lightx2v_cuda — B200 (sm_100a) backend for lightx2v-rs's quantized linear path.

`CudaBackend` mirrors the reference's `Backend` trait for the path; the
compute runs in liblightx2v_cuda.so (hand-written tcgen05 / TMA kernels).
`quant` and `rng` mirror lightx2v-core's weight formats and seeded RNG.
"""
from . import _lib
from .backend import Act, Buf, CudaBackend, Weight
from .quant import Fp8E4M3, Q4, Q8, WeightQuant

BF16 = _lib.BF16
F32 = _lib.F32

__all__ = ["Act", "Buf", "CudaBackend", "Weight", "Q8", "Q4", "Fp8E4M3", "WeightQuant", "BF16",
           "F32"]
