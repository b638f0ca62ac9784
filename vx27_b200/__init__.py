"""vx27_b200: the vx27 attention hot path (Gated DeltaNet + gated GQA with a BF16 KV
cache) as hand-written CUDA for B200 (sm_100a), behind the reference's C interface.

libvx27cuda.so (built from csrc/ by build.py) is the product; this package binds it
with ctypes (ops.py) and drives batched decode (hybrid.py)."""
from ._lib import LIB_PATH, Vx27Error, load  # noqa: F401

__all__ = ["LIB_PATH", "Vx27Error", "load"]
