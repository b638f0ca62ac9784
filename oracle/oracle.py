"""ctypes wrapper of the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg as
the checker; never imported by the vx27_b200 package. Builds liboracle.so from the
committed C sources on first use (gcc), and oracle/_ref/libvx27ref.so (the reference's
own sources) when they are available.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libvx27ref.so")
REF_PMAT_LIB = os.path.join(HERE, "_ref", "libvx27ref_pmat.so")

F_ACT_BF16, F_OUT_BF16, F_NORM_1P = 0x1, 0x2, 0x4

_p, _i, _f, _d, _sz, _u64 = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_size_t, C.c_uint64
_PROTOS = {
    "orc_f32_to_bf16": (C.c_uint16, [_f]),
    "orc_bf16_to_f32": (_f, [C.c_uint16]),
    "orc_update_ref": (None, [_p, _p, _p, _f, _i]),
    "orc_retrieve_ref": (None, [_p, _p, _p, _i]),
    "orc_l2norm": (None, [_p, _p, _i]),
    "orc_softplus": (_d, [_d]),
    "orc_gate_params": (None, [_d, _d, _d, _d, C.POINTER(_d), C.POINTER(_d)]),
    "orc_step_exact": (None, [_p, _p, _p, _p, _d, _d, _p, _i]),
    "orc_conv1d_step": (None, [_p, _p, _p, _p, _i, _i]),
    "orc_kv_for_q": (_i, [_i, _i, _i]),
    "orc_rmsnorm": (None, [_p, _p, _p, _i, _f, _i]),
    "orc_rope_cos_sin": (None, [_i, _p, _p, _i, _f, _f]),
    "orc_rope_apply": (None, [_p, _i, _i, _i, _p, _p]),
    "orc_attn_1q": (None, [_p, _p, _p, _i, _i, _i, _i, _p]),
    "orc_kv_elems": (_u64, [_i]),
    "orc_kv_gb": (_d, [_i, _d]),
    "orc_deltanet_decode_batch": (None, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i,
                                         _i]),
    "orc_deltanet_decode_batch_mt": (None, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i,
                                            _i, _i, _i]),
    "orc_gqa_append": (None, [_p, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _i, _i, _i, _f, _f,
                              _i]),
    "orc_gqa_attend": (None, [_p, _p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i]),
    "orc_gqa_attend_mt": (None, [_p, _p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _i]),
    "orc_gqa_partial": (None, [_p, _p, _p, _i, _i, _i, _p, _p, _i, _i, _i]),
    "orc_gqa_combine": (None, [_p, _p, _i, _p, _p, _i, _i, _i]),
    "orc_gate_params_grid": (None, [_p, _p, _p, _p, _i, _i, _p, _p]),
    "orc_gated_rmsnorm": (None, [_p, _p, _p, _p, _i, _i]),
    "orc_deltanet_recurrent": (None, [_p, _p, _p, _p, C.c_long, _p, _p, _p, _i, _i, _i]),
    "orc_gqa_prefill_rows": (None, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _f, _p, _i,
                                    _p, _i]),
    "orc_fill_normal_f32": (None, [_p, _sz, _u64, _u64, _f, _f]),
    "orc_fill_normal_bf16": (None, [_p, _sz, _u64, _u64, _f, _f]),
    "orc_fill_uniform_f32": (None, [_p, _sz, _u64, _u64, _f, _f]),
    "orc_bp3_scale": (_f, [C.c_uint16]),
    "orc_pmat_batch": (None, [_p, C.c_uint32, _p, _p, _i, _i, _i]),
    "orc_use_reference": (_i, [C.c_char_p]),
    "orc_impl_is_reference": (_i, []),
}

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def build_ref() -> bool:
    """Builds oracle/_ref/ from the reference sources; False if they are absent."""
    r = subprocess.run(["make", "-s", "-C", HERE, "ref"], capture_output=True, text=True)
    return r.returncode == 0 and os.path.exists(REF_LIB)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB) or any(
                os.path.getmtime(os.path.join(HERE, f)) > os.path.getmtime(LIB)
                for f in ("vx27_oracle.c", "vx27_oracle.h", "threadpool_posix.c")):
            build()
        l = C.CDLL(LIB)
        for n, (r, a) in _PROTOS.items():
            fn = getattr(l, n)
            fn.restype, fn.argtypes = r, a
        _lib = l
    return _lib


def P(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)  # keeps the array alive with the pointer


def to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits (uint16), round to nearest even (same rule as the library)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def from_bf16(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def normal(n, seed: int, stream: int, mean: float = 0.0, std: float = 1.0, bf16: bool = False):
    shape = (n,) if isinstance(n, int) else tuple(n)
    cnt = int(np.prod(shape))
    if bf16:
        out = np.empty(cnt, dtype=np.uint16)
        lib().orc_fill_normal_bf16(P(out), cnt, seed, stream, mean, std)
    else:
        out = np.empty(cnt, dtype=np.float32)
        lib().orc_fill_normal_f32(P(out), cnt, seed, stream, mean, std)
    return out.reshape(shape)


def uniform(n, seed: int, stream: int, lo: float, hi: float):
    shape = (n,) if isinstance(n, int) else tuple(n)
    out = np.empty(int(np.prod(shape)), dtype=np.float32)
    lib().orc_fill_uniform_f32(P(out), out.size, seed, stream, lo, hi)
    return out.reshape(shape)


def use_reference(enable: bool = True) -> bool:
    if not enable:
        lib().orc_use_reference(None)
        return False
    if not os.path.exists(REF_LIB):
        return False
    return lib().orc_use_reference(REF_LIB.encode()) == 0


# ---- packed weights (the layouts src/vx27_pmat.c reads) ------------------------------
PMAT_F32, PMAT_Q8K, PMAT_BP3 = 0, 2, 4


def pmat_row_bytes(dtype: int, cols: int) -> int:
    return cols * 4 if dtype == PMAT_F32 else (cols // 256) * 292 if dtype == PMAT_Q8K \
        else (cols // 128) * 52


def packed_weights(dtype: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Random packed weights as raw bytes [rows * row_bytes]: F32 ~N(0, 0.02); Q8_K with
    d ~ U(1e-4, 1e-3) and uniform int8 codes; BP3_128 with uniform 3-bit codes and fp16
    scales ~ U(0.005, 0.05), some of them fp16 subnormals (the reference maps those with
    exponent 1, which the oracle and the device reproduce)."""
    rng = np.random.default_rng(seed)
    if dtype == PMAT_F32:
        return (rng.standard_normal(rows * cols).astype(np.float32) * 0.02).view(np.uint8)
    if dtype == PMAT_Q8K:
        nb = rows * (cols // 256)
        blk = np.zeros((nb, 292), np.uint8)
        blk[:, 0:4] = rng.uniform(1e-4, 1e-3, nb).astype(np.float32).view(np.uint8).reshape(nb, 4)
        blk[:, 4:260] = rng.integers(-127, 128, (nb, 256)).astype(np.int8).view(np.uint8)
        return blk.reshape(-1)
    ng = rows * (cols // 128)
    g = np.zeros((ng, 52), np.uint8)
    g[:, 0:48] = rng.integers(0, 256, (ng, 48), dtype=np.uint8)
    sc = rng.uniform(0.005, 0.05, ng).astype(np.float16)
    sub = rng.random(ng) < 0.05
    sc[sub] = (rng.integers(1, 1024, int(sub.sum())).astype(np.uint16)).view(np.float16)
    g[:, 48:50] = sc.view(np.uint8).reshape(ng, 2)
    return g.reshape(-1)


def pmat_batch(W: np.ndarray, dtype: int, xb: np.ndarray, rows: int, cols: int, B: int):
    y = np.empty(B * rows, np.float32)
    lib().orc_pmat_batch(P(W), dtype, P(np.ascontiguousarray(xb, np.float32)), P(y), rows,
                         cols, B)
    return y
