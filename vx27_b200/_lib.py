"""ctypes binding of libvx27cuda.so (the C ABI declared in include/*.h).

The library is loaded from this package directory. It is the only compute path: if it
is missing the import fails loudly instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvx27cuda.so")

_f, _d, _i, _u64, _sz = C.c_float, C.c_double, C.c_int, C.c_uint64, C.c_size_t
_p, _fp, _dp, _ip, _cp = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_double), \
    C.POINTER(C.c_int), C.c_char_p

# name -> (restype, argtypes); every entry point of include/*.h
PROTOTYPES: dict[str, tuple] = {
    # vx27cuda.h
    "vx27cuda_version": (_i, []),
    "vx27cuda_last_error": (_cp, []),
    "vx27cuda_device_status": (_i, [_p, C.POINTER(C.c_uint32), _i, _cp, _sz]),
    "vx27cuda_num_sms": (_i, []),
    "vx27cuda_fill_normal": (_i, [_p, _sz, _i, _u64, _u64, _u64, _f, _f, _p, _cp, _sz]),
    "vx27cuda_fill_uniform": (_i, [_p, _sz, _u64, _u64, _f, _f, _p, _cp, _sz]),
    "vx27cuda_fill_int": (_i, [_p, _sz, _i, _p, _cp, _sz]),
    "vx27cuda_add_int": (_i, [_p, _sz, _i, _p, _cp, _sz]),
    # vx27_deltanet.h -- reference entry points
    "vx27_deltanet_state_per_layer": (_i, []),
    "vx27_deltanet_state_total": (_i, []),
    "vx27_deltanet_state_mb": (_d, [_i]),
    "vx27_deltanet_update_ref": (None, [_p, _p, _p, _f, _i]),
    "vx27_deltanet_retrieve_ref": (None, [_p, _p, _p, _i]),
    "vx27_deltanet_update_tiled": (None, [_p, _p, _p, _f, _i]),
    "vx27_deltanet_retrieve_tiled": (None, [_p, _p, _p, _i]),
    "vx27_deltanet_update_avx2": (None, [_p, _p, _p, _f, _i]),
    "vx27_deltanet_retrieve_avx2": (None, [_p, _p, _p, _i]),
    "vx27_deltanet_l2norm": (None, [_p, _p, _i]),
    "vx27_deltanet_step_exact": (None, [_p, _p, _p, _p, _d, _d, _p, _i]),
    "vx27_deltanet_gate_params": (None, [_d, _d, _d, _d, _dp, _dp]),
    "vx27_conv1d_step": (None, [_p, _p, _p, _p, _i, _i]),
    # vx27_deltanet.h -- batched tier
    "vx27_deltanet_decode_batch": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i,
                                        _i, _p, _cp, _sz]),
    "vx27_deltanet_decode_batch_gated": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                              _i, _i, _i, _i, _i, _p, _cp, _sz]),
    "vx27_deltanet_gate_params_dev": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p, _cp,
                                           _sz]),
    "vx27_deltanet_decode_tokens": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i,
                                         _i, _i, _i, _p, _cp, _sz]),
    "vx27_deltanet_prefill_workspace_size": (_sz, [_i, _i, _i, _i]),
    "vx27_deltanet_prefill_chunked": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _i, _i,
                                           _i, _i, _i, _p, _cp, _sz]),
    "vx27_deltanet_conv_import": (_i, [_p, _p, _p, _i, _i, _p, _cp, _sz]),
    "vx27_deltanet_conv_export": (_i, [_p, _p, _p, _i, _i, _p, _cp, _sz]),
    # vx27_gqa.h
    "vx27_gqa_kv_for_q": (_i, [_i]),
    "vx27_rmsnorm": (None, [_p, _p, _p, _i, _f]),
    "vx27_attn_1q": (None, [_p, _p, _p, _i, _p]),
    "vx27_gqa_append": (_i, [_p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _p, _i, _p, _i, _i, _i, _i,
                             _i, _f, _i, _p, _cp, _sz]),
    "vx27_gqa_append_grouped": (_i, [_p, _p, _p, _p, _p, _i, _p, _i, _p, _i, _p, _p, _i, _p, _i,
                                     _i, _i, _i, _i, _f, _i, _p, _cp, _sz]),
    "vx27_gqa_decode_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i]),
    "vx27_gqa_decode_batch": (_i, [_p, _p, _p, _p, _i, _p, _p, _p, _sz, _i, _i, _i, _i, _i, _i,
                                   _p, _cp, _sz]),
    "vx27_gqa_decode_plan": (_i, [_i, _i, _i, _i, _i, _sz, _i, _i, _ip, _ip]),
    "vx27_gqa_decode_fused": (_i, [_p, _p, _p, _p, _p, _p, _i, _p, _p, _p, _i, _p, _p, _p, _sz,
                                   _i, _i, _i, _i, _i, _f, _i, _i, _p, _cp, _sz]),
    "vx27_gqa_decode_batch_noalloc": (_i, [_p, _p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _i,
                                           _p, _cp, _sz]),
    "vx27_gqa_prefill_workspace_size": (_sz, [_i, _i, _i]),
    "vx27_gqa_prefill": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _p, _p, _i, _p, _p, _sz, _i, _i,
                              _i, _i, _i, _f, _i, _p, _cp, _sz]),
    "vx27_gqa_partial_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "vx27_gqa_partial": (_i, [_p, _p, _p, _i, _i, _i, _p, _i, _i, _i, _i, _p, _sz, _p, _cp,
                              _sz]),
    "vx27_gqa_combine": (_i, [_p, _i, _sz, _p, _p, _i, _i, _i, _i, _p, _cp, _sz]),
    # vx27_pmat.h
    "vx27_pmat_row_bytes": (_sz, [C.c_uint32, _i]),
    "vx27_pmat_batch_dev": (_i, [_p, C.c_uint32, _p, _p, _i, _i, _i, _p, _cp, _sz]),
    "vx27_pmat_multi_dev": (_i, [_i, _p, C.c_uint32, _p, _p, _p, _i, _i, _p, _cp, _sz]),
    # vx27_kv.h
    "vx27_kv_elems": (_u64, [_i]),
    "vx27_kv_gb": (_d, [_i, _d]),
    "vx27_kv_fits": (_i, [_i, _d, _d]),
    "vx27_kv_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "vx27_kv_create": (_i, [C.POINTER(_p), _i, _i, _i, _i, _i, _cp, _sz]),
    "vx27_kv_destroy": (None, [_p]),
    "vx27_kv_layer": (_i, [_p, _i, C.POINTER(_p), C.POINTER(_p)]),
    "vx27_kv_capacity": (_i, [_p]),
    "vx27_kv_store_f32": (_i, [_p, _i, _i, _i, _i, _p, _p, _cp, _sz]),
    "vx27_kv_load_f32": (_i, [_p, _i, _i, _i, _i, _p, _p, _cp, _sz]),
    # vx27_rope.h
    "vx27_rope_cos_sin": (None, [_i, _p, _p, _i, _f, _f]),
    "vx27_rope_apply": (None, [_p, _i, _i, _i, _p, _p]),
    "vx27_mrope_cos_sin_text": (None, [_i, _p, _p]),
    "vx27_rope_table_build": (_i, [_p, _i, _i, _f, _f, _cp, _sz]),
}

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Loads libvx27cuda.so (building it first if it is absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        _build.build()
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libvx27cuda.so not found at {LIB_PATH}")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class Vx27Error(RuntimeError):
    pass


def check(rc: int, err: C.Array) -> None:
    if rc != 0:
        raise Vx27Error(err.value.decode(errors="replace") or "libvx27cuda call failed")


def errbuf() -> C.Array:
    return C.create_string_buffer(512)
