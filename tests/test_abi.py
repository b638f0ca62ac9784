"""C-ABI checks that need no GPU: the library loads, exports every entry point that
include/*.h declares, and its host-side entry points (sizing, gate mapping, head map,
RoPE tables) are bit-identical to the reference's golden vectors."""
import ctypes as C
import glob
import os
import re
import subprocess

import numpy as np

from conftest import ROOT


def header_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(vx27\w*)\s*\(", src, flags=re.M):
            syms.add(m.group(1))
    return syms


def test_every_declared_symbol_is_exported(vxlib):
    from vx27_b200 import _lib
    syms = header_symbols()
    assert len(syms) > 40
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = sorted(syms - exported)
    assert not missing, missing
    # the ctypes prototype table covers the whole ABI
    assert syms == set(_lib.PROTOTYPES), sorted(syms ^ set(_lib.PROTOTYPES))


def test_reference_signatures_match_reference_headers():
    """Every reference entry point keeps its reference signature (parsed from the copy of
    the prototypes in the reference headers' own order, declared in include/)."""
    ref = {
        "vx27_deltanet_update_ref": "void(float*,const float*,const float*,float,int)",
        "vx27_deltanet_retrieve_ref": "void(const float*,const float*,float*,int)",
        "vx27_deltanet_step_exact":
            "void(float*,const float*,const float*,const float*,double,double,float*,int)",
        "vx27_deltanet_gate_params": "void(double,double,double,double,double*,double*)",
        "vx27_conv1d_step": "void(float*,const float*,const float*,float*,int,int)",
        "vx27_rmsnorm": "void(const float*,const float*,float*,int,float)",
        "vx27_attn_1q": "void(const float*,const float*,const float*,int,float*)",
        "vx27_rope_cos_sin": "void(int,float*,float*,int,float,float)",
        "vx27_rope_apply": "void(float*,int,int,int,const float*,const float*)",
        "vx27_kv_elems": "uint64_t(int)",
    }
    text = " ".join(re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
                    for h in glob.glob(os.path.join(ROOT, "include", "*.h")))
    for name, sig in ref.items():
        m = re.search(r"([\w]+)\s+\*?\s*" + name + r"\s*\(([^)]*)\)", text)
        assert m, name
        params = [re.sub(r"\s*\b\w+$", "", p.strip()) for p in m.group(2).split(",")]
        params = [re.sub(r"\s*\*\s*", "*", re.sub(r"\s+", " ", p)) for p in params]
        got = m.group(1) + "(" + ",".join(params) + ")"
        assert got == sig, (name, got)


def test_host_entry_points_bit_exact(vxlib, golden):
    L = vxlib
    for (a, al, b, dt), (be_ref, g_ref) in zip(golden["gate_in"], golden["gate_out"]):
        be, gg = C.c_double(), C.c_double()
        L.vx27_deltanet_gate_params(a, al, b, dt, C.byref(be), C.byref(gg))
        assert be.value == be_ref and gg.value == g_ref
    assert [L.vx27_gqa_kv_for_q(h) for h in range(24)] == list(golden["headmap"])
    for c, e, g in zip(golden["kv_ctx"], golden["kv_elems"], golden["kv_gb"]):
        assert L.vx27_kv_elems(int(c)) == int(e) and L.vx27_kv_gb(int(c), 2.0) == g
    fits = [L.vx27_kv_fits(int(c), b_, 2.5) for c in golden["kv_ctx"] for b_ in (0.5, 2.0)]
    assert fits == list(golden["kv_fits"])
    assert [L.vx27_deltanet_state_per_layer(), L.vx27_deltanet_state_total()] == \
        list(golden["sizes"])
    assert [L.vx27_deltanet_state_mb(2), L.vx27_deltanet_state_mb(4)] == list(golden["state_mb"])
    for n, (p, yf) in enumerate(zip(golden["rope_pos"], golden["rope_yarn"])):
        c, s = np.zeros(32, np.float32), np.zeros(32, np.float32)
        L.vx27_rope_cos_sin(int(p), c.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p),
                            64, 1e7, float(yf))
        assert np.array_equal(c, golden["rope_cos"][n]) and np.array_equal(s, golden["rope_sin"][n])
    c, s = np.zeros(32, np.float32), np.zeros(32, np.float32)
    L.vx27_mrope_cos_sin_text(7, c.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p))
    c2, s2 = np.zeros(32, np.float32), np.zeros(32, np.float32)
    L.vx27_rope_cos_sin(7, c2.ctypes.data_as(C.c_void_p), s2.ctypes.data_as(C.c_void_p), 64, 1e7, 1.0)
    assert np.array_equal(c, c2) and np.array_equal(s, s2)


def test_batched_entry_points_reject_bad_shapes_without_gpu(vxlib):
    """Argument validation happens on the host, before any CUDA call."""
    err = C.create_string_buffer(256)
    rc = vxlib.vx27_deltanet_decode_batch(None, None, None, None, None, None, None, None, None,
                                          None, 1, 16, 16, 64, 0, None, err, 256)
    assert rc == -1 and b"hd=64" in err.value
    rc = vxlib.vx27_gqa_decode_batch(None, None, None, None, 16, None, None, None, 0, 1, 24, 5,
                                     256, 0, 0, None, err, 256)
    assert rc == -1 and b"bad shape" in err.value
    assert vxlib.vx27_gqa_decode_workspace_size(2, 24, 4, 256, 4096, 3) == 3 * 2 * 24 * 258 * 4
    rc = vxlib.vx27_pmat_multi_dev(5, None, 4, None, None, None, 128, 1, None, err, 256)
    assert rc == -1 and b"n=5 projections" in err.value
    # the fused decode on the tensor cores: a RoPE width that 8-dim lanes cannot pair up;
    # on the CUDA cores (one thread per dim): an odd one (checked before any CUDA call; the
    # pointers are never dereferenced)
    rec = 1 * 24 * 258 * 4
    rc = vxlib.vx27_gqa_decode_fused(16, 16, 16, 16, 16, 16, 64, None, 16, 16, 64, 16, 16, 16, rec,
                                     1, 24, 4, 256, 20, 1e-6, 1, 0x100, None, err, 256)
    assert rc == -1 and b"rope_dim=20" in err.value
    rc = vxlib.vx27_gqa_decode_fused(16, 16, 16, 16, 16, 16, 64, None, 16, 16, 64, 16, 16, 16, rec,
                                     1, 24, 4, 256, 21, 1e-6, 1, 0x80, None, err, 256)
    assert rc == -1 and b"rope_dim=21" in err.value
    # the multi-token DeltaNet decode: the pre-normalisation needs the gated entry point
    rc = vxlib.vx27_deltanet_decode_tokens(16, 16, 16, 16, 16, 16, 16, 16, 16, 16, None, None,
                                           4, 16, 16, 128, 0x20, None, err, 256)
    assert rc == -1 and b"VX27_F_QK_PRENORM" in err.value
    rc = vxlib.vx27_deltanet_decode_tokens(None, 16, 16, 16, 16, 16, 16, 16, 16, 16, None, None,
                                           4, 16, 16, 128, 0, None, err, 256)
    assert rc == -1 and b"null pointer" in err.value
    # the combine reads each record's (m, l) as 8-byte pairs: an odd record stride or an
    # unaligned parts pointer is refused before any launch
    P = C.c_void_p
    rc = vxlib.vx27_gqa_combine(P(16), 2, C.c_size_t(rec // 4 + 1), None, P(16), 1, 24, 256, 0,
                                None, err, 256)
    assert rc == -1 and b"part_stride even" in err.value
    rc = vxlib.vx27_gqa_combine(P(20), 2, C.c_size_t(0), None, P(16), 1, 24, 256, 0, None, err,
                                256)
    assert rc == -1 and b"8-byte aligned" in err.value


def test_flag_values_match_the_header():
    """The Python wrappers' flag constants are the values include/vx27cuda.h defines."""
    import os
    import re
    from vx27_b200 import ops
    hdr = open(os.path.join(os.path.dirname(__file__), "..", "include", "vx27cuda.h")).read()
    defs = {m.group(1): int(m.group(2), 16)
            for m in re.finditer(r"#define VX27_(F_\w+)\s+(0x[0-9a-fA-F]+)", hdr)}
    assert {"F_ACT_BF16", "F_OUT_BF16", "F_PREFETCH_KV", "F_DECODE_CC", "F_DECODE_TC",
            "F_PREFILL_CTA1"} <= defs.keys()
    for name, value in defs.items():
        if hasattr(ops, name):
            assert getattr(ops, name) == value, name


def test_ddmath_host_matches_c_library_nearly_always():
    """The correctly rounded exp/log used for device-side gates (csrc/ddmath.h), compiled
    for the host: agreement with the C library on seeded inputs, and the listed
    disagreements are C-library misroundings (checked against 60-digit arithmetic)."""
    src = os.path.join(ROOT, "tests", "ddmath_check.c")
    exe = os.path.join(ROOT, "vx27_b200", "_build", "ddmath_check")
    os.makedirs(os.path.dirname(exe), exist_ok=True)
    subprocess.run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-I",
                    os.path.join(ROOT, "vx27_b200", "csrc"), "-o", exe, src, "-lm"], check=True)
    out = subprocess.run([exe, "200000"], capture_output=True, text=True, check=True).stdout
    stats = dict(line.split("=") for line in out.split() if "=" in line)
    n = int(stats["n"])
    # the C library misrounds exp/log on a small fraction of inputs; ddmath does not
    assert int(stats["gate_mismatch"]) < 0.01 * n
    from decimal import Decimal, getcontext
    from fractions import Fraction
    getcontext().prec = 60
    for line in out.splitlines():
        if line.startswith("exp "):
            _, x, mine, libc = line.split()
            exact = Decimal(float.fromhex(x)).exp()  # Decimal(float) is exact
            assert float(Fraction(exact)).hex() == float.fromhex(mine).hex()
        elif line.startswith("log "):
            _, x, mine, libc = line.split()
            exact = Decimal(float.fromhex(x)).ln()
            assert float(Fraction(exact)).hex() == float.fromhex(mine).hex()


def test_wrappers_reject_wrong_dtypes_and_sizes_before_any_launch():
    """The Python wrappers check dtype, size and device of every tensor before its pointer
    reaches a kernel (which would otherwise read or write past it). CPU tensors here: the
    checks run first or _t() rejects the host tensor, so nothing is launched."""
    import pytest
    import torch
    from vx27_b200 import ops
    B, nq, nkv, hd, cap = 2, 24, 4, 256, 64
    q = torch.zeros(B, nq, hd)
    kc = torch.zeros(B, nkv, cap, hd, dtype=torch.bfloat16)
    pos = torch.zeros(B, dtype=torch.int32)
    out = torch.zeros(B, nq, hd)
    ws = torch.zeros(16)
    with pytest.raises(ops.Vx27Error, match="k_cache: dtype"):
        ops.gqa_decode_batch(q, None, kc.float(), kc, pos, out, ws)
    with pytest.raises(ops.Vx27Error, match="pos: dtype"):
        ops.gqa_decode_batch(q, None, kc, kc, pos.long(), out, ws)
    with pytest.raises(ops.Vx27Error, match="out: .* elements"):
        ops.gqa_decode_batch(q, None, kc, kc, pos, out[:1], ws)
    nqk = nv = 16
    C_ = (2 * nqk + nv) * 128
    S = torch.zeros(B, nv, 128, 128)
    ring = torch.zeros(B, 4, C_)
    qkv = torch.zeros(B, C_, dtype=torch.float16)  # neither fp32 nor bf16
    a = torch.zeros(B, nv)
    with pytest.raises(ops.Vx27Error, match="qkv: dtype"):
        ops.deltanet_decode_batch(S, ring, qkv, a, a, torch.zeros(nv), torch.zeros(nv),
                                  torch.zeros(C_, 4), pos, torch.zeros(B, nv, 128), nqk, nv)
    with pytest.raises(ops.Vx27Error, match="expected a contiguous CUDA tensor"):
        ops.deltanet_decode_batch(S, ring, qkv.float(), a, a, torch.zeros(nv), torch.zeros(nv),
                                  torch.zeros(C_, 4), pos, torch.zeros(B, nv, 128), nqk, nv)
    # the fused GQA decode: activations of one dtype, caches bf16
    q_in = torch.zeros(B, nq, hd, dtype=torch.bfloat16)
    kv_in = torch.zeros(B, nkv, hd, dtype=torch.bfloat16)
    w = torch.zeros(hd)
    rope = torch.zeros(cap, 64)
    with pytest.raises(ops.Vx27Error, match="k_in: dtype"):
        ops.gqa_decode_fused(q_in, kv_in.float(), kv_in, w, w, rope, q_in, kc, kc, pos, out, ws)
    with pytest.raises(ops.Vx27Error, match="gate: dtype"):
        ops.gqa_decode_fused(q_in, kv_in, kv_in, w, w, rope, q_in.float(), kc, kc, pos, out, ws)
    with pytest.raises(ops.Vx27Error, match="v_cache: .* elements"):
        ops.gqa_decode_fused(q_in, kv_in, kv_in, w, w, rope, q_in, kc, kc[:1], pos, out, ws)
    # grouped projections: one output and one row count per weight set, at most four
    x = torch.zeros(B, 1024)
    Wb = torch.zeros(10 * 8 * 52, dtype=torch.uint8)
    y = torch.zeros(B, 10)
    with pytest.raises(ops.Vx27Error, match="1..4 projections"):
        ops.pmat_multi([Wb] * 5, ops.PMAT_BP3_128, x, [y] * 5, [10] * 5, 1024)
    with pytest.raises(ops.Vx27Error, match="1..4 projections"):
        ops.pmat_multi([Wb, Wb], ops.PMAT_BP3_128, x, [y], [10, 10], 1024)
    with pytest.raises(ops.Vx27Error, match="fewer than 11 packed rows"):
        ops.pmat_multi([Wb], ops.PMAT_BP3_128, x, [torch.zeros(B, 11)], [11], 1024)
    with pytest.raises(ops.Vx27Error, match=r"y\[0\]: .* elements"):
        ops.pmat_multi([Wb], ops.PMAT_BP3_128, x, [y[:1]], [10], 1024)
