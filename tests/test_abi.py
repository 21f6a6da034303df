"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects invalid arguments on the host before launching anything.

Mirrors the reference's host-side contract checks (norm_quant.cu:247-255,
convrot_register_v2.cu:202-205, runtime.py:68-71 for the 1/0 GEMM convention).
"""
import ctypes as ct
import re
from pathlib import Path

import pytest

from h3_speedkit import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "h3sk_b200.h"
INVALID = 1   # cudaErrorInvalidValue


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(h3[a-z0-9_]*)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/h3sk_b200.h but not exported"
    assert set(names) == set(_lib.EXPORTS), "the ctypes table and the header must list the same symbols"


def test_manifest_and_aliases():
    import json
    native = _lib.NATIVE
    manifest = json.loads((native / "build.json").read_text())
    assert manifest["schema"] == 1
    for name in ("norm", "residual", "convrot", "fc1", "gate", "qkv", "sample", "anchor"):
        alias = native / f"{name}.so"
        assert alias.exists() and alias.resolve() == (native / _lib.LIB_NAME).resolve()
        assert manifest["kernels"][name]["sha256"]


def test_abi_versions_and_resource_sizes():
    lib = _lib.load()
    assert lib.h3_norm_quant_abi() == 1 and lib.h3_norm_quant_abi_ex() == 2
    assert lib.h3_convrot_register_abi() == 1
    assert lib.h3_norm_quant_resources_size() == 13 * 8
    assert lib.h3_residual_quant_abi() == 1 and lib.h3_residual_quant_resources_size() == 13 * 8
    assert lib.h3_convrot_register_resources_size() == 14 * 8
    assert b"sm_100a" in lib.h3sk_version()
    assert lib.h3_norm_quant_error(INVALID)


def _nq(lib, **kw):
    args = dict(x=16, w=16, shift=16, scale=16, rows=16, q=16, qscale=16, dn=None, dr=None, drs=None,
                m=4, xs=5376, ss=5376, cs=5376, eps=1e-6, table_dtype=1, debug=0)
    args.update(kw)
    return lib.h3_norm_quant_run(args["x"], args["w"], args["shift"], args["scale"], args["rows"], args["q"],
                                 args["qscale"], args["dn"], args["dr"], args["drs"], args["m"], args["xs"],
                                 args["ss"], args["cs"], ct.c_float(args["eps"]), args["table_dtype"],
                                 args["debug"], 0)


@pytest.mark.parametrize("bad", [dict(x=None), dict(m=0), dict(m=2**31), dict(xs=5375), dict(xs=5378),
                                 dict(ss=100), dict(eps=0.0), dict(eps=float("nan")), dict(eps=1e-45),
                                 dict(table_dtype=2), dict(debug=1), dict(dn=16), dict(x=12),
                                 dict(q=4), dict(qscale=2), dict(shift=1)])
def test_norm_quant_rejects_before_launch(bad):
    """Every invalid argument is caught on the host (no device memory is touched:
    the pointers here are fake and a launch would fault)."""
    assert _nq(_lib.load(), **bad) == INVALID


def test_norm_quant_k_variant_rejects_bad_widths():
    lib = _lib.load()
    for k in (0, 128, 300, 16640):
        rc = lib.h3_norm_quant_run_k(16, 16, 16, 16, 16, 16, 16, None, None, None, 4, k, k, k, k,
                                     ct.c_float(1e-6), 1, 0, 0)
        assert rc == INVALID


@pytest.mark.parametrize("args", [
    (None, 16, 16, None, 4, 4096, 0), (16, 16, 16, None, 0, 4096, 0), (16, 16, 16, None, 4, 4000, 0),
    (16, None, 16, None, 4, 4096, 0), (16, 16, 16, None, 4, 4096, 1), (8, 16, 16, None, 4, 4096, 0),
    (16, 12, 16, None, 4, 4096, 0), (16, 16, 16, None, 4, 4096, 3), (16, 16, 16, None, 4, 20000, 0)])
def test_convrot_register_rejects_before_launch(args):
    x, q, scale, rotated, rows, k, mode = args
    assert _lib.load().h3_convrot_register_run(x, q, scale, rotated, rows, k, mode, 0) == INVALID


def test_convrot_act_rejects_before_launch():
    lib = _lib.load()
    assert lib.h3_convrot_quant_act(16, 4096, 16, 16, 4, 4096, 3, 0) == INVALID        # act
    assert lib.h3_convrot_quant_act(16, 4096, 16, 16, 4, 4096, 2, 0) == INVALID        # SwiGLU needs xs >= 2k
    assert lib.h3_convrot_quant_act(16, 4100, 16, 16, 4, 4096, 0, 0) == INVALID        # xs % 8
    assert lib.h3_convrot_quant_act(8, 4096, 16, 16, 4, 4096, 0, 0) == INVALID         # 16-byte x


def test_rotating_gemm_and_codes_entry_points_reject_before_launch():
    """h3_int8_gelu_rot and h3_convrot_codes check their operands before any CUDA
    call (and before the row maxima are reset)."""
    lib = _lib.load()
    #                       A   B   xs  ws  bias  V  rowmax  M    N    K    ldv
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 16, None, 128, 256, 128, 256, 0) == 0    # no rowmax
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 16, 18, 128, 256, 128, 256, 0) == 0      # rowmax % 4
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 16, 16, 128, 264, 128, 264, 0) == 0      # N % 256
    assert b"256" in lib.h3_int8_error()
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 16, 16, 128, 256, 100, 256, 0) == 0      # K % 16
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 8, 16, 128, 256, 128, 256, 0) == 0       # 16-byte V
    assert lib.h3_int8_gelu_rot(16, 16, 16, 16, None, 16, 16, 128, 256, 128, 200, 0) == 0      # ldv < N
    #                  A   B   xs  ws  bias D  rowmax M    N    K    ldd  gelu rot_n0
    assert lib.h3_int8_rot(16, 16, 16, 16, None, 16, 16, 128, 768, 128, 768, 0, 100, 0) == 0   # rot_n0 % 256
    assert lib.h3_int8_rot(16, 16, 16, 16, None, 16, 16, 128, 768, 128, 768, 0, 768, 0) == 0   # rot_n0 >= N
    assert lib.h3_int8_rot(16, 16, 16, 16, None, 16, 16, 128, 768, 128, 768, 2, 512, 0) == 0   # gelu 0 / 1
    assert lib.h3_int8_rot(16, 16, 16, 16, None, 16, None, 128, 768, 128, 768, 0, 512, 0) == 0  # no rowmax
    #                       v   vs    rowmax q   scale rows k
    assert lib.h3_convrot_codes(16, 4096, 16, 16, 16, 4, 4000, 0) == INVALID    # k % 256
    assert lib.h3_convrot_codes(16, 4096, 16, 16, 16, 4, 32768, 0) == INVALID   # k > 16384
    assert lib.h3_convrot_codes(16, 4000, 16, 16, 16, 4, 4096, 0) == INVALID    # vs < k
    assert lib.h3_convrot_codes(16, 4100, 16, 16, 16, 4, 4096, 0) == INVALID    # vs % 8
    assert lib.h3_convrot_codes(8, 4096, 16, 16, 16, 4, 4096, 0) == INVALID     # 16-byte v
    assert lib.h3_convrot_codes(16, 4096, 16, 8, 16, 4, 4096, 0) == INVALID     # 16-byte q
    assert lib.h3_convrot_codes(16, 4096, 18, 16, 16, 4, 4096, 0) == INVALID    # rowmax % 4
    assert lib.h3_convrot_codes(16, 4096, None, 16, 16, 4, 4096, 0) == INVALID  # no rowmax
    assert lib.h3_convrot_codes(16, 4096, 16, 16, 16, 0, 4096, 0) == INVALID    # rows < 1


def test_gemm_returns_zero_with_a_reason():
    lib = _lib.load()
    # K % 16 != 0
    assert lib.h3_int8(16, 16, 16, 16, 16, 128, 256, 100, 3, 0) == 0
    assert lib.h3_int8_last_error() == INVALID
    assert b"invalid" in lib.h3_int8_error().lower()
    # N % 8 != 0, null operand, misaligned D, config out of range
    assert lib.h3_int8(16, 16, 16, 16, 16, 128, 250, 128, 3, 0) == 0
    assert lib.h3_int8(None, 16, 16, 16, 16, 128, 256, 128, 3, 0) == 0
    assert lib.h3_int8(16, 16, 16, 16, 8, 128, 256, 128, 3, 0) == 0
    assert lib.h3_int8(16, 16, 16, 16, 16, 128, 256, 128, 99, 0) == 0
    # gate without a residual / rows
    assert lib.h3_int8_gate(16, 16, 16, 16, 16, 16, None, 16, 128, 256, 128, 13, 0) == 0
    # extended forms
    assert lib.h3_int8_ex(16, 16, 16, 16, None, 16, 128, 256, 128, 200, 0, 0) == 0   # ldd < N
    assert lib.h3_int8_ex(16, 16, 16, 16, None, 16, 128, 256, 128, 256, 7, 0) == 0   # epilogue
    assert lib.h3_int8_gate_ex(16, 16, 16, 16, None, 16, 16, 16, 16, 16, None, 128, 256, 128, 0) == 0
    assert lib.h3_int8_gate_ex(16, 16, 16, 16, None, 16, 16, 16, 16, 16, 16, 128, 200, 128, 0) == 0


def test_diagnostics_reject_bad_arguments():
    lib = _lib.load()
    status = ct.c_int(0)
    assert lib.h3sk_wait_selftest(0, ct.byref(status), 0) == INVALID
    assert lib.h3sk_wait_selftest(10, None, 0) == INVALID
    tops = ct.c_double(0)
    assert lib.h3sk_int8_mma_peak(1, ct.byref(tops), 0) == INVALID
    assert lib.h3sk_pipeline_status(None, 0, 0) == INVALID


def _qkv(lib, **kw):
    args = dict(A=16, B=16, xs=16, ws=16, D=16, freqs=16, qw=16, kw=16, eps=1e-6, QI=16, QS=16, VP=16, KI=16,
                KS=16, SK=16, anchors=16, M=4)
    args.update(kw)
    return lib.h3_qkv_quant_kv(*(args[k] for k in ("A", "B", "xs", "ws", "D", "freqs", "qw", "kw")),
                               ct.c_float(args["eps"]),
                               *(args[k] for k in ("QI", "QS", "VP", "KI", "KS", "SK", "anchors", "M")), 0)


@pytest.mark.parametrize("bad", [dict(A=None), dict(D=None), dict(M=0), dict(M=200001), dict(D=8),
                                 dict(QI=None), dict(KS=None), dict(QI=18), dict(SK=None),
                                 dict(eps=float("nan")), dict(eps=-1.0)])
def test_qkv_rejects_before_launch(bad):
    """h3_qkv_quant_kv keeps the reference's 1 / 0 convention (r84_kfourwarp.cu:385-388)
    and rejects on the host: null operands, M outside [1, 200000] (the reference's
    bound), a D that a TMA store cannot address, SK without anchors."""
    lib = _lib.load()
    assert _qkv(lib, **bad) == 0
    assert lib.h3_int8_last_error() == INVALID and lib.h3_int8_error()


def test_qkv_sample_entry_points_reject_before_launch():
    lib = _lib.load()
    eps = ct.c_float(1e-6)
    # the reference's h3_sample_konly accepts M == 9 only (r82_sample_konly.cu:339)
    assert lib.h3_sample_konly(16, 16, 16, 16, 16, 16, 16, 16, eps, None, None, None, 8, 0) == 0
    assert lib.h3_sample_konly_ex(16, 16, 16, 16, 16, 16, 16, 16, eps, 9, 56, 5370, None, 0) == 0
    assert lib.h3_sample_gather(16, 16, 16, 16, 16, 16, 0, 0) == 0
    assert lib.h3_sample_gather(16, 18, 16, 16, 16, 16, 9, 0) == 0
    assert lib.h3_sample_anchor_ex(16, 16, 0, 0) == 0
    assert lib.h3_sample_anchor_ex(17, 16, 56, 0) == 0
    assert lib.h3_quant_v(16, 16, 16, 16, 16, 0, 56, 0) == 0
    assert lib.h3_quant_v(16, 8, 16, 16, 16, 9, 56, 0) == 0
