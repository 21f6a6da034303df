"""Loader for the sm_100a kernel library ``_native/libh3sk_b200.so``.

There is no fallback: if the library is missing or does not export the
declared ABI, every op raises.  ``EXPORTS`` mirrors ``include/h3sk_b200.h``
one-to-one (the CPU test suite checks that every declared symbol is exported).
"""
from __future__ import annotations

import ctypes as ct
import threading
from pathlib import Path

NATIVE = Path(__file__).resolve().parent / "_native"
LIB_NAME = "libh3sk_b200.so"

_P, _I, _I64, _F, _SZ = ct.c_void_p, ct.c_int, ct.c_int64, ct.c_float, ct.c_size_t

# symbol -> (argtypes, restype); the order of include/h3sk_b200.h
EXPORTS = {
    "h3_norm_quant_abi": ([], _I),
    "h3_norm_quant_abi_ex": ([], _I),
    "h3_norm_quant_resources_size": ([], _SZ),
    "h3_norm_quant_error": ([_I], ct.c_char_p),
    "h3_norm_quant_query": ([_I, _I, _P, _SZ], _I),
    "h3_norm_quant_query_k": ([_I64, _I, _I, _P, _SZ], _I),
    "h3_norm_quant_run": ([_P] * 10 + [_I64] * 4 + [_F, _I, _I, _SZ], _I),
    "h3_norm_quant_run_k": ([_P] * 10 + [_I64] * 5 + [_F, _I, _I, _SZ], _I),
    "h3_norm_quant_run_t": ([_P] * 10 + [_I64] * 6 + [_F, _I, _I, _SZ], _I),
    "h3_residual_quant_abi": ([], _I),
    "h3_residual_quant_resources_size": ([], _SZ),
    "h3_residual_quant_error": ([_I], ct.c_char_p),
    "h3_residual_quant_query": ([_I, _I, _I, _P, _SZ], _I),
    "h3_residual_quant_query_k": ([_I64, _I, _I, _I, _P, _SZ], _I),
    "h3_residual_quant_run": ([_P] * 12 + [_I64] * 4 + [_F, _I, _I, _I, _SZ], _I),
    "h3_residual_quant_run_k": ([_P] * 12 + [_I64] * 5 + [_F, _I, _I, _I, _SZ], _I),
    "h3_residual_quant_run_t": ([_P] * 12 + [_I64] * 6 + [_F, _I, _I, _I, _SZ], _I),
    "h3_convrot_register_abi": ([], _I),
    "h3_convrot_register_resources_size": ([], _SZ),
    "h3_convrot_register_error": ([_I], ct.c_char_p),
    "h3_convrot_register_query": ([_I, _P, _SZ], _I),
    "h3_convrot_register_run": ([_P] * 4 + [_I64, _I, _I, _SZ], _I),
    "h3_convrot_quant_act": ([_P, _I64, _P, _P, _I64, _I, _I, _SZ], _I),
    "h3_convrot_codes": ([_P, _I64, _P, _P, _P, _I64, _I, _SZ], _I),
    "h3_int8": ([_P] * 5 + [_I] * 4 + [_SZ], _I),
    "h3_int8_gate": ([_P] * 8 + [_I] * 4 + [_SZ], _I),
    "h3_int8_ex": ([_P] * 6 + [_I] * 3 + [_I64, _I, _SZ], _I),
    "h3_int8_gate_ex": ([_P] * 11 + [_I] * 3 + [_SZ], _I),
    "h3_int8_gelu_rot": ([_P] * 7 + [_I] * 3 + [_I64, _SZ], _I),
    "h3_int8_rot": ([_P] * 7 + [_I] * 3 + [_I64, _I, _I, _SZ], _I),
    "h3_int8_last_error": ([], _I),
    "h3_int8_error": ([], ct.c_char_p),
    "h3_qkv_quant_kv": ([_P] * 8 + [_F] + [_P] * 7 + [_I, _SZ], _I),
    "h3_qkv_quant_kv_ex": ([_P] * 8 + [_F] + [_P] * 7 + [_I, _I, _I, _P, _SZ], _I),
    "h3_sample_konly": ([_P] * 8 + [_F] + [_P] * 3 + [_I, _SZ], _I),
    "h3_sample_konly_ex": ([_P] * 8 + [_F] + [_I, _I, _I, _P, _SZ], _I),
    "h3_sample_gather": ([_P] * 6 + [_I, _SZ], _I),
    "h3_sample_gather_ex": ([_P] * 6 + [_I, _I, _SZ], _I),
    "h3_sample_anchor": ([_P, _P, _SZ], _I),
    "h3_sample_anchor_ex": ([_P, _P, _I, _SZ], _I),
    "h3_quant_v": ([_P] * 5 + [_I, _I, _SZ], _I),
    "h3_qkv_noalloc": ([_P] * 8 + [_F] + [_P] * 7 + [_I, _I, _I, _SZ], _I),
    "h3_dense_args_size": ([], _SZ),
    "h3_dense_query_group": ([], _I),
    "h3_dense_error_string": ([_I], ct.c_char_p),
    "h3_dense_launch_window": ([_P, _SZ, ct.c_uint32], _I),
    "h3_dense_launch": ([_P, _SZ], _I),
    "h3_dense_resources": ([_P], _I),
    "h3sk_pipeline_status": ([_P, _I, _SZ], _I),
    "h3sk_wait_selftest": ([_I, _P, _SZ], _I),
    "h3sk_int8_mma_peak": ([_I, _P, _SZ], _I),
    "h3sk_ex2_peak": ([_I, _P, _SZ], _I),
    "h3sk_version": ([], ct.c_char_p),
}

_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return NATIVE / LIB_NAME


def load(path: Path | None = None) -> ct.CDLL:
    """Load the kernel library once and bind every exported symbol."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else library_path()
        if not target.exists():
            raise RuntimeError(
                f"H3 SpeedKit B200 kernel library not found at {target}; build it with "
                "`python comfyui-h3-speedkit_b200/csrc/build.py` (no CPU fallback exists)")
        so = ct.CDLL(str(target), mode=ct.RTLD_LOCAL)
        for name, (args, res) in EXPORTS.items():
            fn = getattr(so, name)
            fn.argtypes, fn.restype = args, res
        if so.h3_norm_quant_abi() != 1 or so.h3_norm_quant_abi_ex() != 2 or so.h3_convrot_register_abi() != 1:
            raise RuntimeError("H3 SpeedKit B200 C/ctypes ABI mismatch")
        if path is None:
            _lib = so
        return so


def check_int8(code: int) -> None:
    """GEMM entry points return 1 on success (runtime.py:68-71 convention)."""
    if code != 1:
        lib = load()
        raise RuntimeError("SpeedKit GEMM failed; the request is aborted, never retried after mutation: "
                           + lib.h3_int8_error().decode())


def pipeline_status(stream: int = 0, clear: bool = True) -> int:
    lib = load()
    value = ct.c_int(0)
    rc = lib.h3sk_pipeline_status(ct.byref(value), int(clear), stream)
    if rc:
        raise RuntimeError(f"h3sk_pipeline_status failed with CUDA error {rc}")
    return int(value.value)
