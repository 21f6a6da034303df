"""ctypes binding of the C restatement (``h3_oracle.c``).  TEST INFRASTRUCTURE ONLY.

BF16 arrays are carried as ``numpy.uint16`` bit patterns.  Each wrapper names
the reference lines its C function restates (see ``h3_oracle.c`` for the full
arithmetic and the documented departures: rsqrt, fast division, libm tanh/exp).
"""
from __future__ import annotations

import ctypes as ct
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None

_P = ct.c_void_p
_I64 = ct.c_int64


def lib():
    """Load ``libh3_oracle.so`` (building it with gcc when it is missing)."""
    global _LIB
    if _LIB is None:
        path = HERE / "libh3_oracle.so"
        if not path.exists():
            from oracle.build import build_c
            build_c()
        so = ct.CDLL(str(path))
        sig = {
            "h3o_quant_rows": ([_P, _I64, _I64, _P, _P, ct.c_int], None),
            "h3o_convrot_rows": ([_P, _I64, _I64, ct.c_int], None),
            "h3o_rms_variance": ([_P, _I64], ct.c_float),
            "h3o_norm_quant": ([_P, _I64, _P, _P, _P, ct.c_int, _I64, _I64, _P, _I64, _I64, ct.c_float,
                                _P, _P, _P, _P, _P, _P, ct.c_int], ct.c_int),
            "h3o_convrot_quant": ([_P, _I64, _I64, _I64, ct.c_int, _P, _P, _P, ct.c_int], ct.c_int),
            "h3o_gemm_s32": ([_P, _P, _I64, _I64, _I64, _P, ct.c_int], None),
            "h3o_dequant": ([_P, _P, _P, _P, _I64, _I64, ct.c_int, _P, _I64, ct.c_int], None),
            "h3o_gate": ([_P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _P, ct.c_int], None),
            "h3o_residual_update": ([_P, _P, _P, ct.c_int, _I64, _P, _I64, _I64, ct.c_int], ct.c_int),
            "h3o_max_threads": ([], ct.c_int),
        }
        for name, (args, res) in sig.items():
            fn = getattr(so, name)
            fn.argtypes, fn.restype = args, res
        _LIB = so
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def threads_default() -> int:
    return int(os.environ.get("H3SK_ORACLE_THREADS", "0"))


# ---- BF16 helpers -------------------------------------------------------------
def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (cvt.rn.bf16.f32)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- Restated functions ---------------------------------------------------------
def norm_quant(x, w, shift, scale, rows, eps, *, xs=None, rrms=None, debug=False, threads=None):
    """Fused prologue, kernels/norm_quant/norm_quant.cu:51-213.

    x uint16 [m, >=k] (BF16 bits), w uint16 [k], shift/scale [T, k] float32 or
    uint16, rows int32 [m].  ``rrms`` (float32 [m]) replaces the CPU rsqrt with
    given values (e.g. the GPU kernel's debug output).  Returns (q, qscale) or,
    with debug, (q, qscale, norm_bits, rotated, rstd).
    """
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m = x.shape[0]
    k = w.shape[0]
    xs = x.shape[1] if xs is None else xs
    table_dtype = 1 if shift.dtype == np.uint16 else 0
    shift = np.ascontiguousarray(shift)
    scale = np.ascontiguousarray(scale)
    if shift.dtype != scale.dtype or shift.dtype not in (np.uint16, np.float32):
        raise ValueError("shift/scale tables must both be float32 or both BF16 bits")
    rows = _c(rows, np.int32)
    w = _c(w, np.uint16)
    q = np.empty((m, k), np.int8)
    qs = np.empty((m,), np.float32)
    dn = np.empty((m, k), np.uint16) if debug else None
    dr = np.empty((m, k), np.float32) if debug else None
    drs = np.empty((m,), np.float32) if debug else None
    rr = None if rrms is None else _c(rrms, np.float32)
    rc = lib().h3o_norm_quant(_ptr(x), xs, _ptr(w), _ptr(shift), _ptr(scale), table_dtype, shift.shape[1],
                              scale.shape[1], _ptr(rows), m, k, float(eps), _ptr(rr), _ptr(q), _ptr(qs),
                              _ptr(dn), _ptr(dr), _ptr(drs), threads_default() if threads is None else threads)
    if rc:
        raise ValueError("oracle norm_quant rejected its arguments")
    return (q, qs, dn, dr, drs) if debug else (q, qs)


def residual_update(x, branch, gate, rows, *, threads=None) -> np.ndarray:
    """x <- bf(fma(branch, bf(gate[rows]), x)) (residual_quant.cu:59-78) on a copy.

    x, branch uint16 [m, k] (BF16 bits); gate [T, >=k] float32 or uint16."""
    x = np.array(x, dtype=np.uint16, copy=True, order="C")
    branch = _c(branch, np.uint16)
    gate = np.ascontiguousarray(gate)
    if gate.dtype not in (np.uint16, np.float32):
        raise ValueError("gate table must be float32 or BF16 bits")
    m, k = x.shape
    rc = lib().h3o_residual_update(_ptr(x), _ptr(branch), _ptr(gate), 1 if gate.dtype == np.uint16 else 0,
                                   gate.shape[1], _ptr(_c(rows, np.int32)), m, k,
                                   threads_default() if threads is None else threads)
    if rc:
        raise ValueError("oracle residual_update rejected its arguments")
    return x


def residual_quant(x, branch, w, gate, shift, scale, rows, eps, *, rrms=None, debug=False, threads=None):
    """Fused residual prologue, kernels/residual_quant/residual_quant.cu:59-224:
    the residual update, then the prologue on the updated rows.  Returns
    (x_new, q, qscale) or, with debug, (x_new, q, qscale, norm_bits, rotated, rstd)."""
    x_new = residual_update(x, branch, gate, rows, threads=threads)
    out = norm_quant(x_new, w, shift, scale, rows, eps, rrms=rrms, debug=debug, threads=threads)
    return (x_new,) + tuple(out)


def rms_variance(x_row) -> float:
    """The reference's RMS statistic for one BF16 row (norm_quant.cu:51-78)."""
    x_row = _c(x_row, np.uint16)
    return float(lib().h3o_rms_variance(_ptr(x_row), x_row.shape[0]))


def convrot_quant(x, k=None, act=0, *, rotated=False, quant=True, threads=None):
    """ConvRot256 + per-token INT8 with input act (convrot64_exact.cuh:913-1027).

    x uint16 [m, xs] BF16 bits; act 0 none, 1 GELU-tanh, 2 SwiGLU ([gate|up]).
    Returns (q, scale[, rotated]).
    """
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, xs = x.shape
    if k is None:
        k = xs // 2 if act == 2 else xs
    q = np.empty((m, k), np.int8) if quant else None
    sc = np.empty((m,), np.float32) if quant else None
    rot = np.empty((m, k), np.float32) if rotated else None
    rc = lib().h3o_convrot_quant(_ptr(x), xs, m, k, act, _ptr(q), _ptr(sc), _ptr(rot),
                                 threads_default() if threads is None else threads)
    if rc:
        raise ValueError("oracle convrot_quant rejected its arguments")
    out = (q, sc)
    return out + (rot,) if rotated else out


def convrot_rows(v, threads=None) -> np.ndarray:
    """ConvRot256 of FP32 rows (rotation only)."""
    v = np.array(v, dtype=np.float32, copy=True, order="C")
    lib().h3o_convrot_rows(_ptr(v), v.shape[0], v.shape[1], threads_default() if threads is None else threads)
    return v


def quant_rows(rot, threads=None):
    """Row scale + codes of already-rotated FP32 rows."""
    rot = _c(rot, np.float32)
    m, k = rot.shape
    q = np.empty((m, k), np.int8)
    sc = np.empty((m,), np.float32)
    lib().h3o_quant_rows(_ptr(rot), m, k, _ptr(q), _ptr(sc), threads_default() if threads is None else threads)
    return q, sc


def gemm_s32(a, b, *, use_torch=True, threads=None) -> np.ndarray:
    """Exact int32 A[M,K] . B[N,K]^T (fc1.cu:60-101).  torch._int_mm on CPU is
    exact and much faster; the C triple loop is the cross-check."""
    a = _c(a, np.int8)
    b = _c(b, np.int8)
    m, k = a.shape
    n = b.shape[0]
    if use_torch:
        import torch
        if m >= 17 and k % 8 == 0 and n % 8 == 0:
            return torch._int_mm(torch.from_numpy(a), torch.from_numpy(b).t()).numpy()
    c = np.empty((m, n), np.int32)
    lib().h3o_gemm_s32(_ptr(a), _ptr(b), m, n, k, _ptr(c), threads_default() if threads is None else threads)
    return c


def dequant(acc, xs, ws, bias=None, *, gelu=False, threads=None) -> np.ndarray:
    """bf(((acc*xs)*ws)+bias) [then bf(gelu)] -> BF16 bits (fc1.cu:83-90; r84:240-241)."""
    acc = _c(acc, np.int32)
    m, n = acc.shape
    out = np.empty((m, n), np.uint16)
    lib().h3o_dequant(_ptr(acc), _ptr(_c(xs, np.float32)), _ptr(_c(ws, np.float32)),
                      _ptr(None if bias is None else _c(bias, np.uint16)), m, n, int(gelu), _ptr(out), n,
                      threads_default() if threads is None else threads)
    return out


def gate_residual(acc, xs, ws, gate, rows, residual, bias=None, threads=None) -> np.ndarray:
    """bf(fmaf(bf(dequant), gate[rows[m]], residual)) -> BF16 bits (gate.cu:33-41, 100-104)."""
    acc = _c(acc, np.int32)
    m, n = acc.shape
    gate = _c(gate, np.uint16)
    out = np.empty((m, n), np.uint16)
    lib().h3o_gate(_ptr(acc), _ptr(_c(xs, np.float32)), _ptr(_c(ws, np.float32)),
                   _ptr(None if bias is None else _c(bias, np.uint16)), _ptr(gate), gate.shape[-1],
                   _ptr(_c(rows, np.int32)), _ptr(_c(residual, np.uint16)), m, n, _ptr(out),
                   threads_default() if threads is None else threads)
    return out


def max_threads() -> int:
    return int(lib().h3o_max_threads())
