"""The reference's own CUDA kernels as the GPU oracle.  TEST INFRASTRUCTURE ONLY.

Loads the libraries ``oracle/build.py`` compiled into ``oracle/_ref`` from the
reference sources (norm_quant.cu, residual_quant.cu, convrot_register_v2.cu, the
vendored Kitchen quantiser, the K anchor detector, the sample-row gather, and the
CUTLASS GEMMs fc1.cu, gate.cu and r84_kfourwarp.cu, and the INT8 attention of
dense_ring.cu) and runs them on torch CUDA tensors.  Output buffers are
allocated by the caller-side helpers here with torch; nothing in the product
path uses this module.
"""
from __future__ import annotations

import ctypes as ct
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"
_CACHE: dict[str, ct.CDLL] = {}


def available(name: str) -> bool:
    return (REF / name).exists()


def _load(name: str) -> ct.CDLL:
    if name not in _CACHE:
        path = REF / name
        if not path.exists():
            raise FileNotFoundError(f"reference GPU oracle {path} is not built (run oracle/build.py)")
        _CACHE[name] = ct.CDLL(str(path), mode=ct.RTLD_LOCAL)
    return _CACHE[name]


def _stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def norm_widths() -> list[int]:
    return sorted(int(p.stem.split("_k")[1]) for p in REF.glob("ref_norm_k*.so"))


def norm_quant(x, w, shift, scale, rows, eps, *, debug=False):
    """Reference norm_quant_kernel (norm_quant.cu:122-213) at K = x.shape[1]."""
    import torch
    m, k = x.shape
    so = _load(f"ref_norm_k{k}.so")
    fn = so.h3_norm_quant_run
    fn.argtypes = [ct.c_void_p] * 10 + [ct.c_int64] * 4 + [ct.c_float, ct.c_int, ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    dev = x.device
    q = torch.empty((m, k), dtype=torch.int8, device=dev)
    qs = torch.empty((m, 1), dtype=torch.float32, device=dev)
    dn = torch.empty((m, k), dtype=torch.bfloat16, device=dev) if debug else None
    dr = torch.empty((m, k), dtype=torch.float32, device=dev) if debug else None
    drs = torch.empty((m,), dtype=torch.float32, device=dev) if debug else None
    ptrs = [t.data_ptr() if t is not None else None for t in (x, w, shift, scale, rows, q, qs, dn, dr, drs)]
    rc = fn(*ptrs, m, x.stride(0), shift.stride(0), scale.stride(0), float(eps),
            int(shift.dtype == torch.bfloat16), int(debug), _stream(x))
    if rc:
        raise RuntimeError(f"reference norm_quant failed with CUDA error {rc}")
    return (q, qs, dn, dr, drs) if debug else (q, qs)


def convrot_register(x, mode=0):
    """Reference register_rotate_quant (convrot_register_v2.cu:67-138), K in {5376, 7168}."""
    import torch
    m, k = x.shape
    so = _load("ref_convrot.so")
    fn = so.h3_convrot_register_run
    fn.argtypes = [ct.c_void_p] * 4 + [ct.c_int64, ct.c_int, ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    q = torch.empty((m, k), dtype=torch.int8, device=x.device) if mode != 2 else None
    sc = torch.empty((m, 1), dtype=torch.float32, device=x.device) if mode != 2 else None
    rot = torch.empty((m, k), dtype=torch.float32, device=x.device) if mode != 0 else None
    rc = fn(x.data_ptr(), q.data_ptr() if q is not None else None, sc.data_ptr() if sc is not None else None,
            rot.data_ptr() if rot is not None else None, m, k, mode, _stream(x))
    if rc:
        raise RuntimeError(f"reference convrot_register failed with CUDA error {rc}")
    return q, sc, rot


def kitchen_quant(x, act=0):
    """Reference Kitchen quantize_int8_rowwise_convrot64_kernel (convrot64_exact.cuh:942-1027)."""
    import torch
    m, width = x.shape
    k = width // 2 if act == 2 else width
    so = _load("ref_kitchen.so")
    fn = so.ref_kitchen_convrot64_quant
    fn.argtypes = [ct.c_void_p] * 3 + [ct.c_int64, ct.c_int, ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    sc = torch.empty((m,), dtype=torch.float32, device=x.device)
    rc = fn(x.data_ptr(), q.data_ptr(), sc.data_ptr(), m, k, act, _stream(x))
    if rc:
        raise RuntimeError(f"reference Kitchen quantiser failed with CUDA error {rc}")
    return q, sc


def residual_widths() -> list[int]:
    return sorted(int(p.stem.split("_k")[1]) for p in REF.glob("ref_residual_k*.so"))


def residual_quant(x, branch, w, gate, shift, scale, rows, eps, *, debug=False):
    """Reference residual_quant_kernel (residual_quant.cu:134-224) at K = x.shape[1]:
    x <- bf(fma(branch, bf(gate[rows]), x)) in place on a copy of ``x``, then the
    prologue on the updated rows.  Returns (x_new, q, qs[, dn, dr, drs])."""
    import torch
    m, k = x.shape
    so = _load(f"ref_residual_k{k}.so")
    fn = so.h3_residual_quant_run
    fn.argtypes = [ct.c_void_p] * 12 + [ct.c_int64] * 4 + [ct.c_float, ct.c_int, ct.c_int, ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    dev = x.device
    xn = x.clone()
    q = torch.empty((m, k), dtype=torch.int8, device=dev)
    qs = torch.empty((m, 1), dtype=torch.float32, device=dev)
    dn = torch.empty((m, k), dtype=torch.bfloat16, device=dev) if debug else None
    dr = torch.empty((m, k), dtype=torch.float32, device=dev) if debug else None
    drs = torch.empty((m,), dtype=torch.float32, device=dev) if debug else None
    ptrs = [t.data_ptr() if t is not None else None
            for t in (xn, branch, w, gate, shift, scale, rows, q, qs, dn, dr, drs)]
    rc = fn(*ptrs, m, gate.stride(0), shift.stride(0), scale.stride(0), float(eps),
            int(gate.dtype == torch.bfloat16), int(shift.dtype == torch.bfloat16), int(debug), _stream(x))
    if rc:
        raise RuntimeError(f"reference residual_quant failed with CUDA error {rc}")
    return (xn, q, qs, dn, dr, drs) if debug else (xn, q, qs)


def sample_anchor(k):
    """Reference h3_sample_anchor (r79_sample_anchor.cu:467-605, 700-702): the nine
    sampled keys k [56, 9, 128] BF16 -> int32 [56] anchor row (0..8) or -1."""
    import torch
    fn = _load("ref_anchor.so").h3_sample_anchor
    fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t]
    fn.restype = ct.c_int
    if tuple(k.shape) != (56, 9, 128) or not k.is_contiguous():
        raise ValueError("the reference detector is launched for 56 heads x 9 samples x 128")
    anchors = torch.empty((56,), dtype=torch.int32, device=k.device)
    if fn(k.data_ptr(), anchors.data_ptr(), _stream(k)) != 1:
        raise RuntimeError("reference h3_sample_anchor launch failed")
    return anchors


def sample_gather(q, xs, rope):
    """Reference h3_sample_gather (r82_sample_konly.cu:345-357): rows s*(m-1)//8 of
    q [m, 5376] INT8, xs [m, 1] FP32 and the RoPE table [m, 192] BF16."""
    import torch
    fn = _load("ref_gather.so").h3_sample_gather
    fn.argtypes = [ct.c_void_p] * 6 + [ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    m = q.shape[0]
    dev = q.device
    sq = torch.empty((9, 5376), dtype=torch.int8, device=dev)
    sx = torch.empty((9, 1), dtype=torch.float32, device=dev)
    sr = torch.empty((9, 192), dtype=torch.bfloat16, device=dev)
    if fn(q.data_ptr(), xs.data_ptr(), rope.data_ptr(), sq.data_ptr(), sx.data_ptr(), sr.data_ptr(), m,
          _stream(q)) != 1:
        raise RuntimeError("reference h3_sample_gather launch failed")
    return sq, sx, sr


def int8(a, b, xs, ws, *, config=3):
    """Reference h3_int8 (fc1.cu:119-138): D = bf(((acc * xs[m]) * ws[n]) + 0), the
    CUTLASS Sm80 INT8 GEMM; config 3 is the one the runtime uses (runtime.py:155-156)."""
    import torch
    fn = _load("ref_fc1.so").h3_int8
    fn.argtypes = [ct.c_void_p] * 5 + [ct.c_int] * 4 + [ct.c_size_t]
    fn.restype = ct.c_int
    m, k = a.shape
    n = b.shape[0]
    d = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if fn(a.data_ptr(), b.data_ptr(), xs.data_ptr(), ws.data_ptr(), d.data_ptr(), m, n, k, config,
          _stream(a)) != 1:
        raise RuntimeError(f"reference h3_int8 (config {config}) refused or failed")
    return d


def int8_gate(a, b, xs, ws, gate, rows, residual, *, config=13, out=None):
    """Reference h3_int8_gate (gate.cu:136-143): D = bf(fmaf(bf(acc*xs*ws + 0),
    gate[rows[m], n], residual[m, n])).  ``out`` may be ``residual`` itself (the
    runtime's in-place call, runtime.py:117-124); by default D is a new tensor."""
    import torch
    fn = _load("ref_gate.so").h3_int8_gate
    fn.argtypes = [ct.c_void_p] * 8 + [ct.c_int] * 4 + [ct.c_size_t]
    fn.restype = ct.c_int
    m, k = a.shape
    n = b.shape[0]
    d = torch.empty((m, n), dtype=torch.bfloat16, device=a.device) if out is None else out
    if fn(a.data_ptr(), b.data_ptr(), xs.data_ptr(), ws.data_ptr(), d.data_ptr(), gate.data_ptr(),
          rows.data_ptr(), residual.data_ptr(), m, n, k, config, _stream(a)) != 1:
        raise RuntimeError(f"reference h3_int8_gate (config {config}) refused or failed")
    return d


def qkv_quant_kv(a, b, xs, ws, freqs, qw, kw, eps, sk, anchors):
    """Reference h3_qkv_quant_kv (r84_kfourwarp.cu:213-388): the H3 QKV GEMM
    (56 heads x 128, hidden 5376) fused with per-head RMS, RoPE, the Q/K rotation
    and quantisation and the V tile maxima.  Returns dict d, qi, qs, ki, ks, vp
    in the layouts of the reference's own call (ops/qkv.py:63-69)."""
    import torch
    fn = _load("ref_qkv.so").h3_qkv_quant_kv
    fn.argtypes = [ct.c_void_p] * 8 + [ct.c_float] + [ct.c_void_p] * 7 + [ct.c_int, ct.c_size_t]
    fn.restype = ct.c_int
    m = a.shape[0]
    heads, dev = 56, a.device
    parts = (m + 127) // 128
    t = {"d": torch.empty((3, heads, m, 128), dtype=torch.bfloat16, device=dev),
         "qi": torch.empty((heads, m, 128), dtype=torch.int8, device=dev),
         "ki": torch.empty((heads, m, 128), dtype=torch.int8, device=dev),
         "qs": torch.empty((heads, parts * 32), dtype=torch.float32, device=dev),
         "ks": torch.empty((heads, parts * 4), dtype=torch.float32, device=dev),
         "vp": torch.empty((heads, parts, 128), dtype=torch.float32, device=dev)}
    if fn(a.data_ptr(), b.data_ptr(), xs.data_ptr(), ws.data_ptr(), t["d"].data_ptr(), freqs.data_ptr(),
          qw.data_ptr(), kw.data_ptr(), float(eps), t["qi"].data_ptr(), t["qs"].data_ptr(), t["vp"].data_ptr(),
          t["ki"].data_ptr(), t["ks"].data_ptr(), sk.data_ptr(), anchors.data_ptr(), m, _stream(a)) != 1:
        raise RuntimeError("reference h3_qkv_quant_kv refused or failed")
    return t


class DenseArgs(ct.Structure):
    """dense_ring.cu:16-24: seven pointers, seventeen uint32 sizes and strides, sm_scale."""
    _fields_ = ([(n, ct.c_void_p) for n in ("q", "k", "v", "o", "q_scale", "k_scale", "v_scale")]
                + [(n, ct.c_uint32) for n in ("batch", "qo_len", "kv_len", "qo_heads", "kv_heads",
                                               "q_stride_b", "q_stride_h", "q_stride_s",
                                               "k_stride_b", "k_stride_h", "k_stride_s",
                                               "v_stride_b", "v_stride_h", "v_stride_d",
                                               "o_stride_b", "o_stride_h", "o_stride_s")]
                + [("sm_scale", ct.c_float)])


def dense_args(q, k, v, qs, ks, vs, o, sm_scale):
    """The argument block for q [B, H, S, 128], k [B, Hk, Sk, 128], v [B*Hk*128, padded],
    o a BHSD-shaped view (BHSD or BSHD storage)."""
    b, h, s, d = q.shape
    hk, sk = k.shape[1:3]
    padded = v.shape[1]
    return DenseArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), qs.data_ptr(), ks.data_ptr(),
                     vs.data_ptr(), b, s, sk, h, hk, *q.stride()[:3], *k.stride()[:3],
                     hk * d * padded, d * padded, padded, *o.stride()[:3], float(sm_scale))


def dense(q, k, v, qs, ks, vs, sm_scale, *, layout="bshd", start=0):
    """Reference h3_dense_launch_window (dense_ring.cu:32-94): BF16 output, a BHSD view."""
    import torch
    so = _load("ref_dense.so")
    fn = so.h3_dense_launch_window
    fn.argtypes = [ct.POINTER(DenseArgs), ct.c_size_t, ct.c_uint32]
    fn.restype = ct.c_int
    b, h, s, d = q.shape
    if layout == "bshd":
        o = torch.empty((b, s, h, d), dtype=torch.bfloat16, device=q.device).transpose(1, 2)
    else:
        o = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=q.device)
    args = dense_args(q, k, v, qs, ks, vs, o, sm_scale)
    rc = fn(ct.byref(args), _stream(q), start)
    if rc:
        raise RuntimeError(f"reference h3_dense_launch_window failed with CUDA error {rc}")
    return o
