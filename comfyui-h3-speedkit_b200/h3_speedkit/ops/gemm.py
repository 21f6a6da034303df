"""Current-stream bindings of the tcgen05 INT8 GEMMs (B200).

The reference calls the C symbols ``h3_int8`` / ``h3_int8_gate`` directly from
``Backend`` (runtime.py:61-66, 117-124, 150-157); the same symbols are exported
by libh3sk_b200.so with the same argument order and 1-on-success convention.
These helpers add host-side validation (before anything is enqueued) and the
extended forms: bias, GELU epilogue, raw int32 accumulators, requantised copy
of a gate-residual output.

Layouts: A INT8 [M, K] row-major (the quantised activation), W INT8 [N, K]
row-major (per-output-channel rows, i.e. K-major), xs FP32 [M] or [M, 1],
ws FP32 [N].
"""
from __future__ import annotations

import torch

from .. import _lib

EPI_DEQUANT, EPI_GELU, EPI_ACC = 0, 1, 3


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_operands(a, w, xs, ws):
    if a.dtype != torch.int8 or w.dtype != torch.int8 or a.ndim != 2 or w.ndim != 2:
        raise ValueError('A and W must be INT8 matrices')
    m, k = a.shape
    n, kw = w.shape
    if kw != k or k % 16 or n % 8 or m < 1:
        raise ValueError(f'Unsupported GEMM geometry M={m} N={n} K={k} (K % 16 == 0, N % 8 == 0)')
    for name, t in (('A', a), ('W', w)):
        if not t.is_cuda or not t.is_contiguous() or t.data_ptr() % 16:
            raise ValueError(f'{name} must be a contiguous, 16-byte aligned CUDA tensor')
    if xs is not None:
        if xs.dtype != torch.float32 or xs.numel() != m or not xs.is_contiguous():
            raise ValueError('xs must be contiguous FP32 with M elements')
        if ws.dtype != torch.float32 or ws.numel() != n or not ws.is_contiguous():
            raise ValueError('ws must be contiguous FP32 with N elements')
    if any(t.device != a.device for t in (w,) + tuple(t for t in (xs, ws) if t is not None)):
        raise ValueError('All operands must be on one CUDA device')
    return m, n, k


def int8_linear(a, w, xs, ws, *, bias=None, gelu=False, out=None):
    """BF16 [M, N] = bf(((A.W^T * xs) * ws) + bias) [then bf(gelu_tanh)]."""
    m, n, k = _check_operands(a, w, xs, ws)
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or out.stride(1) != 1 or out.data_ptr() % 16:
        raise ValueError('out must be BF16 [M, N] with unit columns and 16-byte alignment')
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError('bias must be contiguous BF16 with N elements')
    lib = _lib.load()
    code = lib.h3_int8_ex(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(),
                          bias.data_ptr() if bias is not None else None, out.data_ptr(), m, n, k,
                          out.stride(0), EPI_GELU if gelu else EPI_DEQUANT, _stream(a))
    _lib.check_int8(code)
    return out


def int8_linear_gelu_quant(a, w, xs, ws, *, bias=None, rotated=None, rowmax=None, out=None, out_scale=None):
    """FC1 + GELU straight to the FC2 input: the ConvRot256 + per-token INT8 codes
    of bf(gelu_tanh(bf(((A.W^T * xs) * ws) + bias))), equal bit for bit to
    ``quantize_int8_rowwise_convrot64(int8_linear(..., gelu=True))``.  The
    rotation runs in the GEMM's epilogue (``h3_int8_gelu_rot``), the codes in a
    light pass over the rotated rows (``h3_convrot_codes``).  ``rotated`` (BF16
    [M, N]) and ``rowmax`` (int32 [M]) are the scratch between the two.
    Returns (q INT8 [M, N], scale FP32 [M, 1])."""
    m, n, k = _check_operands(a, w, xs, ws)
    if n % 256 or n > 16384:
        raise ValueError(f'N must be a multiple of 256 up to 16384 (got {n})')
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError('bias must be contiguous BF16 with N elements')
    dev = a.device
    rotated = torch.empty((m, n), dtype=torch.bfloat16, device=dev) if rotated is None else rotated
    rowmax = torch.empty((m,), dtype=torch.int32, device=dev) if rowmax is None else rowmax
    q = torch.empty((m, n), dtype=torch.int8, device=dev) if out is None else out
    s = torch.empty((m, 1), dtype=torch.float32, device=dev) if out_scale is None else out_scale
    for name, t, dt, shape in (('rotated', rotated, torch.bfloat16, (m, n)), ('rowmax', rowmax, torch.int32, (m,)),
                               ('out', q, torch.int8, (m, n)), ('out_scale', s, torch.float32, (m, 1))):
        if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous() or t.data_ptr() % 16 or t.device != dev:
            raise ValueError(f'{name} must be a contiguous, 16-byte aligned {dt} {list(shape)} tensor on {dev}')
    lib = _lib.load()
    stream = _stream(a)
    code = lib.h3_int8_gelu_rot(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(),
                                bias.data_ptr() if bias is not None else None, rotated.data_ptr(),
                                rowmax.data_ptr(), m, n, k, n, stream)
    _lib.check_int8(code)
    code = lib.h3_convrot_codes(rotated.data_ptr(), n, rowmax.data_ptr(), q.data_ptr(), s.data_ptr(), m, n,
                                stream)
    if code:
        raise RuntimeError(f'h3_convrot_codes: CUDA error {code}')
    return q, s


def int8_accumulators(a, w, out=None):
    """Raw int32 accumulators A.W^T (debug epilogue, bit-exact checks)."""
    m, n, k = _check_operands(a, w, None, None)
    if out is None:
        out = torch.empty((m, n), dtype=torch.int32, device=a.device)
    lib = _lib.load()
    code = lib.h3_int8_ex(a.data_ptr(), w.data_ptr(), None, None, None, out.data_ptr(), m, n, k, out.stride(0),
                          EPI_ACC, _stream(a))
    _lib.check_int8(code)
    return out


def int8_gate_residual(a, w, xs, ws, x, gate, rows, *, bias=None, requant=False, out=None):
    """x[m, n] <- bf(fmaf(bf(dequant + bias), gate[rows[m], n], x[m, n])), in place
    unless ``out`` is given.  With ``requant`` also returns the ConvRot256 +
    per-token INT8 copy of the updated rows (q [M, N], scale [M, 1])."""
    m, n, k = _check_operands(a, w, xs, ws)
    if x.dtype != torch.bfloat16 or tuple(x.shape) != (m, n) or not x.is_contiguous() or x.data_ptr() % 16:
        raise ValueError('residual must be contiguous BF16 [M, N], 16-byte aligned')
    if gate.dtype != torch.bfloat16 or gate.shape[-1] != n or not gate.is_contiguous() or gate.data_ptr() % 16:
        raise ValueError('gate must be a contiguous BF16 [G, N] table, 16-byte aligned')
    if rows.dtype != torch.int32 or rows.numel() != m or not rows.is_contiguous():
        raise ValueError('rows must be contiguous int32 [M]')
    dst = x if out is None else out
    if dst is not x and (dst.shape != x.shape or dst.dtype != x.dtype or not dst.is_contiguous()):
        raise ValueError('out must match the residual')
    q = s = None
    if requant:
        q = torch.empty((m, n), dtype=torch.int8, device=x.device)
        s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    code = lib.h3_int8_gate_ex(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(),
                               bias.data_ptr() if bias is not None else None, dst.data_ptr(), gate.data_ptr(),
                               rows.data_ptr(), x.data_ptr(), q.data_ptr() if q is not None else None,
                               s.data_ptr() if s is not None else None, m, n, k, _stream(a))
    _lib.check_int8(code)
    torch.autograd.graph.increment_version(dst)
    return (dst, q, s) if requant else dst
