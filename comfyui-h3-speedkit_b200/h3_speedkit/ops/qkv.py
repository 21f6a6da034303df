"""QKV projection -> pre-quantised INT8 attention operands (B200).

Mirrors the reference's ``QKV`` op (h3_speedkit/ops/qkv.py:9-83 of H3 SpeedKit):
the same constructor argument (the directory of the kernel libraries), the same
operand checks and error texts, and the same launch sequence on the current
stream:

  1. ``h3_sample_gather``  the nine sample rows s*(m-1)//8 of q, xs and the RoPE rows;
  2. ``h3_sample_konly``   their K plane, normalised and roped;
  3. ``h3_sample_anchor``  the per-head anchor row (or -1) from those keys;
  4. ``h3_qkv_quant_kv``   the QKV GEMM into head-major planes with the Q/K/V epilogue;
  5. ``h3_quant_v``        the V quantiser (the reference runs two Triton kernels,
                           quant_v.py:57-104; here it is CUDA in the same library).

The result is the reference's ``PrequantizedInt8Attention`` when comfy_kitchen is
importable, else a dataclass with the same fields.  ``QKV.run`` is the
geometry-generic form the tests use (any head count / hidden size) and returns
every intermediate.
"""
from __future__ import annotations

import ctypes as ct
from dataclasses import dataclass
from pathlib import Path

import torch

from .. import _lib

HEADS, HEAD, HIDDEN, SAMPLES = 56, 128, 5376, 9


@dataclass
class PrequantizedInt8Attention:
    """Field-for-field stand-in for comfy_kitchen.sage_attention.PrequantizedInt8Attention."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    q_scale: torch.Tensor
    k_scale: torch.Tensor
    v_scale: torch.Tensor
    original_head_dim: int
    input_dtype: torch.dtype
    attention_scale: float
    cta_k: int
    attn_mask: object


def _result_type():
    try:
        from comfy_kitchen.sage_attention import PrequantizedInt8Attention as kitchen_type
        return kitchen_type
    except Exception:
        return PrequantizedInt8Attention


class QKV:
    def __init__(self, directory=None):
        # The reference loads qkv.so, sample.so and anchor.so from `directory`; all
        # of them are aliases of the one B200 library here.
        if directory is not None:
            lib_path = Path(directory) / "qkv.so"
            self.lib = _lib.load(lib_path if lib_path.exists() else None)
        else:
            self.lib = _lib.load()

    @staticmethod
    def _check(code):
        if code != 1:
            raise RuntimeError("R85 QKV launch failed; request aborted without retry")

    def __call__(self, q, w, xs, ws, rope, qw, kw, eps):
        m = q.shape[0]
        if q.shape != (m, HIDDEN) or w.shape != (3 * HEADS * HEAD, HIDDEN):
            raise ValueError("QKV requires the H3 56 x 128, hidden=5376 geometry")
        if rope.shape != (1, m, 1, 48, 2, 2):
            raise ValueError("QKV requires the pinned partial split-half RoPE layout")
        expected = ((q, torch.int8, (m, HIDDEN)), (w, torch.int8, (3 * HEADS * HEAD, HIDDEN)),
                    (xs, torch.float32, (m, 1)), (ws, torch.float32, (3 * HEADS * HEAD, 1)),
                    (rope, torch.bfloat16, (1, m, 1, 48, 2, 2)),
                    (qw, torch.bfloat16, (HEAD,)), (kw, torch.bfloat16, (HEAD,)))
        if any(t.dtype != dtype or tuple(t.shape) != shape for t, dtype, shape in expected):
            raise ValueError("QKV operand dtype/shape does not match the CUDA ABI: " +
                             str([(str(t.dtype), tuple(t.shape), str(dtype), shape)
                                  for t, dtype, shape in expected]))
        return self.pack(self.run(q, w, xs, ws, rope, qw, kw, eps, heads=HEADS), m, HEADS)

    @staticmethod
    def pack(out, m, heads):
        """The attention operands of a ``run`` result, as the reference's QKV op
        returns them (ops/qkv.py:80-83): codes and scales viewed [1, H, ...]."""
        parts = (m + 127) // 128
        return _result_type()(
            q=out["qi"].view(1, heads, m, HEAD), k=out["ki"].view(1, heads, m, HEAD), v=out["vi"],
            q_scale=out["qs"].view(1, heads, parts * 32), k_scale=out["ks"].view(1, heads, parts * 4),
            v_scale=out["vs"], original_head_dim=HEAD, input_dtype=torch.bfloat16,
            attention_scale=HEAD ** -0.5, cta_k=128, attn_mask=None)

    def run(self, q, w, xs, ws, rope, qw, kw, eps, *, heads=None, debug=False):
        """The five launches for any geometry (N = 3 * heads * 128); returns a dict with
        sq, sx, sr, sd, sk, anchors, d, qi, qs, ki, ks, vp, vi, vs, vinv (and rrms,
        sample_rrms when ``debug``)."""
        m, hidden = q.shape
        n = w.shape[0]
        heads = n // (3 * HEAD) if heads is None else heads
        if n != 3 * heads * HEAD or w.shape[1] != hidden or hidden % 16:
            raise ValueError("QKV weight must be [3*heads*128, hidden] with hidden % 16 == 0")
        if q.dtype != torch.int8 or w.dtype != torch.int8 or xs.dtype != torch.float32 or ws.dtype != torch.float32:
            raise ValueError("q / w must be INT8 and xs / ws FP32")
        if xs.numel() != m or ws.numel() != n or rope.numel() != m * 192 or rope.dtype != torch.bfloat16:
            raise ValueError("xs [m], ws [N] FP32 and rope [m, 192] BF16 required")
        if qw.numel() != HEAD or kw.numel() != HEAD or qw.dtype != torch.bfloat16 or kw.dtype != torch.bfloat16:
            raise ValueError("qw / kw must be BF16 [128]")
        device = q.device
        inputs = (q, w, xs, ws, rope, qw, kw)
        if any(not x.is_cuda or x.device != device or not x.is_contiguous() for x in inputs):
            raise ValueError("QKV operands must be contiguous and on one CUDA device")
        stream = torch.cuda.current_stream(device)
        st = stream.cuda_stream
        parts = (m + 127) // 128
        bf, i8, f32 = torch.bfloat16, torch.int8, torch.float32
        t = {
            "sq": torch.empty((SAMPLES, hidden), device=device, dtype=i8),
            "sx": torch.empty((SAMPLES, 1), device=device, dtype=f32),
            "sr": torch.empty((SAMPLES, 192), device=device, dtype=bf),
            "sd": torch.empty((3, heads, SAMPLES, HEAD), device=device, dtype=bf),
            "anchors": torch.empty((heads,), device=device, dtype=torch.int32),
            "d": torch.empty((3, heads, m, HEAD), device=device, dtype=bf),
            "qi": torch.empty((heads, m, HEAD), device=device, dtype=i8),
            "ki": torch.empty((heads, m, HEAD), device=device, dtype=i8),
            "qs": torch.empty((heads, parts * 32), device=device, dtype=f32),
            "ks": torch.empty((heads, parts * 4), device=device, dtype=f32),
            "vp": torch.empty((heads, parts, HEAD), device=device, dtype=f32),
            "vi": torch.empty((heads * HEAD, parts * 128), device=device, dtype=i8),
            "vs": torch.empty((heads * HEAD,), device=device, dtype=f32),
            "vinv": torch.empty((heads * HEAD,), device=device, dtype=f32),
        }
        if debug:
            t["rrms"] = torch.empty((2, heads, m), device=device, dtype=f32)
            t["sample_rrms"] = torch.empty((2, heads, SAMPLES), device=device, dtype=f32)
        owners = (*inputs, *t.values())
        for x in owners:
            x.record_stream(stream)
        p = {k: v.data_ptr() for k, v in t.items()}
        lib = self.lib
        rr, srr = p.get("rrms"), p.get("sample_rrms")
        eps = ct.c_float(eps)
        self._check(lib.h3_sample_gather_ex(q.data_ptr(), xs.data_ptr(), rope.data_ptr(), p["sq"], p["sx"], p["sr"],
                                            m, hidden, st))
        self._check(lib.h3_sample_konly_ex(p["sq"], w.data_ptr(), p["sx"], ws.data_ptr(), p["sd"], p["sr"],
                                           qw.data_ptr(), kw.data_ptr(), eps, SAMPLES, heads, hidden, srr, st))
        t["sk"] = t["sd"][1]
        self._check(lib.h3_sample_anchor_ex(t["sk"].data_ptr(), p["anchors"], heads, st))
        self._check(lib.h3_qkv_quant_kv_ex(q.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), p["d"],
                                           rope.data_ptr(), qw.data_ptr(), kw.data_ptr(), eps, p["qi"], p["qs"],
                                           p["vp"], p["ki"], p["ks"], t["sk"].data_ptr(), p["anchors"], m, heads,
                                           hidden, rr, st))
        self._check(lib.h3_quant_v(p["vp"], t["d"][2].data_ptr(), p["vi"], p["vs"], p["vinv"], m, heads, st))
        return t
