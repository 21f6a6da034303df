"""CPU restatement of one quantized DiT block (linear path, identity attention).
TEST INFRASTRUCTURE ONLY: the checker for the block stack and the timed CPU
baseline / reference arm of bench.py.

Follows the block order of ``Backend.block`` (h3_speedkit/runtime.py:126-164 of
H3 SpeedKit): prologue -> QKV -> (attention: V passthrough) -> ConvRot quant ->
outproj gate-residual -> prologue -> FC1 (+GELU epilogue, or SwiGLU in the next
quantiser) -> ConvRot quant -> FC2 gate-residual.  Each step is the oracle.cpu restatement of the
corresponding kernel; arrays are numpy (BF16 as uint16 bits).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import cpu as ocpu


@dataclass
class NpBlock:
    norm1: np.ndarray
    norm2: np.ndarray
    qkv: np.ndarray
    qkv_s: np.ndarray
    out: np.ndarray
    out_s: np.ndarray
    fc1: np.ndarray
    fc1_s: np.ndarray
    fc2: np.ndarray
    fc2_s: np.ndarray
    shift_msa: np.ndarray
    scale_msa: np.ndarray
    gate_msa: np.ndarray
    shift_mlp: np.ndarray
    scale_mlp: np.ndarray
    gate_mlp: np.ndarray

    @classmethod
    def from_torch(cls, bw) -> "NpBlock":
        import torch

        def conv(t):
            t = t.detach().contiguous().cpu()
            if t.dtype == torch.bfloat16:
                return t.view(torch.int16).numpy().view(np.uint16)
            return t.numpy()
        return cls(**{k: conv(v) for k, v in bw.__dict__.items()})


def block(x: np.ndarray, b: NpBlock, rows: np.ndarray, eps: float = 1e-6, threads=None, skip: int = 0) -> np.ndarray:
    """One block on BF16 rows x (uint16 [M, D]); returns the updated rows.

    ``skip``: the reference's row window (runtime.py:117-160): rows [0, skip)
    get no outproj/FC1/FC2 update and keep their residual.  Every op is
    row-local and attention is the identity here, so the window is the block on
    rows [skip, M) with the rows below copied through.

    The geometry comes from the weights: attention width A = qkv rows / 3 (V is
    columns [2A, 3A) of the QKV output), FFN width F = fc2 columns; an FC1 with
    2F rows is a SwiGLU MLP ([gate | up] halves, the activation applied by the
    FC2-input quantiser, convrot64_exact.cuh:928-937 and runtime.py:159), an FC1
    with F rows the GELU-epilogue MLP."""
    if skip:
        out = np.array(x, copy=True)
        if skip < x.shape[0]:
            out[skip:] = block(np.ascontiguousarray(x[skip:]), b, np.ascontiguousarray(rows[skip:]), eps, threads)
        return out
    attn = b.qkv.shape[0] // 3
    ffn = b.fc2.shape[1]
    swiglu = b.fc1.shape[0] == 2 * ffn
    q, qs = ocpu.norm_quant(x, b.norm1, b.shift_msa, b.scale_msa, rows, eps, threads=threads)
    qkv = ocpu.dequant(ocpu.gemm_s32(q, b.qkv, threads=threads), qs, b.qkv_s, threads=threads)
    v = np.ascontiguousarray(qkv[:, 2 * attn:3 * attn])
    aq, as_ = ocpu.convrot_quant(v, threads=threads)
    x = ocpu.gate_residual(ocpu.gemm_s32(aq, b.out, threads=threads), as_, b.out_s, b.gate_msa, rows, x,
                           threads=threads)
    q, qs = ocpu.norm_quant(x, b.norm2, b.shift_mlp, b.scale_mlp, rows, eps, threads=threads)
    h = ocpu.dequant(ocpu.gemm_s32(q, b.fc1, threads=threads), qs, b.fc1_s, gelu=not swiglu, threads=threads)
    if swiglu:
        hq, hs = ocpu.convrot_quant(h, k=ffn, act=2, threads=threads)
    else:
        hq, hs = ocpu.convrot_quant(h, threads=threads)
    return ocpu.gate_residual(ocpu.gemm_s32(hq, b.fc2, threads=threads), hs, b.fc2_s, b.gate_mlp, rows, x,
                              threads=threads)


def stack(x: np.ndarray, blocks: list[NpBlock], rows: np.ndarray, eps: float = 1e-6, threads=None,
          skip: int = 0) -> np.ndarray:
    """All blocks; ``skip`` is the last block's row window (runtime.py:296)."""
    for i, b in enumerate(blocks):
        x = block(x, b, rows, eps, threads, skip=skip if i == len(blocks) - 1 else 0)
    return x
