"""Seeded synthetic inputs with the shapes and value distributions of the five
benchmark configurations of the quantized DiT-block linear path.

The reference measures on private model weights and media; these generators
stand in for them.  Every generator draws on CPU from
``torch.Generator().manual_seed(1000 + cfg)`` (so a given ``rows`` always yields
the same tensors) and returns CPU tensors; callers move them to the device.
``rows`` (the token count M) may be reduced for tests: row r of a reduced draw is
not row r of the full draw, but the distributions are the same.

  cfg 1  single W8A8 linear: X [1024, 2048] ~N(0,1) with 8 outlier channels x30,
         W [2048, 2048] ~N(0, 0.02^2), bias [2048] ~N(0, 0.01^2)
  cfg 2  prologue: x [6144, 4096] ~N(0,1), 16 outlier channels x20,
         RMS weight ~U(0.5, 1.5), eps 1e-6, shift/scale [1, 4096] BF16 ~N(0, 0.1^2)
  cfg 3  FC1: A INT8 [24576, 4096] ~U[-127,127], xs ~U(0.005, 0.05),
         W INT8 [16384, 4096], ws ~U(0.0005, 0.005), bias [16384] ~N(0, 0.01^2), GELU
  cfg 4  FC2: A INT8 [24576, 16384], W INT8 [4096, 16384], scales as cfg 3,
         bias [4096], residual [24576, 4096] ~N(0,1), gate [4096] ~N(0, 0.3^2)
  cfg 5  8 blocks, D 4096, FFN 16384, M 98304 tokens, INT8 weights + per-channel scales
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

FULL_ROWS = {1: 1024, 2: 6144, 3: 24576, 4: 24576, 5: 98304}


def generator(cfg: int, salt: int = 0, device="cpu") -> torch.Generator:
    return torch.Generator(device=device).manual_seed(1000 + cfg + 7919 * salt)


def outlier_normal(rows: int, cols: int, n_outliers: int, factor: float, g: torch.Generator) -> torch.Tensor:
    x = torch.randn((rows, cols), generator=g, dtype=torch.float32, device=g.device)
    channels = torch.randperm(cols, generator=g, device=g.device)[:n_outliers]
    x[:, channels] *= factor
    return x.to(torch.bfloat16)


def int8_uniform(rows: int, cols: int, g: torch.Generator) -> torch.Tensor:
    return torch.randint(-127, 128, (rows, cols), generator=g, dtype=torch.int8, device=g.device)


def uniform(n: int, lo: float, hi: float, g: torch.Generator) -> torch.Tensor:
    return torch.rand((n,), generator=g, dtype=torch.float32, device=g.device) * (hi - lo) + lo


def normal_bf16(shape, std: float, g: torch.Generator) -> torch.Tensor:
    return (torch.randn(shape, generator=g, dtype=torch.float32, device=g.device) * std).to(torch.bfloat16)


def cfg1(rows: int = FULL_ROWS[1], k: int = 2048, n: int = 2048):
    g = generator(1)
    x = outlier_normal(rows, k, 8, 30.0, g)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
    bias = normal_bf16((n,), 0.01, g)
    return {"x": x, "w": w, "bias": bias}


def cfg2(rows: int = FULL_ROWS[2], k: int = 4096):
    g = generator(2)
    x = outlier_normal(rows, k, 16, 20.0, g)
    weight = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16)
    shift = normal_bf16((1, k), 0.1, g)
    scale = normal_bf16((1, k), 0.1, g)
    row_map = torch.zeros((rows,), dtype=torch.int32)
    return {"x": x, "weight": weight, "shift": shift, "scale": scale, "rows": row_map, "eps": 1e-6}


def cfg3(rows: int = FULL_ROWS[3], k: int = 4096, n: int = 16384):
    g = generator(3)
    a = int8_uniform(rows, k, g)
    xs = uniform(rows, 0.005, 0.05, g)
    w = int8_uniform(n, k, g)
    ws = uniform(n, 0.0005, 0.005, g)
    bias = normal_bf16((n,), 0.01, g)
    return {"a": a, "xs": xs, "w": w, "ws": ws, "bias": bias}


def cfg4(rows: int = FULL_ROWS[4], k: int = 16384, n: int = 4096):
    g = generator(4)
    a = int8_uniform(rows, k, g)
    xs = uniform(rows, 0.005, 0.05, g)
    w = int8_uniform(n, k, g)
    ws = uniform(n, 0.0005, 0.005, g)
    bias = normal_bf16((n,), 0.01, g)
    residual = torch.randn((rows, n), generator=g).to(torch.bfloat16)
    gate = normal_bf16((1, n), 0.3, g)
    row_map = torch.zeros((rows,), dtype=torch.int32)
    return {"a": a, "xs": xs, "w": w, "ws": ws, "bias": bias, "residual": residual, "gate": gate,
            "rows": row_map}


@dataclass
class BlockWeights:
    """INT8 weights (per-output-channel rows) and FP32 per-channel scales of one block."""
    norm1: torch.Tensor
    norm2: torch.Tensor
    qkv: torch.Tensor
    qkv_s: torch.Tensor
    out: torch.Tensor
    out_s: torch.Tensor
    fc1: torch.Tensor
    fc1_s: torch.Tensor
    fc2: torch.Tensor
    fc2_s: torch.Tensor
    # adaLN tables [T, D]: shift/scale for the two prologues and the two gates
    shift_msa: torch.Tensor
    scale_msa: torch.Tensor
    gate_msa: torch.Tensor
    shift_mlp: torch.Tensor
    scale_mlp: torch.Tensor
    gate_mlp: torch.Tensor

    def to(self, device) -> "BlockWeights":
        return BlockWeights(**{k: v.to(device) for k, v in self.__dict__.items()})


def cfg5_block(index: int, d: int = 4096, ffn: int = 16384, tables: int = 1, device="cpu", *,
               attn: int | None = None, swiglu: bool = False) -> BlockWeights:
    """Block `index` of the cfg-5 stack, drawn on `device` (a CPU draw and a CUDA
    draw of the same block differ: each device has its own generator stream).

    attn: attention width (QKV N = 3 attn, outproj K = attn; default d).
    swiglu: FC1 has 2 ffn rows ([gate | up]) and the FC2-input quantiser applies
    SwiGLU (the H3 MLP); otherwise FC1 has ffn rows and a GELU epilogue."""
    g = generator(5, salt=1 + index, device=device)
    attn = d if attn is None else attn
    n1 = 2 * ffn if swiglu else ffn
    return BlockWeights(
        norm1=(torch.rand((d,), generator=g, device=g.device) + 0.5).to(torch.bfloat16),
        norm2=(torch.rand((d,), generator=g, device=g.device) + 0.5).to(torch.bfloat16),
        qkv=int8_uniform(3 * attn, d, g), qkv_s=uniform(3 * attn, 0.0005, 0.005, g),
        out=int8_uniform(d, attn, g), out_s=uniform(d, 0.0005, 0.005, g),
        fc1=int8_uniform(n1, d, g), fc1_s=uniform(n1, 0.0005, 0.005, g),
        fc2=int8_uniform(d, ffn, g), fc2_s=uniform(d, 0.0005, 0.005, g),
        shift_msa=normal_bf16((tables, d), 0.1, g), scale_msa=normal_bf16((tables, d), 0.1, g),
        gate_msa=normal_bf16((tables, d), 0.3, g), shift_mlp=normal_bf16((tables, d), 0.1, g),
        scale_mlp=normal_bf16((tables, d), 0.1, g), gate_mlp=normal_bf16((tables, d), 0.3, g),
    )


# The H3 model's own block geometry (hidden 5376, attention 7168, SwiGLU MLP of
# width 14336: FC1 N = 28672, FC2 K = 14336), runtime.py:150-160 of H3 SpeedKit.
H3_GEOMETRY = {"d": 5376, "attn": 7168, "ffn": 14336, "swiglu": True}


def h3_block(index: int, tables: int = 1, device="cpu") -> BlockWeights:
    """Block `index` at the H3 model geometry (synthetic weights)."""
    g = H3_GEOMETRY
    return cfg5_block(index, g["d"], g["ffn"], tables, device, attn=g["attn"], swiglu=g["swiglu"])


def cfg5_tokens(rows: int = FULL_ROWS[5], d: int = 4096, device="cpu") -> torch.Tensor:
    g = generator(5, device=device)
    return torch.randn((rows, d), generator=g, device=g.device).to(torch.bfloat16)
