"""Generate the golden fixtures from the reference's own CUDA kernels.

Run on a B200 box from the repository root after ``oracle/build.py`` has built
``oracle/_ref`` (the reference's norm_quant.cu, residual_quant.cu,
convrot_register_v2.cu, the vendored Kitchen quantiser, r79_sample_anchor.cu and
the gather of r82_sample_konly.cu, compiled from the reference sources):

    python tests/golden/make_golden.py [name-prefix ...]

With prefixes, only the fixtures whose names start with one of them are written.

Inputs are seeded CPU draws; every fixture stores the inputs (BF16 as uint16
bits) and the reference kernel's outputs.  The CPU oracle is pinned against
these files by tests/test_golden.py; the CUDA kernels by tests/test_gpu_golden.py.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT)]

from oracle import ref_gpu  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def norm_case(name, k, m, tables, table_dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[:16]] *= 20.0
    x = x.to(torch.bfloat16)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16)
    shift = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype)
    scale = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32)
    dev = torch.device("cuda")
    q, qs, dn, _, drs = ref_gpu.norm_quant(x.to(dev), w.to(dev), shift.to(dev), scale.to(dev), rows.to(dev), 1e-6,
                                           debug=True)
    torch.cuda.synchronize()
    tab = (lambda t: bits(t)) if table_dtype == torch.bfloat16 else (lambda t: t.numpy())
    np.savez_compressed(HERE / f"{name}.npz", kind="norm_quant", k=k, eps=np.float32(1e-6), x=bits(x), w=bits(w),
                        shift=tab(shift), scale=tab(scale), rows=rows.numpy(), q=q.cpu().numpy(),
                        qscale=qs.cpu().numpy().reshape(-1), norm=bits(dn), rstd=drs.cpu().numpy())


def convrot_case(name, k, m, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn((m, k), generator=g) * 3).to(torch.bfloat16)
    q, sc, _ = ref_gpu.convrot_register(x.cuda(), mode=0)
    torch.cuda.synchronize()
    np.savez_compressed(HERE / f"{name}.npz", kind="convrot_register", k=k, act=0, x=bits(x), q=q.cpu().numpy(),
                        scale=sc.cpu().numpy().reshape(-1))


def kitchen_case(name, k, m, act, seed):
    g = torch.Generator().manual_seed(seed)
    width = 2 * k if act == 2 else k
    x = (torch.randn((m, width), generator=g) * 2).to(torch.bfloat16)
    q, sc = ref_gpu.kitchen_quant(x.cuda(), act)
    torch.cuda.synchronize()
    np.savez_compressed(HERE / f"{name}.npz", kind="kitchen_quant", k=k, act=act, x=bits(x), q=q.cpu().numpy(),
                        scale=sc.cpu().numpy().reshape(-1))


def residual_case(name, k, m, tables, gate_dtype, table_dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[:16]] *= 20.0
    x = x.to(torch.bfloat16)
    branch = (torch.randn((m, k), generator=g) * 2).to(torch.bfloat16)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16)
    gate = (torch.randn((tables, k), generator=g) * 0.3).to(gate_dtype)
    shift = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype)
    scale = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32)
    dev = torch.device("cuda")
    xn, q, qs, dn, _, drs = ref_gpu.residual_quant(x.to(dev), branch.to(dev), w.to(dev), gate.to(dev), shift.to(dev),
                                                   scale.to(dev), rows.to(dev), 1e-6, debug=True)
    torch.cuda.synchronize()

    def tab(t):
        return bits(t) if t.dtype == torch.bfloat16 else t.numpy()

    np.savez_compressed(HERE / f"{name}.npz", kind="residual_quant", k=k, eps=np.float32(1e-6), x=bits(x),
                        branch=bits(branch), w=bits(w), gate=tab(gate), shift=tab(shift), scale=tab(scale),
                        rows=rows.numpy(), x_new=bits(xn), q=q.cpu().numpy(), qscale=qs.cpu().numpy().reshape(-1),
                        norm=bits(dn), rstd=drs.cpu().numpy())


def anchor_case(name, seed):
    """The K anchor detector (r79_sample_anchor.cu:467-605) on three sets of 56 x 9
    sampled keys: plain, with a shared per-head offset, and with one outlier sample."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((3, 56, 9, 128), generator=g)
    k[1] += torch.randn((56, 1, 128), generator=g) * 4
    k[2, :, 4] *= 30
    k = k.to(torch.bfloat16)
    anchors = torch.stack([ref_gpu.sample_anchor(k[i].cuda()) for i in range(3)])
    torch.cuda.synchronize()
    np.savez_compressed(HERE / f"{name}.npz", kind="sample_anchor", k=bits(k), anchors=anchors.cpu().numpy())


def gather_case(name, m, seed):
    """The sample-row gather (r82_sample_konly.cu:345-357), hidden 5376."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (m, 5376), generator=g, dtype=torch.int8)
    xs = torch.rand((m, 1), generator=g)
    rope = torch.randn((m, 192), generator=g).to(torch.bfloat16)
    sq, sx, sr = ref_gpu.sample_gather(q.cuda(), xs.cuda(), rope.cuda())
    torch.cuda.synchronize()
    np.savez_compressed(HERE / f"{name}.npz", kind="sample_gather", q=q.numpy(), xs=xs.numpy(), rope=bits(rope),
                        sq=sq.cpu().numpy(), sx=sx.cpu().numpy(), sr=bits(sr))


CASES = [
    ("norm_k4096_bf16", lambda n: norm_case(n, 4096, 8, 2, torch.bfloat16, 101)),
    ("norm_k5376_f32", lambda n: norm_case(n, 5376, 6, 3, torch.float32, 102)),
    ("norm_k2048_bf16", lambda n: norm_case(n, 2048, 8, 1, torch.bfloat16, 103)),
    ("convrot_k5376", lambda n: convrot_case(n, 5376, 6, 104)),
    ("convrot_k7168", lambda n: convrot_case(n, 7168, 4, 105)),
    ("kitchen_k4096_none", lambda n: kitchen_case(n, 4096, 8, 0, 106)),
    ("kitchen_k4096_gelu", lambda n: kitchen_case(n, 4096, 8, 1, 107)),
    ("kitchen_k2048_swiglu", lambda n: kitchen_case(n, 2048, 8, 2, 108)),
    ("residual_k5376_bf16", lambda n: residual_case(n, 5376, 6, 2, torch.bfloat16, torch.bfloat16, 109)),
    ("residual_k4096_f32", lambda n: residual_case(n, 4096, 8, 3, torch.float32, torch.float32, 110)),
    ("anchor_k56x9", lambda n: anchor_case(n, 111)),
    ("gather_m20", lambda n: gather_case(n, 20, 112)),
]


def main(prefixes):
    for name, make in CASES:
        if not prefixes or any(name.startswith(p) for p in prefixes):
            make(name)
    print("golden fixtures:", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main(sys.argv[1:])
