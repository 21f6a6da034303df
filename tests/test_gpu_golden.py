"""The CUDA kernels reproduce the reference kernels' golden vectors bit for bit
(no reference code is needed at test time: the fixtures are committed)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import bits_to_bf16
from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64
from h3_speedkit.ops.norm_quant import NormQuant

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _tensor(a, device):
    if a.dtype == np.uint16:
        return bits_to_bf16(a).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("norm_*.npz")))
def test_prologue_reproduces_golden(device, name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    x, w = _tensor(g["x"], device), _tensor(g["w"], device)
    shift, scale, rows = _tensor(g["shift"], device), _tensor(g["scale"], device), _tensor(g["rows"], device)
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=device)
    rstd = torch.empty((m,), dtype=torch.float32, device=device)
    NormQuant().bind(x, w, shift, scale, rows, q, qs, eps=float(g["eps"]),
                     debug_norm=torch.empty((m, k), dtype=torch.bfloat16, device=device),
                     debug_rotated=torch.empty((m, k), dtype=torch.float32, device=device), debug_rstd=rstd)()
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(qs.cpu().numpy().reshape(-1), g["qscale"])
    assert np.array_equal(rstd.cpu().numpy(), g["rstd"])


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("*.npz") if p.stem.startswith(("convrot_", "kitchen_"))))
def test_quantiser_reproduces_golden(device, name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    act = int(g["act"])
    q, s = quantize_int8_rowwise_convrot64(_tensor(g["x"], device), 256,
                                           input_act=[None, "gelu_tanh", "swiglu"][act])
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(s.cpu().numpy().reshape(-1), g["scale"])


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("residual_*.npz")))
@pytest.mark.parametrize("debug", [False, True])
def test_residual_prologue_reproduces_golden(device, name, debug):
    from h3_speedkit.ops.residual_quant import ResidualQuant
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    x, branch, w = _tensor(g["x"], device), _tensor(g["branch"], device), _tensor(g["w"], device)
    gate, shift, scale = _tensor(g["gate"], device), _tensor(g["shift"], device), _tensor(g["scale"], device)
    rows = _tensor(g["rows"], device)
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=device)
    dbg = {}
    if debug:
        dbg = dict(debug_norm=torch.empty((m, k), dtype=torch.bfloat16, device=device),
                   debug_rotated=torch.empty((m, k), dtype=torch.float32, device=device),
                   debug_rstd=torch.empty((m,), dtype=torch.float32, device=device))
    ResidualQuant().bind(x, branch, w, gate, shift, scale, rows, q, qs, eps=float(g["eps"]), **dbg)()
    torch.cuda.synchronize()
    assert np.array_equal(x.cpu().view(torch.int16).numpy().view(np.uint16), g["x_new"])
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(qs.cpu().numpy().reshape(-1), g["qscale"])
    if debug:
        assert np.array_equal(dbg["debug_rstd"].cpu().numpy(), g["rstd"])
        assert np.array_equal(dbg["debug_norm"].cpu().view(torch.int16).numpy().view(np.uint16), g["norm"])


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("anchor_*.npz")))
def test_anchor_detector_reproduces_golden(device, name):
    from h3_speedkit import _lib
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    lib = _lib.load()
    for i in range(g["k"].shape[0]):
        k = _tensor(g["k"][i], device)
        out = torch.empty((56,), dtype=torch.int32, device=device)
        assert lib.h3_sample_anchor(k.data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream) == 1
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), g["anchors"][i])


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("gather_*.npz")))
def test_sample_gather_reproduces_golden(device, name):
    from h3_speedkit import _lib
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    q, xs, rope = _tensor(g["q"], device), _tensor(g["xs"], device), _tensor(g["rope"], device)
    sq = torch.empty((9, 5376), dtype=torch.int8, device=device)
    sx = torch.empty((9, 1), dtype=torch.float32, device=device)
    sr = torch.empty((9, 192), dtype=torch.bfloat16, device=device)
    assert _lib.load().h3_sample_gather(q.data_ptr(), xs.data_ptr(), rope.data_ptr(), sq.data_ptr(), sx.data_ptr(),
                                        sr.data_ptr(), q.shape[0], torch.cuda.current_stream().cuda_stream) == 1
    torch.cuda.synchronize()
    assert np.array_equal(sq.cpu().numpy(), g["sq"]) and np.array_equal(sx.cpu().numpy(), g["sx"])
    assert np.array_equal(sr.cpu().view(torch.int16).numpy().view(np.uint16), g["sr"])
