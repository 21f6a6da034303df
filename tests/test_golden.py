"""Pin the CPU oracle to golden vectors produced by the reference's own CUDA
kernels (tests/golden/make_golden.py; norm_quant.cu, convrot_register_v2.cu and
the vendored Kitchen quantiser compiled from the reference sources).

Exact: the normalised/modulated BF16 values (with the reference's rrms, which
comes from the hardware rsqrt.approx), the ConvRot row scales, and codes except
where the reference's fast division lands a quotient on the other side of a
BF16 rounding tie (at most 1 code, at a rate below 1e-3).  GELU-tanh/SwiGLU
inputs go through the device tanhf/expf, so their scales are compared to 1e-6
relative and their codes by the same +-1 rule.
"""
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_codes_close
from oracle import cpu as ocpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def test_fixtures_present():
    assert len(CASES) >= 8


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("norm_")])
def test_oracle_prologue_matches_reference_kernel(name):
    g = load(name)
    q, qs, norm, _, _ = ocpu.norm_quant(g["x"], g["w"], g["shift"], g["scale"], g["rows"], float(g["eps"]),
                                        rrms=g["rstd"], debug=True)
    assert np.array_equal(norm, g["norm"]), "normalised/modulated BF16 values"
    assert np.array_equal(qs, g["qscale"]), "row scales"
    assert_codes_close(q, g["q"], 1e-3, name)
    # without the injected rrms: 1/sqrt in double stands in for rsqrt.approx
    _, _, _, _, rstd = ocpu.norm_quant(g["x"], g["w"], g["shift"], g["scale"], g["rows"], float(g["eps"]),
                                       debug=True)
    ulps = np.abs(rstd.view(np.int32).astype(np.int64) - g["rstd"].view(np.int32).astype(np.int64))
    assert ulps.max() <= 2


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith(("convrot_", "kitchen_"))])
def test_oracle_quantiser_matches_reference_kernel(name):
    g = load(name)
    q, s = ocpu.convrot_quant(g["x"], int(g["k"]), int(g["act"]))
    if int(g["act"]) == 0:
        assert np.array_equal(s, g["scale"])
    else:
        assert np.allclose(s, g["scale"], rtol=1e-6, atol=0)
    assert_codes_close(q, g["q"], 1e-3, name)


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("residual_")])
def test_oracle_residual_prologue_matches_reference_kernel(name):
    """residual_quant.cu fixtures: the updated rows bit for bit, then the prologue
    on them as above (rrms injected from the reference's hardware rsqrt)."""
    g = load(name)
    x_new, q, qs, norm, _, _ = ocpu.residual_quant(g["x"], g["branch"], g["w"], g["gate"], g["shift"], g["scale"],
                                                   g["rows"], float(g["eps"]), rrms=g["rstd"], debug=True)
    assert np.array_equal(x_new, g["x_new"]), "residual-updated rows"
    assert np.array_equal(norm, g["norm"]), "normalised/modulated BF16 values"
    assert np.array_equal(qs, g["qscale"]), "row scales"
    assert_codes_close(q, g["q"], 1e-3, name)


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("anchor_")])
def test_oracle_anchor_detector_matches_reference_kernel(name):
    """r79_sample_anchor.cu fixtures: the anchor row of each head, exactly."""
    from oracle import qkv as oqkv
    g = load(name)
    for i in range(g["k"].shape[0]):
        assert np.array_equal(oqkv.sample_anchor(g["k"][i]), g["anchors"][i]), f"key set {i}"
    assert (g["anchors"][1] >= 0).all() and (g["anchors"][0] == -1).all()


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("gather_")])
def test_oracle_sample_rows_match_reference_kernel(name):
    from oracle import qkv as oqkv
    g = load(name)
    sq, sx, sr = oqkv.gather(g["q"], g["xs"], g["rope"])
    assert np.array_equal(sq, g["sq"]) and np.array_equal(sx, g["sx"]) and np.array_equal(sr, g["sr"])
