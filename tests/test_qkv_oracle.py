"""CPU checks of the QKV op's restatement (oracle/qkv.py, h3_oracle.c).

The reference's QKV epilogue only exists inside a CUTLASS kernel the oracle
build cannot compile (kernels/gemm/r84_kfourwarp.cu:193-375), so these tests
tie the restatement to the mathematics it must implement, in float64:
  * D: Q/K rows RMS-normalised with the head weight and roped on pairs
    (d, d + 48), d < 48 (r84:262-281), V raw;
  * codes: dequantising QI / KI with their group scales and undoing the signed,
    normalised 128-point Hadamard (an orthogonal map) gives back the roped rows
    (K minus its anchor row) to within half a quantisation step;
  * the scale groups are the reference's: 4 rows {base + 8j} for Q, 32 rows
    {tr : tr % 8 in {2kg, 2kg+1}} for K, per 128-row tile;
  * the V quantiser's output is channel-major with the token permutation
    [0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15] inside every run of 16 (quant_v.py:95-99).
The bit-level agreement with the GPU kernels is tests/test_gpu_qkv.py.
"""
import numpy as np
import pytest

from oracle import cpu as ocpu
from oracle import qkv as oqkv

SIGNS = (0x1035997B, 0x8087F5EE, 0xEE2E4E1A, 0x71132418)


def _sign_vector():
    s = np.empty(128)
    for ch in range(128):
        lane, c = divmod(ch, 4)
        flip = ((SIGNS[lane >> 3] >> ((lane & 7) * 4 + c)) & 1) ^ 1
        s[ch] = -1.0 if flip else 1.0
    return s


def _hadamard(n):
    h = np.array([[1.0]])
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def _rotation(full):
    """The 128x128 matrix the restatement applies to a row (row vector on the left)."""
    blocks = np.kron(np.eye(32), _hadamard(4) * 0.5)   # per-lane 4-point block
    if not full:
        return blocks
    # lane butterflies: lane index bits 0..4 -> channel bits 2..6
    lane_h = np.kron(_hadamard(32), np.eye(4)) * 0.1767766952966369
    return np.diag(_sign_vector()) @ blocks.T @ lane_h.T


def _operands(m, heads, hidden, seed, offset=0.0):
    rng = np.random.default_rng(seed)
    n = 3 * heads * 128
    base = rng.integers(-60, 61, (1, hidden)) * offset
    q = np.clip(np.round(rng.integers(-127, 128, (m, hidden)) * (1 - offset) + base), -127, 127).astype(np.int8)
    w = rng.integers(-127, 128, (n, hidden), dtype=np.int8)
    xs = rng.uniform(0.001, 0.01, (m, 1)).astype(np.float32)
    ws = rng.uniform(0.0005, 0.005, (n, 1)).astype(np.float32)
    ang = rng.uniform(0, 6.283, (m, 48))
    rope = np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).reshape(m, 192).astype(np.float32)
    rope = ocpu.f32_to_bf16_bits(rope)
    qw = ocpu.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    kw = ocpu.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    return q, w, xs, ws, rope, qw, kw


def _f(bits):
    return ocpu.bf16_bits_to_f32(bits).astype(np.float64)


@pytest.mark.parametrize("m,offset", [(300, 0.0), (200, 0.8), (1, 0.0)])
def test_qkv_restatement_against_float64_math(m, offset):
    heads, hidden, eps = 2, 256, 1e-6
    q, w, xs, ws, rope, qw, kw = _operands(m, heads, hidden, m, offset)
    out = oqkv.qkv(q, w, xs, ws, rope, qw, kw, eps)
    y = _f(ocpu.dequant(ocpu.gemm_s32(q, w), xs, ws)).reshape(m, 3, heads, 128).transpose(1, 2, 0, 3)
    d = _f(out["d"])
    # V raw
    assert np.array_equal(out["d"][2], ocpu.f32_to_bf16_bits(y[2].astype(np.float32)))
    fr = _f(rope).reshape(m, 48, 4)
    for g, wt in ((0, _f(qw)), (1, _f(kw))):
        x = y[g] / np.sqrt((y[g] ** 2).mean(-1, keepdims=True) + eps) * wt
        ref = x.copy()
        a, b, c, e = (fr[None, :, :, i] for i in range(4))
        ref[..., :48] = a * x[..., :48] + b * x[..., 48:96]
        ref[..., 48:96] = c * x[..., :48] + e * x[..., 48:96]
        assert np.abs(d[g] - ref).max() <= 0.02 * np.abs(ref).max()
    # codes undo to the roped rows; scale groups as the reference forms them
    rot_inv = np.linalg.inv(_rotation(m > 256))
    parts = (m + 127) // 128
    for h in range(heads):
        for tm in range(parts):
            for sub in range(32):
                base = (sub // 8) * 32 + sub % 8
                rows = [tm * 128 + base + 8 * j for j in range(4) if tm * 128 + base + 8 * j < m]
                sc = out["qs"][h, tm * 32 + sub]
                if not rows:
                    assert sc == np.float32(1e-7)
                    continue
                back = (out["qi"][h, rows].astype(np.float64) * sc) @ rot_inv
                assert np.abs(back - d[0, h, rows]).max() <= 0.5 * sc * np.sqrt(128) + 1e-6
            bias = np.zeros(128)
            if out["anchors"][h] >= 0:
                bias = _f(out["sk"][h, out["anchors"][h]])
            for kg in range(4):
                rows = [tm * 128 + (i // 2) * 8 + kg * 2 + (i & 1) for i in range(32)]
                rows = [r for r in rows if r < m]
                sc = out["ks"][h, tm * 4 + kg]
                if not rows:
                    continue
                back = (out["ki"][h, rows].astype(np.float64) * sc) @ rot_inv
                assert np.abs(back - (d[1, h, rows] - bias)).max() <= 0.5 * sc * np.sqrt(128) + 1e-6


def test_offset_keys_choose_an_anchor_and_plain_keys_do_not():
    rng = np.random.default_rng(1)
    plain = rng.standard_normal((4, 9, 128)).astype(np.float32)
    shifted = plain + 5 * rng.standard_normal((4, 1, 128)).astype(np.float32)
    assert (oqkv.sample_anchor(ocpu.f32_to_bf16_bits(plain)) == -1).all()
    assert (oqkv.sample_anchor(ocpu.f32_to_bf16_bits(shifted)) >= 0).all()


def test_v_quantiser_layout_and_scales():
    rng = np.random.default_rng(2)
    heads, m = 2, 300
    v = ocpu.f32_to_bf16_bits(rng.standard_normal((heads, m, 128)).astype(np.float32))
    parts = (m + 127) // 128
    vp = np.zeros((heads, parts, 128), np.float32)
    vf = ocpu.bf16_bits_to_f32(v)
    for p in range(parts):
        vp[:, p] = np.abs(vf[:, p * 128:(p + 1) * 128]).max(1)
    vi, vs = oqkv.quant_v(v, vp)
    assert vi.shape == (heads * 128, parts * 128) and vs.shape == (heads * 128,)
    perm = [0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15]
    src = np.array([(d // 16) * 16 + perm[d % 16] for d in range(parts * 128)])
    expect = np.zeros((heads, 128, parts * 128))
    valid = src < m
    expect[:, :, valid] = vf[:, src[valid], :].transpose(0, 2, 1)
    sc = vs.reshape(heads, 128, 1).astype(np.float64)
    assert np.allclose(vs.reshape(heads, 128), np.abs(vf).max(1) / 127, rtol=1e-6)
    assert np.abs(vi.reshape(heads, 128, -1) * sc - expect).max() <= 0.5 * sc.max() * 1.0001
    assert (vi.reshape(heads, 128, -1)[:, :, ~valid] == 0).all()


def test_sample_rows_follow_the_reference_formula():
    assert oqkv.sample_rows(1) == [0] * 9
    assert oqkv.sample_rows(9) == list(range(9))
    assert oqkv.sample_rows(98304) == [s * 98303 // 8 for s in range(9)]
