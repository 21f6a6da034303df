"""The QKV op's outputs mean what the attention that consumes them needs.

The codes are only useful if the INT8 attention downstream recovers the
attention of the unquantised Q, K, V from them.  On the CPU restatement (whose
outputs the GPU kernels reproduce, tests/test_gpu_qkv.py), in float64:

  * scores from the dequantised Q and K codes, with their per-group scales laid
    out as the reference lays them (Q: one scale per 4 rows {base + 8j} of a
    128-row tile; K: one per 32 rows {tr % 8 in {2kg, 2kg+1}}), equal the scores
    of the roped Q and K up to a per-query constant: the shared rotation is
    orthogonal (Q . K^T is kept) and centring K on its anchor row subtracts
    q . anchor from every score of a query -- softmax is unchanged;
  * the V codes, undone through the token permutation and the per-channel
    scales, give back V, and softmax(scores) . V matches the float attention.

This is the attention the reference's INT8 kernel approximates
(kernels/dense/qk_int_sv_i8_cuda.cuh), here in exact arithmetic.
"""
import numpy as np
import pytest

from oracle import cpu as ocpu
from oracle import qkv as oqkv

PERM = [0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15]


def _operands(m, heads, hidden, seed, offset, angle=6.283):
    rng = np.random.default_rng(seed)
    n = 3 * heads * 128
    base = rng.integers(-60, 61, (1, hidden)) * offset
    q = np.clip(np.round(rng.integers(-127, 128, (m, hidden)) * (1 - offset) + base), -127, 127).astype(np.int8)
    w = rng.integers(-127, 128, (n, hidden), dtype=np.int8)
    xs = rng.uniform(0.001, 0.01, (m, 1)).astype(np.float32)
    ws = rng.uniform(0.0005, 0.005, (n, 1)).astype(np.float32)
    ang = rng.uniform(0, angle, (m, 48))
    rope = np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).reshape(m, 192).astype(np.float32)
    return (q, w, xs, ws, ocpu.f32_to_bf16_bits(rope),
            ocpu.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 128).astype(np.float32)),
            ocpu.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 128).astype(np.float32)))


def _f(bits):
    return ocpu.bf16_bits_to_f32(bits).astype(np.float64)


def _q_scale_index(r):
    tm, tr = divmod(r, 128)
    return tm * 32 + (tr // 32) * 8 + tr % 8


def _k_scale_index(r):
    tm, tr = divmod(r, 128)
    return tm * 4 + (tr % 8) // 2


def _softmax(s):
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    return e / e.sum(-1, keepdims=True)


@pytest.mark.parametrize("m,offset,angle", [(300, 0.0, 6.283), (300, 0.9, 0.05), (200, 0.5, 6.283)])
def test_dequantised_operands_give_the_float_attention(m, offset, angle):
    """angle 0.05: nearly unrotated RoPE keeps the keys' shared offset, so the
    anchor centring is active."""
    heads, hidden = 2, 256
    out = oqkv.qkv(*_operands(m, heads, hidden, 7 * m, offset, angle), 1e-6)
    d = _f(out["d"])                       # [3, H, m, 128]: roped Q, roped K, V
    rows = np.arange(m)
    scale = 128 ** -0.5
    for h in range(heads):
        qd = out["qi"][h].astype(np.float64) * out["qs"][h][[_q_scale_index(r) for r in rows]][:, None]
        kd = out["ki"][h].astype(np.float64) * out["ks"][h][[_k_scale_index(r) for r in rows]][:, None]
        s_codes = qd @ kd.T * scale
        s_float = d[0, h] @ d[1, h].T * scale
        # equal up to a per-query constant (the anchor term), within quantisation error
        diff = (s_codes - s_codes.mean(1, keepdims=True)) - (s_float - s_float.mean(1, keepdims=True))
        assert np.abs(diff).max() < 0.05 * np.abs(s_float).max() + 0.05
        p_codes, p_float = _softmax(s_codes), _softmax(s_float)
        assert np.abs(p_codes - p_float).max() < 0.03
        # V from its codes: row h*128 + c, column dst holds token src(dst)
        parts = (m + 127) // 128
        src = np.array([(t // 16) * 16 + PERM[t % 16] for t in range(parts * 128)])
        vdq = np.zeros((m, 128))
        valid = src < m
        vdq[src[valid]] = (out["vi"][h * 128:(h + 1) * 128, valid].astype(np.float64)
                           * out["vs"][h * 128:(h + 1) * 128, None]).T
        assert np.abs(vdq - d[2, h]).max() <= 0.5 * out["vs"][h * 128:(h + 1) * 128].max() * 1.0001
        o_codes, o_float = p_codes @ vdq, p_float @ d[2, h]
        assert np.abs(o_codes - o_float).max() < 0.03 * np.abs(d[2, h]).max()
    if angle < 1:
        assert (out["anchors"] >= 0).all(), "offset keys are centred on a sample"
