"""CPU checks of the C oracle's arithmetic against independent formulations.

These pin the restatement (oracle/h3_oracle.c) on the host: the ConvRot256 stage
order against the dense normalised Hadamard matrix, the RMS reduction tree
against a float64 evaluation of the same tree, BF16 rounding against torch, the
int32 GEMM against torch._int_mm, and the epilogue formulas against exact
float64 evaluations.  The GPU-side pins (reference kernels, golden fixtures)
are in test_golden.py and the -m gpu suite.
"""
import numpy as np
import pytest
import torch

from oracle import cpu as ocpu

H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)


def hadamard256() -> np.ndarray:
    h = H4
    for _ in range(3):
        h = np.kron(h, H4)
    return h / 16.0


def test_convrot_is_normalised_h4_kronecker_power():
    rng = np.random.default_rng(0)
    v = rng.standard_normal((8, 512)).astype(np.float32)
    out = ocpu.convrot_rows(v)
    h = hadamard256()
    for g in range(2):
        ref = v[:, 256 * g:256 * (g + 1)].astype(np.float64) @ h.T
        assert np.abs(out[:, 256 * g:256 * (g + 1)] - ref).max() < 1e-5


def test_convrot_is_an_involution_up_to_rounding():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal((4, 1024)) * 3).astype(np.float32)
    back = ocpu.convrot_rows(ocpu.convrot_rows(v))
    assert np.abs(back - v).max() < 1e-5 * np.abs(v).max()


def _fht_float32(v: np.ndarray) -> np.ndarray:
    """Independent numpy restatement: four radix-4 stages, float32 ops left to right."""
    v = v.astype(np.float32).copy()
    half = np.float32(0.5)
    for s in (1, 4, 16, 64):
        q = v.reshape(v.shape[0], 256 // (4 * s), 4, s)
        x0, x1, x2, x3 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
        d = np.stack([((x0 + x1) + x2) - x3, ((x0 + x1) - x2) + x3,
                      ((x0 - x1) + x2) + x3, ((-x0 + x1) + x2) + x3], axis=2) * half
        v = d.reshape(v.shape)
    return v


def test_convrot_rounding_order_matches_independent_restatement():
    rng = np.random.default_rng(11)
    v = (rng.standard_normal((16, 256)) * np.logspace(-3, 3, 256)).astype(np.float32)
    v[0, :4] = [1e8, 1.0, -1e8, 3.0]     # additions whose result depends on their order
    assert np.array_equal(ocpu.convrot_rows(v).view(np.uint32), _fht_float32(v).view(np.uint32))


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, np.inf, -np.inf], np.float32)])
    mine = ocpu.f32_to_bf16_bits(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(mine, theirs)


def test_row_scale_and_codes_contract():
    rot = np.zeros((3, 256), np.float32)
    rot[0, 0] = 127.0          # absmax 127.3: scale 1.0024 rounds to BF16 1.0
    rot[0, 1] = -127.3         # bf16(-127.3) = -127.5 -> rint half-even -128: reachable
    rot[1, :] = 0.0            # all-zero row: scale 1e-30, codes 0
    rot[2, 5] = 3.0e38         # near BF16 max: scale min(absmax, BF16_MAX) / 127
    q, s = ocpu.quant_rows(rot)
    assert s[0] == np.float32(127.3) * np.float32(1.0 / 127.0)
    assert q[0, 0] == 127 and q[0, 1] == -128
    assert s[1] == np.float32(1e-30) and not q[1].any()
    assert s[2] == np.float32(3.0e38) * np.float32(1.0 / 127.0)
    assert q[2, 5] == 127


def _rms_tree_float64(row_bits: np.ndarray) -> float:
    """The reference's reduction tree, evaluated with float32 rounding per step."""
    x = (row_bits.astype(np.uint32) << 16).view(np.float32)
    k = x.shape[0]
    lanes = []
    for t in range(128):
        s = np.float32(0.0)
        for c in range(t, k // 4, 128):
            for e in range(4):
                v = np.float64(x[4 * c + e])
                s = np.float32(np.float64(s) + v * v)   # fma: exact product, one rounding
        lanes.append(s)
    warps = []
    for w in range(4):
        s = lanes[32 * w:32 * w + 32]
        for off in (16, 8, 4, 2, 1):
            s = [np.float32(s[l] + s[l + off]) if l + off < 32 else s[l] for l in range(32)]
        warps.append(s[0])
    total = np.float32(np.float32(warps[0] + warps[2]) + np.float32(warps[1] + warps[3]))
    return float(np.float32(total / np.float32(k)))


@pytest.mark.parametrize("k", [512, 4096, 5376])
def test_rms_statistic_follows_the_reference_tree(k):
    rng = np.random.default_rng(k)
    x = ocpu.f32_to_bf16_bits((rng.standard_normal(k) * 2).astype(np.float32))
    assert ocpu.rms_variance(x) == _rms_tree_float64(x)


def test_int32_gemm_matches_torch_int_mm():
    rng = np.random.default_rng(3)
    a = rng.integers(-127, 128, (64, 272), dtype=np.int8)
    b = rng.integers(-127, 128, (48, 272), dtype=np.int8)
    c_loop = ocpu.gemm_s32(a, b, use_torch=False)
    c_torch = torch._int_mm(torch.from_numpy(a), torch.from_numpy(b).t().contiguous()).numpy()
    assert np.array_equal(c_loop, c_torch)
    assert np.array_equal(c_loop, a.astype(np.int64) @ b.astype(np.int64).T)


def test_dequant_is_the_reference_formula():
    rng = np.random.default_rng(4)
    acc = rng.integers(-2**27, 2**27, (32, 64)).astype(np.int32)
    xs = rng.uniform(0.005, 0.05, 32).astype(np.float32)
    ws = rng.uniform(0.0005, 0.005, 64).astype(np.float32)
    bias = ocpu.f32_to_bf16_bits(rng.normal(0, 0.01, 64).astype(np.float32))
    out = ocpu.dequant(acc, xs, ws, bias)
    b = ocpu.bf16_bits_to_f32(bias)
    y = ((acc.astype(np.float32) * xs[:, None]).astype(np.float32) * ws[None, :]).astype(np.float32)
    y = (y + b[None, :]).astype(np.float32)
    assert np.array_equal(out, ocpu.f32_to_bf16_bits(y))


def test_gate_residual_is_one_fused_rounding():
    rng = np.random.default_rng(5)
    acc = rng.integers(-2**26, 2**26, (16, 32)).astype(np.int32)
    xs = rng.uniform(0.005, 0.05, 16).astype(np.float32)
    ws = rng.uniform(0.0005, 0.005, 32).astype(np.float32)
    gate = ocpu.f32_to_bf16_bits(rng.normal(0, 0.3, (3, 32)).astype(np.float32))
    rows = rng.integers(0, 3, 16).astype(np.int32)
    res = ocpu.f32_to_bf16_bits(rng.normal(0, 1, (16, 32)).astype(np.float32))
    out = ocpu.gate_residual(acc, xs, ws, gate, rows, res)
    y = ocpu.bf16_bits_to_f32(ocpu.dequant(acc, xs, ws)).astype(np.float64)
    g = ocpu.bf16_bits_to_f32(gate)[rows].astype(np.float64)
    r = ocpu.bf16_bits_to_f32(res).astype(np.float64)
    # y*g is exact in float64 (8-bit x 8-bit significands); one rounding to FP32,
    # then BF16, equals fmaf's single rounding followed by BF16 (double rounding
    # through FP32 is innocuous for a sum of two values at this precision)
    ref = ocpu.f32_to_bf16_bits((y * g + r).astype(np.float32))
    assert np.array_equal(out, ref)


def test_norm_quant_matches_a_numpy_restatement_given_rrms():
    rng = np.random.default_rng(6)
    m, k = 5, 1024
    x = ocpu.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    w = ocpu.f32_to_bf16_bits(rng.uniform(0.5, 1.5, k).astype(np.float32))
    shift = rng.normal(0, 0.1, (2, k)).astype(np.float32)
    scale = rng.normal(0, 0.1, (2, k)).astype(np.float32)
    rows = np.array([0, 1, 1, 0, 1], np.int32)
    rrms = rng.uniform(0.9, 1.1, m).astype(np.float32)
    q, qs, norm, rot, rstd = ocpu.norm_quant(x, w, shift, scale, rows, 1e-6, rrms=rrms, debug=True)
    bf = lambda a: ocpu.bf16_bits_to_f32(ocpu.f32_to_bf16_bits(a))
    xf, wf = ocpu.bf16_bits_to_f32(x), ocpu.bf16_bits_to_f32(w)
    n = bf((wf[None, :] * (rrms[:, None] * xf).astype(np.float32)).astype(np.float32))
    one_c = bf((np.float32(1.0) + bf(scale[rows])).astype(np.float32))
    n = bf((bf((n * one_c).astype(np.float32)) + bf(shift[rows])).astype(np.float32))
    assert np.array_equal(norm, ocpu.f32_to_bf16_bits(n))
    assert np.array_equal(rot, ocpu.convrot_rows(n))
    assert np.array_equal(rstd, rrms)
    q2, s2 = ocpu.quant_rows(rot)
    assert np.array_equal(q, q2) and np.array_equal(qs, s2)


def test_swiglu_and_gelu_inputs():
    rng = np.random.default_rng(7)
    x = ocpu.f32_to_bf16_bits(rng.standard_normal((3, 512)).astype(np.float32))
    _, _, rot_g = ocpu.convrot_quant(x, act=1, rotated=True)
    xf = ocpu.bf16_bits_to_f32(x).astype(np.float64)
    gelu = 0.5 * xf * (1 + np.tanh(0.7978845608028654 * (xf + 0.044715 * xf ** 3)))
    assert np.abs(rot_g - ocpu.convrot_rows(gelu.astype(np.float32))).max() < 1e-5
    _, _, rot_s = ocpu.convrot_quant(x, act=2, rotated=True)
    g, u = xf[:, :256], xf[:, 256:]
    sw = g / (1 + np.exp(-g)) * u
    assert rot_s.shape == (3, 256)
    assert np.abs(rot_s - ocpu.convrot_rows(sw.astype(np.float32))).max() < 1e-5
