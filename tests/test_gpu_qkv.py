"""GPU parity of the QKV op: projection -> pre-quantised attention operands.

The QKV GEMM with its head epilogue is pinned to the reference's own
r84_kfourwarp.cu in tests/test_gpu_ref_gemm.py.  Here:
  * the sample-row gather (r82_sample_konly.cu:345-357) and the K anchor
    detector (r79_sample_anchor.cu:467-605) run from oracle/_ref on the same
    inputs and must give the same bits;
  * the whole op (any head count and hidden size) is checked against the CPU
    restatement (oracle/qkv.py, h3_oracle.c) with the GPU's rrms injected: D,
    the scales, the V maxima, V scales and the anchors must be bit-exact; the
    INT8 codes may differ by 1 where rcp.approx (GPU) and the correctly rounded
    1/scale (CPU) put v * inv on opposite sides of a rounding boundary;
  * the head epilogue fused into the GEMM's epilogue warps equals the two-kernel
    form (GEMM, then the separate head kernel) bit for bit.
"""
import numpy as np
import pytest
import torch

from helpers import assert_codes_close, bf16_bits, np_
from h3_speedkit import _lib
from h3_speedkit.ops import gemm
from h3_speedkit.ops.qkv import QKV
from oracle import cpu as ocpu
from oracle import qkv as oqkv
from oracle import ref_gpu

pytestmark = pytest.mark.gpu

CODE_RATE = 2e-3


def _inputs(m, heads, hidden, seed, device, offset=0.0):
    """Seeded operands; ``offset`` adds a row-common component to q so every key
    shares a bias (the case the anchor centring is for)."""
    g = torch.Generator().manual_seed(seed)
    n = 3 * heads * 128
    base = torch.randint(-60, 61, (1, hidden), generator=g).float() * offset
    q = (torch.randint(-127, 128, (m, hidden), generator=g).float() * (1 - offset) + base).round().clamp(-127, 127)
    q = q.to(torch.int8)
    w = torch.randint(-127, 128, (n, hidden), generator=g, dtype=torch.int8)
    xs = (torch.rand((m, 1), generator=g) * 0.009 + 0.001).float()
    ws = (torch.rand((n, 1), generator=g) * 0.0045 + 0.0005).float()
    ang = torch.rand((m, 48), generator=g) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    rope = rope.to(torch.bfloat16)
    qw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    kw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    cpu_args = (q, w, xs, ws, rope, qw, kw)
    return tuple(t.to(device) for t in cpu_args), cpu_args


def _oracle(cpu_args, eps, out):
    q, w, xs, ws, rope, qw, kw = cpu_args
    return oqkv.qkv(q.numpy(), w.numpy(), xs.numpy(), ws.numpy(), bf16_bits(rope).reshape(-1, 192),
                    bf16_bits(qw), bf16_bits(kw), eps, rrms=np_(out["rrms"]), sample_rrms=np_(out["sample_rrms"]))


def _compare(out, ref, q):
    assert np.array_equal(np_(out["sq"]), q.numpy()[oqkv.sample_rows(q.shape[0])]), "sample rows"
    assert np.array_equal(bf16_bits(out["sk"]), ref["sk"]), "sampled keys"
    assert np.array_equal(np_(out["anchors"]), ref["anchors"]), "anchors"
    assert np.array_equal(bf16_bits(out["d"]), ref["d"]), "D (normalised, roped Q/K and raw V)"
    assert np.array_equal(np_(out["qs"]), ref["qs"]), "Q scales"
    assert np.array_equal(np_(out["ks"]), ref["ks"]), "K scales"
    assert np.array_equal(np_(out["vp"]), ref["vp"]), "V tile maxima"
    assert np.array_equal(np_(out["vs"]), ref["vs"]), "V scales"
    assert_codes_close(np_(out["qi"]), ref["qi"], CODE_RATE, "Q codes")
    assert_codes_close(np_(out["ki"]), ref["ki"], CODE_RATE, "K codes")
    assert_codes_close(np_(out["vi"]), ref["vi"], CODE_RATE, "V codes")


@pytest.mark.parametrize("m,heads,hidden,offset", [(300, 2, 256, 0.0), (1000, 3, 512, 0.7), (200, 2, 256, 0.7),
                                                   (129, 1, 1024, 0.0), (1, 2, 256, 0.0), (257, 2, 256, 0.9)])
def test_qkv_matches_cpu_restatement(device, m, heads, hidden, offset):
    """Small geometries: the m > 256 signed-H128 path, the m <= 256 4-point path,
    ragged last tiles, a single row, and offset keys that make anchors fire."""
    args, cpu_args = _inputs(m, heads, hidden, 17 * m + heads, device, offset)
    out = QKV().run(*args, 1e-6, debug=True)
    torch.cuda.synchronize()
    ref = _oracle(cpu_args, 1e-6, out)
    _compare(out, ref, cpu_args[0])
    # rrms is the hardware rsqrt: within 2 ulp of the correctly rounded value
    exact = oqkv.heads_epilogue(ocpu.dequant(ocpu.gemm_s32(cpu_args[0].numpy(), cpu_args[1].numpy()),
                                             cpu_args[2].numpy(), cpu_args[3].numpy()),
                                heads, bf16_bits(cpu_args[4]).reshape(-1, 192), bf16_bits(cpu_args[5]),
                                bf16_bits(cpu_args[6]), 1e-6, planes=3, quant=False)["rrms"]
    ulps = np.abs(np_(out["rrms"]).view(np.int32).astype(np.int64) - exact.view(np.int32).astype(np.int64))
    assert ulps.max() <= 2


def test_anchor_fires_on_offset_keys(device):
    args, cpu_args = _inputs(1000, 3, 512, 5, device, 0.9)
    out = QKV().run(*args, 1e-6, debug=True)
    torch.cuda.synchronize()
    anchors = np_(out["anchors"])
    assert (anchors >= 0).any(), "offset keys should be centred on a sample"
    ref = _oracle(cpu_args, 1e-6, out)
    _compare(out, ref, cpu_args[0])


def test_v_plane_is_the_row_major_gemm(device):
    """The head-major planes of D are the dequant GEMM's columns, bit for bit."""
    args, _ = _inputs(777, 2, 512, 3, device)
    q, w, xs, ws = args[:4]
    out = QKV().run(*args, 1e-6)
    y = gemm.int8_linear(q, w, xs.view(-1), ws.view(-1))
    torch.cuda.synchronize()
    v = y[:, 2 * 2 * 128:].reshape(777, 2, 128).permute(1, 0, 2)
    assert torch.equal(out["d"][2].view(torch.int16), v.contiguous().view(torch.int16))


@pytest.mark.parametrize("m", [1, 2, 9, 1000, 98304])
def test_sample_gather_matches_reference_kernel(device, m):
    g = torch.Generator().manual_seed(m)
    q = torch.randint(-127, 128, (m, 5376), generator=g, dtype=torch.int8).to(device)
    xs = torch.rand((m, 1), generator=g).to(device)
    rope = torch.randn((m, 192), generator=g).to(torch.bfloat16).to(device)
    ref = ref_gpu.sample_gather(q, xs, rope)
    lib = _lib.load()
    sq = torch.empty((9, 5376), dtype=torch.int8, device=device)
    sx = torch.empty((9, 1), dtype=torch.float32, device=device)
    sr = torch.empty((9, 192), dtype=torch.bfloat16, device=device)
    st = torch.cuda.current_stream().cuda_stream
    assert lib.h3_sample_gather(q.data_ptr(), xs.data_ptr(), rope.data_ptr(), sq.data_ptr(), sx.data_ptr(),
                                sr.data_ptr(), m, st) == 1
    torch.cuda.synchronize()
    assert torch.equal(sq, ref[0]) and torch.equal(sx, ref[1]) and torch.equal(sr.view(torch.int16),
                                                                             ref[2].view(torch.int16))


@pytest.mark.parametrize("seed", range(6))
def test_sample_anchor_matches_reference_kernel(device, seed):
    """56 heads x 9 sampled keys: plain, shared offsets (centring wins), one huge
    outlier sample (centring raises the max: -1), and ties."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((56, 9, 128), generator=g)
    if seed % 3 == 1:
        k += torch.randn((56, 1, 128), generator=g) * 4
    if seed % 3 == 2:
        k[:, 4] *= 30
    if seed == 5:
        k[:8] = k[:8, :1]         # identical samples: every distance ties
    k = k.to(torch.bfloat16).to(device)
    ref = ref_gpu.sample_anchor(k)
    ours = torch.empty((56,), dtype=torch.int32, device=device)
    assert _lib.load().h3_sample_anchor(k.data_ptr(), ours.data_ptr(), torch.cuda.current_stream().cuda_stream) == 1
    torch.cuda.synchronize()
    assert torch.equal(ours, ref)
    assert np.array_equal(np_(ours), oqkv.sample_anchor(bf16_bits(k)))


def test_h3_geometry_call_matches_cpu_restatement(device):
    """The reference's own call (56 heads x 128, hidden 5376, RoPE [1, m, 1, 48, 2, 2])
    returning the attention operands object."""
    m = 300
    args, cpu_args = _inputs(m, 56, 5376, 11, device, 0.5)
    op = QKV()
    res = op(*args, 1e-6)
    dbg = op.run(*args, 1e-6, debug=True)
    torch.cuda.synchronize()
    assert res.q.shape == (1, 56, m, 128) and res.k.shape == (1, 56, m, 128)
    assert res.v.shape == (56 * 128, 384) and res.v_scale.shape == (56 * 128,)
    assert res.q_scale.shape == (1, 56, 96) and res.k_scale.shape == (1, 56, 12)
    assert res.cta_k == 128 and res.original_head_dim == 128
    assert torch.equal(res.q.view(56, m, 128), dbg["qi"]) and torch.equal(res.v, dbg["vi"])
    ref = _oracle(cpu_args, 1e-6, dbg)
    _compare(dbg, ref, cpu_args[0])
    with pytest.raises(ValueError, match="H3 56 x 128"):
        op(args[0][:, :256].contiguous(), *args[1:], 1e-6)


@pytest.mark.parametrize("m,heads,hidden,offset", [(300, 2, 256, 0.5), (200, 2, 256, 0.7), (1, 2, 256, 0.0),
                                                   (1000, 4, 512, 0.8), (129, 2, 1024, 0.0), (257, 6, 256, 0.9),
                                                   (4096, 56, 5376, 0.6)])
def test_fused_head_epilogue_equals_the_two_kernel_form(device, m, heads, hidden, offset):
    """h3_qkv_quant_kv_ex runs the head epilogue inside the GEMM's epilogue warps
    for an even head count; with the rrms debug output it runs the GEMM and the
    separate head kernel instead.  Both forms (and the anchors they share) must
    give the same bits: D, Q/K codes and scales, V maxima."""
    args, _ = _inputs(m, heads, hidden, 31 * m + heads, device, offset)
    op = QKV()
    fused = op.run(*args, 1e-6)
    split = op.run(*args, 1e-6, debug=True)
    torch.cuda.synchronize()
    assert torch.equal(fused["anchors"], split["anchors"])
    assert torch.equal(fused["d"].view(torch.int16), split["d"].view(torch.int16)), "D planes"
    for key in ("qi", "ki", "qs", "ks", "vp", "vs", "vi"):
        assert torch.equal(fused[key], split[key]), key
