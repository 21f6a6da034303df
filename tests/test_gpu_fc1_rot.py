"""FC1 + GELU with the FC2-input quantiser's rotation in the GEMM epilogue.

``h3_int8_gelu_rot`` + ``h3_convrot_codes`` must give the same INT8 codes and
per-token scales, bit for bit, as the unfused pair FC1 + GELU (``h3_int8_ex``)
then the Kitchen quantiser (``h3_convrot_quant_act``, act none), which are
themselves pinned to the reference's ``fc1.cu`` and ``convrot64_exact.cuh``
kernels elsewhere.  Covers the single-CTA (M <= 128) and CTA-pair forms, ragged
last row tiles, several tiles per CTA pair, bias, and inputs that overflow BF16
(inf and NaN in the rotated rows).
"""
import ctypes as ct

import pytest
import torch

from h3_speedkit import _lib
from h3_speedkit.ops import gemm
from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64

pytestmark = pytest.mark.gpu


def _operands(m, n, k, seed, device, xs_hi=0.05):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    xs = torch.rand((m,), generator=g) * (xs_hi - 0.005) + 0.005
    ws = torch.rand((n,), generator=g) * 0.0045 + 0.0005
    bias = (torch.randn((n,), generator=g) * 0.01).to(torch.bfloat16)
    return [t.to(device) for t in (a, w, xs, ws, bias)]


def _unfused(a, w, xs, ws, bias):
    h = gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True)
    return quantize_int8_rowwise_convrot64(h)


@pytest.mark.parametrize("m,n,k,use_bias", [(77, 512, 256, False), (128, 256, 1024, True), (129, 1024, 512, True),
                                            (300, 2048, 4096, False), (1000, 4096, 1024, True),
                                            (4096, 16384, 4096, False), (2500, 16384, 512, True)])
def test_fused_rotation_equals_fc1_then_quantiser(device, m, n, k, use_bias):
    a, w, xs, ws, bias = _operands(m, n, k, m * 31 + n + k, device)
    b = bias if use_bias else None
    q_ref, s_ref = _unfused(a, w, xs, ws, b)
    rowmax = torch.full((m,), 0x7F7FFFFF, dtype=torch.int32, device=device)   # the call resets it
    q, s = gemm.int8_linear_gelu_quant(a, w, xs, ws, bias=b, rowmax=rowmax)
    torch.cuda.synchronize()
    assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    assert torch.equal(q, q_ref)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("m,attn,k", [(300, 1024, 512), (4096, 4096, 4096), (77, 256, 256), (1000, 7168, 1024)])
def test_qkv_v_rotation_equals_plain_qkv_then_quantiser(device, m, attn, k):
    """h3_int8_rot with the dequant epilogue and rot_n0 = 2 attn (the QKV
    projection whose V third feeds the next quantiser): the Q and K columns equal
    the plain dequant GEMM bit for bit, and the codes pass over the rotated V
    third gives the quantiser's codes and scales of the plain V third."""
    n = 3 * attn
    a, w, xs, ws, _ = _operands(m, n, k, m + attn + k, device)
    plain = gemm.int8_linear(a, w, xs, ws)
    q_ref, s_ref = quantize_int8_rowwise_convrot64(plain[:, 2 * attn:])
    d = torch.empty((m, n), dtype=torch.bfloat16, device=device)
    vmax = torch.empty((m,), dtype=torch.int32, device=device)
    q = torch.empty((m, attn), dtype=torch.int8, device=device)
    s = torch.empty((m, 1), dtype=torch.float32, device=device)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check_int8(lib.h3_int8_rot(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), None, d.data_ptr(),
                                    vmax.data_ptr(), m, n, k, n, 0, 2 * attn, st))
    assert lib.h3_convrot_codes(d[:, 2 * attn:].data_ptr(), n, vmax.data_ptr(), q.data_ptr(), s.data_ptr(), m, attn,
                                st) == 0
    torch.cuda.synchronize()
    assert torch.equal(d[:, :2 * attn].view(torch.int16), plain[:, :2 * attn].view(torch.int16))
    assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    assert torch.equal(q, q_ref)


def test_fused_rotation_overflowing_rows(device):
    """Large activation scales drive some GELU outputs past the BF16 range (inf),
    whose rotations give inf and NaN; scales clamp at BF16_MAX / 127 and the
    codes of inf / NaN follow the quantiser's rules in both paths."""
    m, n, k = 512, 1024, 4096
    a, w, xs, ws, bias = _operands(m, n, k, 5, device)
    xs = xs.clone()
    xs[::7] = 3.0e36
    q_ref, s_ref = _unfused(a, w, xs, ws, bias)
    q, s = gemm.int8_linear_gelu_quant(a, w, xs, ws, bias=bias)
    torch.cuda.synchronize()
    assert not torch.isfinite(gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True).float()).all()
    assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    assert torch.equal(q, q_ref)


def test_fused_rotation_rejects_before_launch(device):
    """N % 256 != 0 is refused by the C entry point before anything runs: the
    rotated rows and the row maxima keep their sentinel contents."""
    m, n, k = 256, 264, 256
    a, w, xs, ws, _ = _operands(m, n, k, 3, device)
    v = torch.full((m, n), 7, dtype=torch.int16, device=device).view(torch.bfloat16)
    rowmax = torch.full((m,), 12345, dtype=torch.int32, device=device)
    lib = _lib.load()
    code = lib.h3_int8_gelu_rot(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), None, v.data_ptr(),
                                rowmax.data_ptr(), m, n, k, n, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert code == 0
    assert torch.equal(rowmax, torch.full_like(rowmax, 12345))
    assert torch.equal(v.view(torch.int16), torch.full((m, n), 7, dtype=torch.int16, device=device))
    code = lib.h3_convrot_codes(v.data_ptr(), n, rowmax.data_ptr(), a.data_ptr(), xs.data_ptr(), m, n,
                                torch.cuda.current_stream().cuda_stream)
    assert code != 0
