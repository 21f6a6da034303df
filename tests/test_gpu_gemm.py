"""GPU parity of the tcgen05 INT8 GEMM and its fused epilogues.

int32 accumulators must equal torch._int_mm on CPU (exact); the dequant, bias
and gate-residual epilogues must equal the C restatement bit for bit (all of
their operations are IEEE round-to-nearest and reproducible on the CPU); the
GELU epilogue is within 1 BF16 ulp (the contract: the reference calls CUDA's
tanhf, the CPU restatement libm's; the epilogue's own tanh form equals the CPU
restatement on every finite BF16 input, which the exhaustive test checks).
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from helpers import bf16_bits, bf16_ulp_distance, np_
from h3_speedkit import _lib, synthetic
from h3_speedkit.ops import gemm
from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64
from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu


def _operands(m, n, k, seed, device):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    xs = torch.rand((m,), generator=g) * 0.045 + 0.005
    ws = torch.rand((n,), generator=g) * 0.0045 + 0.0005
    bias = (torch.randn((n,), generator=g) * 0.01).to(torch.bfloat16)
    return [t.to(device) for t in (a, w, xs, ws, bias)]


SHAPES = [(128, 256, 128), (129, 264, 4096), (1, 8, 16), (300, 512, 4096 + 16), (1024, 2048, 2048),
          (256, 4096, 16384)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_accumulators_exact(device, m, n, k):
    a, w, *_ = _operands(m, n, k, m * 7 + n, device)
    acc = gemm.int8_accumulators(a, w)
    torch.cuda.synchronize()
    ref = ocpu.gemm_s32(np_(a), np_(w))
    assert np.array_equal(np_(acc), ref)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 1024), (5000, 1032, 512), (4096, 4096, 8192), (19000, 3848, 8192)])
def test_accumulators_exact_many_tiles(device, m, n, k):
    """Many tiles per CTA pair (every pair walks several tiles, both accumulators
    and every pipeline stage wrap), checked against torch._int_mm (cuBLAS) as the
    reference for int32 accumulators.  (19000, 3848, 8192) takes the dual form
    (two N-tiles per work unit: K >= 8192, an even number of N-tiles -- sixteen,
    the last 8 columns wide -- and at least eight waves of units; 19000 rows
    leave a ragged last M-tile)."""
    a, w, *_ = _operands(m, n, k, m + n + k, device)
    acc = gemm.int8_accumulators(a, w)
    ref = torch._int_mm(a, w.t())
    torch.cuda.synchronize()
    assert torch.equal(acc, ref)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("m,n,k", SHAPES[:5])
@pytest.mark.parametrize("with_bias", [False, True])
def test_dequant_bitexact(device, m, n, k, with_bias):
    a, w, xs, ws, bias = _operands(m, n, k, m + 3 * n + k, device)
    out = gemm.int8_linear(a, w, xs, ws, bias=bias if with_bias else None)
    torch.cuda.synchronize()
    acc = ocpu.gemm_s32(np_(a), np_(w))
    ref = ocpu.dequant(acc, np_(xs), np_(ws), bf16_bits(bias) if with_bias else None)
    assert np.array_equal(bf16_bits(out), ref)


def test_h3_int8_reference_abi(device):
    """The unsuffixed h3_int8 symbol with the reference's argument order and 1/0 result."""
    m, n, k = 256, 512, 1024
    a, w, xs, ws, _ = _operands(m, n, k, 5, device)
    d = torch.empty((m, n), dtype=torch.bfloat16, device=device)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.h3_int8(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), d.data_ptr(), m, n, k, 3, st) == 1
    torch.cuda.synchronize()
    ref = ocpu.dequant(ocpu.gemm_s32(np_(a), np_(w)), np_(xs), np_(ws))
    assert np.array_equal(bf16_bits(d), ref)
    # invalid geometry is rejected on the host with 0 and nothing is launched
    assert lib.h3_int8(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), d.data_ptr(), m, n, 1000, 3, st) == 0
    assert lib.h3_int8_last_error() != 0


@pytest.mark.parametrize("m,n,k", [(256, 512, 1024), (129, 2048, 4096)])
def test_gelu_within_one_ulp(device, m, n, k):
    a, w, xs, ws, bias = _operands(m, n, k, 99 + m, device)
    out = gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True)
    torch.cuda.synchronize()
    ref = ocpu.dequant(ocpu.gemm_s32(np_(a), np_(w)), np_(xs), np_(ws), bf16_bits(bias), gelu=True)
    assert bf16_ulp_distance(bf16_bits(out), ref).max() <= 1


def test_gelu_exhaustive_bf16_inputs(device):
    """Every finite BF16 value through the FC1 GELU epilogue: with A = W = 0 and
    xs = ws = 1 the dequant value of column n is exactly bias[n], so one GEMM
    row with N = 65536 evaluates bf(gelu(v)) for every BF16 input v."""
    bits = np.arange(1 << 16, dtype=np.uint32)
    finite = (bits & 0x7F80) != 0x7F80
    vals = bits[finite].astype(np.uint16)
    n = (len(vals) + 255) // 256 * 256
    bias_bits = np.zeros(n, np.uint16)
    bias_bits[:len(vals)] = vals
    bias = torch.from_numpy(bias_bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    a = torch.zeros((1, 16), dtype=torch.int8, device=device)
    w = torch.zeros((n, 16), dtype=torch.int8, device=device)
    xs = torch.ones((1,), device=device)
    ws = torch.ones((n,), device=device)
    out = gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True)
    torch.cuda.synchronize()
    ref = ocpu.dequant(np.zeros((1, n), np.int32), np.ones(1, np.float32), np.ones(n, np.float32), bias_bits,
                       gelu=True)
    dist = bf16_ulp_distance(bf16_bits(out), ref)[0, :len(vals)]
    assert dist.max() <= 1, f"{int((dist > 1).sum())} inputs beyond 1 ulp, e.g. {vals[np.argmax(dist)]:#06x}"
    assert (dist != 0).mean() < 0.01


@pytest.mark.parametrize("m,n,k,tables", [(256, 512, 1024, 1), (333, 1024, 4096, 4)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gate_residual_in_place_bitexact(device, m, n, k, tables, with_bias):
    a, w, xs, ws, bias = _operands(m, n, k, 7 * m + tables, device)
    g = torch.Generator().manual_seed(m + tables)
    residual = torch.randn((m, n), generator=g).to(torch.bfloat16).to(device)
    gate = (torch.randn((tables, n), generator=g) * 0.3).to(torch.bfloat16).to(device)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32).to(device)
    before = bf16_bits(residual)
    out = gemm.int8_gate_residual(a, w, xs, ws, residual, gate, rows, bias=bias if with_bias else None)
    torch.cuda.synchronize()
    assert out.data_ptr() == residual.data_ptr()
    ref = ocpu.gate_residual(ocpu.gemm_s32(np_(a), np_(w)), np_(xs), np_(ws), bf16_bits(gate), np_(rows), before,
                             bf16_bits(bias) if with_bias else None)
    assert np.array_equal(bf16_bits(residual), ref)


def test_gate_residual_dual_form_bitexact(device):
    """The gate epilogue through the dual form (see test_accumulators_exact_many_tiles),
    with int32 accumulators from torch._int_mm and the epilogue from the C restatement."""
    m, n, k, tables = 19000, 3848, 8192, 2
    a, w, xs, ws, bias = _operands(m, n, k, 4242, device)
    g = torch.Generator().manual_seed(9)
    residual = torch.randn((m, n), generator=g).to(torch.bfloat16).to(device)
    gate = (torch.randn((tables, n), generator=g) * 0.3).to(torch.bfloat16).to(device)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32).to(device)
    before = bf16_bits(residual)
    acc = torch._int_mm(a, w.t())
    gemm.int8_gate_residual(a, w, xs, ws, residual, gate, rows, bias=bias)
    torch.cuda.synchronize()
    assert _lib.pipeline_status() == 0
    ref = ocpu.gate_residual(np_(acc), np_(xs), np_(ws), bf16_bits(gate), np_(rows), before, bf16_bits(bias))
    assert np.array_equal(bf16_bits(residual), ref)


def test_h3_int8_gate_reference_abi(device):
    m, n, k = 200, 1024, 2048
    a, w, xs, ws, _ = _operands(m, n, k, 17, device)
    x = torch.randn((m, n), device=device).to(torch.bfloat16)
    gate = (torch.randn((2, n), device=device) * 0.3).to(torch.bfloat16)
    rows = (torch.arange(m, device=device, dtype=torch.int32) % 2).contiguous()
    before = bf16_bits(x)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.h3_int8_gate(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), x.data_ptr(), gate.data_ptr(),
                          rows.data_ptr(), x.data_ptr(), m, n, k, 13, st)
    assert rc == 1
    torch.cuda.synchronize()
    ref = ocpu.gate_residual(ocpu.gemm_s32(np_(a), np_(w)), np_(xs), np_(ws), bf16_bits(gate), np_(rows), before)
    assert np.array_equal(bf16_bits(x), ref)


def test_gate_requant_matches_quantiser(device):
    m, n, k = 300, 4096, 2048
    a, w, xs, ws, bias = _operands(m, n, k, 23, device)
    x = torch.randn((m, n), device=device).to(torch.bfloat16)
    gate = (torch.randn((1, n), device=device) * 0.3).to(torch.bfloat16)
    rows = torch.zeros((m,), dtype=torch.int32, device=device)
    out, q, s = gemm.int8_gate_residual(a, w, xs, ws, x, gate, rows, bias=bias, requant=True)
    q2, s2 = quantize_int8_rowwise_convrot64(out)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(s, s2)


def _sampled_rows(m, count, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(m, generator=g)[:count]
    return torch.sort(idx).values


def test_cfg3_full_size_sampled(device):
    """FC1 at the benchmark shape; 48 sampled rows checked against the oracle."""
    inp = synthetic.cfg3()
    a, xs, w, ws, bias = (inp[k].to(device) for k in ("a", "xs", "w", "ws", "bias"))
    out = gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True)
    torch.cuda.synchronize()
    idx = _sampled_rows(a.shape[0], 48, 3)
    acc = ocpu.gemm_s32(inp["a"][idx].numpy(), inp["w"].numpy())
    ref = ocpu.dequant(acc, inp["xs"][idx].numpy(), inp["ws"].numpy(), bf16_bits(inp["bias"]), gelu=True)
    assert bf16_ulp_distance(bf16_bits(out[idx.to(device)]), ref).max() <= 1
    assert _lib.pipeline_status() == 0


def test_cfg4_full_size_sampled(device):
    """FC2 gate-residual + requant at the benchmark shape; 32 sampled rows."""
    inp = synthetic.cfg4()
    a, xs, w, ws, bias = (inp[k].to(device) for k in ("a", "xs", "w", "ws", "bias"))
    x = inp["residual"].to(device)
    gate, rows = inp["gate"].to(device), inp["rows"].to(device)
    out, q, s = gemm.int8_gate_residual(a, w, xs, ws, x, gate, rows, bias=bias, requant=True)
    torch.cuda.synchronize()
    idx = _sampled_rows(a.shape[0], 32, 4)
    acc = ocpu.gemm_s32(inp["a"][idx].numpy(), inp["w"].numpy())
    ref = ocpu.gate_residual(acc, inp["xs"][idx].numpy(), inp["ws"].numpy(), bf16_bits(inp["gate"]),
                             inp["rows"][idx].numpy(), bf16_bits(inp["residual"][idx]), bf16_bits(inp["bias"]))
    got = bf16_bits(out[idx.to(device)])
    assert np.array_equal(got, ref)
    oq, os_ = ocpu.convrot_quant(got)
    from helpers import assert_codes_close
    assert np.array_equal(np_(s[idx.to(device)]).reshape(-1), os_)
    assert_codes_close(np_(q[idx.to(device)]), oq, 1e-3, "requant codes vs CPU oracle")


def test_bounded_wait_selftest(device):
    """A wait on an mbarrier nobody arrives at must time out and report, not hang."""
    lib = _lib.load()
    status = ct.c_int(-1)
    rc = lib.h3sk_wait_selftest(20000, ct.byref(status), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert status.value == 1
    assert _lib.pipeline_status() == 0
    # the context is still usable afterwards
    a, w, *_ = _operands(128, 256, 128, 1, device)
    acc = gemm.int8_accumulators(a, w)
    torch.cuda.synchronize()
    assert np.array_equal(np_(acc), ocpu.gemm_s32(np_(a), np_(w)))

