"""GPU parity of the fused residual prologue (h3_residual_quant_*).

x <- bf(fma(branch, bf(gate[rows]), x)) in place, then the prologue on the
updated rows.  Every case runs the reference's own residual_quant.cu kernel
(compiled into oracle/_ref for K = 4096 and 5376) on the same inputs and
requires the same bits: the updated rows, the INT8 codes and the FP32 row
scales (and, in debug mode, the normalised rows and rrms).  Covered: the
streaming kernel with staged tables (run_t), the streaming kernel with the
modulation pass (run_k), the one-CTA-per-row kernel (debug outputs; rows only
8-byte aligned), BF16 / FP32 gate and modulation tables, several table rows,
and ragged row counts that leave CTAs and row teams idle.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from h3_speedkit import _lib
from h3_speedkit.ops.residual_quant import ResidualQuant
from oracle import ref_gpu

pytestmark = pytest.mark.gpu


def _inputs(m, k, tables, gate_dtype, table_dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[:16]] *= 20.0
    x = x.to(torch.bfloat16).to(device)
    branch = (torch.randn((m, k), generator=g) * 2).to(torch.bfloat16).to(device)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16).to(device)
    gate = (torch.randn((tables, k), generator=g) * 0.3).to(gate_dtype).to(device)
    shift = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    scale = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32).to(device)
    return x, branch, w, gate, shift, scale, rows


def _ours(entry, x, branch, w, gate, shift, scale, rows, debug=False, eps=1e-6):
    """One of run / run_k / run_t on a copy of x; returns (x_new, q, qs[, dn, dr, drs])."""
    lib = _lib.load()
    m, k = x.shape
    xn = x.clone()
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    dbg = [None, None, None]
    if debug:
        dbg = [torch.empty((m, k), dtype=torch.bfloat16, device=x.device),
               torch.empty((m, k), dtype=torch.float32, device=x.device),
               torch.empty((m,), dtype=torch.float32, device=x.device)]
    ptrs = [t.data_ptr() if t is not None else None for t in (xn, branch, w, gate, shift, scale, rows, q, qs, *dbg)]
    tail = [ct.c_float(eps), int(gate.dtype == torch.bfloat16), int(shift.dtype == torch.bfloat16), int(debug),
            torch.cuda.current_stream().cuda_stream]
    strides = [gate.stride(0), shift.stride(0), scale.stride(0)]
    if entry == "run":
        rc = lib.h3_residual_quant_run(*ptrs, m, *strides, *tail)
    elif entry == "run_k":
        rc = lib.h3_residual_quant_run_k(*ptrs, m, k, *strides, *tail)
    else:
        rc = lib.h3_residual_quant_run_t(*ptrs, m, k, shift.shape[0], *strides, *tail)
    assert rc == 0, lib.h3_residual_quant_error(rc)
    return (xn, q, qs, *dbg) if debug else (xn, q, qs)


def _assert_same(ours, ref):
    for a, b in zip(ours, ref):
        assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                           b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


@pytest.mark.parametrize("k,m", [(4096, 3001), (5376, 2003)])
@pytest.mark.parametrize("entry", ["run_t", "run_k"])
@pytest.mark.parametrize("gate_dtype,table_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                                    (torch.float32, torch.bfloat16)])
def test_streaming_bitexact_vs_reference_kernel(device, k, m, entry, gate_dtype, table_dtype):
    if k == 5376 and entry == "run_t":
        entry = "run"   # the reference's own K=5376 entry point (T unknown: modulation pass)
    args = _inputs(m, k, 3, gate_dtype, table_dtype, k + m + (gate_dtype == torch.float32), device)
    ours = _ours(entry, *args)
    ref = ref_gpu.residual_quant(*args, 1e-6)
    torch.cuda.synchronize()
    _assert_same(ours, ref)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("k", [4096, 5376])
def test_row_kernel_debug_outputs_vs_reference_kernel(device, k):
    args = _inputs(301, k, 2, torch.bfloat16, torch.float32, 7 * k, device)
    ours = _ours("run_k", *args, debug=True)
    ref = ref_gpu.residual_quant(*args, 1e-6, debug=True)
    torch.cuda.synchronize()
    _assert_same(ours, ref)


@pytest.mark.parametrize("m", [1, 147, 149, 1185])
def test_ragged_rows_vs_reference_kernel(device, m):
    args = _inputs(m, 4096, 1, torch.bfloat16, torch.bfloat16, 55 + m, device)
    ours = _ours("run_t", *args)
    ref = ref_gpu.residual_quant(*args, 1e-6)
    torch.cuda.synchronize()
    _assert_same(ours, ref)


def test_rows_aligned_to_8_bytes_only(device):
    """x and branch 8 bytes off a 16-byte boundary: no TMA, the row kernel runs."""
    m, k = 149, 4096
    x, branch, w, gate, shift, scale, rows = _inputs(m, k, 2, torch.bfloat16, torch.bfloat16, 9, device)
    xb = torch.empty((m * k + 4,), dtype=torch.bfloat16, device=device)
    bb = torch.empty((m * k + 4,), dtype=torch.bfloat16, device=device)
    x2, b2 = xb[4:].view(m, k), bb[4:].view(m, k)
    x2.copy_(x)
    b2.copy_(branch)
    assert x2.data_ptr() % 16 == 8 and b2.data_ptr() % 16 == 8
    ours = _ours("run_t", x2, b2, w, gate, shift, scale, rows)
    ref = ref_gpu.residual_quant(x, branch, w, gate, shift, scale, rows, 1e-6)
    torch.cuda.synchronize()
    _assert_same(ours, ref)


def test_python_binding_updates_x_in_place(device):
    m, k = 513, 4096
    x, branch, w, gate, shift, scale, rows = _inputs(m, k, 3, torch.float32, torch.bfloat16, 21, device)
    ref = ref_gpu.residual_quant(x, branch, w, gate, shift, scale, rows, 1e-6)
    q = torch.empty((m, k), dtype=torch.int8, device=device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=device)
    out = ResidualQuant().bind(x, branch, w, gate, shift, scale, rows, q, qs, eps=1e-6)()
    torch.cuda.synchronize()
    assert out[0].data_ptr() == x.data_ptr()
    _assert_same((x, q, qs), ref)
    with pytest.raises(ValueError, match="overlaps"):
        ResidualQuant().bind(x, x, w, gate, shift, scale, rows, q, qs, eps=1e-6)


def test_invalid_arguments_rejected_before_launch(device):
    lib = _lib.load()
    m, k = 16, 4096
    x, branch, w, gate, shift, scale, rows = _inputs(m, k, 1, torch.bfloat16, torch.bfloat16, 3, device)
    before = x.clone()
    q = torch.empty((m, k), dtype=torch.int8, device=device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=device)
    st = torch.cuda.current_stream().cuda_stream
    ptrs = [t.data_ptr() for t in (x, branch, w, gate, shift, scale, rows, q, qs)] + [None, None, None]
    # gate row stride below K, eps not normal, K not a multiple of 256
    assert lib.h3_residual_quant_run_k(*ptrs, m, k, k - 1, k, k, ct.c_float(1e-6), 1, 1, 0, st) != 0
    assert lib.h3_residual_quant_run_k(*ptrs, m, k, k, k, k, ct.c_float(0.0), 1, 1, 0, st) != 0
    assert lib.h3_residual_quant_run_k(*ptrs, m, k + 8, k + 8, k + 8, k + 8, ct.c_float(1e-6), 1, 1, 0, st) != 0
    torch.cuda.synchronize()
    assert torch.equal(x, before)


@pytest.mark.parametrize("k,m,tables", [(256, 2001, 1), (2048, 3001, 2), (16384, 501, 1)])
def test_streaming_equals_row_kernel_at_other_widths(device, k, m, tables):
    """Widths the reference build does not cover (its K is a compile-time 4096 or
    5376 here): the streaming form (staged tables where they fit; at K=16384 the
    doubled slot leaves room for one row team) against the one-CTA-per-row form
    (debug outputs), and the updated rows against the CPU restatement."""
    from helpers import bf16_bits
    from oracle import cpu as ocpu
    args = _inputs(m, k, tables, torch.bfloat16, torch.bfloat16, 31 * k + m, device)
    stream = _ours("run_t", *args)
    rows_k = _ours("run_k", *args, debug=True)
    torch.cuda.synchronize()
    _assert_same(stream, rows_k[:3])
    x, branch, w, gate, shift, scale, rows = args
    x_new = ocpu.residual_update(bf16_bits(x), bf16_bits(branch), bf16_bits(gate), rows.cpu().numpy())
    assert np.array_equal(bf16_bits(stream[0]), x_new)
