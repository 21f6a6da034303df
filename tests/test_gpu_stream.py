"""GPU parity of the persistent streaming row kernels (TMA ring, row teams).

The streaming kernels serve every 16-byte aligned call without debug outputs;
the one-CTA-per-row kernels serve the debug / diagnostic modes and unaligned
rows.  Both must give the same bits as the reference's own kernels (compiled
into oracle/_ref) on row counts that wrap every team's ring many times, on
ragged counts that leave CTAs and teams idle, and on strided / misaligned
operands.
"""
import ctypes as ct

import pytest
import torch

from h3_speedkit import _lib
from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64
from oracle import ref_gpu

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _register(x, mode):
    """h3_convrot_register_run: mode 0 = streaming kernel, mode 1 = one CTA per row."""
    lib = _lib.load()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    rot = torch.empty((m, k), dtype=torch.float32, device=x.device) if mode else None
    rc = lib.h3_convrot_register_run(x.data_ptr(), q.data_ptr(), s.data_ptr(), rot.data_ptr() if mode else None, m, k,
                                     mode, _stream())
    assert rc == 0, lib.h3_convrot_register_error(rc)
    return q, s


@pytest.mark.parametrize("k,m", [(256, 5003), (2048, 6001), (4096, 9001), (5376, 3001), (16384, 1501)])
def test_quant_stream_equals_row_kernel(device, k, m):
    g = torch.Generator().manual_seed(k + m)
    x = (torch.randn((m, k), generator=g) * 3).to(torch.bfloat16).to(device)
    x[m // 3] = 0          # an all-zero row: scale 1e-30, codes 0
    x[m // 2, 7] = 3.0e38  # a huge value: absmax clamped to the BF16 maximum
    q0, s0 = _register(x, 0)
    q1, s1 = _register(x, 1)
    torch.cuda.synchronize()
    assert torch.equal(s0, s1)
    assert torch.equal(q0, q1)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("m", [1, 147, 149, 1185])
def test_quant_stream_ragged_rows_vs_kitchen(device, m):
    g = torch.Generator().manual_seed(m)
    x = (torch.randn((m, 4096), generator=g) * 2).to(torch.bfloat16).to(device)
    q, s = quantize_int8_rowwise_convrot64(x)
    rq, rs = ref_gpu.kitchen_quant(x, 0)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(s.reshape(-1), rs)


@pytest.mark.parametrize("k,act", [(4096, 1), (2048, 2), (16384, 2), (16384, 1)])
def test_quant_stream_activations_vs_kitchen(device, k, act):
    m = 700
    g = torch.Generator().manual_seed(7 * k + act)
    width = 2 * k if act == 2 else k
    x = (torch.randn((m, width), generator=g) * 2).to(torch.bfloat16).to(device)
    q, s = quantize_int8_rowwise_convrot64(x, 256, input_act=[None, "gelu_tanh", "swiglu"][act])
    rq, rs = ref_gpu.kitchen_quant(x, act)
    torch.cuda.synchronize()
    assert torch.equal(q, rq)
    assert torch.equal(s.reshape(-1), rs)


def test_quant_stream_strided_v_slice_many_rows(device):
    g = torch.Generator().manual_seed(12)
    qkv = torch.randn((3000, 12288), generator=g).to(torch.bfloat16).to(device)
    v = qkv[:, 8192:]
    q1, s1 = quantize_int8_rowwise_convrot64(v)
    rq, rs = ref_gpu.kitchen_quant(v.contiguous(), 0)
    torch.cuda.synchronize()
    assert torch.equal(q1, rq) and torch.equal(s1.reshape(-1), rs)


def _prologue_inputs(m, k, tables, table_dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[:16]] *= 20.0
    x = x.to(torch.bfloat16).to(device)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16).to(device)
    shift = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    scale = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32).to(device)
    return x, w, shift, scale, rows


def _prologue(x, w, shift, scale, rows, debug=False, eps=1e-6):
    """h3_norm_quant_run_k: debug=False takes the streaming kernel for aligned rows."""
    lib = _lib.load()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    dbg = [None, None, None]
    if debug:
        dbg = [torch.empty((m, k), dtype=torch.bfloat16, device=x.device),
               torch.empty((m, k), dtype=torch.float32, device=x.device),
               torch.empty((m,), dtype=torch.float32, device=x.device)]
    rc = lib.h3_norm_quant_run_k(x.data_ptr(), w.data_ptr(), shift.data_ptr(), scale.data_ptr(), rows.data_ptr(),
                                 q.data_ptr(), qs.data_ptr(), *[t.data_ptr() if t is not None else None for t in dbg],
                                 m, k, x.stride(0), shift.stride(0), scale.stride(0), ct.c_float(eps),
                                 1 if shift.dtype == torch.bfloat16 else 0, 1 if debug else 0, _stream())
    assert rc == 0, lib.h3_norm_quant_error(rc)
    return q, qs


@pytest.mark.parametrize("k", [2048, 4096, 5376])
@pytest.mark.parametrize("table_dtype", [torch.bfloat16, torch.float32])
def test_prologue_stream_bitexact_vs_reference_kernel(device, k, table_dtype):
    x, w, shift, scale, rows = _prologue_inputs(2999, k, 3, table_dtype, 100 + k, device)
    q, qs = _prologue(x, w, shift, scale, rows)
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(qs, rqs)
    assert torch.equal(q, rq)
    assert _lib.pipeline_status() == 0


@pytest.mark.parametrize("k,m", [(4096, 9001), (16384, 701), (256, 4001)])
def test_prologue_stream_equals_row_kernel(device, k, m):
    x, w, shift, scale, rows = _prologue_inputs(m, k, 2, torch.bfloat16, 7 + k, device)
    q0, s0 = _prologue(x, w, shift, scale, rows)
    q1, s1 = _prologue(x, w, shift, scale, rows, debug=True)
    torch.cuda.synchronize()
    assert torch.equal(s0, s1)
    assert torch.equal(q0, q1)


@pytest.mark.parametrize("m", [1, 148, 149])
def test_prologue_stream_misaligned_vectors(device, m):
    """W 8 bytes and the tables 4 bytes off a 16-byte boundary: the modulation
    pass takes its narrow-load paths."""
    k = 4096
    x, w, shift, scale, rows = _prologue_inputs(m, k, 2, torch.bfloat16, 55 + m, device)
    w_big = torch.empty((k + 4,), dtype=torch.bfloat16, device=device)
    w_big[4:] = w
    sh_big = torch.empty((2, k + 2), dtype=torch.bfloat16, device=device)
    sc_big = torch.empty((2, k + 2), dtype=torch.bfloat16, device=device)
    sh_big[:, 2:] = shift
    sc_big[:, 2:] = scale
    w2, sh2, sc2 = w_big[4:], sh_big[:, 2:], sc_big[:, 2:]
    assert w2.data_ptr() % 16 == 8 and sh2.data_ptr() % 16 == 4
    q, qs = _prologue(x, w2, sh2, sc2, rows)
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(qs, rqs)


def test_quant_nan_rows_match_reference(device):
    """NaN inputs: the row absmax ignores them (fmaxf semantics) and their codes
    are -128, in the streaming kernel, the row kernel and the reference."""
    g = torch.Generator().manual_seed(3)
    x = (torch.randn((600, 4096), generator=g) * 2).to(torch.bfloat16).to(device)
    x[5, 3] = float("nan")
    x[6, :] = float("nan")
    x[7, 4095] = float("nan")
    q0, s0 = _register(x, 0)
    q1, s1 = _register(x, 1)
    rq, rs = ref_gpu.kitchen_quant(x, 0)
    torch.cuda.synchronize()
    assert torch.equal(s0.reshape(-1).view(torch.int32), rs.view(torch.int32))
    assert torch.equal(s1, s0) and torch.equal(q1, q0)
    assert torch.equal(q0, rq)


def _prologue_t(x, w, shift, scale, rows, eps=1e-6):
    """h3_norm_quant_run_t: T known, so W and the tables are staged when they fit."""
    lib = _lib.load()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    rc = lib.h3_norm_quant_run_t(x.data_ptr(), w.data_ptr(), shift.data_ptr(), scale.data_ptr(), rows.data_ptr(),
                                 q.data_ptr(), qs.data_ptr(), None, None, None, m, k, shift.shape[0], x.stride(0),
                                 shift.stride(0), scale.stride(0), ct.c_float(eps),
                                 1 if shift.dtype == torch.bfloat16 else 0, 0, _stream())
    assert rc == 0, lib.h3_norm_quant_error(rc)
    return q, qs


@pytest.mark.parametrize("k,tables,table_dtype", [(4096, 1, torch.bfloat16), (4096, 3, torch.float32),
                                                   (2048, 2, torch.bfloat16), (5376, 1, torch.float32),
                                                   (5376, 2, torch.bfloat16), (4096, 12, torch.bfloat16)])
def test_prologue_staged_tables_bitexact_vs_reference_kernel(device, k, tables, table_dtype):
    """Staged-table streaming prologue (and, for 12 tables, the fallback when they
    do not fit) against the reference kernel."""
    x, w, shift, scale, rows = _prologue_inputs(3001, k, tables, table_dtype, 300 + k + tables, device)
    q, qs = _prologue_t(x, w, shift, scale, rows)
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(qs, rqs)
    assert torch.equal(q, rq)
    assert _lib.pipeline_status() == 0


def test_prologue_staged_misaligned_vectors(device):
    k, m = 4096, 149
    x, w, shift, scale, rows = _prologue_inputs(m, k, 2, torch.bfloat16, 77, device)
    w_big = torch.empty((k + 4,), dtype=torch.bfloat16, device=device)
    w_big[4:] = w
    sh_big = torch.empty((2, k + 2), dtype=torch.bfloat16, device=device)
    sc_big = torch.empty((2, k + 2), dtype=torch.bfloat16, device=device)
    sh_big[:, 2:] = shift
    sc_big[:, 2:] = scale
    q, qs = _prologue_t(x, w_big[4:], sh_big[:, 2:], sc_big[:, 2:], rows)
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(qs, rqs)
