"""GPU parity of the INT8 GEMMs against the reference's own CUTLASS kernels.

oracle/build.py compiles the reference's kernels/gemm/fc1.cu (``h3_int8``),
gate.cu (``h3_int8_gate``) and r84_kfourwarp.cu (``h3_qkv_quant_kv``) for
sm_100a from its sources; here they run on the same inputs as this build's
tcgen05 kernels and every output must be the same bits:

* ``h3_int8``          D = bf(((acc*xs)*ws)+0)               fc1.cu:79-90,119-138
* ``h3_int8_gate``     D = bf(fmaf(bf(dequant), gate[rows], residual)), in place
                       or not, multi-row gate tables          gate.cu:33-41,100-143
* ``h3_qkv_quant_kv``  head-major D planes, Q/K codes and scales, V tile maxima,
                       both rotation branches (M <= 256: 4-point, else H128)
                                                              r84_kfourwarp.cu:213-388

The reference's int32 accumulation is exact (|acc| <= K*128^2 < 2^31), so its
tile order and Stream-K split do not change a bit; the epilogue order is the
contract.  Timings of the same calls are printed (not asserted).
"""
import numpy as np
import pytest
import torch

from h3_speedkit import _lib
from h3_speedkit.ops import gemm
from oracle import ref_gpu

pytestmark = pytest.mark.gpu


def _need(name):
    if not ref_gpu.available(name):
        pytest.fail(f"oracle/_ref/{name} is missing: build it with oracle/build.py (needs CUTLASS headers)")


def _operands(m, n, k, seed, device):
    """cfg3/cfg4 distributions: codes U[-127, 127], xs U(0.005, 0.05), ws U(0.0005, 0.005)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    xs = torch.rand((m,), generator=g) * 0.045 + 0.005
    ws = torch.rand((n,), generator=g) * 0.0045 + 0.0005
    return [t.to(device) for t in (a, w, xs, ws)]


def _time(fn, reps=5):
    fn()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


@pytest.mark.parametrize("m,n,k", [(1024, 2048, 2048), (1, 8, 16), (129, 264, 4096), (300, 512, 4112),
                                   (4096, 12288, 4096), (24576, 16384, 4096), (8192, 4096, 16384)])
def test_h3_int8_equals_reference_fc1(device, m, n, k):
    """cfg1 [1024, 2048, 2048], ragged rows and columns, the cfg5 QKV shape, the full
    cfg3 FC1 shape and an FC2-like K; the reference's runtime config 3."""
    _need("ref_fc1.so")
    a, w, xs, ws = _operands(m, n, k, m + 7 * n + k, device)
    ref = ref_gpu.int8(a, w, xs, ws, config=3)
    ours = torch.empty_like(ref)
    st = torch.cuda.current_stream().cuda_stream
    lib = _lib.load()
    assert lib.h3_int8(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), ours.data_ptr(), m, n, k, 3, st) == 1
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))
    assert _lib.pipeline_status() == 0
    if m * n * k >= 1 << 36:
        t_ref = _time(lambda: ref_gpu.int8(a, w, xs, ws, config=3))
        t_ours = _time(lambda: gemm.int8_linear(a, w, xs, ws, out=ours))
        ops = 2.0 * m * n * k
        print(f"\nh3_int8 M={m} N={n} K={k}: reference fc1 {t_ref:.3f} ms ({ops / t_ref / 1e9:.0f} TOPS), "
              f"ours {t_ours:.3f} ms ({ops / t_ours / 1e9:.0f} TOPS)")


@pytest.mark.parametrize("config", [0, 1, 2, 4, 5, 6, 7])
def test_h3_int8_every_reference_config_gives_the_same_bits(device, config):
    """Every tile configuration of fc1.cu computes the same D (exact int32, one
    epilogue order), so ours must equal each of them."""
    _need("ref_fc1.so")
    m, n, k = 777, 1024, 2048
    a, w, xs, ws = _operands(m, n, k, 40 + config, device)
    ref = ref_gpu.int8(a, w, xs, ws, config=config)
    ours = gemm.int8_linear(a, w, xs, ws)
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("m,n,k,tables", [(24576, 4096, 16384, 1), (2048, 4096, 4096, 4), (129, 512, 1024, 3),
                                          (1, 256, 256, 1), (1000, 5376, 7168, 2)])
@pytest.mark.parametrize("config", [13, 0])
def test_h3_int8_gate_equals_reference_gate(device, m, n, k, tables, config):
    """The full cfg4 FC2 shape, the cfg5 outproj shape with four gate rows, ragged
    M, one row, the H3 outproj shape; the reference's Stream-K config 13 (what the
    runtime calls, runtime.py:122-123) and config 0.  Both sides update the
    residual in place (D == residual, runtime.py:120)."""
    _need("ref_gate.so")
    a, w, xs, ws = _operands(m, n, k, 3 * m + n + tables, device)
    g = torch.Generator().manual_seed(m + tables)
    residual = torch.randn((m, n), generator=g).to(torch.bfloat16).to(device)
    gate = (torch.randn((tables, n), generator=g) * 0.3).to(torch.bfloat16).to(device)
    rows = torch.randint(0, tables, (m,), generator=g, dtype=torch.int32).to(device)
    ref = residual.clone()
    ref_gpu.int8_gate(a, w, xs, ws, gate, rows, ref, config=config, out=ref)
    ours = residual.clone()
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.load().h3_int8_gate(a.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), ours.data_ptr(),
                                    gate.data_ptr(), rows.data_ptr(), ours.data_ptr(), m, n, k, config, st) == 1
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))
    assert _lib.pipeline_status() == 0
    if config == 13 and m * n * k >= 1 << 36:
        r1, r2 = residual.clone(), residual.clone()
        t_ref = _time(lambda: ref_gpu.int8_gate(a, w, xs, ws, gate, rows, r1, config=13, out=r1))
        t_ours = _time(lambda: gemm.int8_gate_residual(a, w, xs, ws, r2, gate, rows))
        ops = 2.0 * m * n * k
        print(f"\nh3_int8_gate M={m} N={n} K={k}: reference gate {t_ref:.3f} ms ({ops / t_ref / 1e9:.0f} TOPS), "
              f"ours {t_ours:.3f} ms ({ops / t_ours / 1e9:.0f} TOPS)")


def test_h3_int8_gate_out_of_place_equals_reference(device):
    """D separate from the residual: the residual stays untouched on both sides."""
    _need("ref_gate.so")
    m, n, k = 640, 1024, 2048
    a, w, xs, ws = _operands(m, n, k, 91, device)
    g = torch.Generator().manual_seed(92)
    residual = torch.randn((m, n), generator=g).to(torch.bfloat16).to(device)
    keep = residual.clone()
    gate = (torch.randn((2, n), generator=g) * 0.3).to(torch.bfloat16).to(device)
    rows = (torch.arange(m, device=device) % 2).to(torch.int32)
    ref = ref_gpu.int8_gate(a, w, xs, ws, gate, rows, residual)
    ours = gemm.int8_gate_residual(a, w, xs, ws, residual, gate, rows, out=torch.empty_like(residual))
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(residual.view(torch.int16), keep.view(torch.int16))


def _qkv_inputs(m, seed, device, anchored):
    """H3 geometry operands (56 heads x 128, hidden 5376) and sampled keys with a
    per-head anchor row (or -1: no centring for that head)."""
    g = torch.Generator().manual_seed(seed)
    heads, hidden, n = 56, 5376, 3 * 56 * 128
    q = torch.randint(-127, 128, (m, hidden), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, hidden), generator=g, dtype=torch.int8)
    xs = (torch.rand((m, 1), generator=g) * 0.009 + 0.001).float()
    ws = (torch.rand((n, 1), generator=g) * 0.0045 + 0.0005).float()
    ang = torch.rand((m, 48), generator=g) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    rope = rope.to(torch.bfloat16)
    qw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    kw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    sk = (torch.randn((heads, 9, 128), generator=g) * 2).to(torch.bfloat16)
    if anchored:
        anchors = torch.randint(-1, 9, (heads,), generator=g, dtype=torch.int32)
    else:
        anchors = torch.full((heads,), -1, dtype=torch.int32)
    return [t.to(device) for t in (q, w, xs, ws, rope, qw, kw, sk, anchors)]


@pytest.mark.parametrize("m,anchored", [(300, True), (200, True), (256, False), (257, True), (1, True),
                                        (1000, True), (8192, True)])
def test_h3_qkv_quant_kv_equals_reference_r84(device, m, anchored):
    """M > 256 takes the signed H128 rotation, M <= 256 the 4-point one
    (r84_kfourwarp.cu:297,330); ragged last tiles; anchors on a random subset of
    heads.  D, Q/K codes and scales and the V maxima must be the same bits."""
    _need("ref_qkv.so")
    q, w, xs, ws, rope, qw, kw, sk, anchors = _qkv_inputs(m, 5 * m + int(anchored), device, anchored)
    ref = ref_gpu.qkv_quant_kv(q, w, xs, ws, rope, qw, kw, 1e-6, sk, anchors)
    ours = {k: torch.empty_like(v) for k, v in ref.items()}
    st = torch.cuda.current_stream().cuda_stream
    p = {k: v.data_ptr() for k, v in ours.items()}
    rc = _lib.load().h3_qkv_quant_kv(q.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), p["d"],
                                      rope.data_ptr(), qw.data_ptr(), kw.data_ptr(), 1e-6, p["qi"], p["qs"],
                                      p["vp"], p["ki"], p["ks"], sk.data_ptr(), anchors.data_ptr(), m, st)
    assert rc == 1, _lib.load().h3_int8_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(ours["d"].view(torch.int16), ref["d"].view(torch.int16)), "D planes"
    for key in ("qs", "ks", "vp"):
        assert torch.equal(ours[key].view(torch.int32), ref[key].view(torch.int32)), key
    for key in ("qi", "ki"):
        diff = (ours[key].int() - ref[key].int()).abs()
        assert int(diff.max()) == 0, f"{key}: {int((diff != 0).sum())} codes differ"
    if m >= 8192:
        t_ref = _time(lambda: ref_gpu.qkv_quant_kv(q, w, xs, ws, rope, qw, kw, 1e-6, sk, anchors))
        t_ours = _time(lambda: _lib.load().h3_qkv_quant_kv(
            q.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), p["d"], rope.data_ptr(), qw.data_ptr(),
            kw.data_ptr(), 1e-6, p["qi"], p["qs"], p["vp"], p["ki"], p["ks"], sk.data_ptr(), anchors.data_ptr(),
            m, st))
        print(f"\nh3_qkv_quant_kv M={m}: reference r84 {t_ref:.3f} ms, ours {t_ours:.3f} ms")


def test_cfg1_w8a8_linear_end_to_end_against_reference_kernels(device):
    """BASELINE config 1 end to end on its seeded inputs (synthetic.cfg1: X BF16
    [1024, 2048] with 8 outlier channels x30, W [2048, 2048], bias [2048]): X per
    token and W per output channel through ConvRot256 + INT8 (this build's
    quantiser vs the reference's Kitchen kernel: same codes and scales), then the
    INT8 GEMM with the dequant epilogue (this build vs the reference's fc1.cu: same
    BF16 output), and with the bias, which the reference GEMM lacks, against the C
    restatement of r84_kfourwarp.cu:240's explicit formula (same bits)."""
    from h3_speedkit import synthetic
    from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64
    from helpers import bf16_bits, np_
    from oracle import cpu as ocpu
    _need("ref_fc1.so")
    inp = synthetic.cfg1()
    x, w, bias = (inp[k].to(device) for k in ("x", "w", "bias"))
    xq, xs = quantize_int8_rowwise_convrot64(x)
    wq, ws = quantize_int8_rowwise_convrot64(w)
    rxq, rxs = ref_gpu.kitchen_quant(x, 0)
    rwq, rws = ref_gpu.kitchen_quant(w, 0)
    torch.cuda.synchronize()
    assert torch.equal(xq, rxq) and torch.equal(xs.view(-1), rxs.view(-1)), "activation codes / scales"
    assert torch.equal(wq, rwq) and torch.equal(ws.view(-1), rws.view(-1)), "weight codes / scales"
    y = gemm.int8_linear(xq, wq, xs.view(-1), ws.view(-1))
    ref = ref_gpu.int8(rxq, rwq, rxs.view(-1), rws.view(-1), config=3)
    yb = gemm.int8_linear(xq, wq, xs.view(-1), ws.view(-1), bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), "dequant output vs fc1.cu"
    acc = ocpu.gemm_s32(np_(xq), np_(wq))
    want = ocpu.dequant(acc, np_(xs).reshape(-1), np_(ws).reshape(-1), bf16_bits(bias))
    assert np.array_equal(bf16_bits(yb), want), "dequant + bias vs the C restatement"
