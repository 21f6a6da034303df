"""GPU parity of the row quantisers (fused prologue and ConvRot quantiser).

Gate: bit-exact against the reference's own CUDA kernels compiled into
oracle/_ref (norm_quant.cu, convrot_register_v2.cu, the vendored Kitchen
quantiser); then against the C restatement, where everything but the documented
approximations (rsqrt.approx, fast division) is bit-exact.
"""
import numpy as np
import pytest
import torch

from helpers import assert_codes_close, bf16_bits, np_
from h3_speedkit import synthetic
from h3_speedkit.ops.convrot import ConvRotRegister, quantize_int8_rowwise_convrot64
from h3_speedkit.ops.norm_quant import NormQuant
from oracle import cpu as ocpu
from oracle import ref_gpu

pytestmark = pytest.mark.gpu


def _prologue_inputs(rows, k, tables=1, table_dtype=torch.bfloat16, seed=0, xs_pad=0, device="cuda"):
    g = torch.Generator().manual_seed(4242 + seed)
    x = torch.randn((rows, k + xs_pad), generator=g)
    chans = torch.randperm(k, generator=g)[:16]
    x[:, chans] *= 20.0
    x = x.to(torch.bfloat16).to(device)[:, :k] if xs_pad else x.to(torch.bfloat16).to(device)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16).to(device)
    shift = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    scale = (torch.randn((tables, k), generator=g) * 0.1).to(table_dtype).to(device)
    rows_map = torch.randint(0, tables, (rows,), generator=g, dtype=torch.int32).to(device)
    return x, w, shift, scale, rows_map


def _run_ours(x, w, shift, scale, rows_map, eps=1e-6, debug=False):
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    qs = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    dbg = {}
    if debug:
        dbg = dict(debug_norm=torch.empty((m, k), dtype=torch.bfloat16, device=x.device),
                   debug_rotated=torch.empty((m, k), dtype=torch.float32, device=x.device),
                   debug_rstd=torch.empty((m,), dtype=torch.float32, device=x.device))
    NormQuant().bind(x, w, shift, scale, rows_map, q, qs, eps=eps, **dbg)()
    torch.cuda.synchronize()
    return (q, qs, dbg.get("debug_norm"), dbg.get("debug_rotated"), dbg.get("debug_rstd")) if debug else (q, qs)


@pytest.mark.parametrize("k", [2048, 4096, 5376])
@pytest.mark.parametrize("table_dtype", [torch.bfloat16, torch.float32])
def test_prologue_bitexact_vs_reference_kernel(device, k, table_dtype):
    if not ref_gpu.available(f"ref_norm_k{k}.so"):
        pytest.fail(f"reference GPU oracle ref_norm_k{k}.so missing")
    x, w, shift, scale, rows_map = _prologue_inputs(515, k, tables=3, table_dtype=table_dtype, seed=k)
    ours = _run_ours(x, w, shift, scale, rows_map, debug=True)
    ref = ref_gpu.norm_quant(x, w, shift, scale, rows_map, 1e-6, debug=True)
    torch.cuda.synchronize()
    names = ("q", "q_scale", "debug_norm", "debug_rotated", "debug_rstd")
    for name, a, b in zip(names, ours, ref):
        assert torch.equal(a.view(-1).view(torch.uint8) if a.dtype == torch.int8 else a.reshape(-1),
                           b.view(-1).view(torch.uint8) if b.dtype == torch.int8 else b.reshape(-1)), name


def test_prologue_full_cfg2_bitexact(device):
    inp = synthetic.cfg2()
    x, w = inp["x"].to(device), inp["weight"].to(device)
    shift, scale, rows_map = inp["shift"].to(device), inp["scale"].to(device), inp["rows"].to(device)
    q, qs = _run_ours(x, w, shift, scale, rows_map, eps=inp["eps"])
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows_map, inp["eps"])
    torch.cuda.synchronize()
    assert torch.equal(q, rq)
    assert torch.equal(qs, rqs)


@pytest.mark.parametrize("rows", [1, 127, 129])
def test_prologue_ragged_and_strided(device, rows):
    k = 4096
    x, w, shift, scale, rows_map = _prologue_inputs(rows, k, tables=2, seed=rows, xs_pad=4)
    assert x.stride(0) == k + 4 and x.data_ptr() % 16 == 0
    q, qs = _run_ours(x, w, shift, scale, rows_map)
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows_map, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(qs, rqs)
    # the 8-byte path must equal the 16-byte path on a contiguous copy
    q2, qs2 = _run_ours(x.contiguous(), w, shift, scale, rows_map)
    assert torch.equal(q, q2) and torch.equal(qs, qs2)


def test_prologue_unsuffixed_entry_point_k5376(device):
    """h3_norm_quant_run (K fixed at 5376) is the reference entry point itself."""
    import ctypes as ct
    from h3_speedkit import _lib
    lib = _lib.load()
    x, w, shift, scale, rows_map = _prologue_inputs(64, 5376, tables=2, table_dtype=torch.float32, seed=9)
    q = torch.empty((64, 5376), dtype=torch.int8, device=device)
    qs = torch.empty((64, 1), dtype=torch.float32, device=device)
    rc = lib.h3_norm_quant_run(x.data_ptr(), w.data_ptr(), shift.data_ptr(), scale.data_ptr(), rows_map.data_ptr(),
                               q.data_ptr(), qs.data_ptr(), None, None, None, 64, x.stride(0), shift.stride(0),
                               scale.stride(0), ct.c_float(1e-6), 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    rq, rqs = ref_gpu.norm_quant(x, w, shift, scale, rows_map, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(qs, rqs)


def test_prologue_vs_cpu_oracle(device):
    x, w, shift, scale, rows_map = _prologue_inputs(300, 4096, tables=2, seed=77)
    q, qs, dn, dr, drs = _run_ours(x, w, shift, scale, rows_map, debug=True)
    xb, wb = bf16_bits(x), bf16_bits(w)
    sh, sc, rm = bf16_bits(shift), bf16_bits(scale), np_(rows_map)
    # rrms: hardware rsqrt.approx vs double 1/sqrt -> within 2 FP32 ulp
    _, _, _, _, cpu_rstd = ocpu.norm_quant(xb, wb, sh, sc, rm, 1e-6, debug=True)
    gpu_rstd = np_(drs)
    ulps = np.abs(gpu_rstd.view(np.int32).astype(np.int64) - cpu_rstd.view(np.int32).astype(np.int64))
    assert ulps.max() <= 2
    # with the GPU's rrms injected, norm/rotation/scale are bit-exact, codes differ only at rare ties
    oq, oqs, odn, odr, _ = ocpu.norm_quant(xb, wb, sh, sc, rm, 1e-6, rrms=gpu_rstd, debug=True)
    assert np.array_equal(bf16_bits(dn), odn)
    assert np.array_equal(np_(dr).view(np.uint32), odr.view(np.uint32))
    assert np.array_equal(np_(qs).reshape(-1), oqs)
    assert_codes_close(np_(q), oq, 1e-3, "prologue codes vs CPU oracle")


@pytest.mark.parametrize("k", [5376, 7168])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_convrot_register_bitexact_vs_reference(device, k, mode):
    g = torch.Generator().manual_seed(k + mode)
    x = (torch.randn((257, k), generator=g) * 3).to(torch.bfloat16).to(device)
    op = ConvRotRegister()
    q = torch.empty((257, k), dtype=torch.int8, device=device) if mode != 2 else None
    sc = torch.empty((257, 1), dtype=torch.float32, device=device) if mode != 2 else None
    rot = torch.empty((257, k), dtype=torch.float32, device=device) if mode != 0 else None
    op.bind(x, q, sc, rotated=rot, mode=mode)()
    rq, rsc, rrot = ref_gpu.convrot_register(x, mode)
    torch.cuda.synchronize()
    if mode != 2:
        assert torch.equal(q, rq) and torch.equal(sc, rsc)
    if mode != 0:
        assert torch.equal(rot.view(torch.int32), rrot.view(torch.int32))


@pytest.mark.parametrize("k,act", [(4096, 0), (4096, 1), (4096, 2), (16384, 0), (16384, 1), (2048, 2), (256, 0)])
def test_convrot_act_bitexact_vs_kitchen(device, k, act):
    g = torch.Generator().manual_seed(31 * k + act)
    width = 2 * k if act == 2 else k
    x = (torch.randn((129, width), generator=g) * 2).to(torch.bfloat16).to(device)
    q, s = quantize_int8_rowwise_convrot64(x, 256, input_act=[None, "gelu_tanh", "swiglu"][act])
    rq, rs = ref_gpu.kitchen_quant(x, act)
    torch.cuda.synchronize()
    assert torch.equal(q, rq)
    assert torch.equal(s.reshape(-1), rs)


def test_convrot_strided_v_slice(device):
    """V = columns 8192:12288 of a QKV output, quantised in place of a copy."""
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn((200, 12288), generator=g).to(torch.bfloat16).to(device)
    v = qkv[:, 8192:]
    q1, s1 = quantize_int8_rowwise_convrot64(v)
    q2, s2 = quantize_int8_rowwise_convrot64(v.contiguous())
    rq, rs = ref_gpu.kitchen_quant(v.contiguous(), 0)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    assert torch.equal(q1, rq) and torch.equal(s1.reshape(-1), rs)


def test_convrot_vs_cpu_oracle(device):
    g = torch.Generator().manual_seed(11)
    x = (torch.randn((256, 4096), generator=g) * 4).to(torch.bfloat16).to(device)
    rot = torch.empty((256, 4096), dtype=torch.float32, device=device)
    q = torch.empty((256, 4096), dtype=torch.int8, device=device)
    s = torch.empty((256, 1), dtype=torch.float32, device=device)
    ConvRotRegister().bind(x, q, s, rotated=rot, mode=1)()
    torch.cuda.synchronize()
    oq, os_, orot = ocpu.convrot_quant(bf16_bits(x), rotated=True)
    assert np.array_equal(np_(rot).view(np.uint32), orot.view(np.uint32))
    assert np.array_equal(np_(s).reshape(-1), os_)
    assert_codes_close(np_(q), oq, 1e-3, "convrot codes vs CPU oracle")
