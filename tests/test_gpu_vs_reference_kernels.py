"""Same-GPU speed of the row kernels against the reference's own kernels.

The reference's prologue (norm_quant.cu), fused residual prologue
(residual_quant.cu), register ConvRot quantiser (convrot_register_v2.cu) and
Kitchen quantiser (convrot64_exact.cuh), compiled
from their sources for sm_100a into oracle/_ref, run on the same B200 at the
same shapes as this build's kernels.  Each case times both with CUDA events on
the launching stream (3 warm-up launches, then the median of 3 runs of 10
launches each, inputs larger than L2 or rotated through buffer sets that are),
prints both and the ratio and checks the outputs are the same bits.  Speed is
reported, not asserted: on a shared, power-capped GPU a timing is no
correctness gate (the measured ratios are kept under profiles/).

    python -m pytest tests/test_gpu_vs_reference_kernels.py -m gpu -s -q
"""
import ctypes as ct

import pytest
import torch

from h3_speedkit import _lib
from oracle import ref_gpu

pytestmark = pytest.mark.gpu

L2_BYTES = 126 << 20


def _time_ms(fn, sets, warm=3, iters=10, runs=3):
    for i in range(warm):
        fn(i % sets)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    times = []
    for _ in range(runs):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(iters):
            fn(i % sets)
        end.record(stream)
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) / iters)
    return sorted(times)[len(times) // 2]


def _sets(bytes_per_set):
    return max(1, -(-2 * L2_BYTES // bytes_per_set))


def _report(name, nbytes, t_ours, t_ref):
    print(f"\n{name}: ours {t_ours * 1e3:.1f} us ({nbytes / t_ours / 1e6:.0f} GB/s), "
          f"reference {t_ref * 1e3:.1f} us ({nbytes / t_ref / 1e6:.0f} GB/s), speed-up {t_ref / t_ours:.2f}x")


def _ref_fn(so_name, fn_name, argtypes):
    fn = getattr(ref_gpu._load(so_name), fn_name)
    fn.argtypes = argtypes
    fn.restype = ct.c_int
    return fn


@pytest.mark.parametrize("m,k", [(6144, 4096), (98304, 4096), (65536, 5376)])
def test_prologue_against_reference_kernel(device, m, k):
    if f"ref_norm_k{k}.so" not in [p.name for p in ref_gpu.REF.glob("ref_norm_k*.so")]:
        pytest.skip(f"reference prologue for K={k} not built")
    lib = _lib.load()
    ref = _ref_fn(f"ref_norm_k{k}.so", "h3_norm_quant_run", [ct.c_void_p] * 10 + [ct.c_int64] * 4 +
                  [ct.c_float, ct.c_int, ct.c_int, ct.c_size_t])
    nbytes = m * k * 2 + m * k + m * 4 + m * 4 + 3 * k * 2
    sets = _sets(nbytes)
    g = torch.Generator().manual_seed(m + k)
    xs = [(torch.randn((m, k), generator=g) * 2).to(torch.bfloat16).to(device) for _ in range(sets)]
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16).to(device)
    shift = (torch.randn((1, k), generator=g) * 0.1).to(torch.bfloat16).to(device)
    scale = (torch.randn((1, k), generator=g) * 0.1).to(torch.bfloat16).to(device)
    rows = torch.zeros((m,), dtype=torch.int32, device=device)
    q = [torch.empty((m, k), dtype=torch.int8, device=device) for _ in range(2)]
    qs = [torch.empty((m, 1), dtype=torch.float32, device=device) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream

    def ours(i):
        assert lib.h3_norm_quant_run_t(xs[i].data_ptr(), w.data_ptr(), shift.data_ptr(), scale.data_ptr(),
                                       rows.data_ptr(), q[0].data_ptr(), qs[0].data_ptr(), None, None, None, m, k, 1,
                                       k, k, k, ct.c_float(1e-6), 1, 0, st) == 0

    def theirs(i):
        assert ref(xs[i].data_ptr(), w.data_ptr(), shift.data_ptr(), scale.data_ptr(), rows.data_ptr(),
                   q[1].data_ptr(), qs[1].data_ptr(), None, None, None, m, k, k, k, 1e-6, 1, 0, st) == 0

    t_ours, t_ref = _time_ms(ours, sets), _time_ms(theirs, sets)
    ours(0)
    theirs(0)
    torch.cuda.synchronize()
    assert torch.equal(q[0], q[1]) and torch.equal(qs[0], qs[1])
    _report(f"prologue [{m},{k}]", nbytes, t_ours, t_ref)


@pytest.mark.parametrize("m,k,act", [(98304, 4096, 0), (98304, 16384, 0), (32768, 14336, 2), (32768, 16384, 1)])
def test_quantiser_against_reference_kitchen_kernel(device, m, k, act):
    lib = _lib.load()
    ref = _ref_fn("ref_kitchen.so", "ref_kitchen_convrot64_quant", [ct.c_void_p] * 3 +
                  [ct.c_int64, ct.c_int, ct.c_int, ct.c_size_t])
    width = 2 * k if act == 2 else k
    nbytes = m * width * 2 + m * k + m * 4
    sets = _sets(nbytes)
    g = torch.Generator().manual_seed(m + k + act)
    xs = [(torch.randn((m, width), generator=g) * 2).to(torch.bfloat16).to(device) for _ in range(sets)]
    q = [torch.empty((m, k), dtype=torch.int8, device=device) for _ in range(2)]
    sc = [torch.empty((m,), dtype=torch.float32, device=device) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream

    def ours(i):
        assert lib.h3_convrot_quant_act(xs[i].data_ptr(), width, q[0].data_ptr(), sc[0].data_ptr(), m, k, act,
                                        st) == 0

    def theirs(i):
        assert ref(xs[i].data_ptr(), q[1].data_ptr(), sc[1].data_ptr(), m, k, act, st) == 0

    t_ours, t_ref = _time_ms(ours, sets), _time_ms(theirs, sets)
    ours(0)
    theirs(0)
    torch.cuda.synchronize()
    assert torch.equal(q[0], q[1]) and torch.equal(sc[0], sc[1])
    _report(f"Kitchen quantiser [{m},{k}] act {act}", nbytes, t_ours, t_ref)


def test_register_quantiser_against_reference_kernel(device):
    m, k = 65536, 5376
    lib = _lib.load()
    ref = _ref_fn("ref_convrot.so", "h3_convrot_register_run", [ct.c_void_p] * 4 +
                  [ct.c_int64, ct.c_int, ct.c_int, ct.c_size_t])
    nbytes = m * k * 2 + m * k + m * 4
    sets = _sets(nbytes)
    g = torch.Generator().manual_seed(5)
    xs = [(torch.randn((m, k), generator=g) * 2).to(torch.bfloat16).to(device) for _ in range(sets)]
    q = [torch.empty((m, k), dtype=torch.int8, device=device) for _ in range(2)]
    sc = [torch.empty((m, 1), dtype=torch.float32, device=device) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream

    def ours(i):
        assert lib.h3_convrot_register_run(xs[i].data_ptr(), q[0].data_ptr(), sc[0].data_ptr(), None, m, k, 0,
                                           st) == 0

    def theirs(i):
        assert ref(xs[i].data_ptr(), q[1].data_ptr(), sc[1].data_ptr(), None, m, k, 0, st) == 0

    t_ours, t_ref = _time_ms(ours, sets), _time_ms(theirs, sets)
    ours(0)
    theirs(0)
    torch.cuda.synchronize()
    assert torch.equal(q[0], q[1]) and torch.equal(sc[0], sc[1])
    _report(f"register ConvRot quantiser [{m},{k}]", nbytes, t_ours, t_ref)


@pytest.mark.parametrize("m,k", [(98304, 4096), (65536, 5376)])
def test_residual_prologue_against_reference_kernel(device, m, k):
    if f"ref_residual_k{k}.so" not in [p.name for p in ref_gpu.REF.glob("ref_residual_k*.so")]:
        pytest.skip(f"reference residual prologue for K={k} not built")
    lib = _lib.load()
    ref = _ref_fn(f"ref_residual_k{k}.so", "h3_residual_quant_run", [ct.c_void_p] * 12 + [ct.c_int64] * 4 +
                  [ct.c_float, ct.c_int, ct.c_int, ct.c_int, ct.c_size_t])
    # x and branch read, x written back, codes + scale written
    nbytes = 3 * m * k * 2 + m * k + m * 4 + m * 4 + 4 * k * 2
    g = torch.Generator().manual_seed(m + k)
    x0 = (torch.randn((m, k), generator=g) * 2).to(torch.bfloat16).to(device)
    branch = (torch.randn((m, k), generator=g) * 0.1).to(torch.bfloat16).to(device)
    w = (torch.rand((k,), generator=g) + 0.5).to(torch.bfloat16).to(device)
    gate = (torch.randn((1, k), generator=g) * 0.01).to(torch.bfloat16).to(device)
    shift = (torch.randn((1, k), generator=g) * 0.1).to(torch.bfloat16).to(device)
    scale = (torch.randn((1, k), generator=g) * 0.1).to(torch.bfloat16).to(device)
    rows = torch.zeros((m,), dtype=torch.int32, device=device)
    xs = [x0.clone(), x0.clone()]
    q = [torch.empty((m, k), dtype=torch.int8, device=device) for _ in range(2)]
    qs = [torch.empty((m, 1), dtype=torch.float32, device=device) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream

    def ours(i):
        assert lib.h3_residual_quant_run_t(xs[0].data_ptr(), branch.data_ptr(), w.data_ptr(), gate.data_ptr(),
                                           shift.data_ptr(), scale.data_ptr(), rows.data_ptr(), q[0].data_ptr(),
                                           qs[0].data_ptr(), None, None, None, m, k, 1, k, k, k, ct.c_float(1e-6),
                                           1, 1, 0, st) == 0

    def theirs(i):
        assert ref(xs[1].data_ptr(), branch.data_ptr(), w.data_ptr(), gate.data_ptr(), shift.data_ptr(),
                   scale.data_ptr(), rows.data_ptr(), q[1].data_ptr(), qs[1].data_ptr(), None, None, None, m, k, k, k,
                   1e-6, 1, 1, 0, st) == 0

    # x is updated in place by every launch: both kernels see the same sequence
    t_ours, t_ref = _time_ms(ours, 1), _time_ms(theirs, 1)
    torch.cuda.synchronize()
    assert torch.equal(xs[0], xs[1]) and torch.equal(q[0], q[1]) and torch.equal(qs[0], qs[1])
    _report(f"residual prologue [{m},{k}]", nbytes, t_ours, t_ref)
