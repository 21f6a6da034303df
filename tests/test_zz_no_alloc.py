"""The allocation-free QKV entry point ``h3_qkv_noalloc``.

It is for callers that cannot allocate device memory while they run (a serving
loop that forbids cudaMalloc after warm-up, a framework that owns all device
memory).  It runs the same five steps as the QKV op with its intermediates in a
file-scope device array, so its outputs must equal, bit for bit, those of the op built
from the individual entry points with torch-allocated intermediates
(``QKV.run``) -- on two calls in a row, so that stale scratch from the first
call cannot leak into the second.  Collected last so that it also runs after
every other test has used the library.
"""
import ctypes as ct

import pytest
import torch

from h3_speedkit import _lib
from h3_speedkit.ops.qkv import QKV

OUTPUTS = ("d", "qi", "qs", "ki", "ks", "vp", "vi", "vs")


def _inputs(m, heads, hidden, seed, device, offset):
    g = torch.Generator().manual_seed(seed)
    n = 3 * heads * 128
    base = torch.randint(-60, 61, (1, hidden), generator=g).float() * offset
    q = (torch.randint(-127, 128, (m, hidden), generator=g).float() * (1 - offset) + base).round().clamp(-127, 127)
    ang = torch.rand((m, 48), generator=g) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    t = (q.to(torch.int8), torch.randint(-127, 128, (n, hidden), generator=g, dtype=torch.int8),
         torch.rand((m, 1), generator=g) * 0.009 + 0.001, torch.rand((n, 1), generator=g) * 0.0045 + 0.0005,
         rope.to(torch.bfloat16), (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16),
         (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16))
    return tuple(x.to(device) for x in t)


def _noalloc(args, heads, eps):
    q, w, xs, ws, rope, qw, kw = args
    m, hidden = q.shape
    parts = (m + 127) // 128
    dev = q.device
    out = {
        "d": torch.full((3, heads, m, 128), -1, dtype=torch.int16, device=dev).view(torch.bfloat16),
        "qi": torch.full((heads, m, 128), 7, dtype=torch.int8, device=dev),
        "ki": torch.full((heads, m, 128), 7, dtype=torch.int8, device=dev),
        "qs": torch.full((heads, parts * 32), -1.0, device=dev),
        "ks": torch.full((heads, parts * 4), -1.0, device=dev),
        "vp": torch.full((heads, parts, 128), -1.0, device=dev),
        "vi": torch.full((heads * 128, parts * 128), 7, dtype=torch.int8, device=dev),
        "vs": torch.full((heads * 128,), -1.0, device=dev),
    }
    p = {k: v.data_ptr() for k, v in out.items()}
    rc = _lib.load().h3_qkv_noalloc(q.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), p["d"],
                                    rope.data_ptr(), qw.data_ptr(), kw.data_ptr(), ct.c_float(eps), p["qi"],
                                    p["qs"], p["vp"], p["ki"], p["ks"], p["vi"], p["vs"], m, heads, hidden,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 1, _lib.load().h3_int8_error()
    return out


def _same(a, b):
    if a.dtype == torch.bfloat16:
        a, b = a.view(torch.int16), b.view(torch.int16)
    return torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("m,heads,hidden,offset", [(1000, 56, 5376, 0.6), (300, 2, 256, 0.9), (129, 3, 512, 0.0)])
def test_noalloc_equals_the_op_on_two_calls_in_a_row(device, m, heads, hidden, offset):
    """The second call gets other inputs (different anchors, sample rows and V
    scales) so a scratch value left from the first call would show."""
    first = _inputs(m, heads, hidden, 3 * m + heads, device, offset)
    second = _inputs(m + 37, heads, hidden, 5 * m + heads, device, 0.9 - offset)
    ref1 = QKV().run(*first, 1e-6, heads=heads)
    ref2 = QKV().run(*second, 1e-6, heads=heads)
    got1 = _noalloc(first, heads, 1e-6)
    got2 = _noalloc(second, heads, 1e-6)
    torch.cuda.synchronize()
    for ref, got in ((ref1, got1), (ref2, got2)):
        for k in OUTPUTS:
            assert _same(got[k], ref[k]), k


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """Rejected on the host before any device work (fake pointers would fault)."""
    lib = _lib.load()
    eps = ct.c_float(1e-6)
    for heads, hidden in ((65, 5376), (56, 8208), (0, 5376), (56, 5370)):
        assert lib.h3_qkv_noalloc(16, 16, 16, 16, 16, 16, 16, 16, eps, 16, 16, 16, 16, 16, 16, 16, 100, heads,
                                  hidden, 0) == 0
        assert b"h3_qkv_noalloc" in lib.h3_int8_error()


@pytest.mark.gpu
@pytest.mark.parametrize("fault", ["B", "D", "KS", "VI_misaligned", "xs_misaligned"])
def test_noalloc_rejects_before_any_launch(device, fault):
    """A call with one bad operand (a null weight, output or scale buffer, or a
    misaligned one) is rejected on the host before the first of its five
    launches: it returns 0 and every sentinel-filled output stays as it was."""
    m, heads, hidden = 300, 2, 256
    q, w, xs, ws, rope, qw, kw = _inputs(m, heads, hidden, 77, device, 0.5)
    parts = (m + 127) // 128
    out = {
        "d": torch.full((3, heads, m, 128), -1, dtype=torch.int16, device=device).view(torch.bfloat16),
        "qi": torch.full((heads, m, 128), 7, dtype=torch.int8, device=device),
        "ki": torch.full((heads, m, 128), 7, dtype=torch.int8, device=device),
        "qs": torch.full((heads, parts * 32), -1.0, device=device),
        "ks": torch.full((heads, parts * 4), -1.0, device=device),
        "vp": torch.full((heads, parts, 128), -1.0, device=device),
        "vi": torch.full((heads * 128 * parts * 128 + 16,), 7, dtype=torch.int8, device=device),
        "vs": torch.full((heads * 128,), -1.0, device=device),
    }
    keep = {k: v.clone() for k, v in out.items()}
    xs_big = torch.zeros((m + 4,), device=device)
    xs_big[1:m + 1] = xs.view(-1)
    p = {k: v.data_ptr() for k, v in out.items()}
    b_ptr = None if fault == "B" else w.data_ptr()
    if fault == "D":
        p["d"] = None
    if fault == "KS":
        p["ks"] = None
    if fault == "VI_misaligned":
        p["vi"] += 1
    xs_ptr = xs_big.data_ptr() + 4 if fault == "xs_misaligned" else xs.data_ptr()
    if fault == "xs_misaligned":
        xs_ptr += 2   # FP32 scales two bytes off their alignment
    torch.cuda.synchronize()
    lib = _lib.load()
    rc = lib.h3_qkv_noalloc(q.data_ptr(), b_ptr, xs_ptr, ws.data_ptr(), p["d"], rope.data_ptr(), qw.data_ptr(),
                            kw.data_ptr(), ct.c_float(1e-6), p["qi"], p["qs"], p["vp"], p["ki"], p["ks"], p["vi"],
                            p["vs"], m, heads, hidden, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    assert lib.h3_int8_last_error() != 0 and lib.h3_int8_error()
    for k in out:
        assert _same(out[k], keep[k]), f"{k} was written by a rejected call"


@pytest.mark.parametrize("fault", ["B", "D", "KS", "VI_misaligned", "xs_misaligned", "A_misaligned", "eps"])
def test_noalloc_checks_run_before_any_cuda_call(fault):
    """The same rejections with stand-in pointer values on any host: each one is
    caught by a validation message before the entry point makes its first CUDA
    call (an accepted call would go on to look up the scratch address and, with
    no GPU, fail with a different message)."""
    lib = _lib.load()
    ptr = {k: 0x10000 * (i + 1) for i, k in enumerate(
        ("A", "B", "xs", "ws", "D", "freqs", "qw", "kw", "QI", "QS", "VP", "KI", "KS", "VI", "VS"))}
    eps = 1e-6
    if fault in ("B", "D", "KS"):
        ptr[fault] = None
    elif fault == "VI_misaligned":
        ptr["VI"] += 1
    elif fault == "xs_misaligned":
        ptr["xs"] += 2
    elif fault == "A_misaligned":
        ptr["A"] += 8
    else:
        eps = float("nan")
    rc = lib.h3_qkv_noalloc(ptr["A"], ptr["B"], ptr["xs"], ptr["ws"], ptr["D"], ptr["freqs"], ptr["qw"], ptr["kw"],
                            ct.c_float(eps), ptr["QI"], ptr["QS"], ptr["VP"], ptr["KI"], ptr["KS"], ptr["VI"],
                            ptr["VS"], 300, 2, 256, 0)
    assert rc == 0
    msg = lib.h3_int8_error().decode()
    assert "scratch address" not in msg and ("h3_qkv" in msg), msg
