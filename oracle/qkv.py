"""CPU restatement of the reference's QKV op.  TEST INFRASTRUCTURE ONLY.

The op (h3_speedkit/ops/qkv.py:24-83 of H3 SpeedKit) is five steps:
  1. gather the nine sample rows s*(m-1)//8 of q, xs and the RoPE table
     (r82_sample_konly.cu:345-357);
  2. the K plane of the QKV GEMM on those rows, RMS-normalised and roped
     (r82_sample_konly.cu:193-330, launched for M = 9);
  3. the K anchor detector on the nine sampled keys (r79_sample_anchor.cu:467-605);
  4. the full QKV GEMM with its fused head epilogue: Q/K normalised and roped,
     Q and K (centred on the anchor) rotated and quantised, V per-tile maxima
     (r84_kfourwarp.cu:193-375);
  5. the V quantiser on the V plane (h3_speedkit/ops/quant_v.py:57-110).
The arithmetic of each step lives in ``h3_oracle.c`` (h3o_qkv_heads,
h3o_sample_anchor, h3o_quant_v) with its documented departures (rsqrt and rcp
are hardware approximations on the GPU; here they are correctly rounded unless
the caller injects the GPU's rrms).  BF16 arrays are ``numpy.uint16`` bits.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from oracle import cpu

HEAD = 128          # channels per head
ROPE_PAIRS = 48     # rotated pairs (d, d + 48) per head; channels 96..127 are not rotated
SAMPLES = 9

_P, _I64 = ct.c_void_p, ct.c_int64
_SIGS = {
    "h3o_qkv_heads": ([_P, _I64, _I64, _P, _P, _P, ct.c_float, _P, _P, _P, ct.c_int, _P, _P, _P, _P, _P, _P, _P,
                       ct.c_int], None),
    "h3o_sample_anchor": ([_P, _I64, _P], None),
    "h3o_quant_v": ([_P, _I64, _I64, _P, _P, _P, ct.c_int], None),
}


def _lib():
    so = cpu.lib()
    for name, (args, res) in _SIGS.items():
        fn = getattr(so, name)
        fn.argtypes, fn.restype = args, res
    return so


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data


def sample_rows(m: int) -> list[int]:
    """r82_sample_konly.cu:347-349: row s*(m-1)/8 in int64 arithmetic."""
    return [s * (m - 1) // 8 for s in range(SAMPLES)]


def gather(q, xs, rope):
    """The nine sample rows of q [m, K] INT8, xs [m, 1] and rope [m, 192] (BF16 bits)."""
    rows = sample_rows(q.shape[0])
    return q[rows].copy(), xs[rows].copy(), rope[rows].copy()


def heads_epilogue(y, heads, freqs, qw, kw, eps, sk=None, anchors=None, *, planes=7, quant=True, rrms=None,
                   threads=None):
    """The fused head epilogue on the dequantised rows y [m, 3*heads*128] (BF16 bits).

    Returns a dict with d [3, heads, m, 128] (planes not requested stay zero), and
    for the requested planes qi, qs (Q), ki, ks (K), vp (V) and rrms [2, heads, m].
    ``quant=False`` is the sample form: normalised, roped rows only.
    """
    y = _c(y, np.uint16)
    m = y.shape[0]
    if y.shape[1] != 3 * heads * HEAD:
        raise ValueError("y must be [m, 3*heads*128]")
    parts = (m + 127) // 128
    d = np.zeros((3, heads, m, HEAD), np.uint16)
    out = {"d": d, "rrms": np.zeros((2, heads, m), np.float32)}
    if planes & 1 and quant:
        out["qi"] = np.zeros((heads, m, HEAD), np.int8)
        out["qs"] = np.zeros((heads, parts * 32), np.float32)
    if planes & 2 and quant:
        out["ki"] = np.zeros((heads, m, HEAD), np.int8)
        out["ks"] = np.zeros((heads, parts * 4), np.float32)
    if planes & 4 and quant:
        out["vp"] = np.zeros((heads, parts, HEAD), np.float32)
    if anchors is None:
        anchors = np.full((heads,), -1, np.int32)
    sk = None if sk is None else _c(sk, np.uint16)
    rr = None if rrms is None else _c(rrms, np.float32)
    _lib().h3o_qkv_heads(_ptr(y), m, heads, _ptr(_c(freqs, np.uint16)), _ptr(_c(qw, np.uint16)),
                         _ptr(_c(kw, np.uint16)), float(eps), _ptr(sk), _ptr(_c(anchors, np.int32)), _ptr(rr),
                         int(planes), _ptr(d), _ptr(out.get("qi")), _ptr(out.get("qs")), _ptr(out.get("ki")),
                         _ptr(out.get("ks")), _ptr(out.get("vp")), _ptr(out["rrms"]),
                         cpu.threads_default() if threads is None else threads)
    return out


def sample_anchor(k) -> np.ndarray:
    """Anchor row (0..8) or -1 per head from the sampled keys k [heads, 9, 128]."""
    k = _c(k, np.uint16)
    heads = k.shape[0]
    anchors = np.empty((heads,), np.int32)
    _lib().h3o_sample_anchor(_ptr(k), heads, _ptr(anchors))
    return anchors


def quant_v(v, vp, *, threads=None):
    """V plane v [heads, m, 128] (BF16 bits) and its tile maxima vp -> (vi, vs)."""
    v = _c(v, np.uint16)
    heads, m, _ = v.shape
    parts = (m + 127) // 128
    vi = np.empty((heads * HEAD, parts * 128), np.int8)
    vs = np.empty((heads * HEAD,), np.float32)
    _lib().h3o_quant_v(_ptr(v), m, heads, _ptr(_c(vp, np.float32)), _ptr(vi), _ptr(vs),
                       cpu.threads_default() if threads is None else threads)
    return vi, vs


def qkv(q, w, xs, ws, rope, qw, kw, eps, *, heads=None, rrms=None, sample_rrms=None, threads=None):
    """The whole op: returns a dict with sk [heads, 9, 128], anchors, d, qi, qs, ki,
    ks, vp, vi, vs.  q [m, K] INT8, w [3*heads*128, K] INT8, xs [m, 1], ws [N, 1],
    rope [m, 192] BF16 bits, qw / kw [128] BF16 bits."""
    q = _c(q, np.int8)
    w = _c(w, np.int8)
    m = q.shape[0]
    heads = w.shape[0] // (3 * HEAD) if heads is None else heads
    xs = _c(xs, np.float32).reshape(-1)
    ws = _c(ws, np.float32).reshape(-1)
    rope = _c(rope, np.uint16).reshape(m, 4 * ROPE_PAIRS)
    sq, sx, sr = gather(q, xs, rope)
    kplane = slice(heads * HEAD, 2 * heads * HEAD)
    ys = np.zeros((SAMPLES, 3 * heads * HEAD), np.uint16)
    ys[:, kplane] = cpu.dequant(cpu.gemm_s32(sq, w[kplane], threads=threads), sx, ws[kplane], threads=threads)
    sample = heads_epilogue(ys, heads, sr, qw, kw, eps, planes=2, quant=False, rrms=sample_rrms, threads=threads)
    sk = sample["d"][1]
    anchors = sample_anchor(sk)
    y = cpu.dequant(cpu.gemm_s32(q, w, threads=threads), xs, ws, threads=threads)
    out = heads_epilogue(y, heads, rope, qw, kw, eps, sk, anchors, planes=7, rrms=rrms, threads=threads)
    vi, vs = quant_v(out["d"][2], out["vp"], threads=threads)
    out.update(sk=sk, anchors=anchors, vi=vi, vs=vs, sample_rrms=sample["rrms"])
    return out
