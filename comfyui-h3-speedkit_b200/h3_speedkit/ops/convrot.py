"""Preallocated, current-stream bindings of the ConvRot256 INT8 quantiser (B200).

``ConvRotRegister`` stands in for h3_speedkit/ops/convrot.py of H3 SpeedKit
(:39-111): same modes (0 production, 1 diagnostic, 2 rotation oracle), same
error texts and error behaviour, any K % 256 == 0 up to 16384 (reference: 5376
and 7168) on a B200.  Its operand checks are a rule table (see ``_contract``).

``quantize_int8_rowwise_convrot64`` replaces the Kitchen call the reference's
block makes for the FC2 input, ``cuda.quantize_int8_rowwise_convrot64(hidden,
256, input_act=...)`` (runtime.py:159), with input activations none / gelu_tanh /
swiglu, and accepts a strided row view (used for the V slice of a QKV output).
"""
from __future__ import annotations

import ctypes as ct

import torch

from .. import _lib
from ._contract import INT32_MAX, Call, Launch, Rule, all_finite, enforce, first_overlap
from .norm_quant import DEVICE_CAPABILITY, MAX_K

ACT_CODES = {None: 0, 'none': 0, 'gelu_tanh': 1, 'gelu': 1, 'swiglu': 2}


class Resources(ct.Structure):
    """h3_convrot_register_query's report (field order of convrot_register_v2.cu:140-144)."""
    _fields_ = [(n, ct.c_int64) for n in (
        'abi', 'bytes', 'k', 'threads', 'warps', 'num_regs', 'static_shared_bytes',
        'local_bytes', 'max_threads_per_block', 'active_blocks_per_sm',
        'sm_count', 'max_threads_per_sm', 'binary_version', 'ptx_version')]


def finite_bounded(x, rows=128):
    if rows < 1:
        raise ValueError('finite-check row chunk must be positive')
    if not all_finite(x, rows):
        raise ValueError('NaN/Inf lies outside this finite-input replay contract')


def _buffer_rules(name, shape, dtype):
    """A dense, element-aligned CUDA buffer `name` of `dtype` and shape(call) on x's device."""
    def placed(c):
        t = c[name]
        return (isinstance(t, torch.Tensor) and tuple(t.shape) == tuple(shape(c)) and t.dtype == dtype
                and t.is_cuda and t.device == c['x'].device and t.is_contiguous())
    return [Rule(placed, lambda c: f"{name} requires contiguous {dtype} {tuple(shape(c))} on {c['x'].device}"),
            Rule(lambda c: c[name].data_ptr() % c[name].element_size() == 0, f'{name} is not element-aligned')]


def _when(pred, rules):
    return [Rule(lambda c, r=r: not pred(c) or r.ok(c), r.message) for r in rules]


def _x_dims(c):
    x = c['x']
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.bfloat16 and x.ndim == 2
            and x.is_contiguous()):
        return False
    c.dims.update(m=x.shape[0], k=x.shape[1])
    return True


_MK = lambda c: (c.dims['m'], c.dims['k'])
_M1 = lambda c: (c.dims['m'], 1)

RULES = [
    Rule(_x_dims, 'X requires contiguous CUDA BF16 [M,K]'),
    Rule(lambda c: 1 <= c.dims['m'] <= INT32_MAX and c.dims['k'] % 256 == 0 and 256 <= c.dims['k'] <= MAX_K
         and c.dims['act_code'] == 0,
         f'Only M=1..INT32_MAX, K%256==0 (<= {MAX_K}), ACT=none is supported'),
    Rule(lambda c: c.dims['mode'] in (0, 1, 2), 'Mode must be production=0, diagnostic=1 or oracle=2'),
    *_buffer_rules('x', _MK, torch.bfloat16),
    Rule(lambda c: c['x'].data_ptr() % 16 == 0, 'x must be 16-byte aligned'),
    *_when(lambda c: c.dims['mode'] != 2,
           _buffer_rules('q', _MK, torch.int8) + _buffer_rules('scale', _M1, torch.float32)),
    Rule(lambda c: c.dims['mode'] != 2 or (c['q'] is None and c['scale'] is None),
         'Oracle mode accepts only X and rotated output'),
    *_when(lambda c: c.dims['mode'] != 0, _buffer_rules('rotated', _MK, torch.float32)),
    Rule(lambda c: c.dims['mode'] != 0 or c['rotated'] is None, 'Production mode does not accept rotated output'),
]


def _disjoint(c):
    """Every present buffer must own its bytes (x included: it is never written,
    but an output over it would be read after it is written)."""
    bufs = [(n, c[n]) for n in ('x', 'q', 'scale', 'rotated') if c[n] is not None]
    hit = first_overlap([], bufs)
    if hit is not None:
        raise ValueError(f'Overlapping buffers: {hit[1]} and {hit[0]}')


def _check_device(device):
    with torch.cuda.device(device):
        if torch.cuda.get_device_capability(device) != DEVICE_CAPABILITY:
            raise RuntimeError('This binary is restricted to B200 (sm_100)')


class ConvRotRegister:
    """ctypes front of h3_convrot_register_* (libh3sk_b200.so)."""

    def __init__(self, library=None):
        self.lib = _lib.load(library)
        if self.lib.h3_convrot_register_resources_size() != ct.sizeof(Resources):
            raise RuntimeError('C/ctypes resource layout mismatch')

    def check(self, code):
        if code:
            raise RuntimeError(f'ConvRot CUDA error {code}: ' + self.lib.h3_convrot_register_error(code).decode())

    def query(self, k):
        report = Resources()
        self.check(self.lib.h3_convrot_register_query(k, ct.byref(report), ct.sizeof(report)))
        values = {n: int(getattr(report, n)) for n, _ in report._fields_}
        values['active_warps_per_sm'] = values['active_blocks_per_sm'] * values['warps']
        values['theoretical_occupancy'] = (values['active_blocks_per_sm'] * values['threads']
                                           / values['max_threads_per_sm'])
        return values

    def bind(self, x, q=None, scale=None, *, rotated=None, mode=0, act_code=0, check_finite=True):
        call = Call({'x': x, 'q': q, 'scale': scale, 'rotated': rotated}, {'mode': mode, 'act_code': act_code})
        enforce(RULES, call)
        _disjoint(call)
        _check_device(x.device)
        if check_finite:
            finite_bounded(x)
        launch = Bound(self.lib.h3_convrot_register_run, x.device,
                       [None if t is None else t.data_ptr() for t in (x, q, scale, rotated)] + [*x.shape, mode],
                       (x, q, scale, rotated), (q, scale, rotated),
                       rotated if mode == 2 else (q, scale), self.check)
        launch.mode, launch.resources = mode, self.query(x.shape[1])
        return launch


Bound = Launch


def quantize_int8_rowwise_convrot64(x, groupsize=256, input_act=None, *, out=None, out_scale=None):
    """ConvRot256 + per-token INT8 of a BF16 [M, W] row view, with an optional
    input activation absorbed on the way in.

    W = K, or 2K for ``input_act='swiglu'`` ([gate | up] rows).  ``x`` may be a
    column slice of a wider tensor (row stride a multiple of 8 elements, 16-byte
    aligned start).  Returns (q INT8 [M, K], scale FP32 [M, 1]).
    """
    if groupsize != 256:
        raise ValueError('ConvRot group size must be 256')
    act = ACT_CODES.get(input_act)
    if act is None:
        raise ValueError(f'Unsupported input_act {input_act!r}')
    if not isinstance(x, torch.Tensor) or x.dtype != torch.bfloat16 or x.ndim != 2 or not x.is_cuda:
        raise ValueError('x requires a CUDA BF16 [M, W] tensor')
    m, width = x.shape
    k = width // 2 if act == 2 else width
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16 or (act == 2 and width % 2):
        raise ValueError('x requires unit columns, row stride % 8 == 0 and 16-byte alignment')
    if k % 256 or not 256 <= k <= MAX_K or m < 1:
        raise ValueError(f'K must be a multiple of 256 in [256, {MAX_K}]')
    q = torch.empty((m, k), dtype=torch.int8, device=x.device) if out is None else out
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device) if out_scale is None else out_scale
    outputs = Call({'x': x, 'q': q, 'scale': s}, {'m': m, 'k': k})
    enforce(_buffer_rules('q', _MK, torch.int8) + _buffer_rules('scale', _M1, torch.float32), outputs)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device)
        code = lib.h3_convrot_quant_act(x.data_ptr(), x.stride(0), q.data_ptr(), s.data_ptr(), m, k, act,
                                        stream.cuda_stream)
    if code:
        raise RuntimeError(f'ConvRot CUDA error {code}: ' + lib.h3_convrot_register_error(code).decode())
    return q, s
