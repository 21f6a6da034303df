"""Preallocated, current-stream bindings of the ConvRot256 INT8 quantiser (B200).

``ConvRotRegister`` is the drop-in for h3_speedkit/ops/convrot.py of H3 SpeedKit
(:39-111): same modes (0 production, 1 diagnostic, 2 rotation oracle), same
validation and error behaviour, any K % 256 == 0 up to 16384 (reference: 5376
and 7168) on a B200.

``quantize_int8_rowwise_convrot64`` replaces the Kitchen call the reference's
block makes for the FC2 input, ``cuda.quantize_int8_rowwise_convrot64(hidden,
256, input_act=...)`` (runtime.py:159), with input activations none / gelu_tanh /
swiglu, and accepts a strided row view (used for the V slice of a QKV output).
"""
from __future__ import annotations

import ctypes as ct

import torch

from .. import _lib
from .norm_quant import DEVICE_CAPABILITY, MAX_K

ACT_CODES = {None: 0, 'none': 0, 'gelu_tanh': 1, 'gelu': 1, 'swiglu': 2}


class Resources(ct.Structure):
    _fields_ = [(n, ct.c_int64) for n in (
        'abi', 'bytes', 'k', 'threads', 'warps', 'num_regs', 'static_shared_bytes',
        'local_bytes', 'max_threads_per_block', 'active_blocks_per_sm',
        'sm_count', 'max_threads_per_sm', 'binary_version', 'ptx_version')]


def finite_bounded(x, rows=128):
    if rows < 1:
        raise ValueError('finite-check row chunk must be positive')
    for start in range(0, x.shape[0], rows):
        if not bool(torch.isfinite(x[start:start + rows]).all().item()):
            raise ValueError('NaN/Inf lies outside this finite-input replay contract')


def _validate(t, shape, dtype, device, name):
    if (not isinstance(t, torch.Tensor) or tuple(t.shape) != tuple(shape) or t.dtype != dtype
            or not t.is_cuda or t.device != device or not t.is_contiguous()):
        raise ValueError(f'{name} requires contiguous {dtype} {tuple(shape)} on {device}')
    if t.data_ptr() % t.element_size():
        raise ValueError(f'{name} is not element-aligned')


def _no_alias(tensors):
    spans = sorted((t.data_ptr(), t.data_ptr() + t.numel() * t.element_size(), n)
                   for n, t in tensors if t is not None)
    for left, right in zip(spans, spans[1:]):
        if left[1] > right[0]:
            raise ValueError(f'Overlapping buffers: {left[2]} and {right[2]}')


def _check_device(device):
    with torch.cuda.device(device):
        if torch.cuda.get_device_capability(device) != DEVICE_CAPABILITY:
            raise RuntimeError('This binary is restricted to B200 (sm_100)')


class ConvRotRegister:
    def __init__(self, library=None):
        self.lib = _lib.load(library)
        if self.lib.h3_convrot_register_resources_size() != ct.sizeof(Resources):
            raise RuntimeError('C/ctypes resource layout mismatch')

    def check(self, code):
        if code:
            raise RuntimeError(f'ConvRot CUDA error {code}: ' + self.lib.h3_convrot_register_error(code).decode())

    def query(self, k):
        resource = Resources()
        self.check(self.lib.h3_convrot_register_query(k, ct.byref(resource), ct.sizeof(resource)))
        values = {n: int(getattr(resource, n)) for n, _ in resource._fields_}
        values['active_warps_per_sm'] = values['active_blocks_per_sm'] * values['warps']
        values['theoretical_occupancy'] = (values['active_blocks_per_sm'] * values['threads']
                                           / values['max_threads_per_sm'])
        return values

    def bind(self, x, q=None, scale=None, *, rotated=None, mode=0, act_code=0, check_finite=True):
        if (not isinstance(x, torch.Tensor) or not x.is_cuda or x.dtype != torch.bfloat16
                or x.ndim != 2 or not x.is_contiguous()):
            raise ValueError('X requires contiguous CUDA BF16 [M,K]')
        m, k = x.shape
        if m < 1 or m > 0x7fffffff or k % 256 or not 256 <= k <= MAX_K or act_code != 0:
            raise ValueError(f'Only M=1..INT32_MAX, K%256==0 (<= {MAX_K}), ACT=none is supported')
        if mode not in (0, 1, 2):
            raise ValueError('Mode must be production=0, diagnostic=1 or oracle=2')
        _validate(x, (m, k), torch.bfloat16, x.device, 'x')
        if x.data_ptr() % 16:
            raise ValueError('x must be 16-byte aligned')
        if mode != 2:
            _validate(q, (m, k), torch.int8, x.device, 'q')
            _validate(scale, (m, 1), torch.float32, x.device, 'scale')
        elif q is not None or scale is not None:
            raise ValueError('Oracle mode accepts only X and rotated output')
        if mode != 0:
            _validate(rotated, (m, k), torch.float32, x.device, 'rotated')
        elif rotated is not None:
            raise ValueError('Production mode does not accept rotated output')
        _no_alias([('x', x), ('q', q), ('scale', scale), ('rotated', rotated)])
        _check_device(x.device)
        if check_finite:
            finite_bounded(x)
        return Bound(self, x, q, scale, rotated, mode, self.query(k))


class Bound:
    """Owns tensor refs and records allocator stream use; caller orders producers."""

    def __init__(self, library, x, q, scale, rotated, mode, resources):
        self.library, self.x, self.q, self.scale = library, x, q, scale
        self.rotated, self.mode, self.resources = rotated, mode, resources
        self.owners = tuple(t for t in (x, q, scale, rotated) if t is not None)
        self.pointers = tuple(t.data_ptr() if t is not None else None for t in (x, q, scale, rotated))

    def __call__(self):
        with torch.cuda.device(self.x.device):
            stream = torch.cuda.current_stream(self.x.device)
            for owner in self.owners:
                owner.record_stream(stream)
            self.library.check(self.library.lib.h3_convrot_register_run(
                *self.pointers, *self.x.shape, self.mode, stream.cuda_stream))
        return self.rotated if self.mode == 2 else (self.q, self.scale)


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
    _validate(q, (m, k), torch.int8, x.device, 'q')
    _validate(s, (m, 1), torch.float32, x.device, 'scale')
    lib = _lib.load()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device)
        code = lib.h3_convrot_quant_act(x.data_ptr(), x.stride(0), q.data_ptr(), s.data_ptr(), m, k, act,
                                        stream.cuda_stream)
    if code:
        raise RuntimeError(f'ConvRot CUDA error {code}: ' + lib.h3_convrot_register_error(code).decode())
    return q, s
