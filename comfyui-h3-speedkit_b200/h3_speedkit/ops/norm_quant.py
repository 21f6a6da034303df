"""Preallocated, current-stream binding of the fused prologue (B200).

RMSNorm -> adaLN x*(1+scale)+shift -> ConvRot256 -> per-token INT8, one pass.
Drop-in for h3_speedkit/ops/norm_quant.py of H3 SpeedKit: the same class and
function names, argument meaning, validation messages and error behaviour
(``validate`` at :57-105, ``NormQuant`` at :108-146, ``Bound`` at :149-164), with
two deliberate differences: the hidden width K is taken from ``x`` (any
K % 256 == 0 up to 16384, reference: 5376 only) and the device must be a B200
(capability 10.0, reference: SM120).

The bound object owns the Torch tensors; rows are immutable after validation;
callers order producers before bind/launch.  Returned q/q_scale are the
prequantised Linear input.
"""
from __future__ import annotations

import ctypes as ct
import math

import torch

from .. import _lib

K = 5376                      # width of the reference geometry (unsuffixed C entry point)
MAX_K = 16384
DEVICE_CAPABILITY = (10, 0)   # B200


class Resources(ct.Structure):
    _fields_ = [(name, ct.c_int64) for name in (
        'abi', 'bytes', 'k', 'threads', 'warps', 'num_regs',
        'static_shared_bytes', 'local_bytes', 'active_blocks_per_sm',
        'sm_count', 'max_threads_per_sm', 'binary_version', 'ptx_version')]


def span(tensor):
    """Address interval [start, end) a strided tensor can touch."""
    if tensor.numel() == 0:
        return tensor.data_ptr(), tensor.data_ptr()
    last = sum((size - 1) * stride for size, stride in zip(tensor.shape, tensor.stride()))
    return tensor.data_ptr(), tensor.data_ptr() + (last + 1) * tensor.element_size()


def check_disjoint(inputs, outputs):
    """Outputs may overlap neither an input nor each other."""
    spans_out = [(name, *span(t)) for name, t in outputs]
    spans_in = [(name, *span(t)) for name, t in inputs]
    for i, (name, lo, hi) in enumerate(spans_out):
        for other, a, b in spans_in:
            if lo < b and a < hi:
                raise ValueError(f'Output {name} overlaps input {other}')
        for other, a, b in spans_out[:i]:
            if lo < b and a < hi:
                raise ValueError(f'Outputs {name} and {other} overlap')


def finite_bounded(tensor, rows=128):
    """Reject NaN/Inf, scanning 2-D tensors in bounded row chunks."""
    chunks = [tensor] if tensor.ndim < 2 else (tensor[i:i + rows] for i in range(0, tensor.shape[0], rows))
    for chunk in chunks:
        if not bool(torch.isfinite(chunk).all().item()):
            raise ValueError('Nonfinite input is outside the contract')


def validate(x, weight, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None,
             check_values=True, require_cuda=True):
    """Metadata checks; runnable on CPU tensors with require_cuda=False."""
    inputs = [('x', x), ('weight', weight), ('shift', shift), ('scale', scale), ('rows', rows)]
    outputs = [('q', q), ('q_scale', q_scale)]
    debug = (debug_norm, debug_rotated, debug_rstd)
    if any(t is not None for t in debug):
        if any(t is None for t in debug):
            raise ValueError('Debug requires norm, rotated, and rstd outputs together')
        outputs.extend(zip(('debug_norm', 'debug_rotated', 'debug_rstd'), debug))
    if any(type(t) is not torch.Tensor for _, t in inputs + outputs):
        raise ValueError('All operands must be original plain Torch tensors')
    if (require_cuda and not x.is_cuda) or any(t.device != x.device for _, t in inputs + outputs):
        raise ValueError('All operands must use one CUDA device')
    if any(t.requires_grad for _, t in inputs + outputs):
        raise ValueError('Inference only; detach only after validating model autograd policy')
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        raise ValueError('X requires BF16 [M,K], unit columns, XS % 4 == 0, 8B alignment')
    m, k = x.shape
    if (k % 256 or not 256 <= k <= MAX_K or not 1 <= m <= 0x7fffffff or x.stride(1) != 1
            or x.stride(0) < k or x.stride(0) % 4 or x.data_ptr() % 8):
        raise ValueError('X requires BF16 [M,K], unit columns, XS % 4 == 0, 8B alignment')

    def dense(name, t, shape, dtype, alignment):
        if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous() or t.data_ptr() % alignment:
            raise ValueError(f'{name} requires contiguous {dtype} {tuple(shape)} and {alignment}B alignment')

    dense('weight', weight, (k,), torch.bfloat16, 8)
    if (shift.ndim != 2 or shift.shape[1] != k or shift.shape[0] < 1
            or scale.shape != shift.shape or shift.dtype != scale.dtype
            or shift.dtype not in (torch.bfloat16, torch.float32)):
        raise ValueError(f'Tables require matching nonempty FP32/BF16 [T,{k}]')
    for t in (shift, scale):
        if t.stride(1) != 1 or t.stride(0) < k or t.data_ptr() % t.element_size():
            raise ValueError('Tables require dense hidden axes and nonoverlapping rows')
    dense('rows', rows, (m,), torch.int32, 4)
    dense('q', q, (m, k), torch.int8, 8)
    dense('q_scale', q_scale, (m, 1), torch.float32, 4)
    if debug_norm is not None:
        dense('debug_norm', debug_norm, (m, k), torch.bfloat16, 2)
        dense('debug_rotated', debug_rotated, (m, k), torch.float32, 4)
        dense('debug_rstd', debug_rstd, (m,), torch.float32, 4)
    tiny, big = torch.finfo(torch.float32).tiny, torch.finfo(torch.float32).max
    if not math.isfinite(float(eps)) or not tiny <= float(eps) <= big:
        raise ValueError('Epsilon must be finite, positive, normal FP32')
    check_disjoint(inputs, outputs)
    if check_values:
        if int(rows.min().item()) < 0 or int(rows.max().item()) >= shift.shape[0]:
            raise ValueError('Rows outside modulation table')
        for _, tensor in inputs[:4]:
            finite_bounded(tensor)
    return tuple(inputs), tuple(outputs)


class NormQuant:
    """ctypes front of h3_norm_quant_* (libh3sk_b200.so)."""

    def __init__(self, library=None):
        self.lib = _lib.load(library)
        self.path = _lib.library_path() if library is None else library
        if self.lib.h3_norm_quant_resources_size() != ct.sizeof(Resources):
            raise RuntimeError('NormQuant C/ctypes ABI mismatch')

    def check(self, code):
        if code:
            raise RuntimeError(f'NormQuant CUDA error {code}: ' + self.lib.h3_norm_quant_error(code).decode())

    def query(self, table_dtype=0, debug=0, k=K):
        data = Resources()
        self.check(self.lib.h3_norm_quant_query_k(k, table_dtype, debug, ct.byref(data), ct.sizeof(data)))
        return {name: int(getattr(data, name)) for name, _ in data._fields_}

    def bind(self, x, weight, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None, check_values=True):
        inputs, outputs = validate(x, weight, shift, scale, rows, q, q_scale, eps=eps,
                                   debug_norm=debug_norm, debug_rotated=debug_rotated,
                                   debug_rstd=debug_rstd, check_values=check_values)
        with torch.cuda.device(x.device):
            if torch.cuda.get_device_capability(x.device) != DEVICE_CAPABILITY:
                raise RuntimeError('Only the intended B200 (sm_100) device is supported')
            if torch.compiler.is_compiling():
                raise RuntimeError('NormQuant requires eager execution')
        pointers = [t.data_ptr() for t in (x, weight, shift, scale, rows, q, q_scale)]
        pointers += [t.data_ptr() if t is not None else None for t in (debug_norm, debug_rotated, debug_rstd)]
        args = pointers + [x.shape[0], x.shape[1], shift.shape[0], x.stride(0), shift.stride(0), scale.stride(0),
                           float(eps), int(shift.dtype == torch.bfloat16), int(debug_norm is not None)]
        return Bound(self, x.device, inputs, outputs, args, (q, q_scale))


class Bound:
    """A validated launch: owns its tensors, records allocator stream use."""

    def __init__(self, library, device, inputs, outputs, args, result):
        self.library, self.device, self.inputs, self.outputs = library, device, inputs, outputs
        self.args, self.result = args, result
        self.owners = tuple(t for _, t in inputs + outputs)

    def __call__(self):
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            for owner in self.owners:
                owner.record_stream(stream)
            code = self.library.lib.h3_norm_quant_run_t(*self.args, stream.cuda_stream)
            # Stores may already be queued when an error is reported: never retried.
            torch.autograd.graph.increment_version(tuple(t for _, t in self.outputs))
            self.library.check(code)
        return self.result
